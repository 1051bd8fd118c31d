"""Benchmark: train samples/s of the full MLP step (forward + backward + update)
on 1..8 B200, with the roofline of the dominant kernel and the CPU baseline.

Default workload: the wide MLP
4096 -> 8192 -> 8192 -> 8192 -> 1000, ReLU, softmax-CE, bf16 operands with f32
accumulate and f32 master weights, Adam(lr 1e-3), batch 8192 per GPU
(weak scaling: at 8 GPUs the global batch is 65536, configs[4]).  Synthetic
seeded data: X ~ N(0,1), labels uniform in [0,1000), Kaiming-uniform W, zero b.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config wide|small] [--global-batch B]

Multi-GPU: launch one process per GPU with torch.distributed.run; dW/db are
summed with NCCL inside the captured step (rt_mlp_set_comm).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # wide MLP, bf16/f32-acc, Adam 1e-3, batch 8192 per GPU
    "wide": dict(dims=[4096, 8192, 8192, 8192, 1000], batch=8192, dtype="bf16", optimizer="adam", lr=1e-3),
    # 512 -> 1024 -> 1024 -> 10, f32, SGD 0.01, batch 2048
    "small": dict(dims=[512, 1024, 1024, 10], batch=2048, dtype="f32", optimizer="sgd", lr=0.01),
    # profiling case for ncu: one 8192 -> 8192 layer of the wide MLP (its
    # step is a forward GEMM, the softmax-CE and one dW GEMM with the Adam
    # update fused into its epilogue), 1.6 GB on the device
    "probe_dw": dict(dims=[8192, 8192], batch=8192, dtype="bf16", optimizer="adam", lr=1e-3),
}
# the fixed global batch of the strong-scaling leg
STRONG_GLOBAL_BATCH = 65536
# Rows of the one-thread CPU baseline step (the full batch where that is quick)
CPU_SAMPLE_ROWS = {"wide": 256, "small": 2048, "probe_dw": 256}
# DRAM bytes (read + write) per launch of the step's dominant kernels, each
# from one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of an
# 8192 x 8192 x 8192 launch (2 * 8192^3 algorithmic FLOPs), scaled to the
# step's launches of that label by their FLOPs (every such launch of the wide
# step has k = 8192, so its bytes grow with its FLOPs):
#   dw_gemm       `bench.py --gemm TN --mnk 8192 8192 8192` (plain dW GEMM)
#   dw_gemm_adam  the dW GEMM of `bench.py --config probe_dw` (Adam fused in
#                 the epilogue; the [W; b] block of one 8192 -> 8192 layer)
#   fwd_gemm_bias_relu_split  `bench.py --gemm NN --split --mnk 8192 8192 8192`
#                 (A as bf16 hi + lo planes, bias + ReLU, bf16 output with its
#                 lo plane: the forward GEMM of a hidden layer that feeds another)
TRAFFIC_PER_LAUNCH = {
    "dw_gemm": (1.099e9 + 0.251e9, "bench.py --gemm TN --mnk 8192 8192 8192"),
    "dw_gemm_adam": (2.087e9 + 1.182e9, "the dW launch of bench.py --config probe_dw"),
    "fwd_gemm_bias_relu_split": (1.742e9 + 0.255e9, "bench.py --gemm NN --split --mnk 8192 8192 8192"),
}
TRAFFIC_FLOPS = 2.0 * 8192 ** 3


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"], bf16_sus=d.get("bf16_tflops_sustained"),
                    source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, source="fallback")


def exact_flops(dims, n):
    """fwd + dW for every layer, dX for every layer but the first."""
    f = 0
    for l in range(len(dims) - 1):
        dm = dims[l] * dims[l + 1]
        f += 4 * n * dm
        if l > 0:
            f += 2 * n * dm
    return float(f)


def make_weights(cfg, seed):
    """Kaiming-uniform W, zero b (bf16 configs: W rounded to bf16 values, the
    configs' bf16 weights; the f32 masters start equal to their shadows)."""
    rng = np.random.default_rng(seed)
    dims = cfg["dims"]
    params = []
    for l in range(len(dims) - 1):
        lim = np.float32(np.sqrt(6.0 / dims[l]))
        w = rng.uniform(-lim, lim, size=(dims[l], dims[l + 1])).astype(np.float32)
        if cfg["dtype"] == "bf16":
            w = bf16_values(w)
        params.append(w)
        params.append(np.zeros((1, dims[l + 1]), np.float32))
    return params


def make_data(cfg, rows, seed):
    """X ~ N(0,1) (bf16 values for bf16 configs), labels uniform in [0, classes)."""
    rng = np.random.default_rng(seed)
    dims = cfg["dims"]
    x = rng.standard_normal((rows, dims[0]), dtype=np.float32)
    if cfg["dtype"] == "bf16":
        x = bf16_values(x)
    labels = rng.integers(0, dims[-1], size=rows, dtype=np.uint32)
    return x, labels


def make_inputs(cfg, rows, seed):
    x, labels = make_data(cfg, rows, seed + 1)
    return make_weights(cfg, seed), x, labels


def bf16_values(a):
    """Nearest-even bf16 value of each f32 element, as f32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32).reshape(a.shape)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region.

    nvidia-smi takes a while to print its first sample, so the sampler is
    started before the warm-up and waits for that first line; every sample is
    time-stamped on arrival and only those between mark_start() and stop()
    are kept (the window is widened to the warm-up when the timed region is
    too short to hold one)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []
        self.t_open = self.t0 = None

    def start(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return

        def reader():
            for line in self.proc.stdout:
                self.lines.append((time.monotonic(), line))

        threading.Thread(target=reader, daemon=True).start()
        t_end = time.monotonic() + 10.0
        while not self.lines and time.monotonic() < t_end and self.proc.poll() is None:
            time.sleep(0.02)
        self.t_open = time.monotonic()

    def mark_start(self):
        self.t0 = time.monotonic()

    def stop(self):
        if not self.proc:
            return None
        t1 = time.monotonic()
        time.sleep(0.06)  # the sample that covers the region's last moments
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        window = "timed"
        lines = [ln for t, ln in self.lines if self.t0 is not None and self.t0 <= t <= t1 + 0.06]
        if not lines:
            window = "warm-up and timed"
            lines = [ln for t, ln in self.lines if self.t_open is not None and self.t_open <= t <= t1 + 0.06]
        sm, mx, reasons = [], None, set()
        for line in lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for name, v in zip(self.NAMES, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "window": window}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


class CpuStep:
    """rtensor's CPU train step (the oracle's C++ restatement of the
    reference's CPU backend: forward, tape backward, optimiser) of the
    config's whole model on `rows` rows, on `threads` host threads.  Every
    timed step is a real step; nothing is extrapolated."""

    def __init__(self, cfg, rows, threads):
        import oracle

        self.O = oracle
        self.cfg = cfg
        self.rows = min(rows, cfg["batch"])
        self.threads = threads
        params, self.x, self.labels = make_inputs(cfg, self.rows, 99)
        self.nparams = sum(p.size for p in params)
        self.m = oracle.Mlp(cfg["dims"])
        self.m.set_params(params)
        self.opt = oracle.OPT_ADAM if cfg["optimizer"] == "adam" else oracle.OPT_SGD

    def step(self, rows=None):
        n = self.rows if rows is None else rows
        t0 = time.perf_counter()
        self.m.train_step(self.x[:n], self.labels[:n], self.opt, self.cfg["lr"], threads=self.threads)
        return time.perf_counter() - t0

    def describe(self):
        part = "the full batch" if self.rows >= self.cfg["batch"] else f"a {self.rows}-row sample of the {self.cfg['batch']}-row batch"
        return (f"one train step of the whole model on {part} (forward, tape backward, {self.cfg['optimizer']} over all "
                f"{self.nparams} parameters), {self.threads} thread{'s' if self.threads > 1 else ''}")


def cpu_baseline(cfg_name, cfg):
    """The reference CPU step timed on this host: the primary figure on one
    thread (rtensor's CPU backend is single-threaded) on a bounded sample of
    rows, and a secondary full-batch step on every host thread (the oracle
    splits each matmul's rows; per-element summation order, and so the
    result, is unchanged, but the threading is not the reference's)."""
    host_threads = os.cpu_count() or 1
    one = CpuStep(cfg, CPU_SAMPLE_ROWS[cfg_name], 1)
    one.step(min(64, one.rows))  # warm-up: pages in weights and moments
    t1 = min(one.step() for _ in range(2))
    out = {"value": one.rows / t1, "unit": "samples/s", "cores": 1, "kind": "port",
           "sample": f"{one.describe()}; {t1:.2f} s per step, best of 2 after a warm-up step",
           "cpu_model": cpu_model(), "host_threads": host_threads}
    del one
    if host_threads > 1:
        full = CpuStep(cfg, cfg["batch"], host_threads)
        full.step(min(64, full.rows))
        tf = full.step()
        out["all_threads"] = {"value": full.rows / tf, "unit": "samples/s", "cores": host_threads,
                              "label": "non-reference (multi-threaded oracle; the reference CPU backend uses 1 thread)",
                              "sample": f"{full.describe()}; {tf:.1f} s for the step"}
    return out


# The reference arm's full-batch steps stop once another would end past this
# many seconds of stepping (at least one step always runs).
REFERENCE_BUDGET_S = 150.0


def run_reference(args, cfg_name, cfg, rank):
    """--impl reference: the reference's CPU implementation of the step (the
    oracle port: the Rust crate cannot be built here) on every host thread,
    on the arm's config.  Each timed step is a full-batch step; as many run
    as --steps asks for or REFERENCE_BUDGET_S allows, and the line reports how
    many did."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    c = CpuStep(cfg, cfg["batch"], threads)
    c.step(min(64, c.rows))  # warm-up: a 64-row step pages in weights and moments
    times = []
    t_start = time.perf_counter()
    while len(times) < args.steps:
        times.append(c.step())
        spent = time.perf_counter() - t_start
        if spent + times[-1] > REFERENCE_BUDGET_S:
            break
    sec = sum(times) / len(times)
    value = c.rows / sec
    line = {
        "impl": "reference", "metric": "train samples/sec (fwd+bwd+update)", "value": value,
        "unit": "samples/s", "n_gpus": args.gpus, "steps": len(times), "steps_requested": args.steps,
        "warmup": 1, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": config_dict(cfg_name, cfg, args.gpus, cfg["batch"] * args.gpus),
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                         "sample": (f"{c.describe()}; {len(times)} timed full-batch steps "
                                    f"({'all requested' if len(times) == args.steps else f'the {REFERENCE_BUDGET_S:.0f} s budget'}), "
                                    "after one 64-row warm-up step"),
                         "cpu_model": cpu_model()},
        "timed_region_s": sum(times),
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_gemm_only(args):
    """One tensor-core GEMM repeated `reps` times (the small case for ncu
    captures of the dominant kernel).  Operands are N(0,1) bf16 (or f32 on the
    3xTF32 path with --gemm-dtype f32); the output is bf16 except for TN and
    f32 operands."""
    import torch

    import rgpu_b200

    m, n, k = args.mnk
    gpu = rgpu_b200.Gpu(0)
    if args.l2_group:
        gpu.set_grupo_l2(args.l2_group)
    rng = np.random.default_rng(0)
    shape_a = (k, m) if args.gemm == "TN" else (m, k)
    shape_b = (n, k) if args.gemm == "NT" else (k, n)
    if args.split:
        # the split-activation forward GEMM of a hidden layer: A as bf16 hi
        # and lo planes, bias + ReLU, bf16 output with its lo plane
        from rgpu_b200 import gpu as G

        assert args.gemm == "NN" and args.gemm_dtype == "bf16", "--split profiles the NN bf16 forward GEMM"
        xa = np.maximum(rng.standard_normal(shape_a, dtype=np.float32), 0)
        hi = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(xa))
        a, a_lo = gpu.upload(hi, "bf16"), gpu.upload(xa - hi, "bf16")
        b = gpu.upload(rng.standard_normal(shape_b, dtype=np.float32) * np.float32(0.01), "bf16")
        bias = gpu.upload(np.zeros((1, n), np.float32))
        c, c_lo = gpu.zeros((m, n), "bf16"), gpu.zeros((m, n), "bf16")
        args_g = G.GemmArgs(G.RT_NN, G.RT_BF16, G.RT_BF16, m, n, k, a.ptr, a.ld, b.ptr, b.ld, c.ptr, c.ld,
                            G.RT_EPI_BIAS_RELU, bias.ptr, None, 0, 1, None, 0)
        args_g.a_lo, args_g.c_lo = a_lo.ptr, c_lo.ptr

        def fn(*_):
            gpu.gemm(args_g)
    else:
        a = gpu.upload(rng.standard_normal(shape_a, dtype=np.float32), args.gemm_dtype)
        b = gpu.upload(rng.standard_normal(shape_b, dtype=np.float32), args.gemm_dtype)
        c = gpu.zeros((m, n), "f32" if args.gemm == "TN" or args.gemm_dtype == "f32" else "bf16")
        fn = {"NN": gpu.matmul, "NT": gpu.matmul_a_bt, "TN": gpu.matmul_at_b}[args.gemm]
    fn(a, b, c)
    gpu.sync()
    st = torch.cuda.ExternalStream(gpu.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        torch.cuda._sleep(20000000)  # the host enqueues the timed launches meanwhile
    e0.record(st)
    for _ in range(args.reps):
        fn(a, b, c)
    e1.record(st)
    gpu.sync()
    ms = e0.elapsed_time(e1) / args.reps
    mma_flops = 2.0 * m * n * k * (2 if args.split else 1)
    print(json.dumps({"gemm": args.gemm, "dtype": args.gemm_dtype, "split": bool(args.split), "m": m, "n": n, "k": k,
                      "ms": ms, "tflops": 2.0 * m * n * k / (ms / 1e3) / 1e12,
                      "tensor_tflops": mma_flops / (ms / 1e3) / 1e12}), flush=True)
    gpu.close()


SWEEP_M = (1024, 4096, 8192)
SWEEP_N = (512, 4096, 8192)
SWEEP_K = (1, 8, 32, 128, 512, 2048, 16384)


def run_dw_sweep(args):
    """dW = X^T dY in isolation (rt_gemm, layout TN) over
    M in {1024,4096,8192} x N in {512,4096,8192} x K (the batch) in
    {1,...,16384}, f32 (3xTF32 tensor cores) and bf16 operands, f32 output,
    split-K chosen by the library.  Entries N(0,1).  Each point is timed with
    CUDA events around the GEMM alone, with L2 flushed before every
    repetition: a 256 MB write, then a 256 MB read of another buffer, so the
    GEMM starts from a cold L2 that holds no dirty lines (a write flush alone
    leaves ~126 MB to be written back during the GEMM, a 50 % surcharge on
    the output-write-bound small-K points).  Roofline time = max(2MNK / peak,
    ((M+N) K s_in + 4 M N) / HBM); the f32 peak is the bf16 figure / 2 (tf32
    rate) / 3 (three products).  Each timed span holds one rt_gemm call: the
    operand split (f32), the GEMM and the split-K reduction when it splits."""
    import torch

    import rgpu_b200
    from rgpu_b200 import gpu as G

    pk = peaks()
    gpu = rgpu_b200.Gpu(0)
    dev = torch.device("cuda", 0)
    st = torch.cuda.ExternalStream(gpu.stream(), device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    flush_sum = torch.empty((), dtype=torch.float32, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    dtypes = args.sweep_dtypes.split(",")
    ks = [int(k) for k in args.sweep_k.split(",")] if args.sweep_k else SWEEP_K
    points = []
    for dt in dtypes:
        tdt = torch.bfloat16 if dt == "bf16" else torch.float32
        s_in = 2 if dt == "bf16" else 4
        peak = pk["bf16"] if dt == "bf16" else pk["bf16"] / 6.0
        for m in SWEEP_M:
            for n in SWEEP_N:
                for k in ks:
                    x = torch.randn((k, m), generator=gen, device=dev, dtype=torch.float32).to(tdt)
                    dy = torch.randn((k, n), generator=gen, device=dev, dtype=torch.float32).to(tdt)
                    c = torch.empty((m, n), device=dev, dtype=torch.float32)
                    a = G.GemmArgs()
                    a.layout, a.in_dtype, a.out_dtype = G.RT_TN, G.RT_BF16 if dt == "bf16" else G.RT_F32, G.RT_F32
                    a.m, a.n, a.k = m, n, k
                    a.a, a.lda, a.b, a.ldb, a.c, a.ldc = x.data_ptr(), m, dy.data_ptr(), n, c.data_ptr(), n
                    a.split_k = 0
                    wsb = gpu.gemm_workspace_size(a)
                    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
                    a.workspace, a.workspace_bytes = ws.data_ptr(), wsb
                    torch.cuda.synchronize()
                    for _ in range(2):
                        gpu.gemm(a)
                    gpu.sync()
                    flops = 2.0 * m * n * k
                    reps = max(3, min(20, int(2e12 / max(flops, 1.0))))
                    # flush, event, GEMM, event on the library's stream, all
                    # enqueued behind a device sleep: the GPU starts only once
                    # the host has enqueued every repetition, so host-side
                    # launch cost stays out of the timed spans
                    evs = []
                    with torch.cuda.stream(st):
                        torch.cuda._sleep(40000000)
                        for _ in range(reps):
                            flush.fill_(1)
                            torch.sum(flush_rd, dim=None, out=flush_sum)
                            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                            e0.record(st)
                            gpu.gemm(a)
                            e1.record(st)
                            evs.append((e0, e1))
                    gpu.sync()
                    torch.cuda.synchronize()
                    ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs)
                    byts = (m + n) * k * s_in + 4.0 * m * n
                    roof_ms = max(flops / (peak * 1e12), byts / (pk["hbm"] * 1e9)) * 1e3
                    pt = {"dtype": dt, "M": m, "N": n, "K": k, "ms": round(ms, 5),
                          "tflops": round(flops / (ms / 1e3) / 1e12, 2),
                          "gbs": round(byts / (ms / 1e3) / 1e9, 1), "roofline_ms": round(roof_ms, 5),
                          "frac": round(roof_ms / ms, 3),
                          "bound": "tensor" if flops / (peak * 1e12) > byts / (pk["hbm"] * 1e9) else "hbm",
                          "workspace_bytes": wsb}
                    points.append(pt)
                    print(json.dumps(pt), flush=True)
                    del x, dy, c, ws
    for dt in dtypes:
        fr = [p["frac"] for p in points if p["dtype"] == dt]
        if fr:
            print(json.dumps({"summary": dt, "points": len(fr), "frac_median": statistics.median(fr),
                              "frac_min": min(fr), "peak_source": pk["source"]}), flush=True)
    gpu.close()


def run_op(args):
    """One HBM-bound kernel of the step on its own (the small case for ncu
    captures of the elementwise kernels): `adam` updates an [rows, cols] f32
    parameter (30 algorithmic bytes per element: theta, m, v, g read; theta, m,
    v written; no shadow here, so 28), `xent` is the softmax-CE of [rows, cols]
    f32 logits (4 C + 4 bytes read, 4 C + 4 written per row)."""
    import torch

    import rgpu_b200

    gpu = rgpu_b200.Gpu(0)
    rows, cols = args.op_shape
    rng = np.random.default_rng(0)
    st = torch.cuda.ExternalStream(gpu.stream())
    if args.op == "adam":
        z = lambda: gpu.upload(rng.standard_normal((rows, cols)).astype(np.float32))  # noqa: E731
        theta, m, v, g = z(), gpu.zeros((rows, cols)), gpu.zeros((rows, cols)), z()
        t = [0]

        def fn():
            t[0] += 1
            gpu.adam(theta, m, v, g, 1e-3, t[0])

        nbytes = 28.0 * rows * cols
    else:
        logits = gpu.upload(rng.standard_normal((rows, cols)).astype(np.float32))
        labels = rgpu_b200.upload_labels(gpu, rng.integers(0, cols, rows))
        delta, loss = gpu.zeros((rows, cols)), gpu.zeros((1, rows))

        def fn():
            gpu.softmax_xent(logits, labels, delta, loss)

        nbytes = rows * (8.0 * cols + 8.0)
    for _ in range(3):
        fn()
    gpu.sync()
    with torch.cuda.stream(st):
        torch.cuda._sleep(20000000)  # the host enqueues the timed launches meanwhile
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(args.reps):
            fn()
        e1.record(st)
    gpu.sync()
    ms = e0.elapsed_time(e1) / args.reps
    pk = peaks()
    print(json.dumps({"op": args.op, "rows": rows, "cols": cols, "ms": ms, "bytes": nbytes,
                      "gbs": nbytes / (ms / 1e3) / 1e9, "frac_of_hbm": nbytes / (ms / 1e3) / 1e9 / pk["hbm"],
                      "peak_source": pk["source"]}), flush=True)
    gpu.close()


INFER_BATCHES = (1, 32, 512, 4096)


def glorot_weights(dims, seed):
    """Dense::new's Glorot-uniform W (limit sqrt(6 / (in + out))), zero b."""
    rng = np.random.default_rng(seed)
    params = []
    for l in range(len(dims) - 1):
        lim = np.float32(np.sqrt(6.0 / (dims[l] + dims[l + 1])))
        params.append(rng.uniform(-lim, lim, size=(dims[l], dims[l + 1])).astype(np.float32))
        params.append(np.zeros((1, dims[l + 1]), np.float32))
    return params


def suite_data(n, d):
    """examples/suite.rs:27-32: x[i, j] = sin(0.01 i + 0.03 j)."""
    i = np.arange(n, dtype=np.float32).reshape(n, 1)
    j = np.arange(d, dtype=np.float32).reshape(1, d)
    return np.sin(i * np.float32(0.01) + j * np.float32(0.03)).astype(np.float32)


def run_infer(args):
    """Inference (the forward pass alone) as examples/suite.rs:204-240 times
    it: the MLP 512 -> 1024 -> 1024 -> 10, f32, Glorot weights, suite.rs's
    sin data, at batch 1 / 32 / 512 / 4096.  Per batch: GpuMlp.forward_only
    on a device-resident input (the captured forward graph), each of --steps
    calls timed by its own CUDA events with L2 flushed before it; the same through rt_mlp_forward_host (H2D of
    x and D2H of the logits inside the timed span); and the CPU reference's
    Sequential::predict (the oracle port, 1 thread as rtensor's CPU backend)
    on the same batch.  One JSON line per batch."""
    import torch

    import oracle
    import rgpu_b200

    dims = [512, 1024, 1024, 10]
    params = glorot_weights(dims, 7)
    gpu = rgpu_b200.Gpu(0)
    st = torch.cuda.ExternalStream(gpu.stream())
    cpu_model_ = oracle.Mlp(dims)
    cpu_model_.set_params(params)
    # the model (6 MB) fits in L2: flush it before every timed forward, outside
    # that forward's events (a 256 MB write, then a 256 MB read)
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    flush_s = torch.empty((), dtype=torch.float32, device="cuda")
    for batch in INFER_BATCHES:
        x = suite_data(batch, dims[0])
        mlp = rgpu_b200.GpuMlp.from_params(gpu, params, batch, 0.0, optimizer="none")
        x_dev = gpu.upload(x)
        x_pin = torch.from_numpy(x).pin_memory()
        out_pin = torch.zeros((batch, dims[-1]), dtype=torch.float32).pin_memory()
        for _ in range(max(3, args.warmup)):
            mlp.forward_only(x_dev)
            mlp.forward_host_ptr(x_pin.data_ptr(), "f32", out_pin.data_ptr())
        gpu.sync()

        def span(fn):
            gpu.sync()
            evs = []
            for _ in range(args.steps):
                with torch.cuda.stream(st):
                    flush_w.fill_(1)
                    torch.sum(flush_r, dim=None, out=flush_s)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                fn()
                e1.record(st)
                evs.append((e0, e1))
            gpu.sync()
            return sum(a.elapsed_time(b) for a, b in evs) / args.steps

        l0 = gpu.launch_count()
        ms_dev = span(lambda: mlp.forward_only(x_dev))
        launches = (gpu.launch_count() - l0) // args.steps
        ms_e2e = span(lambda: mlp.forward_host_ptr(x_pin.data_ptr(), "f32", out_pin.data_ptr()))
        reps = 20 if batch < 512 else 5
        cpu_model_.forward(x, threads=1)
        t0 = time.perf_counter()
        for _ in range(reps):
            cpu_model_.forward(x, threads=1)
        t_cpu = (time.perf_counter() - t0) / reps
        line = {"mode": "infer", "metric": "inference samples/sec (forward_only)", "batch": batch,
                "value": batch / (ms_dev / 1e3), "unit": "samples/s", "ms_per_forward": ms_dev, "steps": args.steps,
                "higher_is_better": True, "dtype": "f32", "data": "synthetic (examples/suite.rs sin data)",
                "config": {"workload": "MLP " + "->".join(map(str, dims)), "batch": batch,
                           "weights": "Glorot-uniform, zero bias", "reference": "examples/suite.rs:204-240",
                           "l2": "model smaller than L2: L2 flushed before every timed forward, each timed by its own events"},
                "e2e": {"value": batch / (ms_e2e / 1e3), "unit": "samples/s", "ms_per_forward": ms_e2e,
                        "h2d_bytes_per_step": x.nbytes, "d2h_bytes_per_step": batch * dims[-1] * 4},
                "gpu_launches": int(launches),
                "cpu_baseline": {"value": batch / t_cpu, "unit": "samples/s", "cores": 1, "kind": "port",
                                 "ms_per_forward": t_cpu * 1e3, "cpu_model": cpu_model(),
                                 "sample": f"Sequential::predict on the same {batch} rows, 1 thread, mean of {reps}"}}
        print(json.dumps(line), flush=True)
        mlp.close()
    gpu.close()


# B200 L2: a step whose working set is smaller runs with L2 flushed before each
# timed step (flush_l2_between_steps); larger ones stream it every step.
L2_BYTES = 126 << 20


def dominant_kernel_roofline(ops, cfg, pk):
    """`roofline` of the step's dominant kernel: the GEMM label with the
    largest total time.  `ops` holds (label, algorithmic FLOPs, mean ms) per
    launch of one step, `pk` the peaks (`peaks()`)."""
    by_label = {}
    for lab, fl, t in ops:
        a = by_label.setdefault(lab, [0.0, 0.0, 0])
        a[0] += fl
        a[1] += t
        a[2] += 1
    dom = max(by_label.items(), key=lambda kv: kv[1][1]) if by_label else None
    roof = None
    if dom:
        lab, (fl, t, cnt) = dom
        ach = fl / (t / 1e3) / 1e12 if t > 0 else 0.0
        # The denominator is the burst bf16 figure (cuBLAS timed alone): the
        # timed region is a fraction of a second, shorter than the seconds-long
        # loop behind the sustained figure.  The wide step does reach the power
        # cap (sw_power_cap in its clock record), so the sustained figure is
        # given beside it.  f32 GEMMs run as 3xTF32: three tf32 products at
        # half the bf16 rate.
        scale = 1.0 if cfg["dtype"] == "bf16" else 1.0 / 6.0
        peak = pk["bf16"] * scale
        sustained = pk["bf16_sus"] * scale if cfg["dtype"] == "bf16" and pk["bf16_sus"] else None
        traffic, traffic_src = None, None
        if cfg["dtype"] == "bf16" and lab in TRAFFIC_PER_LAUNCH:
            tb, traffic_src = TRAFFIC_PER_LAUNCH[lab]
            traffic = tb * (fl / cnt) / TRAFFIC_FLOPS
        # split-activation forward GEMMs run two bf16 products per algorithmic one
        executed = 2.0 if lab.endswith("_split") else 1.0
        roof = {"bound": "tensor", "kernel": lab, "launches_per_step": cnt, "achieved": ach, "peak": peak,
                "unit": "TFLOP/s", "frac": ach / peak, "peak_sustained": sustained,
                "frac_of_sustained": ach / sustained if sustained else None,
                "executed_tensor_tflops": ach * executed, "executed_frac": ach * executed / peak,
                "traffic": traffic,
                "traffic_note": (f"DRAM bytes per launch: ncu capture of {traffic_src}, scaled by FLOPs"
                                 if traffic_src else "no ncu capture for this kernel"),
                "peak_source": pk["source"] + (" bf16 dense burst (cuBLAS timed alone)" if cfg["dtype"] == "bf16"
                                               else " bf16 dense burst / 2 (tf32 rate) / 3 (3xTF32 products)")}
    return roof


# Child runs that put BASELINE configs[1] (the f32 batch-2048 step) and
# configs[3] (the dW sweep) into the default benchmark line, each bounded by
# its own time limit (seconds).
EXTRA_RUNS = {
    "config2_small": (["--config", "small"], 120),
    "config4_dw_sweep": (["--sweep"], 240),
}


def summarize_extra(key, lines):
    """The part of a child run's JSON lines that goes into the main line."""
    if key == "config2_small":
        d = lines[-1]
        return {k: d.get(k) for k in ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "dtype", "config",
                                      "e2e", "roofline", "cpu_baseline", "gpu_launches", "clocks")}
    pts = [d for d in lines if "summary" not in d]
    return {"summaries": [d for d in lines if "summary" in d], "points": len(pts),
            "columns": ["dtype", "M", "N", "K", "ms", "tflops", "frac_of_roofline", "bound"],
            "per_point": [[d["dtype"], d["M"], d["N"], d["K"], d["ms"], d["tflops"], d["frac"], d["bound"]]
                          for d in pts]}


def run_extra(key, cmd, limit):
    """Runs one child benchmark; its JSON lines are summarised, and a failure
    or an overrun comes back as {"error": ...} instead of an exception."""
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=limit, cwd=ROOT)
    except subprocess.TimeoutExpired:
        return {"error": f"did not finish within {limit} s"}
    except Exception as e:
        return {"error": f"could not start: {e}"}
    lines = []
    for ln in r.stdout.splitlines():
        if ln.startswith("{"):
            try:
                lines.append(json.loads(ln))
            except ValueError:
                pass
    if r.returncode != 0 or not lines:
        return {"error": f"exit {r.returncode}: {r.stderr.strip()[-300:]}"}
    try:
        return summarize_extra(key, lines)
    except Exception as e:
        return {"error": f"unreadable output: {e}"}


def run_extra_configs(args):
    """configs[1] and configs[3] as child processes of the default 1-GPU run,
    after its own timed regions: the f32 step with the driver's step counts,
    and the whole dW sweep."""
    out = {}
    for key, (extra, limit) in EXTRA_RUNS.items():
        cmd = [sys.executable, os.path.abspath(__file__)] + extra
        if key == "config2_small":
            cmd += ["--steps", str(args.steps), "--warmup", str(max(3, args.warmup))]
        out[key] = run_extra(key, cmd, limit)
    return out


def working_set_bytes(cfg, rows):
    """Bytes a train step touches: parameters with their gradients and
    optimiser state, the input rows, and each layer's activations and
    adjoints."""
    dims, es = cfg["dims"], 2 if cfg["dtype"] == "bf16" else 4
    params = sum((dims[l] + 1) * dims[l + 1] for l in range(len(dims) - 1))
    per_param = 4 + 4 + (8 if cfg["optimizer"] == "adam" else 0) + (2 if cfg["dtype"] == "bf16" else 0)
    return params * per_param + rows * dims[0] * es + rows * sum(dims[1:]) * es * 2


def flush_l2_between_steps(cfg, rows):
    return working_set_bytes(cfg, rows) < L2_BYTES


def config_dict(cfg_name, cfg, n, global_batch):
    d = cfg["dims"]
    rows = global_batch // n
    l2 = ("working set smaller than L2: L2 flushed (256 MB write, then 256 MB read) before every timed step, "
          "each step timed by its own events" if flush_l2_between_steps(cfg, rows)
          else "inputs larger than L2 (each step streams several GB)")
    return {"workload": ("wide MLP " if cfg_name == "wide" else "MLP ") + "->".join(map(str, d)),
            "global_batch": global_batch, "batch_per_gpu": rows, "dtype_policy":
            "bf16 operands, f32 accumulate, f32 master weights" if cfg["dtype"] == "bf16" else "f32",
            "optimizer": f"{cfg['optimizer']}(lr={cfg['lr']})", "parallelism": f"dp{n}", "l2": l2}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="wide", choices=sorted(CONFIGS))
    ap.add_argument("--global-batch", type=int, default=0, help="strong scaling: fixed global batch")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-strong", action="store_true", help="skip the fixed-global-batch (65536) leg")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the configs[1] step and the configs[3] sweep that the default 1-GPU run adds")
    ap.add_argument("--gemm", choices=["NN", "NT", "TN"], help="profile one bf16 GEMM instead of the step")
    ap.add_argument("--mnk", type=int, nargs=3, default=[8192, 8192, 8192], metavar=("M", "N", "K"))
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--l2-group", type=int, default=0, help="GEMM raster group (tile rows), 0 = library default")
    ap.add_argument("--gemm-dtype", default="bf16", choices=["bf16", "f32"], help="operand dtype of --gemm")
    ap.add_argument("--split", action="store_true", help="--gemm NN with split (hi + lo) A and C planes")
    ap.add_argument("--sweep", action="store_true", help="dW = X^T dY sweep (BASELINE configs[3])")
    ap.add_argument("--infer", action="store_true", help="inference at batch 1/32/512/4096 (examples/suite.rs)")
    ap.add_argument("--op", choices=["adam", "xent"], help="time one HBM-bound kernel alone")
    ap.add_argument("--op-shape", type=int, nargs=2, default=[8192, 8192], metavar=("ROWS", "COLS"))
    ap.add_argument("--sweep-dtypes", default="f32,bf16")
    ap.add_argument("--sweep-k", default="", help="comma-separated K values (default: the full sweep)")
    ap.add_argument("--activations", default="split", choices=["split", "bf16"],
                    help="bf16 plans: hidden activations as a bf16 hi + lo pair (default) or one bf16 rounding")
    args = ap.parse_args()
    if args.sweep:
        run_dw_sweep(args)
        return
    if args.infer:
        run_infer(args)
        return
    if args.op:
        run_op(args)
        return
    if args.gemm:
        run_gemm_only(args)
        return
    cfg = CONFIGS[args.config]
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, args.config, cfg, rank)
        return

    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    import rgpu_b200

    if args.global_batch:
        batch = args.global_batch // world
        scaling = "strong"
    else:
        batch = cfg["batch"]
        scaling = "weak"
    global_batch = batch * world
    dims = cfg["dims"]

    gpu = rgpu_b200.Gpu(local)
    if args.l2_group:
        gpu.set_grupo_l2(args.l2_group)
    # Data parallelism: every rank starts from the same weights (one seed)
    # and takes its own rows of the global batch (seeded per rank).
    params = make_weights(cfg, 1234)
    x, labels = make_data(cfg, batch, 5678 + rank)
    mlp = rgpu_b200.GpuMlp.from_params(gpu, params, batch, cfg["lr"], dtype=cfg["dtype"],
                                       optimizer=cfg["optimizer"], global_batch=global_batch,
                                       activations=args.activations)
    comm = None
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(rgpu_b200.Comm.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = rgpu_b200.Comm(gpu, rank, world, bytes(uid.cpu().numpy().tobytes()))
        mlp.set_comm(comm)

    # inputs: device copy (value) and pinned host copy (e2e)
    x_dtype = cfg["dtype"]
    if x_dtype == "bf16":
        xh = rgpu_b200.f32_to_bf16(x)
    else:
        xh = x
    x_dev = torch.from_numpy(xh.view(np.int16) if x_dtype == "bf16" else xh).cuda(local)
    lab_dev = torch.from_numpy(labels.view(np.int32)).cuda(local)
    x_pin = torch.from_numpy(xh.view(np.int16) if x_dtype == "bf16" else xh).pin_memory()
    lab_pin = torch.from_numpy(labels.view(np.int32)).pin_memory()
    loss_pin = torch.zeros(batch, dtype=torch.float32).pin_memory()
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(gpu.stream(), device=torch.device("cuda", local))

    def step_dev():
        mlp.step_ptr(x_dev.data_ptr(), x_dtype, lab_dev.data_ptr())

    def step_host():
        mlp.step_host_ptr(x_pin.data_ptr(), x_dtype, lab_pin.data_ptr(), loss_pin.data_ptr())

    def barrier():
        if dist:
            dist.barrier()
        gpu.sync()
        torch.cuda.synchronize()

    cold = flush_l2_between_steps(cfg, batch)
    if cold:
        flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=torch.device("cuda", local))
        flush_r = torch.ones(64 << 20, dtype=torch.float32, device=torch.device("cuda", local))
        flush_s = torch.empty((), dtype=torch.float32, device=torch.device("cuda", local))

    def flush_l2():
        # a write larger than L2, then a read of another buffer, so the next step
        # starts with an L2 that holds none of its data and no dirty lines
        with torch.cuda.stream(stream):
            flush_w.fill_(1)
            torch.sum(flush_r, dim=None, out=flush_s)

    def timed(fn, k):
        barrier()
        if cold:
            # small working set: L2 flushed before every step, outside its events
            evs = []
            for _ in range(k):
                flush_l2()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                evs.append((e0, e1))
            gpu.sync()
            ms = sum(a.elapsed_time(b) for a, b in evs)
        else:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(k):
                fn()
            e1.record(stream)
            gpu.sync()
            ms = e0.elapsed_time(e1)
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        barrier()
        return float(t.item())

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(args.warmup):
        step_dev()
    gpu.sync()

    # ---- timed region: device-resident inputs (the captured step as shipped)
    clocks.mark_start()
    launches0 = gpu.launch_count()
    ms = timed(step_dev, args.steps)
    launches = gpu.launch_count() - launches0
    clk = clocks.stop()

    # ---- end-to-end: host buffers, H2D + D2H inside the timed region
    for _ in range(2):
        step_host()
    gpu.sync()
    ms_e2e = timed(step_host, args.steps)

    # ---- second timed region of the same steps with a CUDA event between
    # consecutive kernels of the captured step (the per-kernel times behind
    # the roofline), read back after every step and averaged over the steps;
    # the events cost a little, so `value` comes from the region above
    mlp.enable_timing(True)
    for _ in range(2):
        step_dev()
    gpu.sync()
    barrier()
    op_sum = None
    for _ in range(args.steps):
        if cold:
            flush_l2()
        step_dev()
        gpu.sync()
        ops_i = mlp.op_times()
        if op_sum is None:
            op_sum = [[lab, fl, 0.0] for lab, fl, _ in ops_i]
        for acc_op, (lab, fl, t) in zip(op_sum, ops_i):
            acc_op[2] += t
    barrier()
    ops = [(lab, fl, t / args.steps) for lab, fl, t in op_sum]  # mean device ms per kernel
    ms_events = sum(t for _, _, t in ops) * args.steps

    # ---- the same model at a fixed global batch of
    # 65536 rows split over the ranks (strong scaling), device-resident
    # inputs, timed like the main region; the 1-GPU run gives the baseline
    # of the scaling efficiency at the same global batch.
    grad_sync = mlp.comm_mode()
    strong = None
    if args.config == "wide" and not args.global_batch and not args.no_strong:
        mlp.close()
        sb = STRONG_GLOBAL_BATCH // world
        smlp = rgpu_b200.GpuMlp.from_params(gpu, params, sb, cfg["lr"], dtype=cfg["dtype"],
                                            optimizer=cfg["optimizer"], global_batch=sb * world,
                                            activations=args.activations)
        if comm:
            smlp.set_comm(comm)
        gen = torch.Generator(device=torch.device("cuda", local))
        gen.manual_seed(91 + rank)
        sx = torch.randn((sb, dims[0]), generator=gen, device=torch.device("cuda", local)).to(torch.bfloat16)
        sl = torch.randint(0, dims[-1], (sb,), generator=gen, device=torch.device("cuda", local), dtype=torch.int32)
        torch.cuda.synchronize()

        def step_strong():
            smlp.step_ptr(sx.data_ptr(), "bf16", sl.data_ptr())

        for _ in range(max(3, args.warmup)):
            step_strong()
        gpu.sync()
        ms_s = timed(step_strong, args.steps)
        strong = {"global_batch": sb * world, "batch_per_gpu": sb, "n_gpus": world, "steps": args.steps,
                  "ms_per_step": ms_s / args.steps, "value": sb * world / (ms_s / args.steps / 1e3),
                  "unit": "samples/s", "scaling": "strong",
                  "note": "BASELINE configs[4]: fixed global batch over the ranks; device-resident N(0,1) bf16 inputs"}
        smlp.close()
        mlp = None
        del sx, sl

    ms_step = ms / args.steps
    value = global_batch / (ms_step / 1e3)
    e2e_value = global_batch / (ms_e2e / args.steps / 1e3)
    pk = peaks()
    step_flops = exact_flops(dims, batch)
    roof = dominant_kernel_roofline(ops, cfg, pk)
    gemm_t = sum(t for lab, fl, t in ops if fl > 0)
    gemm_f = sum(fl for lab, fl, t in ops if fl > 0)
    step_tflops = step_flops / (ms_step / 1e3) / 1e12

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            try:
                cpu = cpu_baseline(args.config, cfg)
            except Exception as e:  # the baseline must not hide the GPU line
                cpu = {"value": None, "unit": "samples/s", "cores": 1, "kind": "port", "sample": f"failed: {e}"}
        extra = None
        if world == 1 and args.config == "wide" and not args.global_batch and not args.no_extra:
            extra = run_extra_configs(args)
        in_bytes = xh.nbytes + labels.nbytes
        line = {
            "metric": "train samples/sec (fwd+bwd+update)", "value": value, "unit": "samples/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": cfg["dtype"],
            "data": "synthetic (seeded N(0,1) inputs, uniform labels, Kaiming-uniform weights)",
            "config": dict(config_dict(args.config, cfg, world, global_batch), grad_sync=grad_sync,
                           activations=(args.activations if cfg["dtype"] == "bf16" else "f32")),
            "roofline": roof,
            "ms_per_step_with_kernel_events": ms_events / args.steps,
            "roofline_window": f"per-kernel CUDA events, mean over {args.steps} timed steps",
            "step_tensor_frac": {"achieved_tflops": step_tflops, "peak": pk["bf16"], "frac": step_tflops / pk["bf16"],
                                 "peak_sustained": pk["bf16_sus"],
                                 "frac_of_sustained": step_tflops / pk["bf16_sus"] if pk["bf16_sus"] else None,
                                 "flops_per_step_per_gpu": step_flops,
                                 "gemm_tflops": gemm_f / (gemm_t / 1e3) / 1e12 if gemm_t > 0 else None},
            "cpu_baseline": cpu,
            "strong_scaling": strong,
            "e2e": {"value": e2e_value, "unit": "samples/s", "h2d_bytes_per_step": in_bytes,
                    "d2h_bytes_per_step": batch * 4},
            "gpu_launches": int(launches),
            "clocks": clk,
            "kernels_mean_over_steps": [{"label": lab, "ms": round(t, 4),
                                         "tflops": round(fl / (t / 1e3) / 1e12, 1) if fl and t else None}
                                        for lab, fl, t in ops],
        }
        if extra is not None:
            line["other_configs"] = extra
        print(json.dumps(line), flush=True)

    if mlp:
        mlp.close()
    if comm:
        comm.close()
    gpu.close()
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
