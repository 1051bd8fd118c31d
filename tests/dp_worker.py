"""One rank of the data-parallel parity check (launched by tests/test_gpu_dp.py
with torch.distributed.run, one process per GPU).

Every rank holds the full model, takes rows [r*n/p, (r+1)*n/p) of the global
batch, scales its softmax-CE adjoint by 1/n_global, and the plan sums dW/db
over ranks with NCCL inside the captured step.  Rank 0 also runs the whole
global batch on its GPU without a communicator and on the CPU oracle (the
reference's CPU step); the summed DP gradients must equal the single-GPU
result and the oracle's within the north-star bars (and the replicas must
stay identical under Adam).  x and W are bf16 values, so the f32 and bf16
plans and the oracle all start from identical inputs and weights.  Results
go to the JSON file named by argv[1].
"""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import oracle  # noqa: E402
import rgpu_b200  # noqa: E402
from tests.helpers import bf16_round  # noqa: E402


def main():
    out_path = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    gpu = rgpu_b200.Gpu(local)
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(rgpu_b200.Comm.unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    comm = rgpu_b200.Comm(gpu, rank, world, bytes(uid.cpu().numpy().tobytes()))

    rng = np.random.default_rng(7)
    # 1025 rows of [W_0; b_0]: the plan can cut the first layer's dW GEMM into
    # 4 chunks on 256-row edges (RTGPU_FIRST_LAYER_CHUNKS=4 below), whose
    # allreduces and updates then run per chunk
    # (and 513 rows of layer 1: 2 chunks under RTGPU_DW_CHUNKS=2)
    dims = [1024, 512, 192, 10]
    params = []
    for l in range(len(dims) - 1):
        lim = np.sqrt(6.0 / dims[l])
        params += [bf16_round(rng.uniform(-lim, lim, (dims[l], dims[l + 1])).astype(np.float32)),
                   rng.uniform(-0.1, 0.1, (1, dims[l + 1])).astype(np.float32)]
    n_global = 512
    x = bf16_round(rng.standard_normal((n_global, dims[0])).astype(np.float32))
    labels = rng.integers(0, dims[-1], n_global).astype(np.uint32)
    g_oracle = None
    if rank == 0:
        cpu = oracle.Mlp(dims)
        cpu.set_params(params)
        loss_oracle = cpu.train_step(x, labels, threads=os.cpu_count() or 4, input_grad=False)
        g_oracle = cpu.grads()
    per = n_global // world
    xs, ls = x[rank * per:(rank + 1) * per], labels[rank * per:(rank + 1) * per]
    result = {}
    cases = (("f32", "1", "1", "f32"), ("bf16", "1", "1", "f32"), ("f32_chunked", "4", "2", "f32"),
             ("bf16_gradcomm", "4", "2", "bf16"))
    for dtype, chunks, dw_chunks, grad_comm in cases:
        os.environ["RTGPU_FIRST_LAYER_CHUNKS"] = chunks
        os.environ["RTGPU_DW_CHUNKS"] = dw_chunks
        os.environ["RTGPU_GRAD_COMM"] = grad_comm
        dtype_name = dtype
        dtype = dtype.split("_")[0]
        mlp = rgpu_b200.GpuMlp.from_params(gpu, params, per, 0.0, dtype=dtype, optimizer="none",
                                           global_batch=n_global)
        mlp.set_comm(comm)
        mlp.step(gpu.upload(xs), rgpu_b200.upload_labels(gpu, ls))
        g_dp = mlp.grads()
        loss_dp = mlp.global_loss()
        mlp.close()
        if rank == 0:
            ref = rgpu_b200.GpuMlp.from_params(gpu, params, n_global, 0.0, dtype=dtype, optimizer="none")
            ref.step(gpu.upload(x), rgpu_b200.upload_labels(gpu, labels))
            g_ref = ref.grads()
            loss_ref = ref.last_loss()
            ref.close()
            result[dtype_name] = [float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
                                  for a, b in zip(g_dp, g_ref)]
            result[dtype_name + "_oracle"] = [float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
                                              for a, b in zip(g_dp, g_oracle)]
            result[dtype_name + "_loss"] = [loss_dp, loss_ref, loss_oracle]
    # Adam with chunked dW GEMMs and bf16 gradient sums: replicas stay bit-identical.
    os.environ["RTGPU_FIRST_LAYER_CHUNKS"] = "4"
    os.environ["RTGPU_DW_CHUNKS"] = "2"
    os.environ["RTGPU_GRAD_COMM"] = "bf16"
    mlp = rgpu_b200.GpuMlp.from_params(gpu, params, per, 1e-3, dtype="bf16", optimizer="adam", global_batch=n_global)
    mlp.set_comm(comm)
    gx, gl = gpu.upload(xs), rgpu_b200.upload_labels(gpu, ls)
    for _ in range(5):
        mlp.step(gx, gl)
    w = np.concatenate([a.ravel() for a in mlp.weights()])
    mlp.close()
    wt = torch.from_numpy(w).cuda()
    gathered = [torch.zeros_like(wt) for _ in range(world)]
    dist.all_gather(gathered, wt)
    if rank == 0:
        result["replicas_identical"] = all(torch.equal(gathered[0], g) for g in gathered[1:])
    # Sharded optimiser (bf16 + Adam, f32 gradient sums) with each exchange:
    # NCCL reduce-scatter + all-gather, the dW GEMMs' peer scatter, and the
    # copy-engine copies between mapped buffers.  Five steps give the
    # replicated update's weights, gradients and checkpoint, and replicas that
    # agree bit for bit.
    os.environ["RTGPU_GRAD_COMM"] = "f32"
    runs = {}
    for sharded in ("0", "1", "p2p", "ce"):
        os.environ["RTGPU_SHARDED_OPT"] = "0" if sharded == "0" else "1"
        os.environ["RTGPU_P2P_RS"] = "1" if sharded == "p2p" else "0"
        os.environ["RTGPU_CE_EXCHANGE"] = "1" if sharded == "ce" else "0"
        mlp = rgpu_b200.GpuMlp.from_params(gpu, params, per, 1e-3, dtype="bf16", optimizer="adam",
                                           global_batch=n_global)
        mlp.set_comm(comm)
        mode = mlp.comm_mode()
        for _ in range(5):
            mlp.step(gx, gl)
        runs[sharded] = (mode, np.concatenate([a.ravel() for a in mlp.weights()]),
                         np.concatenate([a.ravel() for a in mlp.grads()]),
                         np.frombuffer(mlp.save_state(), np.uint8))
        mlp.close()
    os.environ.pop("RTGPU_SHARDED_OPT")
    os.environ.pop("RTGPU_P2P_RS")
    os.environ.pop("RTGPU_CE_EXCHANGE")
    mode0, w0, g0, s0 = runs["0"]
    rel = lambda a, b: float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))  # noqa: E731
    hdr = 24 + 8 * len(dims)
    for key, name in (("1", "sharded"), ("p2p", "sharded_p2p"), ("ce", "sharded_ce")):
        mode1, w1, g1, s1 = runs[key]
        wt = torch.from_numpy(w1).cuda()
        gathered = [torch.zeros_like(wt) for _ in range(world)]
        dist.all_gather(gathered, wt)
        if rank == 0:
            result[name] = {"modes": [mode0, mode1], "weights": rel(w1, w0), "grads": rel(g1, g0),
                            "state": rel(s1[hdr:].view(np.float32), s0[hdr:].view(np.float32)),
                            "header_equal": bool(np.array_equal(s1[:hdr], s0[:hdr])),
                            "replicas_identical": all(torch.equal(gathered[0], g) for g in gathered[1:])}
    if rank == 0:
        json.dump(result, open(out_path, "w"))
    comm.close()
    gpu.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
