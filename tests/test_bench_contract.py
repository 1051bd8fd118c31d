"""The benchmark's JSON contract, checked on CPU: `bench.py --impl reference`
(the reference's CPU step, restated by the oracle) on the small config prints
one JSON line with the keys the benchmark driver reads, times real steps, and
reports how many it ran.  Also the L2 rule: a config whose working set fits in
L2 is timed with L2 flushed before every step, and says so."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_complete_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "small",
                        "--steps", "2", "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "samples/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["steps_requested"] == 2
    assert d["value"] > 0 and abs(d["value"] - 2048 / (d["ms_per_step"] / 1e3)) < 1e-6 * d["value"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["cpu_model"]
    assert d["e2e"] == {"value": d["value"], "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "MLP 512->1024->1024->10"


def test_l2_rule_follows_the_working_set():
    sys.path.insert(0, ROOT)
    import bench

    small, wide = bench.CONFIGS["small"], bench.CONFIGS["wide"]
    assert bench.flush_l2_between_steps(small, small["batch"])
    assert not bench.flush_l2_between_steps(wide, wide["batch"])
    assert "flushed" in bench.config_dict("small", small, 1, small["batch"])["l2"]
    assert "larger than L2" in bench.config_dict("wide", wide, 1, wide["batch"])["l2"]


def test_roofline_names_the_dominant_kernel_against_the_burst_peak():
    sys.path.insert(0, ROOT)
    import bench

    f = 2.0 * 8192 ** 3
    # (label, algorithmic FLOPs, mean ms) per launch, shaped like a wide step
    ops = [("fwd_gemm_bias_relu_split", f, 1.385), ("fwd_gemm_bias_relu_split", f, 1.346),
           ("dw_gemm_adam", f, 0.970), ("dw_gemm_adam", f, 0.965), ("softmax_xent", 0.0, 0.063)]
    pk = {"hbm": 6553.6, "bf16": 1642.0, "bf16_sus": 1380.2, "source": "measured"}
    r = bench.dominant_kernel_roofline(ops, bench.CONFIGS["wide"], pk)
    assert r["kernel"] == "fwd_gemm_bias_relu_split" and r["launches_per_step"] == 2
    ach = 2 * f / ((1.385 + 1.346) / 1e3) / 1e12
    assert abs(r["achieved"] - ach) < 1e-9 * ach
    assert r["peak"] == 1642.0 and abs(r["frac"] - ach / 1642.0) < 1e-12
    assert abs(r["frac_of_sustained"] - ach / 1380.2) < 1e-12
    assert abs(r["executed_tensor_tflops"] - 2 * ach) < 1e-9 * ach  # two bf16 products per algorithmic one
    tb = bench.TRAFFIC_PER_LAUNCH["fwd_gemm_bias_relu_split"][0]
    assert abs(r["traffic"] - tb) < 1e-6 * tb  # each launch is one 8192^3 GEMM
    # f32 configs: the 3xTF32 rate, no sustained figure
    r32 = bench.dominant_kernel_roofline([("fwd_gemm_bias_relu", 1e9, 0.01)], bench.CONFIGS["small"], pk)
    assert abs(r32["peak"] - 1642.0 / 6) < 1e-9 and r32["peak_sustained"] is None and r32["traffic"] is None
    assert bench.dominant_kernel_roofline([], bench.CONFIGS["small"], pk) is None


def test_other_configs_are_summarised_and_failures_reported():
    sys.path.insert(0, ROOT)
    import bench

    # a child that prints a sweep's lines
    pts = [{"dtype": "bf16", "M": 1024, "N": 512, "K": k, "ms": 0.01, "tflops": 1.0, "gbs": 1.0, "roofline_ms": 0.005,
            "frac": 0.5, "bound": "hbm", "workspace_bytes": 0} for k in (1, 8)]
    lines = pts + [{"summary": "bf16", "points": 2, "frac_median": 0.5, "frac_min": 0.5, "peak_source": "measured"}]
    script = "import json\n" + "".join(f"print(json.dumps({d!r}))\n" for d in lines)
    r = bench.run_extra("config4_dw_sweep", [sys.executable, "-c", script], 60)
    assert r["points"] == 2 and r["summaries"][0]["frac_median"] == 0.5
    assert r["per_point"][1] == ["bf16", 1024, 512, 8, 0.01, 1.0, 0.5, "hbm"]
    # the f32 step's line keeps its measurement keys
    step = {"metric": "m", "value": 6.6e6, "unit": "samples/s", "ms_per_step": 0.31, "steps": 5, "warmup": 3,
            "dtype": "f32", "config": {"workload": "w"}, "e2e": {}, "roofline": {}, "cpu_baseline": None,
            "gpu_launches": 40, "clocks": None, "kernels_mean_over_steps": []}
    r = bench.run_extra("config2_small", [sys.executable, "-c", f"print({json.dumps(json.dumps(step))})"], 60)
    assert r["value"] == 6.6e6 and r["gpu_launches"] == 40 and "kernels_mean_over_steps" not in r
    # failures and overruns come back as errors, not exceptions
    r = bench.run_extra("config2_small", [sys.executable, "-c", "import sys; sys.exit(3)"], 60)
    assert r["error"].startswith("exit 3")
    r = bench.run_extra("config2_small", [sys.executable, "-c", "import time; time.sleep(30)"], 1)
    assert "within 1 s" in r["error"]
    r = bench.run_extra("config2_small", [sys.executable, "-c", "print('{not json')"], 60)
    assert "error" in r
