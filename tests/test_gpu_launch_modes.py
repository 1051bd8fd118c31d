"""The plan's launch modes change when and where tiles run, never what they
compute.

- Programmatic dependent launch (RTGPU_PDL) lets a GEMM start while the kernel
  before it drains.
- The dynamic tile schedule (RTGPU_DYN_TILES) hands the pair kernel's tiles
  out through an atomic counter instead of round robin. By default it is on
  only under data parallelism; here it is forced on a single device, so that
  its ring of tile ids in shared memory runs on a one-GPU box too.

Every tile is still computed by one CTA pair with the same k order, and every
epilogue is unchanged. So plans built on contexts with these switches must
give the same weights, moments and losses bit for bit, over several Adam
steps.
"""
import os

import numpy as np
import pytest

import rgpu_b200
from tests.helpers import bf16_baseline_inputs, baseline_inputs

pytestmark = pytest.mark.gpu

MODES = [
    {"RTGPU_PDL": "0", "RTGPU_DYN_TILES": "0"},
    {"RTGPU_PDL": "1", "RTGPU_DYN_TILES": "1"},
    {"RTGPU_PDL": "0", "RTGPU_DYN_TILES": "1"},
]


def _run(env, dims, n, dtype, optimizer, steps):
    """Steps of a plan on a fresh context created under `env`; returns the
    weights, the checkpoint (weights, moments, step count) and the losses."""
    saved = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        gpu = rgpu_b200.Gpu(0)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    try:
        if dtype == "bf16":
            model, x, labels = bf16_baseline_inputs(dims, n, 77)
        else:
            model, x, labels = baseline_inputs(dims, n, 77)
        mlp = rgpu_b200.GpuMlp.from_params(gpu, model.params(), n, 1e-3, dtype=dtype, optimizer=optimizer)
        gx, gy = gpu.upload(x, dtype), rgpu_b200.upload_labels(gpu, labels)
        losses = []
        for _ in range(steps):
            mlp.step(gx, gy)
            losses.append(mlp.last_loss())
        weights = [w.copy() for w in mlp.weights()]
        state = mlp.save_state()
        mlp.close()
        return weights, state, losses
    finally:
        gpu.close()


@pytest.mark.parametrize("dtype,optimizer", [("bf16", "adam"), ("f32", "sgd")])
def test_launch_modes_are_bit_identical(dtype, optimizer):
    # Layers wide enough for the two-CTA kernel: a few hundred tiles per GEMM
    # and, for bf16, the split-activation forward GEMMs and the fused update.
    dims = [512, 1024, 1024, 100]
    n = 1024
    ref = _run({"RTGPU_PDL": "1", "RTGPU_DYN_TILES": "0"}, dims, n, dtype, optimizer, 3)
    for env in MODES:
        got = _run(env, dims, n, dtype, optimizer, 3)
        for i, (a, b) in enumerate(zip(ref[0], got[0])):
            assert np.array_equal(a, b), f"{env}: param {i} differs"
        assert ref[1] == got[1], f"{env}: checkpoints differ"
        assert ref[2] == got[2], f"{env}: losses differ"
