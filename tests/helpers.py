"""Shared helpers for the parity tests."""
import numpy as np

import oracle


def erro_rel(a, b) -> float:
    """Max relative distance of crates/rtensor/tests/gpu.rs:53-60:
    max |x - y| / (1 + max(|x|, |y|))."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    assert a.shape == b.shape
    if a.size == 0:
        return 0.0
    return float(np.max(np.abs(a - b) / (1.0 + np.maximum(np.abs(a), np.abs(b)))))


def rel_l2(x, ref) -> float:
    """||x - ref||_2 / ||ref||_2, the north-star parity metric."""
    x = np.asarray(x, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    den = np.linalg.norm(ref)
    num = np.linalg.norm(x - ref)
    return float(num / den) if den > 0 else float(num)


def quadrant_data(n, d):
    """tests/gpu.rs:21-30: x_i = sin(0.37 i), label = quadrant of (x0, x1)."""
    x = np.sin(np.arange(n * d, dtype=np.float32) * np.float32(0.37)).astype(np.float32).reshape(n, d)
    labels = (x[:, 0] > 0).astype(np.uint32) + 2 * (x[:, 1] > 0).astype(np.uint32)
    return x, labels


def glorot_model(dims, seed):
    """Dense::new Glorot weights drawn layer by layer from Rng::new(seed)."""
    m = oracle.Mlp(dims)
    m.init_glorot(oracle.Rng(seed))
    return m


def baseline_inputs(dims, batch, seed):
    """X ~ N(0,1), labels uniform in [0, C), Kaiming-uniform
    W, zero b, all from rtensor's Rng seeded with `seed`."""
    rng = oracle.Rng(seed)
    m = oracle.Mlp(dims)
    m.init_kaiming(rng)
    x = rng.normal(batch * dims[0]).reshape(batch, dims[0])
    labels = rng.below(dims[-1], batch)
    return m, x, labels


def bf16_round(a) -> np.ndarray:
    """Nearest-even bf16 value of each f32 element, widened back to f32."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(a.shape)


def bf16_baseline_inputs(dims, batch, seed):
    """baseline_inputs for the bf16 configs ("bf16 inputs/weights with fp32
    accumulate and fp32 master weights"): x and W are rounded to bf16 values,
    so the CPU reference and the GPU plan start from identical inputs and
    weights, and the f32 masters begin equal to their bf16 shadows."""
    m, x, labels = baseline_inputs(dims, batch, seed)
    params = m.params()
    for l in range(0, len(params), 2):
        params[l] = bf16_round(params[l])
    m.set_params(params)
    return m, bf16_round(x), labels
