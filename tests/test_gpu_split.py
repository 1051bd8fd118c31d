"""Split bf16 planes of the GEMMs (rt_gemm_args.a_lo / c_lo) on every kernel
path: the two-CTA and one-CTA tensor-core kernels (a second k segment over
A's low-order plane), the SIMT kernel and the skinny CUDA-core kernels (hi +
lo summed exactly in f32 before the product).

An f32 operand X stored as hi = bf16(X), lo = bf16(X - hi) keeps ~16
significant bits, so (hi + lo) B must track the exact product of X with the
bf16 operand B far closer than hi B does; and a bf16 output with a low-order
plane must give back v to ~2^-16 through hi + lo.  These are the two halves of
the split-activation MLP plan (a hidden layer's output is written as hi and lo
planes, the next layer's forward GEMM reads both).
"""
import numpy as np
import pytest

import rgpu_b200
from rgpu_b200 import gpu as G
from tests.helpers import bf16_round, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    g = rgpu_b200.Gpu(0)
    yield g
    g.close()


def _split(x):
    hi = bf16_round(x)
    return hi, bf16_round(x - hi)


# (m, n, k): which kernel each shape lands on with fast GEMM on
CASES = [
    (2048, 2048, 512),  # two-CTA kernel, 256-wide tiles
    (2048, 1024, 320),  # two-CTA kernel, 128-wide tiles
    (2000, 1500, 136),  # two-CTA kernel, 256-wide tiles, ragged m, n and k
    (1000, 1200, 200),  # two-CTA kernel, 128-wide tiles, ragged m, n and k
    (512, 384, 1000),   # one-CTA kernel, 128 x 64 tiles (few tiles)
    (200, 136, 72),     # one-CTA kernel, ragged edges
    (300, 10, 512),     # skinny narrow-N kernel (n <= 16)
    (300, 200, 16),     # narrow K: tensor cores (bf16, one k block)
]


def _run(gpu, m, n, k, epi, seed, layout=G.RT_NN):
    rng = np.random.default_rng(seed)
    x = np.maximum(rng.standard_normal((m, k)), 0).astype(np.float32)  # ReLU-like activations
    b = bf16_round(rng.uniform(-0.05, 0.05, (k, n)).astype(np.float32))
    bias = rng.uniform(-0.1, 0.1, (1, n)).astype(np.float32)
    hi, lo = _split(x)
    ghi, glo, gb = gpu.upload(hi, "bf16"), gpu.upload(lo, "bf16"), gpu.upload(b, "bf16")
    gbias = gpu.upload(bias)
    c = gpu.zeros((m, n))
    args = G.GemmArgs(layout, G.RT_BF16, G.RT_F32, m, n, k, ghi.ptr, ghi.ld, gb.ptr, gb.ld, c.ptr, c.ld, epi,
                      gbias.ptr, None, 0, 1, None, 0)
    args.a_lo = glo.ptr
    gpu.gemm(args)
    ref = x.astype(np.float64) @ b.astype(np.float64)
    if epi in (G.RT_EPI_BIAS, G.RT_EPI_BIAS_RELU):
        ref = ref + bias
    if epi == G.RT_EPI_BIAS_RELU:
        ref = np.maximum(ref, 0)
    plain = hi.astype(np.float64) @ b.astype(np.float64)
    return gpu.download(c), ref, plain, (hi, lo, b, bias)


@pytest.mark.parametrize("fast", [True, False])
@pytest.mark.parametrize("m,n,k", CASES)
def test_split_a_tracks_the_f32_operand(gpu, fast, m, n, k):
    gpu.set_fast_gemm(fast)
    try:
        got, ref, plain, _ = _run(gpu, m, n, k, G.RT_EPI_NONE, m + n + k)
    finally:
        gpu.set_fast_gemm(True)
    e_split = rel_l2(got, ref)
    e_plain = rel_l2(plain, ref)
    # hi B alone is ~1e-3 off the f32 operand's product; (hi + lo) B must be
    # within what hi + lo leaves of x (lo's own rounding, <= 2^-18 |x|, about
    # 1.3e-6 rms) plus the tensor cores' accumulation error (two k segments,
    # 2k deep)
    assert e_plain > 1e-4
    assert e_split <= 3e-6 + 3.2e-9 * k, f"{m}x{n}x{k} fast={fast}: {e_split:.2e} (plain bf16 {e_plain:.2e})"


@pytest.mark.parametrize("m,n,k", [(300, 200, 16), (512, 384, 8)])
def test_split_a_on_the_narrow_k_cuda_core_kernel(monkeypatch, m, n, k):
    # RTGPU_SKINNY_K_MAX keeps narrow-K bf16 GEMMs on the CUDA-core kernel.
    monkeypatch.setenv("RTGPU_SKINNY_K_MAX", "16")
    g = rgpu_b200.Gpu(0)
    try:
        got, ref, _, _ = _run(g, m, n, k, G.RT_EPI_NONE, 3)
        assert rel_l2(got, ref) <= 3e-6
    finally:
        g.close()


@pytest.mark.parametrize("fast", [True, False])
@pytest.mark.parametrize("m,n,k", [(2048, 2048, 512), (2048, 1024, 320), (2000, 1500, 136), (1000, 1200, 200),
                                   (512, 384, 1000), (200, 136, 72), (300, 200, 16)])
def test_c_lo_plane_carries_the_rounding_residual(gpu, fast, m, n, k):
    # bias + ReLU epilogue with a bf16 output and its low-order plane: the
    # forward GEMM of a hidden layer in the split-activation plan, whose
    # input is itself split.
    gpu.set_fast_gemm(fast)
    try:
        rng = np.random.default_rng(k)
        x = np.maximum(rng.standard_normal((m, k)), 0).astype(np.float32)
        b = bf16_round(rng.uniform(-0.05, 0.05, (k, n)).astype(np.float32))
        bias = rng.uniform(-0.1, 0.1, (1, n)).astype(np.float32)
        hi, lo = _split(x)
        ghi, glo, gb, gbias = gpu.upload(hi, "bf16"), gpu.upload(lo, "bf16"), gpu.upload(b, "bf16"), gpu.upload(bias)
        chi, clo = gpu.zeros((m, n), "bf16"), gpu.zeros((m, n), "bf16")
        args = G.GemmArgs(G.RT_NN, G.RT_BF16, G.RT_BF16, m, n, k, ghi.ptr, ghi.ld, gb.ptr, gb.ld, chi.ptr, chi.ld,
                          G.RT_EPI_BIAS_RELU, gbias.ptr, None, 0, 1, None, 0)
        args.a_lo = glo.ptr
        args.c_lo = clo.ptr
        assert clo.ld == chi.ld
        gpu.gemm(args)
        h, l = gpu.download(chi), gpu.download(clo)
    finally:
        gpu.set_fast_gemm(True)
    ref = np.maximum(x.astype(np.float64) @ b.astype(np.float64) + bias, 0)
    # hi alone is the bf16 rounding (~2^-9 relative); hi + lo keeps all but
    # lo's own rounding (<= 2^-18), on the input's split and on the output's
    assert rel_l2(h, ref) > 1e-4
    assert rel_l2(h.astype(np.float64) + l, ref) <= 5e-6 + 3.2e-9 * k, f"{rel_l2(h.astype(np.float64) + l, ref):.2e}"
    # lo is a rounding residual: at most half a bf16 ulp of hi, zero where hi is
    assert np.all(np.abs(l) <= np.abs(h) * 2.0 ** -8)
    assert np.all(l[h == 0] == 0)


def test_split_planes_are_checked(gpu):
    a, b, c = gpu.zeros((64, 64)), gpu.zeros((64, 64)), gpu.zeros((64, 64))
    args = G.GemmArgs(G.RT_NN, G.RT_F32, G.RT_F32, 64, 64, 64, a.ptr, a.ld, b.ptr, b.ld, c.ptr, c.ld,
                      G.RT_EPI_NONE, None, None, 0, 1, None, 0)
    args.a_lo = a.ptr
    with pytest.raises(rgpu_b200.RtError) as e:
        gpu.gemm(args)
    assert "a_lo" in str(e.value)
    args.a_lo = None
    args.c_lo = c.ptr
    with pytest.raises(rgpu_b200.RtError) as e:
        gpu.gemm(args)
    assert "c_lo" in str(e.value)
