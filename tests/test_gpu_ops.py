"""Op-level parity of the CUDA kernels against the CPU oracle.

Mirrors crates/rtensor/tests/gpu.rs (round trip, GEMM in every layout on
ragged shapes, split-K, mixed precision) and adds the kernels the reference
has only on the CPU (SGD) or that the B200 design fuses (bias/ReLU/mask
epilogues).  Every call goes through librtgpu.so's C ABI.
"""
import numpy as np
import pytest

import oracle
import rgpu_b200
from rgpu_b200 import gpu as G
from tests.helpers import erro_rel, rel_l2

pytestmark = pytest.mark.gpu

# gpu.rs:250-258: degenerate (1), below a tile (17), one tile (64), just past
# (65), unaligned (130, 199) and a larger multiple.
SHAPES = [(1, 1, 1), (17, 33, 65), (64, 64, 64), (65, 64, 63), (130, 96, 80), (199, 130, 71), (256, 512, 128)]


@pytest.fixture(scope="module")
def gpu():
    g = rgpu_b200.Gpu(0)
    yield g
    g.close()


def _ab(m, n, k):
    a = np.sin(np.arange(m * k, dtype=np.float32) * np.float32(0.013)).reshape(m, k).astype(np.float32)
    b = np.cos(np.arange(k * n, dtype=np.float32) * np.float32(0.007)).reshape(k, n).astype(np.float32)
    return a, b


def test_upload_download_roundtrip(gpu):
    # gpu.rs:215-221
    t = (np.arange(15, dtype=np.float32) * 0.5 - 3.0).reshape(3, 5)
    assert np.array_equal(gpu.download(gpu.upload(t)), t)


def test_matmul_37x23x19(gpu):
    # gpu.rs:223-240
    a = np.sin(np.arange(37 * 23, dtype=np.float32) * np.float32(0.11)).reshape(37, 23)
    b = np.cos(np.arange(23 * 19, dtype=np.float32) * np.float32(0.07)).reshape(23, 19)
    ga, gb, gc = gpu.upload(a), gpu.upload(b), gpu.zeros((37, 19))
    gpu.matmul(ga, gb, gc)
    assert erro_rel(oracle.matmul(a, b), gpu.download(gc)) < 1e-5


@pytest.mark.parametrize("fast", [False, True])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_all_layouts_f32(gpu, fast, m, n, k):
    # gpu.rs:244-295: all three variants, f32, error < 1e-5 against the CPU.
    gpu.set_fast_gemm(fast)
    try:
        a, b = _ab(m, n, k)
        want = oracle.matmul(a, b)
        ga, gb = gpu.upload(a), gpu.upload(b)
        gat, gbt = gpu.upload(np.ascontiguousarray(a.T)), gpu.upload(np.ascontiguousarray(b.T))
        c1, c2, c3 = gpu.zeros((m, n)), gpu.zeros((m, n)), gpu.zeros((m, n))
        gpu.matmul(ga, gb, c1)
        gpu.matmul_at_b(gat, gb, c2)
        gpu.matmul_a_bt(ga, gbt, c3)
        for name, c in (("mm", c1), ("mm_atb", c2), ("mm_abt", c3)):
            e = erro_rel(want, gpu.download(c))
            assert e < 1e-5, f"{name} {m}x{n}x{k} fast={fast}: {e:.2e}"
    finally:
        gpu.set_fast_gemm(True)


@pytest.mark.parametrize("m,n,k", [(64, 64, 64), (256, 128, 512), (512, 512, 256), (200, 136, 72)])
def test_gemm_bf16_operands(gpu, m, n, k):
    # gpu.rs:445-503 (f16 there): error < 10 sqrt(K) 2^-8 for bf16's 8-bit mantissa.
    a, b = _ab(m, n, k)
    want = oracle.matmul(a, b)
    bound = 10.0 * np.sqrt(k) * 2.0 ** -8
    ga, gb = gpu.upload(a, "bf16"), gpu.upload(b, "bf16")
    gat = gpu.upload(np.ascontiguousarray(a.T), "bf16")
    gbt = gpu.upload(np.ascontiguousarray(b.T), "bf16")
    for name, fn, x, y in (("A.B", gpu.matmul, ga, gb), ("At.B", gpu.matmul_at_b, gat, gb),
                           ("A.Bt", gpu.matmul_a_bt, ga, gbt)):
        c = gpu.zeros((m, n))
        fn(x, y, c)
        e = erro_rel(want, gpu.download(c))
        assert e < bound, f"{name} {m}x{n}x{k}: {e:.2e} >= {bound:.2e}"


@pytest.mark.parametrize("m,n,k", [(64, 1000, 8192), (128, 256, 4096), (128, 64, 8192), (300, 200, 2048),
                                   (256, 512, 520)])
def test_tensor_core_gemm_accuracy_deep_k(gpu, m, n, k):
    # Against the exact (f64) product of the bf16-rounded operands.  The
    # tensor cores truncate while accumulating, so the error grows ~linearly
    # with k: measured 9e-6 at k = 8192.
    rng = np.random.default_rng(k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    qa = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(a)).astype(np.float64)
    qb = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(b)).astype(np.float64)
    ref = qa @ qb
    bound = 1e-6 + 1.6e-9 * k
    ga, gb = gpu.upload(a, "bf16"), gpu.upload(b, "bf16")
    gat = gpu.upload(np.ascontiguousarray(a.T), "bf16")
    gbt = gpu.upload(np.ascontiguousarray(b.T), "bf16")
    for name, fn, x, y in (("NN", gpu.matmul, ga, gb), ("TN", gpu.matmul_at_b, gat, gb),
                           ("NT", gpu.matmul_a_bt, ga, gbt)):
        c = gpu.zeros((m, n))
        fn(x, y, c)
        e = rel_l2(gpu.download(c), ref)
        assert e <= bound, f"{name} {m}x{n}x{k}: {e:.2e} > {bound:.2e}"


@pytest.mark.parametrize("m,n,k", [(64, 1000, 8192), (128, 256, 4096), (300, 200, 2048), (513, 1024, 2048),
                                   (2048, 10, 1024), (37, 23, 19)])
def test_f32_tensor_core_gemm_tracks_the_exact_product(gpu, m, n, k):
    # f32 operands on the tensor cores as three tf32 products (3xTF32),
    # against the exact f64 product.  The split itself loses < 2^-20 per
    # product; the rest is the tensor cores' truncating f32 accumulation,
    # which grows linearly with the number of 8-deep MMA steps (k / 8 per
    # segment, twice the bf16 path's k / 16): measured 1.95e-5 at k = 8192,
    # inside the 1e-4 f32 gradient bar up to k ~ 40000.  The SIMT f32 kernel
    # (round-to-nearest FMA) is held to the bf16 test's tighter bound.
    rng = np.random.default_rng(k + m)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    ga, gb = gpu.upload(a), gpu.upload(b)
    gat, gbt = gpu.upload(np.ascontiguousarray(a.T)), gpu.upload(np.ascontiguousarray(b.T))
    try:
        for tensor in (True, False):
            gpu.set_f32_tensor(tensor)
            bound = 1e-6 + (3e-9 if tensor else 1.6e-9) * k
            for name, fn, x, y in (("NN", gpu.matmul, ga, gb), ("TN", gpu.matmul_at_b, gat, gb),
                                   ("NT", gpu.matmul_a_bt, ga, gbt)):
                c = gpu.zeros((m, n))
                fn(x, y, c)
                e = rel_l2(gpu.download(c), ref)
                assert e <= bound, f"{name} {m}x{n}x{k} tensor={tensor}: {e:.2e} > {bound:.2e}"
    finally:
        gpu.set_f32_tensor(True)


def test_f32_gemm_runs_on_the_tensor_cores(gpu):
    # An aligned f32 GEMM is two launches on the tensor-core path (operand
    # split + tcgen05 GEMM) and one on the SIMT path.
    a, b = _ab(256, 512, 128)
    ga, gb, c = gpu.upload(a), gpu.upload(b), gpu.zeros((256, 512))
    try:
        counts = {}
        for tensor in (True, False):
            gpu.set_f32_tensor(tensor)
            before = gpu.launch_count()
            gpu.matmul(ga, gb, c)
            gpu.sync()
            counts[tensor] = gpu.launch_count() - before
            assert erro_rel(oracle.matmul(a, b), gpu.download(c)) < 1e-5
        assert counts == {True: 2, False: 1}, counts
    finally:
        gpu.set_f32_tensor(True)


def test_f32_tensor_core_gemm_non_finite_inputs(gpu):
    # A non-finite operand makes its output row non-finite, as in an f32 GEMM
    # (inf may come out as NaN: the split's hi(A) lo(B) product is inf * 0),
    # and leaves every other row exact.
    a = np.ones((128, 64), np.float32)
    b = np.ones((64, 128), np.float32)
    a[3, 5] = np.inf
    a[7, 9] = np.nan
    c = gpu.zeros((128, 128))
    gpu.matmul(gpu.upload(a), gpu.upload(b), c)
    got = gpu.download(c)
    assert not np.isfinite(got[3]).any() and np.isnan(got[7]).all()
    rest = np.delete(got, [3, 7], axis=0)
    assert np.array_equal(rest, np.full_like(rest, 64.0))


def test_bf16_output_store(gpu):
    a, b = _ab(96, 80, 48)
    ga, gb = gpu.upload(a, "bf16"), gpu.upload(b, "bf16")
    c = gpu.zeros((96, 80), "bf16")
    gpu.matmul(ga, gb, c)
    got = gpu.download(c)
    ref = oracle.matmul(rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(a)),
                        rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(b)))
    assert rel_l2(got, ref) < 4e-3


@pytest.mark.parametrize("relu", [False, True])
def test_matmul_bias_epilogue(gpu, relu):
    # gemm.rs:372-494 (MM_EPILOGO): C = A B + 1 b, ReLU in registers.
    m, n, k = 130, 96, 80
    a, b = _ab(m, n, k)
    bias = np.linspace(-1, 1, n, dtype=np.float32).reshape(1, n)
    want = oracle.matmul(a, b) + bias
    if relu:
        want = np.maximum(want, 0)
    c = gpu.zeros((m, n))
    gpu.matmul_bias(gpu.upload(a), gpu.upload(b), c, gpu.upload(bias), relu)
    assert erro_rel(want, gpu.download(c)) < 1e-5


def test_relu_mask_epilogue_via_rt_gemm(gpu):
    # kernels.rs:119-131 fused into the dX GEMM: C = (A B^T) * 1[mask > 0].
    m, n, k = 199, 130, 71
    a, b = _ab(m, n, k)
    bt = np.ascontiguousarray(b.T)
    mask = np.sin(np.arange(m * n, dtype=np.float32) * 0.5).reshape(m, n).astype(np.float32)
    want = oracle.matmul(a, b) * (mask > 0)
    ga, gbt, gm = gpu.upload(a), gpu.upload(bt), gpu.upload(mask)
    c = gpu.zeros((m, n))
    args = G.GemmArgs(G.RT_NT, G.RT_F32, G.RT_F32, m, n, k, ga.ptr, ga.ld, gbt.ptr, gbt.ld, c.ptr, c.ld,
                      G.RT_EPI_RELU_MASK, None, gm.ptr, gm.ld, 1, None, 0)
    gpu.gemm(args)
    assert erro_rel(want, gpu.download(c)) < 1e-5


SKINNY = [(2048, 10, 1024), (1025, 10, 2048), (2048, 1024, 10), (37, 16, 300), (300, 200, 16), (5, 3, 7),
          (129, 1, 4096), (64, 2000, 1), (70, 203, 5), (70, 204, 9)]


def _skinny_ref(a, b, epi, bias, mask):
    want = a.astype(np.float64) @ b.astype(np.float64)
    if epi in (G.RT_EPI_BIAS, G.RT_EPI_BIAS_RELU):
        want = want + bias
    if epi == G.RT_EPI_BIAS_RELU:
        want = np.maximum(want, 0)
    if epi == G.RT_EPI_RELU_MASK:
        want = want * (mask > 0)
    return want


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("m,n,k", SKINNY)
def test_skinny_gemms_every_layout_and_epilogue(gpu, m, n, k, dtype):
    # n <= 16 or k <= 16 (an output layer's classes) runs on the skinny CUDA-core
    # kernels: narrow N over A K-major (NN, NT), narrow N over A MN-major (TN,
    # with and without k slices), narrow K.  Every layout and epilogue against
    # the exact (f64) result, bf16 on the bf16-rounded operands; the kernels
    # sum k in lane-strided order, so the bound is the SIMT f32 one used for
    # the 3xTF32 test above.
    a, b = _ab(m, n, k)
    if dtype == "bf16":
        a = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(a))
        b = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(b))
    bias = np.linspace(-1, 1, n, dtype=np.float32).reshape(1, n)
    mask = np.sin(np.arange(m * n, dtype=np.float32) * 0.5).reshape(m, n).astype(np.float32)
    ops = {G.RT_NN: (a, b), G.RT_NT: (a, np.ascontiguousarray(b.T)), G.RT_TN: (np.ascontiguousarray(a.T), b)}
    gbias, gmask = gpu.upload(bias), gpu.upload(mask)
    for layout, (x, y) in ops.items():
        gx, gy = gpu.upload(x, dtype), gpu.upload(y, dtype)
        for epi in (G.RT_EPI_NONE, G.RT_EPI_BIAS, G.RT_EPI_BIAS_RELU, G.RT_EPI_RELU_MASK):
            for split in ((1, 4) if layout == G.RT_TN else (1,)):
                c = gpu.zeros((m, n))
                ws = gpu.zeros((split * m, n)) if split > 1 else None
                args = G.GemmArgs(layout, G.RT_BF16 if dtype == "bf16" else G.RT_F32, G.RT_F32, m, n, k,
                                  gx.ptr, gx.ld, gy.ptr, gy.ld, c.ptr, c.ld, epi, gbias.ptr, gmask.ptr, gmask.ld,
                                  split, ws.ptr if ws is not None else None,
                                  split * m * n * 4 if ws is not None else 0)
                gpu.gemm(args)
                e = rel_l2(gpu.download(c), _skinny_ref(a, b, epi, bias, mask))
                assert e <= 1e-6 + 1.6e-9 * k, f"layout {layout} epi {epi} split {split} {m}x{n}x{k} {dtype}: {e:.2e}"


@pytest.mark.parametrize("m,n,k", [(256, 512, 1), (300, 200, 8), (512, 1024, 16), (2048, 1024, 10)])
def test_narrow_k_gemms_on_the_tensor_cores(monkeypatch, m, n, k):
    # RTGPU_SKINNY_K_MAX=0 sends every narrow-K GEMM that the tensor cores
    # can take there (one k-block, zero-filled past k): f32 operands as
    # 3xTF32 in two launches (operand split, GEMM), bf16 in one.  Against the
    # exact product of the (bf16-rounded) operands, with the 3xTF32 bound.
    monkeypatch.setenv("RTGPU_SKINNY_K_MAX", "0")
    g = rgpu_b200.Gpu(0)
    try:
        a0, b0 = _ab(m, n, k)
        mask = np.sin(np.arange(m * n, dtype=np.float32) * 0.5).reshape(m, n).astype(np.float32)
        gmask = g.upload(mask)
        for dtype, launches in (("f32", 2), ("bf16", 1)):
            a, b = a0, b0
            if dtype == "bf16":
                a = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(a))
                b = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(b))
            ops = {G.RT_NN: (a, b), G.RT_NT: (a, np.ascontiguousarray(b.T)), G.RT_TN: (np.ascontiguousarray(a.T), b)}
            for layout, (x, y) in ops.items():
                gx, gy = g.upload(x, dtype), g.upload(y, dtype)
                for epi in (G.RT_EPI_NONE, G.RT_EPI_RELU_MASK):
                    c = g.zeros((m, n))
                    args = G.GemmArgs(layout, G.RT_BF16 if dtype == "bf16" else G.RT_F32, G.RT_F32, m, n, k,
                                      gx.ptr, gx.ld, gy.ptr, gy.ld, c.ptr, c.ld, epi, None, gmask.ptr, gmask.ld,
                                      1, None, 0)
                    before = g.launch_count()
                    g.gemm(args)
                    g.sync()
                    assert g.launch_count() - before == launches, (dtype, layout, epi)
                    e = rel_l2(g.download(c), _skinny_ref(a, b, epi, None, mask))
                    assert e <= 1e-6 + 3e-9 * k, f"layout {layout} epi {epi} {m}x{n}x{k} {dtype}: {e:.2e}"
    finally:
        g.close()


def test_skinny_gemm_is_one_launch(gpu):
    a, b = _ab(2048, 10, 1024)
    ga, gb, c = gpu.upload(a), gpu.upload(b), gpu.zeros((2048, 10))
    before = gpu.launch_count()
    gpu.matmul(ga, gb, c)
    gpu.sync()
    assert gpu.launch_count() - before == 1
    assert rel_l2(gpu.download(c), a.astype(np.float64) @ b.astype(np.float64)) < 3e-6


@pytest.mark.parametrize("m,n,k", [(64, 64, 4096), (32, 96, 2048), (128, 64, 1024)])
def test_split_k_matches_unsplit(gpu, m, n, k):
    # gpu.rs:383-430: 1/2/4/8/16 slices, NN and TN, error <= 3x the unsplit GEMM.
    a, b = _ab(m, n, k)
    want = oracle.matmul(a, b)
    ga, gat, gb = gpu.upload(a), gpu.upload(np.ascontiguousarray(a.T)), gpu.upload(b)
    c0 = gpu.zeros((m, n))
    gpu.matmul(ga, gb, c0)
    e0 = erro_rel(want, gpu.download(c0))
    for slices in (1, 2, 4, 8, 16):
        for transposed, x in ((False, ga), (True, gat)):
            c = gpu.zeros((m, n))
            parts = gpu.zeros((slices * m, n))
            gpu.split_k(x, gb, c, parts, slices, transposed)
            e = erro_rel(want, gpu.download(c))
            assert e < max(3 * e0, 2e-5), f"{m}x{n}x{k} slices={slices} T={transposed}: {e:.2e} vs {e0:.2e}"


def test_gemm_empty_and_zero_k(gpu):
    # k = 0 must give exactly the epilogue of a zero accumulator.
    a = gpu.zeros((5, 0))
    b = gpu.zeros((0, 7))
    c = gpu.upload(np.full((5, 7), 3.0, np.float32))
    gpu.matmul(a, b, c)
    assert np.array_equal(gpu.download(c), np.zeros((5, 7), np.float32))
    e = gpu.zeros((0, 4))
    gpu.matmul(e, gpu.zeros((4, 3)), gpu.zeros((0, 3)))
    gpu.sync()


def test_shape_mismatch_is_an_error_not_a_crash(gpu):
    with pytest.raises(rgpu_b200.RtError) as ei:
        gpu.matmul(gpu.zeros((4, 5)), gpu.zeros((6, 3)), gpu.zeros((4, 3)))
    assert ei.value.code == G.RT_ERR_INVALID


@pytest.mark.parametrize("n,c", [(64, 4), (37, 10), (512, 1000), (3, 1)])
def test_softmax_xent_matches_oracle(gpu, n, c):
    # kernels.rs:138-167 vs losses.rs:99-115
    rng = oracle.Rng(3)
    z = (rng.normal(n * c) * 3).reshape(n, c)
    labels = rng.below(c, n)
    loss_ref, d_ref = oracle.softmax_xent(z, oracle.one_hot(labels, c))
    gz, gl = gpu.upload(z), rgpu_b200.upload_labels(gpu, labels)
    d, loss = gpu.zeros((n, c)), gpu.zeros((n,))
    gpu.softmax_xent(gz, gl, d, loss)
    rows = gpu.download(loss).ravel()
    assert abs(float(np.float32(rows.sum()) / n) - loss_ref) < 1e-5 * max(1, abs(loss_ref))
    assert erro_rel(d_ref, gpu.download(d)) < 1e-6


def test_softmax_xent_saturated_logits(gpu):
    # autodiff.rs:62-72: logits of 100 must stay finite.
    z = np.array([[1, 2, 3], [100, 100, 100], [1000, -1000, 0]], np.float32)
    labels = np.array([2, 0, 1], np.uint32)
    loss_ref, d_ref = oracle.softmax_xent(z, oracle.one_hot(labels, 3))
    d, loss = gpu.zeros((3, 3)), gpu.zeros((3,))
    gpu.softmax_xent(gpu.upload(z), rgpu_b200.upload_labels(gpu, labels), d, loss)
    got = gpu.download(d)
    assert np.all(np.isfinite(got))
    assert erro_rel(d_ref, got) < 1e-6
    assert abs(gpu.download(loss).mean() - loss_ref) < 1e-4


@pytest.mark.parametrize("rows,cols", [(1, 1), (32, 10), (64, 130), (65, 7), (2048, 1024), (8192, 33)])
def test_colsum_matches_reduce_to(gpu, rows, cols):
    # kernels.rs:182-199 vs tensor.rs:410-418
    g = oracle.Rng(11).normal(rows * cols).reshape(rows, cols)
    src, dst = gpu.upload(g), gpu.zeros((1, cols))
    scratch = gpu.zeros((max(1, (rows + 63) // 64), cols))
    gpu.colsum(src, dst, scratch)
    # Both sums round differently (64-row chunks vs one sequential sweep); the
    # GPU's must be at least about as close to the exact sum as the CPU's.
    exact = g.astype(np.float64).sum(0, keepdims=True)
    e_cpu = erro_rel(exact, oracle.reduce_rows(g))
    e_gpu = erro_rel(exact, gpu.download(dst))
    assert e_gpu <= 2 * e_cpu + 1e-6, (e_gpu, e_cpu)


def test_bias_add_relu_relu_bwd(gpu):
    rng = oracle.Rng(2)
    z = rng.normal(50 * 9).reshape(50, 9)
    b = rng.normal(9).reshape(1, 9)
    gz = gpu.upload(z)
    gpu.bias_add(gz, gpu.upload(b))
    assert np.array_equal(gpu.download(gz), z + b)
    y = gpu.zeros((50, 9))
    gpu.relu(gz, y)
    a = np.maximum(z + b, 0)
    assert np.array_equal(gpu.download(y), a)
    dz = rng.normal(50 * 9).reshape(50, 9)
    gdz = gpu.upload(dz)
    gpu.relu_bwd(y, gdz)
    assert np.array_equal(gpu.download(gdz), dz * (a > 0))


@pytest.mark.parametrize("n", [1, 7, 1000, 4099])
def test_adam_is_bit_exact_with_cpu_optimiser(gpu, n):
    # optim.rs:163-198: same rounding sequence, so equal bit for bit.
    rng = oracle.Rng(5)
    theta = rng.normal(n)
    th_ref, m_ref, v_ref = theta.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    gt, gm, gv = gpu.upload(theta), gpu.zeros((n,)), gpu.zeros((n,))
    for t in range(1, 4):
        g = rng.normal(n)
        oracle.adam_update(th_ref, m_ref, v_ref, g, 1e-3, t)
        gpu.adam(gt, gm, gv, gpu.upload(g), 1e-3, t)
    assert np.array_equal(gpu.download(gt).ravel(), th_ref)
    assert np.array_equal(gpu.download(gm).ravel(), m_ref)
    assert np.array_equal(gpu.download(gv).ravel(), v_ref)


def test_sgd_is_bit_exact(gpu):
    rng = oracle.Rng(6)
    theta = rng.normal(1027)
    g = rng.normal(1027)
    ref = theta.copy()
    oracle.sgd_update(ref, g, 0.01)
    gt = gpu.upload(theta)
    gpu.sgd(gt, gpu.upload(g), 0.01)
    assert np.array_equal(gpu.download(gt).ravel(), ref)


def test_cast_rounds_to_nearest_even(gpu):
    x = oracle.Rng(9).normal(333) * 100
    src, dst = gpu.upload(x), gpu.zeros((333,), "bf16")
    gpu.cast(src, dst)
    want = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(x))
    assert np.array_equal(gpu.download(dst).ravel(), want)


@pytest.mark.parametrize("rows,cols", [(8192, 4096), (3, 5), (257, 24), (64, 1000)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_same_dtype_cast_is_an_exact_copy(gpu, rows, cols, dtype):
    # A same-dtype rt_cast copies rows (16-byte vectors when every row start
    # allows them, the element loop otherwise); padding columns stay zero.
    x = np.random.default_rng(rows + cols).standard_normal((rows, cols)).astype(np.float32)
    if dtype == "bf16":
        x = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(x))
    src, dst = gpu.upload(x, dtype), gpu.zeros((rows, cols), dtype)
    gpu.cast(src, dst)
    assert np.array_equal(gpu.download(dst), x)


@pytest.mark.parametrize("m,n,k", [(1, 1024, 512), (5, 1000, 1024), (16, 130, 300), (17, 4096, 257),
                                   (64, 1024, 1024), (32, 8192, 4096)])
def test_few_row_gemms(gpu, m, n, k):
    # Forward GEMMs at small batch (layout NN, m <= 16, or m <= 64 for f32):
    # a cluster of CTAs splits k and sums in a fixed order.  Against the exact
    # product, with the bias and bias + ReLU epilogues; bf16 operands (m <= 16)
    # also with A as hi + lo planes and a lo output plane.
    a, b = _ab(m, n, k)
    bias = np.linspace(-1, 1, n, dtype=np.float32).reshape(1, n)
    gbias = gpu.upload(bias)
    for dtype in ("f32", "bf16"):
        if dtype == "bf16" and m > 16:
            continue
        x = a if dtype == "f32" else rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(a))
        w = b if dtype == "f32" else rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(b))
        gx, gw = gpu.upload(x, dtype), gpu.upload(w, dtype)
        for epi in (G.RT_EPI_NONE, G.RT_EPI_BIAS, G.RT_EPI_BIAS_RELU):
            c = gpu.zeros((m, n))
            args = G.GemmArgs(G.RT_NN, G.RT_BF16 if dtype == "bf16" else G.RT_F32, G.RT_F32, m, n, k,
                              gx.ptr, gx.ld, gw.ptr, gw.ld, c.ptr, c.ld, epi, gbias.ptr, None, 0, 1, None, 0)
            before = gpu.launch_count()
            gpu.gemm(args)
            gpu.sync()
            assert gpu.launch_count() - before == 1
            ref = _skinny_ref(x, w, epi, bias, None)
            got = gpu.download(c)
            e = rel_l2(got, ref)
            # The sin/cos operands of the larger shapes cancel heavily (at
            # 32 x 8192 x 4096 the outputs' rms is 0.23 against sums of |terms|
            # near 1660), so any f32 summation order is ~1e-4 off in relative
            # L2 there (the kernel's order, replayed in numpy float32, gives the
            # same 9.55e-5).  Such cases are held to the f32 forward-error bound
            # instead: the error against |x| |w| (+ |bias|), sqrt(k) units of
            # f32 roundoff, far below what a wrong or missing k slice gives.
            mag = np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64) + np.abs(bias)
            e_mag = float(np.linalg.norm(got - ref) / np.linalg.norm(mag))
            assert e <= 1e-5 or e_mag <= np.sqrt(k) * 2.0**-24, \
                f"{dtype} epi {epi} {m}x{n}x{k}: rel L2 {e:.2e}, against |x||w| {e_mag:.2e}"
    if m <= 16:
        # split A planes and a bf16 output with its lo plane
        hi = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(np.abs(a)))
        lo = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(np.abs(a) - hi))
        w = rgpu_b200.bf16_to_f32(rgpu_b200.f32_to_bf16(b))
        ghi, glo, gw = gpu.upload(hi, "bf16"), gpu.upload(lo, "bf16"), gpu.upload(w, "bf16")
        chi, clo = gpu.zeros((m, n), "bf16"), gpu.zeros((m, n), "bf16")
        args = G.GemmArgs(G.RT_NN, G.RT_BF16, G.RT_BF16, m, n, k, ghi.ptr, ghi.ld, gw.ptr, gw.ld, chi.ptr, chi.ld,
                          G.RT_EPI_BIAS_RELU, gbias.ptr, None, 0, 1, None, 0)
        args.a_lo, args.c_lo = glo.ptr, clo.ptr
        gpu.gemm(args)
        ref = _skinny_ref((hi.astype(np.float64) + lo), w, G.RT_EPI_BIAS_RELU, bias, None)
        got = gpu.download(chi).astype(np.float64) + gpu.download(clo)
        assert rel_l2(got, ref) <= 1e-5, f"split {m}x{n}x{k}: {rel_l2(got, ref):.2e}"


def test_device_wait_timeout_is_reported_and_the_context_stays_usable(gpu):
    # A kernel whose bounded barrier wait runs out (nothing signals the
    # barrier) records a timeout instead of spinning or faulting; the next
    # sync reports RT_ERR_DEVICE_TIMEOUT, clears it, and the context keeps
    # working.
    import time

    t0 = time.perf_counter()
    gpu.selftest_timeout()
    with pytest.raises(rgpu_b200.RtError) as e:
        gpu.sync()
    waited = time.perf_counter() - t0
    assert e.value.code == G.RT_ERR_DEVICE_TIMEOUT and "self-test" in str(e.value)
    assert 1.5 < waited < 30.0, waited  # the 2 s wait limit, not a hang
    gpu.sync()  # the error word was cleared
    a, b = _ab(64, 48, 32)
    c = gpu.zeros((64, 48))
    gpu.matmul(gpu.upload(a), gpu.upload(b), c)
    gpu.sync()
    assert erro_rel(oracle.matmul(a, b), gpu.download(c)) < 1e-5
