"""The allocation-free split-K entry point (rt_matmul_split_k_noalloc).

Some callers cannot allocate device memory at the moment they call in (for
example when a host framework's own allocator owns the device memory, or in
a loop that forbids allocation after start-up), so this variant keeps its
split-K partial sums in a fixed scratch array inside librtgpu.so instead of a
caller buffer.
These tests call it through the C ABI and check it against the existing
rt_matmul_split_k (caller-provided partials) on two calls in a row, within the
split-K tolerance of the other GEMM tests.  This file is named to be
collected last.
"""
import numpy as np
import pytest

import rgpu_b200
from tests.helpers import erro_rel, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    g = rgpu_b200.Gpu(0)
    yield g
    g.close()


def _operands(m, n, k, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((m, k)).astype(np.float32), rng.standard_normal((k, n)).astype(np.float32)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_noalloc_split_k_matches_caller_buffer_version_twice(gpu, dtype):
    cases = [(64, 96, 4096, 8, True), (200, 136, 2048, 4, False)]
    for i, (m, n, k, slices, transposed) in enumerate(cases):
        a, b = _operands(m, n, k, i)
        ga = gpu.upload(np.ascontiguousarray(a.T) if transposed else a, dtype)
        gb = gpu.upload(b, dtype)
        want = gpu.zeros((m, n))
        parts = gpu.zeros((slices * m, n))
        gpu.split_k(ga, gb, want, parts, slices, transposed)
        got = gpu.zeros((m, n))
        gpu.split_k_noalloc(ga, gb, got, slices, transposed)
        w, g = gpu.download(want), gpu.download(got)
        if dtype == "f32":
            # The no-allocation variant keeps f32 operands on the SIMT kernel;
            # the caller-buffer version runs them on the tensor cores (3xTF32)
            # by default, so the two agree within the 3xTF32 GEMM bound of
            # test_gpu_ops.py ...
            assert rel_l2(g, w) <= 1e-6 + 3e-9 * k, f"call {i + 1}: {rel_l2(g, w):.2e}"
            # ... and bit for bit up to the split-K tolerance once the
            # caller-buffer version is put on the same SIMT kernel.
            gpu.set_f32_tensor(False)
            try:
                gpu.split_k(ga, gb, want, parts, slices, transposed)
            finally:
                gpu.set_f32_tensor(True)
            w = gpu.download(want)
        # Same kernels and the same fixed-order reduction: equal within the
        # split-K tolerance used by test_split_k_matches_unsplit (in practice
        # bit-identical).
        assert erro_rel(w, g) < 2e-5, f"call {i + 1}: {erro_rel(w, g):.2e}"


def test_noalloc_rejects_sizes_beyond_the_scratch(gpu):
    cap = rgpu_b200.Gpu.split_k_static_capacity()
    assert cap == 4 << 20
    m = n = 1024
    slices = cap // (m * n) + 1
    a, b = gpu.zeros((m, 64)), gpu.zeros((64, n))
    with pytest.raises(rgpu_b200.RtError) as e:
        gpu.split_k_noalloc(a, b, gpu.zeros((m, n)), slices, False)
    assert "exceed the built-in scratch" in str(e.value)
