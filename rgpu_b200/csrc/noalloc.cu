// Split-K GEMM whose partial-sum scratch lives in a fixed device array
// compiled into this library, so that a call allocates no device memory.
//
// Who needs this: callers that must not allocate device memory when they
// call in.  Two common cases: host runtimes whose own caching allocator owns
// the device memory and must not be bypassed behind its back (a cudaMalloc
// outside it can fail once that allocator has reserved the device, and it
// can synchronise the device, stalling the caller's other streams); and
// latency-bound loops that forbid allocation after start-up.
// rt_matmul_split_k needs the caller to provide the partials buffer; this
// variant does not.
//
// Limits and sharing rules:
//   - the scratch holds kScratchFloats f32 values (16 MiB) per device, held
//     by every device that loads this library until the process exits;
//     a call needs slices * m * n <= kScratchFloats and is rejected otherwise;
//   - every call on a device uses the same array and leaves its partial sums
//     in it.  Nothing needs clearing first: each call writes every partial it
//     later reads.  Two calls whose kernels overlap on the GPU (different
//     streams or contexts) race on the array: serialise them;
//   - the array's host-side name is not a device address; its device address
//     is looked up with cudaGetSymbolAddress, with the context's device
//     current, the first time this entry point runs on a context, and kept in
//     the context (a context created after a cudaDeviceReset looks it up
//     again).  Make that first call on a context before any stream capture
//     begins, so that the lookup is not made while a capture is open.
#include "internal.h"

namespace rt {
int run_gemm(rt_ctx* ctx, GemmDesc g, cudaStream_t stream, size_t ws_bytes);
}  // namespace rt

using namespace rt;

namespace {

constexpr size_t kScratchFloats = size_t(4) << 20;  // 16 MiB of f32 partials

static __device__ __align__(256) float g_splitk_scratch[kScratchFloats];

// Device address of the scratch array for ctx's device (looked up once per
// context, with the device current).
int scratch_for_context(rt_ctx* ctx, float** out) {
    if (!ctx->splitk_static) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_splitk_scratch);
        if (e != cudaSuccess || !p)
            return fail(RT_ERR_CUDA, "cudaGetSymbolAddress(split-K scratch) failed on device %d: %s", ctx->device,
                        cudaGetErrorString(e));
        ctx->splitk_static = static_cast<float*>(p);
    }
    *out = ctx->splitk_static;
    return RT_OK;
}

}  // namespace

extern "C" {

int64_t rt_split_k_static_capacity(void) { return (int64_t)kScratchFloats; }

int rt_matmul_split_k_noalloc(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c, int slices,
                              int transposed) {
    RT_CHECK(ctx && a && b && c, "rt_matmul_split_k_noalloc: NULL argument");
    RT_CHECK(a->ctx == ctx && b->ctx == ctx && c->ctx == ctx, "tensor belongs to another context");
    RT_CHECK(slices >= 1, "slices must be >= 1");
    const int64_t m = transposed ? a->cols : a->rows;
    const int64_t k = transposed ? a->rows : a->cols;
    RT_CHECK(b->rows == k && c->rows == m && c->cols == b->cols, "split_k_noalloc: incompatible shapes");
    RT_CHECK(a->dtype == b->dtype, "split_k_noalloc: operand dtypes differ");
    const int64_t n = b->cols;
    const size_t need = (size_t)slices * (size_t)m * (size_t)n;
    if (need > kScratchFloats)
        return fail(RT_ERR_INVALID,
                    "split_k_noalloc: %d slices x %lld x %lld = %zu partial sums exceed the built-in scratch of "
                    "%zu floats; use fewer slices or rt_matmul_split_k with a caller buffer",
                    slices, (long long)m, (long long)n, need, kScratchFloats);
    RT_CUDA(cudaSetDevice(ctx->device));
    float* scratch = nullptr;
    RT_TRY(scratch_for_context(ctx, &scratch));
    GemmDesc g{};
    g.layout = transposed ? RT_TN : RT_NN;
    g.in_dtype = a->dtype;
    g.out_dtype = c->dtype;
    g.m = m;
    g.n = n;
    g.k = k;
    g.a = a->ptr;
    g.lda = a->ld;
    g.b = b->ptr;
    g.ldb = b->ld;
    g.c = c->ptr;
    g.ldc = c->ld;
    g.epi = RT_EPI_NONE;
    g.split_k = slices;
    g.workspace = scratch;
    g.no_alloc = true;  // f32 operands stay on the SIMT kernel (the 3xTF32 path needs an operand workspace)
    return run_gemm(ctx, g, ctx->stream, kScratchFloats * sizeof(float));
}

}  // extern "C"
