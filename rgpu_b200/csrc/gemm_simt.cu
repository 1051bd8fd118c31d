// Tiled SIMT GEMM (f32 FMA, f32 accumulate) for every layout and epilogue.
//
// This is the counterpart of rtensor's scalar tiled GEMM MM_FAST
// (crates/rtensor/src/gpu/gemm.rs:65-342: mm / mm_atb / mm_abt) and of its
// fused epilogue MM_EPILOGO (gemm.rs:372-494), and of the split-K product
// (splitk.rs:33-237).  On B200 it is the path for operands the tensor-core
// kernel cannot take (rows not 16-byte aligned, odd leading dimensions) and
// the exact-f32 reference path when fast GEMM is switched off
// (Gpu::set_fast_gemm, gpu/mod.rs:442-448).
//
// Tile: 128x128 outputs per 256-thread block, 8 outputs x 8 outputs per
// thread, k depth 8 per stage, register-prefetched double buffer in shared
// memory.
#include "internal.h"

namespace rt {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, THREADS = 256;

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ void store_out(void* c, int64_t idx, float v);
template <>
__device__ __forceinline__ void store_out<float>(void* c, int64_t idx, float v) {
    static_cast<float*>(c)[idx] = v;
}
template <>
__device__ __forceinline__ void store_out<__nv_bfloat16>(void* c, int64_t idx, float v) {
    static_cast<__nv_bfloat16*>(c)[idx] = __float2bfloat16_rn(v);
}

template <typename T>
__device__ __forceinline__ float load_mask(const void* mask, int64_t idx) {
    return to_f(static_cast<const T*>(mask)[idx]);
}

struct SimtParams {
    const void* a;
    const void* a2;  // A's low-order bf16 plane (null = none): A(i,k) = a + a2, exact in f32
    const void* b;
    void* c;
    void* c_lo;      // bf16 output's low-order plane (null = none)
    float* ws;
    const float* bias;
    const void* mask;
    int64_t m, n, k, lda, ldb, ldc, ldmask;
    int64_t k_per_slice;
    int epi;
    int out_bf16;
    OptFuse opt;
};

// Applies the epilogue to one accumulator and stores it.
template <typename TOut>
__device__ __forceinline__ void finish(const SimtParams& p, int64_t i, int64_t j, float v) {
    if (p.epi == RT_EPI_BIAS || p.epi == RT_EPI_BIAS_RELU) v = v + p.bias[j];
    if (p.epi == RT_EPI_BIAS_RELU) v = fmaxf(v, 0.0f);
    if (p.epi == RT_EPI_RELU_MASK) v = v * (load_mask<TOut>(p.mask, i * p.ldmask + j) > 0.0f ? 1.0f : 0.0f);
    store_out<TOut>(p.c, i * p.ldc + j, v);
    if (sizeof(TOut) == 2 && p.c_lo)
        store_out<TOut>(p.c_lo, i * p.ldc + j, v - __bfloat162float(__float2bfloat16_rn(v)));
}

// A_KMAJOR: A(i,k) = a[i*lda + k], else a[k*lda + i].
// B_KMAJOR: B(k,j) = b[j*ldb + k], else b[k*ldb + j].
template <typename TIn, bool A_KMAJOR, bool B_KMAJOR>
__global__ void __launch_bounds__(THREADS) gemm_simt_kernel(SimtParams p) {
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const TIn* A = static_cast<const TIn*>(p.a);
    const TIn* A2 = static_cast<const TIn*>(p.a2);
    const TIn* B = static_cast<const TIn*>(p.b);
    const int tid = threadIdx.x;
    const int64_t m0 = (int64_t)blockIdx.y * BM;
    const int64_t n0 = (int64_t)blockIdx.x * BN;
    const int64_t kbeg = (int64_t)blockIdx.z * p.k_per_slice;
    const int64_t kend = min(p.k, kbeg + p.k_per_slice);

    // Each thread stages 4 elements of A and 4 of B per k tile.
    float ra[4], rb[4];
    auto load_tile = [&](int64_t k0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int row, kk;
            if (A_KMAJOR) {
                row = tid / BK + q * (THREADS / BK);
                kk = tid % BK;
            } else {
                row = tid % BM;
                kk = tid / BM + q * (THREADS / BM);
            }
            int64_t gi = m0 + row, gk = k0 + kk;
            float v = 0.0f;
            if (gi < p.m && gk < kend) {
                const int64_t ai = A_KMAJOR ? gi * p.lda + gk : gk * p.lda + gi;
                v = to_f(A[ai]);
                if (A2) v += to_f(A2[ai]);
            }
            ra[q] = v;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int col, kk;
            if (B_KMAJOR) {
                col = tid / BK + q * (THREADS / BK);
                kk = tid % BK;
            } else {
                col = tid % BN;
                kk = tid / BN + q * (THREADS / BN);
            }
            int64_t gj = n0 + col, gk = k0 + kk;
            float v = 0.0f;
            if (gj < p.n && gk < kend) v = to_f(B_KMAJOR ? B[gj * p.ldb + gk] : B[gk * p.ldb + gj]);
            rb[q] = v;
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int row, kk;
            if (A_KMAJOR) {
                row = tid / BK + q * (THREADS / BK);
                kk = tid % BK;
            } else {
                row = tid % BM;
                kk = tid / BM + q * (THREADS / BM);
            }
            As[buf][kk][row] = ra[q];
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int col, kk;
            if (B_KMAJOR) {
                col = tid / BK + q * (THREADS / BK);
                kk = tid % BK;
            } else {
                col = tid % BN;
                kk = tid / BN + q * (THREADS / BN);
            }
            Bs[buf][kk][col] = rb[q];
        }
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    const int ty = tid / 16, tx = tid % 16;
    int buf = 0;
    if (kbeg < kend) {
        load_tile(kbeg);
        store_tile(0);
    }
    __syncthreads();
    for (int64_t k0 = kbeg; k0 < kend; k0 += BK) {
        bool more = k0 + BK < kend;
        if (more) load_tile(k0 + BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
            float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
            float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (more) {
            store_tile(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int64_t gi = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (gi >= p.m) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int64_t gj = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (gj >= p.n) continue;
            if (p.ws) {
                p.ws[(int64_t)blockIdx.z * p.m * p.n + gi * p.n + gj] = acc[i][j];
            } else if (p.out_bf16) {
                finish<__nv_bfloat16>(p, gi, gj, acc[i][j]);
            } else {
                finish<float>(p, gi, gj, acc[i][j]);
            }
        }
        if (!p.ws && p.opt.kind) {
            // the gradient row segments this thread owns, updated in place
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                int64_t gj0 = n0 + half * 64 + tx * 4;
                int64_t rem = p.n - gj0;
                int cnt = rem < 4 ? (int)rem : 4;
                if (cnt > 0) opt_apply_row<4>(p.opt, gi * p.ldc + gj0, &acc[i][half * 4], cnt);
            }
        }
    }
}

// Deterministic split-K reduction: slices summed in ascending order, then the
// epilogue (splitk.rs:240-256 REDUZ, plus bias/ReLU/mask).
__global__ void splitk_reduce_kernel(SimtParams p, int slices) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    int64_t total = p.m * p.n;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        // slices summed in order; loads issued eight at a time ahead of the adds
        float s = 0.0f;
        for (int z0 = 0; z0 < slices; z0 += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = z0 + u < slices ? __ldg(p.ws + (int64_t)(z0 + u) * total + idx) : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (z0 + u < slices) s += v[u];
        }
        int64_t i = idx / p.n, j = idx % p.n;
        if (p.out_bf16)
            finish<__nv_bfloat16>(p, i, j, s);
        else
            finish<float>(p, i, j, s);
        if (p.opt.kind) opt_apply_row<1>(p.opt, i * p.ldc + j, &s, 1);
    }
}

// The same reduction four columns at a time (n, ldc and, for the epilogue
// inputs, ldmask multiples of 4; f32 output, no optimiser): blockIdx.y walks
// rows, the x threads walk 4-column groups, every load and store 16 bytes.
// Slices are summed in the same fixed order.
__global__ void splitk_reduce4_kernel(SimtParams p, int slices) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    const int64_t total = p.m * p.n;
    const int64_t groups = p.n / 4;
    for (int64_t i = blockIdx.y; i < p.m; i += gridDim.y) {
        for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups;
             g += (int64_t)gridDim.x * blockDim.x) {
            const int64_t j = 4 * g;
            const float* src = p.ws + i * p.n + j;
            float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int z0 = 0; z0 < slices; z0 += 4) {
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    v[u] = z0 + u < slices ? __ldg(reinterpret_cast<const float4*>(src + (int64_t)(z0 + u) * total))
                                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (z0 + u < slices) s.x += v[u].x, s.y += v[u].y, s.z += v[u].z, s.w += v[u].w;
            }
            if (p.epi == RT_EPI_BIAS || p.epi == RT_EPI_BIAS_RELU) {
                s.x += p.bias[j], s.y += p.bias[j + 1], s.z += p.bias[j + 2], s.w += p.bias[j + 3];
                if (p.epi == RT_EPI_BIAS_RELU)
                    s.x = fmaxf(s.x, 0.0f), s.y = fmaxf(s.y, 0.0f), s.z = fmaxf(s.z, 0.0f), s.w = fmaxf(s.w, 0.0f);
            } else if (p.epi == RT_EPI_RELU_MASK) {
                const float4 mk = *reinterpret_cast<const float4*>(static_cast<const float*>(p.mask) + i * p.ldmask + j);
                s.x = s.x * (mk.x > 0.0f ? 1.0f : 0.0f), s.y = s.y * (mk.y > 0.0f ? 1.0f : 0.0f);
                s.z = s.z * (mk.z > 0.0f ? 1.0f : 0.0f), s.w = s.w * (mk.w > 0.0f ? 1.0f : 0.0f);
            }
            *reinterpret_cast<float4*>(static_cast<float*>(p.c) + i * p.ldc + j) = s;
        }
    }
}

SimtParams make_params(const GemmDesc& g) {
    SimtParams p;
    p.a = g.a;
    p.a2 = g.a_lo;
    p.b = g.b;
    p.c = g.c;
    p.c_lo = g.c_lo;
    p.ws = g.split_k > 1 ? g.workspace : nullptr;
    p.bias = g.bias;
    p.mask = g.mask;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.lda = g.lda;
    p.ldb = g.ldb;
    p.ldc = g.ldc;
    p.ldmask = g.ldmask;
    int s = g.split_k > 1 ? g.split_k : 1;
    int64_t kps = (g.k + s - 1) / s;
    kps = (kps + BK - 1) / BK * BK;
    p.k_per_slice = kps > 0 ? kps : BK;
    p.epi = g.epi;
    p.out_bf16 = g.out_dtype == RT_BF16;
    p.opt = g.opt;
    return p;
}

template <typename TIn>
void launch_typed(const GemmDesc& g, const SimtParams& p, dim3 grid, cudaStream_t st) {
    switch (g.layout) {
        case RT_NN: gemm_simt_kernel<TIn, true, false><<<grid, THREADS, 0, st>>>(p); break;
        case RT_NT: gemm_simt_kernel<TIn, true, true><<<grid, THREADS, 0, st>>>(p); break;
        case RT_TN: gemm_simt_kernel<TIn, false, false><<<grid, THREADS, 0, st>>>(p); break;
    }
}

}  // namespace

int launch_gemm_simt(rt_ctx* ctx, const GemmDesc& g, cudaStream_t stream) {
    if (g.m == 0 || g.n == 0) return RT_OK;
    SimtParams p = make_params(g);
    int slices = g.split_k > 1 ? g.split_k : 1;
    dim3 grid((unsigned)((g.n + BN - 1) / BN), (unsigned)((g.m + BM - 1) / BM), (unsigned)slices);
    if (grid.y > 65535u) return fail(RT_ERR_INVALID, "GEMM m=%lld too large for the SIMT grid", (long long)g.m);
    if (g.in_dtype == RT_BF16)
        launch_typed<__nv_bfloat16>(g, p, grid, stream);
    else
        launch_typed<float>(g, p, grid, stream);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    if (slices > 1) return launch_splitk_reduce(ctx, g, stream);
    return RT_OK;
}

int launch_splitk_reduce(rt_ctx* ctx, const GemmDesc& g, cudaStream_t stream) {
    SimtParams p = make_params(g);
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    const bool vec = g.out_dtype == RT_F32 && !g.opt.kind && g.n % 4 == 0 && g.ldc % 4 == 0 && al16(g.c) &&
                     al16(g.workspace) && (g.epi != RT_EPI_RELU_MASK || (g.ldmask % 4 == 0 && al16(g.mask)));
    if (vec) {
        const int64_t groups = g.n / 4;
        const int threads = groups >= 256 ? 256 : (int)((groups + 31) / 32 * 32);
        const int64_t gx = (groups + threads - 1) / threads;
        int64_t gy = g.m < 65535 ? g.m : 65535;
        RT_CUDA(launch_k(ctx->plan_pdl, splitk_reduce4_kernel, dim3((unsigned)gx, (unsigned)gy), dim3(threads), 0, stream, p,
                         g.split_k));
        count_launch(ctx);
        RT_CUDA(cudaGetLastError());
        return RT_OK;
    }
    int64_t total = g.m * g.n;
    int64_t blocks = (total + 255) / 256;
    int64_t cap = (int64_t)ctx->sm_count * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    RT_CUDA(launch_k(ctx->plan_pdl, splitk_reduce_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, p, g.split_k));
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

}  // namespace rt
