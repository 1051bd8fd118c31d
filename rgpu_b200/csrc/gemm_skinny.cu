// GEMMs with one tiny dimension, on CUDA cores with f32 FMA.
//
// The output layer of rtensor's MLPs has as many columns as classes (10 for
// the 512 -> 1024 -> 1024 -> 10 configs), which makes three of a step's
// GEMMs skinny (crates/rtensor/src/gpu/mod.rs:1404-1455):
//   forward  Z_L = A_{L-1} W_L + 1 b_L     n = classes      (narrow N, NN)
//   dW       [dW_L; db_L] = [A, 1]^T delta_L  n = classes   (narrow N, TN)
//   dX       delta_L W_L^T                 k = classes      (narrow K, NT)
// A tensor-core tile wastes most of its width on them and they move few
// bytes, so they run here instead: each is one pass over its large operand
// (or, for narrow K, over its output), with the tiny operand held in L1 or
// shared memory.  Same epilogues as the other GEMM kernels (bias, bias+ReLU,
// ReLU mask, fused optimiser), f32 or bf16 operands and output.
#include "internal.h"

namespace rt {
namespace {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ float ld_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, int64_t i) {
    return __ldg(p + i);
}
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}

struct SkinnyParams {
    const void* a;
    const void* b;
    void* c;
    float* ws;  // [slices][m][n] partial sums (narrow-N TN with slices > 1)
    const float* bias;
    const void* mask;
    int64_t m, n, k, lda, ldb, ldc, ldmask;
    int64_t k_per_slice;
    int epi;
    int out_bf16;
    OptFuse opt;
};

// Epilogue of one output element (the same arithmetic as the tiled kernels').
__device__ __forceinline__ void finish_one(const SkinnyParams& p, int64_t i, int64_t j, float v) {
    if (p.epi == RT_EPI_BIAS || p.epi == RT_EPI_BIAS_RELU) {
        v = v + p.bias[j];
        if (p.epi == RT_EPI_BIAS_RELU) v = fmaxf(v, 0.0f);
    } else if (p.epi == RT_EPI_RELU_MASK) {
        const int64_t mi = i * p.ldmask + j;
        const float mk = p.out_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.mask)[mi])
                                    : static_cast<const float*>(p.mask)[mi];
        v = v * (mk > 0.0f ? 1.0f : 0.0f);
    }
    if (p.opt.kind) opt_apply_row<1>(p.opt, i * p.ldc + j, &v, 1);
    if (p.out_bf16)
        static_cast<__nv_bfloat16*>(p.c)[i * p.ldc + j] = __float2bfloat16_rn(v);
    else
        static_cast<float*>(p.c)[i * p.ldc + j] = v;
}

// Narrow N, A K-major (layouts NN and NT): a block owns ROWS rows of C and
// its 8 warps split k (warp w takes k indices w*32 + lane + 256 i, four at a
// time so that 4 x ROWS loads of A are in flight per lane); a shuffle tree
// sums each warp's lanes and the warps' sums are added in fixed order.  The
// small operand B is read through L1.
template <typename TIn, int NMAX, bool B_KMAJOR, int ROWS>
__global__ void __launch_bounds__(kThreads) skinny_n_kernel(SkinnyParams p) {
    constexpr int U = 4;
    constexpr int WARPS = kThreads / 32;
    __shared__ float red[WARPS][ROWS][NMAX];
    const TIn* A = static_cast<const TIn*>(p.a);
    const TIn* B = static_cast<const TIn*>(p.b);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t i0 = (int64_t)blockIdx.x * ROWS;
    const int n = (int)p.n;
    float acc[ROWS][NMAX];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int j = 0; j < NMAX; ++j) acc[r][j] = 0.0f;
    for (int64_t q0 = (int64_t)warp * 32 + lane; q0 < p.k; q0 += (int64_t)kThreads * U) {
        float a[U][ROWS];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t q = q0 + (int64_t)u * kThreads;
#pragma unroll
            for (int r = 0; r < ROWS; ++r) a[u][r] = (q < p.k && i0 + r < p.m) ? ld_f(A, (i0 + r) * p.lda + q) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t q = q0 + (int64_t)u * kThreads;
            if (q < p.k) {
#pragma unroll
                for (int j = 0; j < NMAX; ++j) {
                    if (j < n) {
                        const float bv = B_KMAJOR ? ld_f(B, (int64_t)j * p.ldb + q) : ld_f(B, q * p.ldb + j);
#pragma unroll
                        for (int r = 0; r < ROWS; ++r) acc[r][j] = fmaf(a[u][r], bv, acc[r][j]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int j = 0; j < NMAX; ++j) {
            float v = acc[r][j];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) red[warp][r][j] = v;
        }
    __syncthreads();
    if (threadIdx.x < ROWS * NMAX) {
        const int r = threadIdx.x / NMAX, j = threadIdx.x % NMAX;
        if (j < n && i0 + r < p.m) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < WARPS; ++w) v += red[w][r][j];
            finish_one(p, i0 + r, j, v);
        }
    }
}

// Narrow N, A MN-major (layout TN, the dW of the output layer): thread i of
// the grid owns row i of C (column i of A's storage); every k row of A is
// read coalesced once (eight rows in flight per thread), the k rows of B are
// broadcast from shared memory.  blockIdx.y takes a k slice; with more than
// one slice the partial sums go to p.ws and the fixed-order split-K reduction
// finishes them.
template <typename TIn, int NMAX>
__global__ void __launch_bounds__(kThreads) skinny_n_tn_kernel(SkinnyParams p) {
    constexpr int KC = 64;  // k rows of B staged per pass
    constexpr int U = 8;
    __shared__ float sb[KC][NMAX];
    const TIn* A = static_cast<const TIn*>(p.a);
    const TIn* B = static_cast<const TIn*>(p.b);
    const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    const int n = (int)p.n;
    const int64_t k0 = (int64_t)blockIdx.y * p.k_per_slice;
    const int64_t k1 = min(p.k, k0 + p.k_per_slice);
    float acc[NMAX];
#pragma unroll
    for (int j = 0; j < NMAX; ++j) acc[j] = 0.0f;
    for (int64_t kc = k0; kc < k1; kc += KC) {
        __syncthreads();
        for (int t = threadIdx.x; t < KC * NMAX; t += kThreads) {
            const int r = t / NMAX, j = t % NMAX;
            sb[r][j] = (kc + r < k1 && j < n) ? ld_f(B, (kc + r) * p.ldb + j) : 0.0f;
        }
        __syncthreads();
        if (i < p.m) {
            const int kn = (int)min((int64_t)KC, k1 - kc);
            for (int r0 = 0; r0 < kn; r0 += U) {
                float a[U];
#pragma unroll
                for (int u = 0; u < U; ++u) a[u] = r0 + u < kn ? ld_f(A, (kc + r0 + u) * p.lda + i) : 0.0f;
#pragma unroll
                for (int u = 0; u < U; ++u)
#pragma unroll
                    for (int j = 0; j < NMAX; ++j) acc[j] = fmaf(a[u], sb[r0 + u][j], acc[j]);
            }
        }
    }
    if (i >= p.m) return;
    if (p.ws) {
        float* dst = p.ws + (int64_t)blockIdx.y * p.m * p.n + i * p.n;
#pragma unroll
        for (int j = 0; j < NMAX; ++j)
            if (j < n) dst[j] = acc[j];
    } else {
#pragma unroll
        for (int j = 0; j < NMAX; ++j)
            if (j < n) finish_one(p, i, j, acc[j]);
    }
}

// Narrow K (k <= KMAX): a block computes a TM x 256 tile of C.  Its threads
// each hold the k x 4 slab of B for four consecutive columns in registers and
// walk down the tile's rows, reading the row's k values of A from shared
// memory (a broadcast) and storing four columns at once when the row is
// aligned for it.
template <typename TIn, int KMAX, bool A_KMAJOR, bool B_KMAJOR>
__global__ void __launch_bounds__(kThreads) skinny_k_kernel(SkinnyParams p) {
    constexpr int TM = 64, TN = 4 * 64;
    __shared__ float sa[TM][KMAX];
    const TIn* A = static_cast<const TIn*>(p.a);
    const TIn* B = static_cast<const TIn*>(p.b);
    const int64_t m0 = (int64_t)blockIdx.y * TM, n0 = (int64_t)blockIdx.x * TN;
    const int k = (int)p.k;
    for (int t = threadIdx.x; t < TM * KMAX; t += kThreads) {
        const int r = t / KMAX, q = t % KMAX;
        const int64_t i = m0 + r;
        sa[r][q] = (i < p.m && q < k) ? ld_f(A, A_KMAJOR ? i * p.lda + q : (int64_t)q * p.lda + i) : 0.0f;
    }
    const int cg = threadIdx.x % 64;        // column group: 4 columns
    const int rg = threadIdx.x / 64;        // row phase: rows rg, rg + 4, ...
    const int64_t j0 = n0 + cg * 4;
    float b[KMAX][4];
#pragma unroll
    for (int q = 0; q < KMAX; ++q)
#pragma unroll
        for (int c = 0; c < 4; ++c)
            b[q][c] = (q < k && j0 + c < p.n) ? ld_f(B, B_KMAJOR ? (j0 + c) * p.ldb + q : (int64_t)q * p.ldb + j0 + c)
                                             : 0.0f;
    __syncthreads();
    if (j0 >= p.n) return;
    const bool plain_vec = p.epi == RT_EPI_NONE && !p.opt.kind && !p.out_bf16 && j0 + 4 <= p.n &&
                           (p.ldc % 4) == 0 && ((reinterpret_cast<uintptr_t>(p.c) & 15) == 0);
    for (int r = rg; r < TM; r += kThreads / 64) {
        const int64_t i = m0 + r;
        if (i >= p.m) break;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q = 0; q < KMAX; ++q) {
            if (q < k) {
                const float av = sa[r][q];
#pragma unroll
                for (int c = 0; c < 4; ++c) v[c] = fmaf(av, b[q][c], v[c]);
            }
        }
        if (plain_vec) {
            *reinterpret_cast<float4*>(static_cast<float*>(p.c) + i * p.ldc + j0) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (j0 + c < p.n) finish_one(p, i, j0 + c, v[c]);
        }
    }
}

SkinnyParams make_params(const GemmDesc& g) {
    SkinnyParams p{};
    p.a = g.a;
    p.b = g.b;
    p.c = g.c;
    p.bias = g.bias;
    p.mask = g.mask;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.lda = g.lda;
    p.ldb = g.ldb;
    p.ldc = g.ldc;
    p.ldmask = g.ldmask;
    p.epi = g.epi;
    p.out_bf16 = g.out_dtype == RT_BF16;
    p.opt = g.opt;
    return p;
}

template <typename TIn>
int launch_typed(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    SkinnyParams p = make_params(g);
    if (g.n <= kSkinnyMax) {
        if (g.layout == RT_TN) {
            int slices = g.split_k > 1 && g.workspace ? g.split_k : 1;
            int64_t kps = (g.k + slices - 1) / slices;
            kps = (kps + 63) / 64 * 64;
            slices = (int)((g.k + kps - 1) / kps);
            p.k_per_slice = kps;
            p.ws = slices > 1 ? g.workspace : nullptr;
            dim3 grid((unsigned)((g.m + kThreads - 1) / kThreads), (unsigned)slices);
            skinny_n_tn_kernel<TIn, kSkinnyMax><<<grid, kThreads, 0, st>>>(p);
            count_launch(ctx);
            RT_CUDA(cudaGetLastError());
            if (slices > 1) {
                GemmDesc gr = g;
                gr.split_k = slices;
                return launch_splitk_reduce(ctx, gr, st);
            }
            return RT_OK;
        }
        constexpr int ROWS = 4;
        const int64_t blocks = (g.m + ROWS - 1) / ROWS;
        if (g.layout == RT_NT)
            skinny_n_kernel<TIn, kSkinnyMax, true, ROWS><<<(unsigned)blocks, kThreads, 0, st>>>(p);
        else
            skinny_n_kernel<TIn, kSkinnyMax, false, ROWS><<<(unsigned)blocks, kThreads, 0, st>>>(p);
    } else {
        dim3 grid((unsigned)((g.n + 255) / 256), (unsigned)((g.m + 63) / 64));
        if (grid.y > 65535u) return fail(RT_ERR_INVALID, "narrow-k GEMM m=%lld too large for its grid", (long long)g.m);
        switch (g.layout) {
            case RT_NN: skinny_k_kernel<TIn, kSkinnyMax, true, false><<<grid, kThreads, 0, st>>>(p); break;
            case RT_NT: skinny_k_kernel<TIn, kSkinnyMax, true, true><<<grid, kThreads, 0, st>>>(p); break;
            case RT_TN: skinny_k_kernel<TIn, kSkinnyMax, false, false><<<grid, kThreads, 0, st>>>(p); break;
        }
    }
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

}  // namespace

bool gemm_skinny_wanted(const GemmDesc& g) {
    return g.m >= 1 && g.k >= 1 && (g.n <= kSkinnyMax || g.k <= kSkinnyMax);
}

int launch_gemm_skinny(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    RT_CHECK(gemm_skinny_wanted(g), "GEMM is not skinny");
    if (g.in_dtype == RT_BF16) return launch_typed<__nv_bfloat16>(ctx, g, st);
    return launch_typed<float>(ctx, g, st);
}

}  // namespace rt
