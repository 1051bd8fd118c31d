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
#include <cooperative_groups.h>

#include "internal.h"

namespace rt {
namespace {

namespace cg = cooperative_groups;

constexpr int kThreads = 256;
constexpr int kSkinnyNSmem = 1024 * 20 * 4;  // skinny_n_kernel's staged B chunk

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

// Four consecutive elements from a 4-element-aligned address, as f32.
__device__ __forceinline__ float4 ld4_f(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 ld4_f(const __nv_bfloat16* p) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}

struct SkinnyParams {
    const void* a;
    const void* a2;  // A's low-order bf16 plane (null = none): A = a + a2, exact in f32
    const void* b;
    void* c;
    void* c_lo;      // bf16 output's low-order plane (null = none)
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
    if (p.out_bf16) {
        static_cast<__nv_bfloat16*>(p.c)[i * p.ldc + j] = __float2bfloat16_rn(v);
        if (p.c_lo)
            static_cast<__nv_bfloat16*>(p.c_lo)[i * p.ldc + j] =
                __float2bfloat16_rn(v - __bfloat162float(__float2bfloat16_rn(v)));
    } else {
        static_cast<float*>(p.c)[i * p.ldc + j] = v;
    }
}

// Vector epilogue of 4 consecutive columns j0..j0+3 of row i (all < n): the
// same arithmetic as finish_one, with 16-byte loads and stores where the
// rows are aligned for them.
__device__ __forceinline__ void finish_four(const SkinnyParams& p, int64_t i, int64_t j0, float (&v)[4], bool vec) {
    if (!vec || p.opt.kind) {
#pragma unroll
        for (int c = 0; c < 4; ++c) finish_one(p, i, j0 + c, v[c]);
        return;
    }
    if (p.epi == RT_EPI_BIAS || p.epi == RT_EPI_BIAS_RELU) {
        const float4 b = *reinterpret_cast<const float4*>(p.bias + j0);
        v[0] += b.x, v[1] += b.y, v[2] += b.z, v[3] += b.w;
        if (p.epi == RT_EPI_BIAS_RELU)
#pragma unroll
            for (int c = 0; c < 4; ++c) v[c] = fmaxf(v[c], 0.0f);
    } else if (p.epi == RT_EPI_RELU_MASK) {
        const int64_t mi = i * p.ldmask + j0;
        float mk[4];
        if (p.out_bf16) {
            const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.mask) + mi);
            const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
            for (int c = 0; c < 4; ++c) mk[c] = __bfloat162float(h[c]);
        } else {
            const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(p.mask) + mi);
            mk[0] = f.x, mk[1] = f.y, mk[2] = f.z, mk[3] = f.w;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = v[c] * (mk[c] > 0.0f ? 1.0f : 0.0f);
    }
    if (p.out_bf16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&lo);
        u.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.c) + i * p.ldc + j0) = u;
        if (p.c_lo) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
                static_cast<__nv_bfloat16*>(p.c_lo)[i * p.ldc + j0 + c] =
                    __float2bfloat16_rn(v[c] - __bfloat162float(__float2bfloat16_rn(v[c])));
        }
    } else {
        *reinterpret_cast<float4*>(static_cast<float*>(p.c) + i * p.ldc + j0) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// 16-byte loads and stores of 4-column groups are legal for this call.
__host__ __device__ __forceinline__ bool four_aligned(const SkinnyParams& p) {
    const int es = p.out_bf16 ? 2 : 4;
    bool ok = (p.ldc % 4) == 0 && (reinterpret_cast<uintptr_t>(p.c) % (4 * es)) == 0;
    if (p.epi == RT_EPI_BIAS || p.epi == RT_EPI_BIAS_RELU) ok = ok && (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0;
    if (p.epi == RT_EPI_RELU_MASK)
        ok = ok && (p.ldmask % 4) == 0 && (reinterpret_cast<uintptr_t>(p.mask) % (4 * es)) == 0;
    return ok;
}

// Sum of v[0..15] over the 32 lanes of a warp, reduce-scattered: at each of
// four levels a lane keeps the half of its values its lane bit selects and
// adds its partner's copy of that half (8 + 4 + 2 + 1 shuffles), then one
// more exchange completes the pair.  Lanes 2c and 2c + 1 end with column c's
// total; the summation order is fixed.
__device__ __forceinline__ float warp_sum16_scatter(float (&v)[16], int lane) {
    float a8[8], a4[4], a2[2], a1;
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1, b1 = (lane >> 1) & 1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float send = b4 ? v[i] : v[8 + i];
        const float keep = b4 ? v[8 + i] : v[i];
        a8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = b3 ? a8[i] : a8[4 + i];
        const float keep = b3 ? a8[4 + i] : a8[i];
        a4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b2 ? a4[i] : a4[2 + i];
        const float keep = b2 ? a4[2 + i] : a4[i];
        a2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    {
        const float send = b1 ? a2[0] : a2[1];
        const float keep = b1 ? a2[1] : a2[0];
        a1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    return a1 + __shfl_xor_sync(0xffffffffu, a1, 1);
}

// Narrow N (n <= 16), A K-major (layouts NN and NT): one warp per row of C,
// eight rows per block.  The block stages B in 1024-row chunks in shared
// memory ([k][16], rows padded to 20 floats so a warp's 16-byte reads of 8
// different rows hit distinct banks); the warp's lanes stride over k reading
// A coalesced, all 32 of a chunk's loads in flight per lane, and accumulate
// the 16 partial dot products, which a reduce-scatter (16 shuffles) leaves in
// lane 2c for column c.  One chunk covers the output layers of the reference
// MLPs (k <= 1024), so their A and B loads are a single round trip.
template <typename TIn, bool B_KMAJOR>
__global__ void __launch_bounds__(kThreads) skinny_n_kernel(SkinnyParams p) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    constexpr int U = 32, KC = 32 * U, BP = 20;  // k rows per chunk, padded row length of staged B
    extern __shared__ __align__(16) float sb_raw[];
    float(*sb)[BP] = reinterpret_cast<float(*)[BP]>(sb_raw);
    const TIn* A = static_cast<const TIn*>(p.a);
    const TIn* B = static_cast<const TIn*>(p.b);
    const int lane = threadIdx.x & 31;
    const int64_t i = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
    const bool row_ok = i < p.m;  // warp-uniform; every warp still helps stage B
    const int n = (int)p.n;
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
    const TIn* arow = A + (row_ok ? i : 0) * p.lda;
    const TIn* arow2 = p.a2 ? static_cast<const TIn*>(p.a2) + (row_ok ? i : 0) * p.lda : nullptr;
    for (int64_t kc = 0; kc < p.k; kc += KC) {
        float a[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t q = kc + lane + 32 * u;
            a[u] = (row_ok && q < p.k) ? ld_f(arow, q) : 0.0f;
        }
        if (arow2) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t q = kc + lane + 32 * u;
                if (row_ok && q < p.k) a[u] += ld_f(arow2, q);
            }
        }
        __syncthreads();  // the previous chunk's reads of sb are done
        const int kn = (int)min((int64_t)KC, p.k - kc);
        if (!B_KMAJOR && sizeof(TIn) == 4 && n == 16 && (p.ldb % 4) == 0 &&
            (reinterpret_cast<uintptr_t>(p.b) & 15) == 0) {
            // whole 16-float B rows as four 16-byte loads
            for (int t = threadIdx.x; t < kn * 4; t += kThreads) {
                const int r = t / 4, c4 = t % 4;
                const float4 v = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(B) +
                                                                       (kc + r) * p.ldb) + c4);
                *reinterpret_cast<float4*>(&sb[r][4 * c4]) = v;
            }
        } else {
            for (int t = threadIdx.x; t < kn * 16; t += kThreads) {
                // NN: consecutive threads walk a B row (16 columns); NT: a B row is a
                // column j of C, so consecutive threads walk k instead
                const int r = B_KMAJOR ? t % kn : t / 16, j = B_KMAJOR ? t / kn : t % 16;
                const int64_t q = kc + r;
                sb[r][j] = j < n ? ld_f(B, B_KMAJOR ? (int64_t)j * p.ldb + q : q * p.ldb + j) : 0.0f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (32 * u >= kn) break;  // a[u] is zero past k; its B rows were not staged
            const float4* br = reinterpret_cast<const float4*>(&sb[lane + 32 * u][0]);
#pragma unroll
            for (int t4 = 0; t4 < 4; ++t4) {
                const float4 b = br[t4];
                acc[4 * t4 + 0] = fmaf(a[u], b.x, acc[4 * t4 + 0]);
                acc[4 * t4 + 1] = fmaf(a[u], b.y, acc[4 * t4 + 1]);
                acc[4 * t4 + 2] = fmaf(a[u], b.z, acc[4 * t4 + 2]);
                acc[4 * t4 + 3] = fmaf(a[u], b.w, acc[4 * t4 + 3]);
            }
        }
    }
    const float v = warp_sum16_scatter(acc, lane);
    const int c = lane >> 1;
    if (row_ok && (lane & 1) == 0 && c < n) finish_one(p, i, c, v);
}

// Narrow N, A MN-major (layout TN, the dW of the output layer): thread i of
// the grid owns row i of C (column i of A's storage); every k row of A is
// read coalesced once (sixteen rows in flight per thread), the k rows of B
// are broadcast from shared memory.  blockIdx.y takes a k slice; with more
// than one slice the partial sums go to p.ws and the fixed-order split-K
// reduction finishes them.
template <typename TIn, int NMAX>
__global__ void __launch_bounds__(kThreads) skinny_n_tn_kernel(SkinnyParams p) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    constexpr int KC = 64;  // k rows of B staged per pass
    constexpr int U = 16;
    __shared__ __align__(16) float sb[KC][NMAX];
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
                if (p.a2) {
#pragma unroll
                    for (int u = 0; u < U; ++u)
                        if (r0 + u < kn) a[u] += ld_f(static_cast<const TIn*>(p.a2), (kc + r0 + u) * p.lda + i);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const float4* br = reinterpret_cast<const float4*>(&sb[r0 + u][0]);  // a broadcast
#pragma unroll
                    for (int t4 = 0; t4 < NMAX / 4; ++t4) {
                        const float4 b = br[t4];
                        acc[4 * t4 + 0] = fmaf(a[u], b.x, acc[4 * t4 + 0]);
                        acc[4 * t4 + 1] = fmaf(a[u], b.y, acc[4 * t4 + 1]);
                        acc[4 * t4 + 2] = fmaf(a[u], b.z, acc[4 * t4 + 2]);
                        acc[4 * t4 + 3] = fmaf(a[u], b.w, acc[4 * t4 + 3]);
                    }
                }
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

// Narrow K (k <= KMAX): a block computes a 32 x 256 tile of C.  Each thread
// holds the k x 4 slab of B for four consecutive columns in registers and
// walks down eight of the tile's rows, reading each row's k values of A from
// shared memory (a 16-byte broadcast per four k) and finishing four columns
// with 16-byte loads and stores.
template <typename TIn, int KMAX, bool A_KMAJOR, bool B_KMAJOR>
__global__ void __launch_bounds__(kThreads) skinny_k_kernel(SkinnyParams p) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    constexpr int TM = 32, TN = 4 * 64, RPT = TM / (kThreads / 64);  // rows per thread
    __shared__ __align__(16) float sa[TM][KMAX];
    const TIn* A = static_cast<const TIn*>(p.a);
    const TIn* B = static_cast<const TIn*>(p.b);
    const int64_t m0 = (int64_t)blockIdx.y * TM, n0 = (int64_t)blockIdx.x * TN;
    const int k = (int)p.k;
    for (int t = threadIdx.x; t < TM * KMAX; t += kThreads) {
        // consecutive threads read consecutive addresses of A
        const int r = A_KMAJOR ? t / KMAX : t % TM, q = A_KMAJOR ? t % KMAX : t / TM;
        const int64_t i = m0 + r;
        float v = 0.0f;
        if (i < p.m && q < k) {
            const int64_t ai = A_KMAJOR ? i * p.lda + q : (int64_t)q * p.lda + i;
            v = ld_f(A, ai);
            if (p.a2) v += ld_f(static_cast<const TIn*>(p.a2), ai);
        }
        sa[r][q] = v;
    }
    const int cg = threadIdx.x % 64;  // column group: 4 columns
    const int rg = threadIdx.x / 64;  // rows rg, rg + 4, ...
    const int64_t j0 = n0 + cg * 4;
    float b[KMAX][4];
    if (!B_KMAJOR && j0 + 4 <= p.n && (p.ldb % 4) == 0 &&
        (reinterpret_cast<uintptr_t>(B) % (4 * sizeof(TIn))) == 0) {
        // a row of B holds this thread's four columns: one vector load per k
#pragma unroll
        for (int q = 0; q < KMAX; ++q) {
            const float4 v = q < k ? ld4_f(B + (int64_t)q * p.ldb + j0) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            b[q][0] = v.x;
            b[q][1] = v.y;
            b[q][2] = v.z;
            b[q][3] = v.w;
        }
    } else {
#pragma unroll
        for (int q = 0; q < KMAX; ++q)
#pragma unroll
            for (int c = 0; c < 4; ++c)
                b[q][c] = (q < k && j0 + c < p.n)
                              ? ld_f(B, B_KMAJOR ? (j0 + c) * p.ldb + q : (int64_t)q * p.ldb + j0 + c)
                              : 0.0f;
    }
    const bool vec = j0 + 4 <= p.n && four_aligned(p);
    // the ReLU-mask epilogue's loads for all of this thread's rows, in flight together
    float4 mk[RPT];
    const bool pre_mask = vec && p.epi == RT_EPI_RELU_MASK && !p.out_bf16 && !p.opt.kind;
    if (pre_mask) {
#pragma unroll
        for (int t = 0; t < RPT; ++t) {
            const int64_t i = m0 + rg + t * (kThreads / 64);
            mk[t] = i < p.m ? *reinterpret_cast<const float4*>(static_cast<const float*>(p.mask) + i * p.ldmask + j0)
                            : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    }
    __syncthreads();
    if (j0 >= p.n) return;
#pragma unroll
    for (int t = 0; t < RPT; ++t) {
        const int r = rg + t * (kThreads / 64);
        const int64_t i = m0 + r;
        if (i >= p.m) break;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q4 = 0; q4 < KMAX; q4 += 4) {
            const float4 a = *reinterpret_cast<const float4*>(&sa[r][q4]);
            const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
                for (int c = 0; c < 4; ++c) v[c] = fmaf(av[t], b[q4 + t][c], v[c]);
        }
        if (pre_mask) {
            const float4 m4 = mk[t];
            *reinterpret_cast<float4*>(static_cast<float*>(p.c) + i * p.ldc + j0) =
                make_float4(v[0] * (m4.x > 0.0f ? 1.0f : 0.0f), v[1] * (m4.y > 0.0f ? 1.0f : 0.0f),
                            v[2] * (m4.z > 0.0f ? 1.0f : 0.0f), v[3] * (m4.w > 0.0f ? 1.0f : 0.0f));
        } else if (vec) {
            finish_four(p, i, j0, v, true);
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (j0 + c < p.n) finish_one(p, i, j0 + c, v[c]);
        }
    }
}

// Few rows (layouts NN and TN, m <= 16, or m <= 64 for f32 operands, whose
// tensor-core path would be three tf32 products behind an operand split: the
// forward pass at small batch, and dW of a layer with few inputs):
// a GEMV-like pass over B.  A cluster of kClusterK CTAs owns 64 columns of C
// (lane l of every warp holds columns 2 l and 2 l + 1) and splits k: CTA r of
// the cluster takes the r-th k range, and its 8 warps split that range again.
// A's rows are staged in shared memory 256 k at a time (hi + lo summed when A
// is split), B is read once per 16-row pass with coalesced 8-byte (f32) or
// 4-byte (bf16) loads, 16 rows' loads in flight per thread.  The warps' sums
// are reduced in shared memory in warp order, then CTA 0 of the cluster adds
// the CTAs' sums in rank order through distributed shared memory and runs
// the epilogue: one launch, no workspace, a fixed summation order.
constexpr int kClusterK = 8;
constexpr int kSkinnyRowsMax = 64;
constexpr int kMRows = 16;  // rows per pass
constexpr int kKChunk = 256;

template <typename TIn>
__device__ __forceinline__ float2 ld2_f(const TIn* p);
template <>
__device__ __forceinline__ float2 ld2_f<float>(const float* p) {
    return __ldg(reinterpret_cast<const float2*>(p));
}
template <>
__device__ __forceinline__ float2 ld2_f<__nv_bfloat16>(const __nv_bfloat16* p) {
    const uint32_t u = __ldg(reinterpret_cast<const unsigned int*>(p));
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}

template <typename TIn, bool A_KM>
__global__ void __cluster_dims__(kClusterK, 1, 1) __launch_bounds__(kThreads)
    skinny_m_kernel(SkinnyParams p) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    // A_KM: A is stored [k, m] (layout TN), else [m, k] (layout NN)
    // sa (A rows of the k chunk) during the k loop; red (the warps' sums)
    // after it, in the same shared memory
    __shared__ __align__(16) float buf[kThreads / 32][kMRows][64];
    __shared__ __align__(16) float part[kMRows][64];
    static_assert(sizeof(float) * kMRows * kKChunk <= sizeof(buf), "A chunk fits the reduction buffer");
    float(*sa)[kKChunk] = reinterpret_cast<float(*)[kKChunk]>(&buf[0][0][0]);
    float(*red)[kMRows][64] = buf;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const TIn* A = static_cast<const TIn*>(p.a);
    const TIn* A2 = static_cast<const TIn*>(p.a2);
    const TIn* B = static_cast<const TIn*>(p.b);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n0 = (int64_t)(blockIdx.x / kClusterK) * 64;
    const int64_t j = n0 + 2 * lane;  // this lane's columns j, j + 1
    // two columns per load where the row stride and base allow an aligned pair
    const bool pair = j + 1 < p.n && (p.ldb & 1) == 0 && (reinterpret_cast<uintptr_t>(B) % (2 * sizeof(TIn))) == 0;
    const int64_t kr = (p.k + kClusterK - 1) / kClusterK;  // this CTA's k range
    const int64_t k_lo = (int64_t)rank * kr, k_hi = min(p.k, k_lo + kr);
    for (int64_t m0 = 0; m0 < p.m; m0 += kMRows) {
        const int rows = (int)min((int64_t)kMRows, p.m - m0);
        float acc[kMRows][2];
#pragma unroll
        for (int i = 0; i < kMRows; ++i) acc[i][0] = acc[i][1] = 0.0f;
        for (int64_t kc = k_lo; kc < k_hi; kc += kKChunk) {
            const int kn = (int)min((int64_t)kKChunk, k_hi - kc);
            __syncthreads();  // the previous chunk's reads of sa are done
            for (int t = threadIdx.x; t < kMRows * kKChunk; t += kThreads) {
                // consecutive threads read consecutive elements of A's stored rows
                const int i = A_KM ? t % kMRows : t / kKChunk, q = A_KM ? t / kMRows : t % kKChunk;
                float v = 0.0f;
                if (i < rows && q < kn) {
                    const int64_t ai = A_KM ? (kc + q) * p.lda + m0 + i : (m0 + i) * p.lda + kc + q;
                    v = ld_f(A, ai);
                    if (A2) v += ld_f(A2, ai);
                }
                sa[i][q] = v;
            }
            __syncthreads();
            // warp w takes k rows w, w + 8, ... of the chunk, 16 at a time
            for (int q0 = warp; q0 < kn; q0 += 16 * (kThreads / 32)) {
                float2 b[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int q = q0 + u * (kThreads / 32);
                    b[u] = make_float2(0.0f, 0.0f);
                    if (q < kn && j < p.n) {
                        const TIn* br = B + (kc + q) * p.ldb + j;
                        if (pair)
                            b[u] = ld2_f(br);
                        else
                            b[u] = make_float2(ld_f(br, 0), j + 1 < p.n ? ld_f(br, 1) : 0.0f);
                    }
                }
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int q = q0 + u * (kThreads / 32);
                    if (q >= kn) break;
#pragma unroll
                    for (int i = 0; i < kMRows; ++i) {
                        const float a = sa[i][q];
                        acc[i][0] = fmaf(a, b[u].x, acc[i][0]);
                        acc[i][1] = fmaf(a, b[u].y, acc[i][1]);
                    }
                }
            }
        }
        __syncthreads();  // every warp is done reading sa, which red overwrites
#pragma unroll
        for (int i = 0; i < kMRows; ++i) {
            red[warp][i][2 * lane] = acc[i][0];
            red[warp][i][2 * lane + 1] = acc[i][1];
        }
        __syncthreads();
        for (int t = threadIdx.x; t < kMRows * 64; t += kThreads) {
            const int i = t / 64, c = t % 64;
            float v = 0.0f;
            for (int w = 0; w < kThreads / 32; ++w) v += red[w][i][c];
            part[i][c] = v;
        }
        cluster.sync();  // every CTA's part is complete
        if (rank == 0) {
            for (int t = threadIdx.x; t < kMRows * 64; t += kThreads) {
                const int i = t / 64, c = t % 64;
                if (i >= rows || n0 + c >= p.n) continue;
                float v = 0.0f;
                for (int r = 0; r < kClusterK; ++r) v += cluster.map_shared_rank(&part[0][0], r)[i * 64 + c];
                finish_one(p, m0 + i, n0 + c, v);
            }
        }
        cluster.sync();  // CTA 0 has read every part before they are rewritten (or the CTAs exit)
    }
}

// The few-row kernel's GEMMs (n and k wider than the skinny limit).
bool few_rows(const GemmDesc& g) {
    if ((g.layout != RT_NN && g.layout != RT_TN) || g.n <= kSkinnyMax || g.k <= kSkinnyMax || g.opt.kind || g.split_k > 1 || g.p2p.world)
        return false;
    return g.m <= kSkinnyMax || (g.in_dtype == RT_F32 && g.m <= kSkinnyRowsMax);
}

SkinnyParams make_params(const GemmDesc& g) {
    SkinnyParams p{};
    p.a = g.a;
    p.a2 = g.a_lo;
    p.b = g.b;
    p.c = g.c;
    p.c_lo = g.c_lo;
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

template <typename TIn, int KMAX>
cudaError_t launch_narrow_k(bool pdl, const GemmDesc& g, const SkinnyParams& p, dim3 grid, cudaStream_t st) {
    switch (g.layout) {
        case RT_NN: return launch_k(pdl, skinny_k_kernel<TIn, KMAX, true, false>, grid, dim3(kThreads), 0, st, p);
        case RT_NT: return launch_k(pdl, skinny_k_kernel<TIn, KMAX, true, true>, grid, dim3(kThreads), 0, st, p);
        case RT_TN: return launch_k(pdl, skinny_k_kernel<TIn, KMAX, false, false>, grid, dim3(kThreads), 0, st, p);
    }
    return cudaErrorInvalidValue;
}

template <typename TIn>
int launch_typed(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    SkinnyParams p = make_params(g);
    if (few_rows(g)) {
        const int64_t groups = (g.n + 63) / 64;
        if (groups * kClusterK > (int64_t)INT32_MAX) return fail(RT_ERR_INVALID, "few-row GEMM n too large");
        const dim3 grid((unsigned)(groups * kClusterK));
        if (g.layout == RT_TN)
            RT_CUDA(launch_k(ctx->plan_pdl, skinny_m_kernel<TIn, true>, grid, dim3(kThreads), 0, st, p));
        else
            RT_CUDA(launch_k(ctx->plan_pdl, skinny_m_kernel<TIn, false>, grid, dim3(kThreads), 0, st, p));
        count_launch(ctx);
        RT_CUDA(cudaGetLastError());
        return RT_OK;
    }
    if (g.n <= kSkinnyMax) {
        if (g.layout == RT_TN) {
            int slices = g.split_k > 1 && g.workspace ? g.split_k : 1;
            int64_t kps = (g.k + slices - 1) / slices;
            kps = (kps + 15) / 16 * 16;
            slices = (int)((g.k + kps - 1) / kps);
            p.k_per_slice = kps;
            p.ws = slices > 1 ? g.workspace : nullptr;
            dim3 grid((unsigned)((g.m + kThreads - 1) / kThreads), (unsigned)slices);
            RT_CUDA(launch_k(ctx->plan_pdl, skinny_n_tn_kernel<TIn, kSkinnyMax>, grid, dim3(kThreads), 0, st, p));
            count_launch(ctx);
            RT_CUDA(cudaGetLastError());
            if (slices > 1) {
                GemmDesc gr = g;
                gr.split_k = slices;
                return launch_splitk_reduce(ctx, gr, st);
            }
            return RT_OK;
        }
        const int64_t blocks = (g.m * 32 + kThreads - 1) / kThreads;  // one warp per row
        if (g.layout == RT_NT)
            RT_CUDA(launch_k(ctx->plan_pdl, skinny_n_kernel<TIn, true>, dim3((unsigned)blocks), dim3(kThreads),
                             kSkinnyNSmem, st, p));
        else
            RT_CUDA(launch_k(ctx->plan_pdl, skinny_n_kernel<TIn, false>, dim3((unsigned)blocks), dim3(kThreads),
                             kSkinnyNSmem, st, p));
    } else {
        dim3 grid((unsigned)((g.n + 255) / 256), (unsigned)((g.m + 31) / 32));
        if (grid.y > 65535u) return fail(RT_ERR_INVALID, "narrow-k GEMM m=%lld too large for its grid", (long long)g.m);
        if (g.k <= 4)
            RT_CUDA((launch_narrow_k<TIn, 4>(ctx->plan_pdl, g, p, grid, st)));
        else if (g.k <= 8)
            RT_CUDA((launch_narrow_k<TIn, 8>(ctx->plan_pdl, g, p, grid, st)));
        else
            RT_CUDA((launch_narrow_k<TIn, 16>(ctx->plan_pdl, g, p, grid, st)));
    }
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

}  // namespace

int gemm_skinny_init() {
    RT_CUDA(cudaFuncSetAttribute(skinny_n_kernel<float, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSkinnyNSmem));
    RT_CUDA(cudaFuncSetAttribute(skinny_n_kernel<float, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSkinnyNSmem));
    RT_CUDA(cudaFuncSetAttribute(skinny_n_kernel<__nv_bfloat16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSkinnyNSmem));
    RT_CUDA(cudaFuncSetAttribute(skinny_n_kernel<__nv_bfloat16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSkinnyNSmem));
    return RT_OK;
}

bool gemm_skinny_wanted(const GemmDesc& g) {
    if (g.m < 1 || g.k < 1) return false;
    return g.n <= kSkinnyMax || g.k <= kSkinnyMax || few_rows(g);
}

int launch_gemm_skinny(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    RT_CHECK(gemm_skinny_wanted(g), "GEMM is not skinny");
    if (g.in_dtype == RT_BF16) return launch_typed<__nv_bfloat16>(ctx, g, st);
    return launch_typed<float>(ctx, g, st);
}

}  // namespace rt
