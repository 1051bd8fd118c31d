// Per-element optimiser arithmetic shared by the stand-alone SGD/Adam kernels
// and by the GEMM epilogues that apply the update to a dW tile as it leaves
// the accumulator.  Rounding sequence of rtensor's CPU optimiser
// (crates/rtensor/src/optim.rs:88-95 SGD, 189-195 Adam): every product and
// sum rounded separately (__fmul_rn / __fadd_rn forbid FMA contraction), so
// the GPU update is bit-identical to the CPU one for the same gradient.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace rt {

// Adam bias-correction scalars for the current step (device memory, written
// once per step by opt_step_begin_kernel).
struct OptScalars {
    int t;
    float inv_c1, inv_c2;
    float pad;
};

// Optimiser update fused into a GEMM epilogue: the GEMM's output tile is the
// gradient g of a parameter block theta with the same [rows, ld] layout.
struct OptFuse {
    int kind;             // 0 none, 1 sgd, 2 adam
    float* theta;         // f32 master
    float* m;             // Adam first moment
    float* v;             // Adam second moment
    __nv_bfloat16* shadow;  // bf16 copy of theta for the next GEMMs (may be null)
    const OptScalars* sc; // Adam step scalars
    float lr, beta1, beta2, eps;
};

__device__ __forceinline__ float adam_one(float th, float g, float& m, float& v, float b1, float b2, float omb1,
                                          float omb2, float inv_c1, float inv_c2, float eps, float lr) {
    m = __fadd_rn(__fmul_rn(m, b1), __fmul_rn(g, omb1));
    v = __fadd_rn(__fmul_rn(v, b2), __fmul_rn(__fmul_rn(g, g), omb2));
    float m_hat = __fmul_rn(m, inv_c1);
    float v_hat = __fmul_rn(v, inv_c2);
    return __fsub_rn(th, __fmul_rn(__fdiv_rn(m_hat, __fadd_rn(__fsqrt_rn(v_hat), eps)), lr));
}

__device__ __forceinline__ float sgd_one(float th, float g, float lr) { return __fsub_rn(th, __fmul_rn(g, lr)); }

// Applies the fused update to n <= N consecutive elements starting at flat
// index idx (gradients in g[0..n)).  Loops are fully unrolled over N with the
// tail predicated, so g stays in registers; vectorised when all 32 of a
// 32-wide chunk are present and the row segment is 16-byte aligned.
template <int N>
__device__ __forceinline__ void opt_apply_row(const OptFuse& o, int64_t idx, const float* g, int n) {
    if (o.kind == 0) return;
    const bool vec = N == 32 && n == 32 && ((idx & 3) == 0);
    if (o.kind == 2) {
        const float b1 = o.beta1, b2 = o.beta2;
        const float omb1 = __fsub_rn(1.0f, b1), omb2 = __fsub_rn(1.0f, b2);
        const float ic1 = o.sc->inv_c1, ic2 = o.sc->inv_c2;
        if (vec) {
#pragma unroll
            for (int q = 0; q < N / 4; ++q) {
                float4 th = reinterpret_cast<const float4*>(o.theta + idx)[q];
                float4 mm = reinterpret_cast<const float4*>(o.m + idx)[q];
                float4 vv = reinterpret_cast<const float4*>(o.v + idx)[q];
                th.x = adam_one(th.x, g[q * 4 + 0], mm.x, vv.x, b1, b2, omb1, omb2, ic1, ic2, o.eps, o.lr);
                th.y = adam_one(th.y, g[q * 4 + 1], mm.y, vv.y, b1, b2, omb1, omb2, ic1, ic2, o.eps, o.lr);
                th.z = adam_one(th.z, g[q * 4 + 2], mm.z, vv.z, b1, b2, omb1, omb2, ic1, ic2, o.eps, o.lr);
                th.w = adam_one(th.w, g[q * 4 + 3], mm.w, vv.w, b1, b2, omb1, omb2, ic1, ic2, o.eps, o.lr);
                reinterpret_cast<float4*>(o.theta + idx)[q] = th;
                reinterpret_cast<float4*>(o.m + idx)[q] = mm;
                reinterpret_cast<float4*>(o.v + idx)[q] = vv;
                if (o.shadow) {
                    __nv_bfloat162 lo = __floats2bfloat162_rn(th.x, th.y);
                    __nv_bfloat162 hi = __floats2bfloat162_rn(th.z, th.w);
                    uint2 pk;
                    pk.x = *reinterpret_cast<uint32_t*>(&lo);
                    pk.y = *reinterpret_cast<uint32_t*>(&hi);
                    reinterpret_cast<uint2*>(o.shadow + idx)[q] = pk;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < N; ++j) {
                if (j < n) {
                    float mm = o.m[idx + j], vv = o.v[idx + j];
                    float th = adam_one(o.theta[idx + j], g[j], mm, vv, b1, b2, omb1, omb2, ic1, ic2, o.eps, o.lr);
                    o.theta[idx + j] = th;
                    o.m[idx + j] = mm;
                    o.v[idx + j] = vv;
                    if (o.shadow) o.shadow[idx + j] = __float2bfloat16_rn(th);
                }
            }
        }
    } else {
        if (vec) {
#pragma unroll
            for (int q = 0; q < N / 4; ++q) {
                float4 th = reinterpret_cast<const float4*>(o.theta + idx)[q];
                th.x = sgd_one(th.x, g[q * 4 + 0], o.lr);
                th.y = sgd_one(th.y, g[q * 4 + 1], o.lr);
                th.z = sgd_one(th.z, g[q * 4 + 2], o.lr);
                th.w = sgd_one(th.w, g[q * 4 + 3], o.lr);
                reinterpret_cast<float4*>(o.theta + idx)[q] = th;
                if (o.shadow) {
                    __nv_bfloat162 lo = __floats2bfloat162_rn(th.x, th.y);
                    __nv_bfloat162 hi = __floats2bfloat162_rn(th.z, th.w);
                    uint2 pk;
                    pk.x = *reinterpret_cast<uint32_t*>(&lo);
                    pk.y = *reinterpret_cast<uint32_t*>(&hi);
                    reinterpret_cast<uint2*>(o.shadow + idx)[q] = pk;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < N; ++j) {
                if (j < n) {
                    float th = sgd_one(o.theta[idx + j], g[j], o.lr);
                    o.theta[idx + j] = th;
                    if (o.shadow) o.shadow[idx + j] = __float2bfloat16_rn(th);
                }
            }
        }
    }
}

}  // namespace rt
