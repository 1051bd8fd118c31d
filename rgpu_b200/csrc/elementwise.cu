// Memory-bound kernels of the training step: softmax cross-entropy, the
// bias-gradient column reduction, bias/ReLU helpers, casts and the SGD/Adam
// updates.  Counterparts of rtensor's WGSL kernels in
// crates/rtensor/src/gpu/kernels.rs (XENT 138-167, COLSUM 182-199, ADAM
// 205-224, VEC 86-112, RELU_BWD 119-131) and mista.rs:326-341 (EMPACOTA), with
// the arithmetic of the CPU optimiser (optim.rs:80-198) that the parity tests
// hold them to.
#include "internal.h"

namespace rt {
namespace {

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ldf<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ void stf(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void stf<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void stf<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float v) {
    p[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------------ xent
// One warp per row (kernels.rs:146-166 uses one thread per row).  Loss is
// -ln(max(p_y, 1e-12)) as losses.rs:104-111 computes it; delta is
// (p - 1[j == y]) * scale (losses.rs:114, scale = g/n).
//
// Rows of up to 32 * VPL classes stay in registers: one read of the logits,
// one exp per element, one write of delta (the generic form below reads a
// row three times and takes each exp twice).  Both forms give the same bits.
template <typename TD, int VPL>
__global__ void xent_reg_kernel(const float* __restrict__ logits, int64_t ldz, const uint32_t* __restrict__ labels,
                                int64_t n, int64_t C, float scale, TD* __restrict__ delta, int64_t ldd,
                                float* __restrict__ loss) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= n) return;
    const float* z = logits + r * ldz;
    float v[VPL];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
        const int64_t j = lane + 32 * k;
        v[k] = j < C ? __ldg(z + j) : -INFINITY;
        mx = fmaxf(mx, v[k]);
    }
    mx = warp_max(mx);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
        const int64_t j = lane + 32 * k;
        if (j < C) {
            v[k] = expf(v[k] - mx);
            s += v[k];
        }
    }
    s = warp_sum(s);
    const uint32_t y = labels[r];
    TD* d = delta + r * ldd;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
        const int64_t j = lane + 32 * k;
        if (j < C) {
            const float p = v[k] / s;
            stf<TD>(d, j, (p - (j == (int64_t)y ? 1.0f : 0.0f)) * scale);
            if (j == (int64_t)y) loss[r] = -logf(fmaxf(p, 1e-12f));
        }
    }
    if (lane == 0 && (int64_t)y >= C) loss[r] = __int_as_float(0x7fc00000);  // label out of range: NaN loss
}

template <typename TD>
__global__ void xent_kernel(const float* __restrict__ logits, int64_t ldz, const uint32_t* __restrict__ labels,
                            int64_t n, int64_t C, float scale, TD* __restrict__ delta, int64_t ldd,
                            float* __restrict__ loss) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= n) return;
    const float* z = logits + r * ldz;
    float mx = -INFINITY;
    for (int64_t j = lane; j < C; j += 32) mx = fmaxf(mx, z[j]);
    mx = warp_max(mx);
    float s = 0.0f;
    for (int64_t j = lane; j < C; j += 32) s += expf(z[j] - mx);
    s = warp_sum(s);
    const uint32_t y = labels[r];
    TD* d = delta + r * ldd;
    for (int64_t j = lane; j < C; j += 32) {
        float p = expf(z[j] - mx) / s;
        stf<TD>(d, j, (p - (j == (int64_t)y ? 1.0f : 0.0f)) * scale);
    }
    if (lane == 0) {
        float l;
        if ((int64_t)y < C)
            l = -logf(fmaxf(expf(z[y] - mx) / s, 1e-12f));
        else
            l = __int_as_float(0x7fc00000);  // label out of range: NaN loss, as a visible error
        loss[r] = l;
    }
}

// --------------------------------------------------------------- colsum
constexpr int kColsumChunk = 64;

template <typename T>
__global__ void colsum_stage_kernel(const T* __restrict__ src, int64_t rows, int64_t cols, int64_t ld,
                                    int64_t chunk, float* __restrict__ dst) {
    int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= cols) return;
    int64_t r0 = (int64_t)blockIdx.y * chunk;
    int64_t r1 = min(rows, r0 + chunk);
    float acc = 0.0f;
    for (int64_t i = r0; i < r1; ++i) acc += ldf<T>(src, i * ld + j);
    dst[(int64_t)blockIdx.y * cols + j] = acc;
}

// ---------------------------------------------------------- elementwise
template <typename T>
__global__ void bias_add_kernel(T* z, int64_t rows, int64_t cols, int64_t ld, const float* b) {
    int64_t total = rows * cols;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = idx / cols, j = idx % cols;
        stf<T>(z, i * ld + j, ldf<T>(z, i * ld + j) + b[j]);
    }
}

template <typename T>
__global__ void relu_kernel(const T* x, T* y, int64_t rows, int64_t cols, int64_t ldx, int64_t ldy) {
    int64_t total = rows * cols;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = idx / cols, j = idx % cols;
        stf<T>(y, i * ldy + j, fmaxf(ldf<T>(x, i * ldx + j), 0.0f));
    }
}

template <typename T>
__global__ void relu_bwd_kernel(const T* a, T* dz, int64_t rows, int64_t cols, int64_t lda, int64_t ldz) {
    int64_t total = rows * cols;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = idx / cols, j = idx % cols;
        float m = ldf<T>(a, i * lda + j) > 0.0f ? 1.0f : 0.0f;
        stf<T>(dz, i * ldz + j, ldf<T>(dz, i * ldz + j) * m);
    }
}

template <typename TS, typename TD>
__global__ void cast_kernel(const TS* s, int64_t lds, TD* d, int64_t ldd, int64_t rows, int64_t cols) {
    int64_t total = rows * cols;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = idx / cols, j = idx % cols;
        stf<TD>(d, i * ldd + j, ldf<TS>(s, i * lds + j));
    }
}

// Same-dtype copy of a row-strided matrix whose rows start 16-byte aligned
// and hold a whole number of 16-byte vectors: a block per row (grid-stride
// over rows), 16-byte loads and stores, no index division.
__global__ void copy_rows_v16_kernel(const uint4* s, int64_t lds16, uint4* d, int64_t ldd16, int64_t rows,
                                     int64_t vecs) {
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint4* sr = s + r * lds16;
        uint4* dr = d + r * ldd16;
        for (int64_t v = threadIdx.x; v < vecs; v += blockDim.x) dr[v] = __ldg(sr + v);
    }
}

// ------------------------------------------------------------ optimisers
struct OptBatch {
    OptTensor t[kMaxOptTensors];
    int count;
};

// f32::powi with a runtime exponent (compiler-rt __powisf2: square and
// multiply), as Adam::step computes beta^t (optim.rs:163-164).
__device__ float powi_f32(float a, int b) {
    bool recip = b < 0;
    float r = 1.0f;
    for (;;) {
        if (b & 1) r = __fmul_rn(r, a);
        b /= 2;
        if (b == 0) break;
        a = __fmul_rn(a, a);
    }
    return recip ? 1.0f / r : r;
}

// Bias-correction scalars of Adam step t (optim.rs:164-172), t from the host.
__global__ void opt_scalars_at_kernel(OptScalars* s, int t, float beta1, float beta2) {
    s->t = t;
    float c1 = __fsub_rn(1.0f, powi_f32(beta1, t));
    float c2 = __fsub_rn(1.0f, powi_f32(beta2, t));
    s->inv_c1 = __fdiv_rn(1.0f, c1);
    s->inv_c2 = __fdiv_rn(1.0f, c2);
}

__global__ void opt_step_begin_kernel(OptScalars* s, float beta1, float beta2) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    int t = s->t + 1;
    s->t = t;
    float c1 = __fsub_rn(1.0f, powi_f32(beta1, t));
    float c2 = __fsub_rn(1.0f, powi_f32(beta2, t));
    s->inv_c1 = __fdiv_rn(1.0f, c1);
    s->inv_c2 = __fdiv_rn(1.0f, c2);
}

// One fused pass per element (adam_one: the rounding sequence of
// optim.rs:189-195), 128-bit vector loads where the buffers allow.
// 128-thread blocks of <= 48 registers per thread: small enough to co-reside
// with a running tensor-core GEMM CTA on the same SM, so a layer's update
// overlaps the next layer's GEMMs.
constexpr int kOptThreads = 128;

__global__ void __launch_bounds__(kOptThreads) adam_kernel(OptBatch batch, const OptScalars* __restrict__ sc, float lr, float b1, float b2,
                            float eps) {
    const OptTensor& T = batch.t[blockIdx.y];
    const float inv_c1 = sc->inv_c1, inv_c2 = sc->inv_c2;
    const float omb1 = __fsub_rn(1.0f, b1), omb2 = __fsub_rn(1.0f, b2);
    const int64_t n = T.n;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    bool vec = ((reinterpret_cast<uintptr_t>(T.theta) | reinterpret_cast<uintptr_t>(T.g) |
                 reinterpret_cast<uintptr_t>(T.m) | reinterpret_cast<uintptr_t>(T.v)) & 15) == 0 &&
               (!T.shadow || (reinterpret_cast<uintptr_t>(T.shadow) & 7) == 0);
    int64_t nv = vec ? n / 4 : 0;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nv; q += stride) {
        float4 th = reinterpret_cast<const float4*>(T.theta)[q];
        float4 g = reinterpret_cast<const float4*>(T.g)[q];
        float4 m = reinterpret_cast<const float4*>(T.m)[q];
        float4 v = reinterpret_cast<const float4*>(T.v)[q];
        th.x = adam_one(th.x, g.x, m.x, v.x, b1, b2, omb1, omb2, inv_c1, inv_c2, eps, lr);
        th.y = adam_one(th.y, g.y, m.y, v.y, b1, b2, omb1, omb2, inv_c1, inv_c2, eps, lr);
        th.z = adam_one(th.z, g.z, m.z, v.z, b1, b2, omb1, omb2, inv_c1, inv_c2, eps, lr);
        th.w = adam_one(th.w, g.w, m.w, v.w, b1, b2, omb1, omb2, inv_c1, inv_c2, eps, lr);
        reinterpret_cast<float4*>(T.theta)[q] = th;
        reinterpret_cast<float4*>(T.m)[q] = m;
        reinterpret_cast<float4*>(T.v)[q] = v;
        if (T.shadow) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(th.x, th.y);
            __nv_bfloat162 hi = __floats2bfloat162_rn(th.z, th.w);
            uint2 packed;
            packed.x = *reinterpret_cast<uint32_t*>(&lo);
            packed.y = *reinterpret_cast<uint32_t*>(&hi);
            reinterpret_cast<uint2*>(T.shadow)[q] = packed;
        }
    }
    for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float m = T.m[i], v = T.v[i];
        float th = adam_one(T.theta[i], T.g[i], m, v, b1, b2, omb1, omb2, inv_c1, inv_c2, eps, lr);
        T.theta[i] = th;
        T.m[i] = m;
        T.v[i] = v;
        if (T.shadow) T.shadow[i] = __float2bfloat16_rn(th);
    }
}

// optim.rs:88-95: theta -= g * lr.
__global__ void __launch_bounds__(kOptThreads) sgd_kernel(OptBatch batch, float lr) {
    const OptTensor& T = batch.t[blockIdx.y];
    const int64_t n = T.n;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    bool vec = ((reinterpret_cast<uintptr_t>(T.theta) | reinterpret_cast<uintptr_t>(T.g)) & 15) == 0 &&
               (!T.shadow || (reinterpret_cast<uintptr_t>(T.shadow) & 7) == 0);
    int64_t nv = vec ? n / 4 : 0;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nv; q += stride) {
        float4 th = reinterpret_cast<const float4*>(T.theta)[q];
        float4 g = reinterpret_cast<const float4*>(T.g)[q];
        th.x = __fsub_rn(th.x, __fmul_rn(g.x, lr));
        th.y = __fsub_rn(th.y, __fmul_rn(g.y, lr));
        th.z = __fsub_rn(th.z, __fmul_rn(g.z, lr));
        th.w = __fsub_rn(th.w, __fmul_rn(g.w, lr));
        reinterpret_cast<float4*>(T.theta)[q] = th;
        if (T.shadow) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(th.x, th.y);
            __nv_bfloat162 hi = __floats2bfloat162_rn(th.z, th.w);
            uint2 packed;
            packed.x = *reinterpret_cast<uint32_t*>(&lo);
            packed.y = *reinterpret_cast<uint32_t*>(&hi);
            reinterpret_cast<uint2*>(T.shadow)[q] = packed;
        }
    }
    for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float th = __fsub_rn(T.theta[i], __fmul_rn(T.g[i], lr));
        T.theta[i] = th;
        if (T.shadow) T.shadow[i] = __float2bfloat16_rn(th);
    }
}

// out[i] = in[i] + in[q_stride + i] + ... + in[(parts - 1) q_stride + i], summed
// in that order (the owner's side of the peer-memory reduce-scatter: one
// partial per source rank), 16-byte accesses where the buffers allow.
__global__ void sum_partials_kernel(float* __restrict__ out, const float* __restrict__ in, int64_t q_stride,
                                    int parts, int64_t n, bool vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t nv = vec ? n / 4 : 0;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nv; q += stride) {
        float4 acc = reinterpret_cast<const float4*>(in)[q];
        for (int r = 1; r < parts; ++r) {
            const float4 x = reinterpret_cast<const float4*>(in + r * q_stride)[q];
            acc.x = __fadd_rn(acc.x, x.x);
            acc.y = __fadd_rn(acc.y, x.y);
            acc.z = __fadd_rn(acc.z, x.z);
            acc.w = __fadd_rn(acc.w, x.w);
        }
        reinterpret_cast<float4*>(out)[q] = acc;
    }
    for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float acc = in[i];
        for (int r = 1; r < parts; ++r) acc = __fadd_rn(acc, in[r * q_stride + i]);
        out[i] = acc;
    }
}

// out[i] = sum over r < parts, in order, of (r == own_rank ? own[i] : in[r * q_stride + i]);
// out may be own (each element reads own[i] before writing out[i]).
__global__ void sum_partials_own_kernel(float* out, const float* own, const float* __restrict__ in,
                                        int64_t q_stride, int parts, int own_rank, int64_t n, bool vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t nv = vec ? n / 4 : 0;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nv; q += stride) {
        float4 acc = own_rank == 0 ? reinterpret_cast<const float4*>(own)[q] : reinterpret_cast<const float4*>(in)[q];
        for (int r = 1; r < parts; ++r) {
            const float4 x = r == own_rank ? reinterpret_cast<const float4*>(own)[q]
                                           : reinterpret_cast<const float4*>(in + r * q_stride)[q];
            acc.x = __fadd_rn(acc.x, x.x);
            acc.y = __fadd_rn(acc.y, x.y);
            acc.z = __fadd_rn(acc.z, x.z);
            acc.w = __fadd_rn(acc.w, x.w);
        }
        reinterpret_cast<float4*>(out)[q] = acc;
    }
    for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float acc = own_rank == 0 ? own[i] : in[i];
        for (int r = 1; r < parts; ++r) acc = __fadd_rn(acc, r == own_rank ? own[i] : in[r * q_stride + i]);
        out[i] = acc;
    }
}

__global__ void axpy_kernel(float* dst, int64_t ldd, const float* src, int64_t lds, int64_t rows, int64_t cols) {
    int64_t total = rows * cols;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = idx / cols, j = idx % cols;
        dst[i * ldd + j] = dst[i * ldd + j] + src[i * lds + j];
    }
}

// out[0] = (sum of rows[0..n)) / n, in a fixed order (one block).
__global__ void mean_rows_kernel(const float* rows, int64_t n, float* out) {
    __shared__ float part[256];
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += rows[i];
    part[threadIdx.x] = s;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[0] = n > 0 ? part[0] / (float)n : 0.0f;
}

template <typename T>
__global__ void fill_column_kernel(T* p, int64_t rows, int64_t ld, int64_t col, float value) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x)
        stf<T>(p, i * ld + col, value);
}

unsigned grid_for(const rt_ctx* ctx, int64_t work, int per_thread = 1) {
    int64_t blocks = (work / per_thread + 255) / 256;
    int64_t cap = (int64_t)ctx->sm_count * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

}  // namespace

int launch_xent(rt_ctx* ctx, const float* logits, int64_t ldz, const uint32_t* labels, int64_t n, int64_t classes,
                float scale, void* delta, rt_dtype ddt, int64_t ldd, float* loss_rows, cudaStream_t st) {
    if (n == 0) return RT_OK;
    unsigned blocks = (unsigned)((n + 7) / 8);
    const bool pdl = ctx->plan_pdl;
    if (classes <= 32 * 32) {
        if (ddt == RT_BF16)
            RT_CUDA(launch_k(pdl, xent_reg_kernel<__nv_bfloat16, 32>, dim3(blocks), dim3(256), 0, st, logits, ldz, labels,
                             n, classes, scale, (__nv_bfloat16*)delta, ldd, loss_rows));
        else
            RT_CUDA(launch_k(pdl, xent_reg_kernel<float, 32>, dim3(blocks), dim3(256), 0, st, logits, ldz, labels, n,
                             classes, scale, (float*)delta, ldd, loss_rows));
    } else if (ddt == RT_BF16) {
        RT_CUDA(launch_k(pdl, xent_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, logits, ldz, labels, n, classes,
                         scale, (__nv_bfloat16*)delta, ldd, loss_rows));
    } else {
        RT_CUDA(launch_k(pdl, xent_kernel<float>, dim3(blocks), dim3(256), 0, st, logits, ldz, labels, n, classes, scale,
                         (float*)delta, ldd, loss_rows));
    }
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int64_t colsum_scratch_rows(int64_t rows) { return (rows + kColsumChunk - 1) / kColsumChunk; }

int launch_colsum(rt_ctx* ctx, const void* src, rt_dtype dt, int64_t rows, int64_t cols, int64_t ld,
                  float* scratch, float* dst, cudaStream_t st) {
    if (cols == 0) return RT_OK;
    if (rows == 0) {
        RT_CUDA(cudaMemsetAsync(dst, 0, (size_t)cols * 4, st));
        return RT_OK;
    }
    dim3 block(256);
    if (rows <= kColsumChunk) {
        dim3 grid((unsigned)((cols + 255) / 256), 1);
        if (dt == RT_BF16)
            colsum_stage_kernel<__nv_bfloat16><<<grid, block, 0, st>>>((const __nv_bfloat16*)src, rows, cols, ld,
                                                                       rows, dst);
        else
            colsum_stage_kernel<float><<<grid, block, 0, st>>>((const float*)src, rows, cols, ld, rows, dst);
        count_launch(ctx);
        RT_CUDA(cudaGetLastError());
        return RT_OK;
    }
    int64_t parts = colsum_scratch_rows(rows);
    if (parts > 65535) return fail(RT_ERR_INVALID, "colsum: %lld rows exceed the two-stage limit", (long long)rows);
    dim3 grid((unsigned)((cols + 255) / 256), (unsigned)parts);
    if (dt == RT_BF16)
        colsum_stage_kernel<__nv_bfloat16><<<grid, block, 0, st>>>((const __nv_bfloat16*)src, rows, cols, ld,
                                                                   kColsumChunk, scratch);
    else
        colsum_stage_kernel<float><<<grid, block, 0, st>>>((const float*)src, rows, cols, ld, kColsumChunk, scratch);
    dim3 grid2((unsigned)((cols + 255) / 256), 1);
    colsum_stage_kernel<float><<<grid2, block, 0, st>>>(scratch, parts, cols, cols, parts, dst);
    count_launch(ctx, 2);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_bias_add(rt_ctx* ctx, void* z, rt_dtype dt, int64_t rows, int64_t cols, int64_t ld, const float* b,
                    cudaStream_t st) {
    if (rows * cols == 0) return RT_OK;
    unsigned g = grid_for(ctx, rows * cols);
    if (dt == RT_BF16)
        bias_add_kernel<__nv_bfloat16><<<g, 256, 0, st>>>((__nv_bfloat16*)z, rows, cols, ld, b);
    else
        bias_add_kernel<float><<<g, 256, 0, st>>>((float*)z, rows, cols, ld, b);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_relu(rt_ctx* ctx, const void* x, void* y, rt_dtype dt, int64_t rows, int64_t cols, int64_t ldx,
                int64_t ldy, cudaStream_t st) {
    if (rows * cols == 0) return RT_OK;
    unsigned g = grid_for(ctx, rows * cols);
    if (dt == RT_BF16)
        relu_kernel<__nv_bfloat16><<<g, 256, 0, st>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, rows, cols, ldx,
                                                      ldy);
    else
        relu_kernel<float><<<g, 256, 0, st>>>((const float*)x, (float*)y, rows, cols, ldx, ldy);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_relu_bwd(rt_ctx* ctx, const void* a, void* dz, rt_dtype dt, int64_t rows, int64_t cols, int64_t lda,
                    int64_t ldz, cudaStream_t st) {
    if (rows * cols == 0) return RT_OK;
    unsigned g = grid_for(ctx, rows * cols);
    if (dt == RT_BF16)
        relu_bwd_kernel<__nv_bfloat16><<<g, 256, 0, st>>>((const __nv_bfloat16*)a, (__nv_bfloat16*)dz, rows, cols,
                                                          lda, ldz);
    else
        relu_bwd_kernel<float><<<g, 256, 0, st>>>((const float*)a, (float*)dz, rows, cols, lda, ldz);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_cast(rt_ctx* ctx, const void* src, rt_dtype sdt, int64_t lds, void* dst, rt_dtype ddt, int64_t ldd,
                int64_t rows, int64_t cols, cudaStream_t st) {
    if (rows * cols == 0) return RT_OK;
    if (sdt == ddt) {
        const int64_t es = sdt == RT_BF16 ? 2 : 4;
        const bool v16 = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0 &&
                         (lds * es) % 16 == 0 && (ldd * es) % 16 == 0 && (cols * es) % 16 == 0;
        if (v16) {
            const int64_t cap = (int64_t)ctx->sm_count * 8;
            const unsigned blocks = (unsigned)(rows < cap ? rows : cap);
            copy_rows_v16_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(src), lds * es / 16,
                                                         static_cast<uint4*>(dst), ldd * es / 16, rows,
                                                         cols * es / 16);
            count_launch(ctx);
            RT_CUDA(cudaGetLastError());
            return RT_OK;
        }
    }
    unsigned g = grid_for(ctx, rows * cols);
    if (sdt == RT_F32 && ddt == RT_BF16)
        cast_kernel<float, __nv_bfloat16><<<g, 256, 0, st>>>((const float*)src, lds, (__nv_bfloat16*)dst, ldd, rows,
                                                             cols);
    else if (sdt == RT_BF16 && ddt == RT_F32)
        cast_kernel<__nv_bfloat16, float><<<g, 256, 0, st>>>((const __nv_bfloat16*)src, lds, (float*)dst, ldd, rows,
                                                             cols);
    else if (sdt == RT_F32 && ddt == RT_F32)
        cast_kernel<float, float><<<g, 256, 0, st>>>((const float*)src, lds, (float*)dst, ldd, rows, cols);
    else if (sdt == RT_BF16 && ddt == RT_BF16)
        cast_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, st>>>((const __nv_bfloat16*)src, lds,
                                                                     (__nv_bfloat16*)dst, ldd, rows, cols);
    else
        return fail(RT_ERR_INVALID, "cast: unsupported dtype pair");
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_axpy_inplace(rt_ctx* ctx, float* dst, int64_t ldd, const float* src, int64_t lds, int64_t rows,
                        int64_t cols, cudaStream_t st) {
    if (rows * cols == 0) return RT_OK;
    axpy_kernel<<<grid_for(ctx, rows * cols), 256, 0, st>>>(dst, ldd, src, lds, rows, cols);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_sum_partials(rt_ctx* ctx, float* out, const float* in, int64_t q_stride, int parts, int64_t n,
                        cudaStream_t st) {
    if (n == 0) return RT_OK;
    const bool vec = ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(in)) & 15) == 0 &&
                     (q_stride & 3) == 0;
    sum_partials_kernel<<<grid_for(ctx, vec ? n / 4 + 1 : n), 256, 0, st>>>(out, in, q_stride, parts, n, vec);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_sum_partials_own(rt_ctx* ctx, float* out, const float* own, const float* in, int64_t q_stride, int parts,
                            int own_rank, int64_t n, cudaStream_t st) {
    if (n == 0) return RT_OK;
    const bool vec = ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(own) |
                       reinterpret_cast<uintptr_t>(in)) & 15) == 0 && (q_stride & 3) == 0;
    sum_partials_own_kernel<<<grid_for(ctx, vec ? n / 4 + 1 : n), 256, 0, st>>>(out, own, in, q_stride, parts,
                                                                              own_rank, n, vec);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_mean_rows(rt_ctx* ctx, const float* rows, int64_t n, float* out, cudaStream_t st) {
    mean_rows_kernel<<<1, 256, 0, st>>>(rows, n, out);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_fill_column(rt_ctx* ctx, void* p, rt_dtype dt, int64_t rows, int64_t ld, int64_t col, float value,
                       cudaStream_t st) {
    if (rows == 0) return RT_OK;
    unsigned g = grid_for(ctx, rows);
    if (dt == RT_BF16)
        fill_column_kernel<__nv_bfloat16><<<g, 256, 0, st>>>((__nv_bfloat16*)p, rows, ld, col, value);
    else
        fill_column_kernel<float><<<g, 256, 0, st>>>((float*)p, rows, ld, col, value);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_opt_step_begin(rt_ctx* ctx, OptScalars* s, float beta1, float beta2, cudaStream_t st) {
    RT_CUDA(launch_k(ctx->plan_pdl, opt_step_begin_kernel, dim3(1), dim3(1), 0, st, s, beta1, beta2));
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_opt_scalars_at(rt_ctx* ctx, OptScalars* s, int t, float beta1, float beta2, cudaStream_t st) {
    opt_scalars_at_kernel<<<1, 1, 0, st>>>(s, t, beta1, beta2);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

static int fill_batch(OptBatch& b, const OptTensor* ts, int count, int64_t& max_n) {
    if (count < 1 || count > kMaxOptTensors)
        return fail(RT_ERR_INVALID, "optimizer: %d tensors (1..%d supported per launch)", count, kMaxOptTensors);
    max_n = 0;
    for (int i = 0; i < count; ++i) {
        b.t[i] = ts[i];
        if (ts[i].n > max_n) max_n = ts[i].n;
    }
    b.count = count;
    return RT_OK;
}

int launch_adam(rt_ctx* ctx, const OptTensor* ts, int count, const OptScalars* s, float lr, float beta1, float beta2,
                float eps, cudaStream_t st) {
    OptBatch b;
    int64_t max_n;
    RT_TRY(fill_batch(b, ts, count, max_n));
    if (max_n == 0) return RT_OK;
    dim3 grid(2 * grid_for(ctx, max_n, 4), (unsigned)count);
    adam_kernel<<<grid, kOptThreads, 0, st>>>(b, s, lr, beta1, beta2, eps);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

int launch_sgd(rt_ctx* ctx, const OptTensor* ts, int count, float lr, cudaStream_t st) {
    OptBatch b;
    int64_t max_n;
    RT_TRY(fill_batch(b, ts, count, max_n));
    if (max_n == 0) return RT_OK;
    dim3 grid(2 * grid_for(ctx, max_n, 4), (unsigned)count);
    sgd_kernel<<<grid, kOptThreads, 0, st>>>(b, lr);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

}  // namespace rt
