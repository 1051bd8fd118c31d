// The rest of rtensor's differentiable ops on the GPU tape
// (crates/rtensor/src/ops.rs:49-309, losses.rs:31-160): broadcasting
// add/sub/mul/div with the adjoint reduced back to each operand's shape
// (tensor.rs:183-246 zip, 399-438 reduce_to), the pointwise family (scale,
// offset, neg, square, sqrt, exp, ln, relu, leaky_relu, sigmoid, tanh), the
// contractions sum / mean / row softmax, and the mse / mae / binary
// cross-entropy losses; plus SGD with momentum (optim.rs:44-116) and
// accuracy (losses.rs:181-185).
//
// Shapes are rank 2 ([rows, cols]; a scalar is [1, 1]); a broadcast operand
// is [1, n] (a row), [m, 1] (a column) or [1, 1] against [m, n], the cases
// tensor.rs's zip and reduce_to handle with dedicated paths.  Every kernel
// computes in f32 with the reference's per-element formulas; sums are
// deterministic (fixed-order block and warp trees, not the reference's
// sequential order, so they differ from the CPU in the last bits).
#include <cmath>

#include "tape_internal.h"

using namespace rt;
using rt::tp::Buf;
using rt::tp::check_var;

namespace {

constexpr int kThreads = 256;

int64_t grid_for(int64_t n, const rt_ctx* ctx) {
    int64_t b = (n + kThreads - 1) / kThreads;
    const int64_t cap = (int64_t)ctx->sm_count * 8;
    if (b > cap) b = cap;
    return b < 1 ? 1 : b;
}

// ------------------------------------------------------------ pointwise
// Forward value (ops.rs:132-227).
__device__ __forceinline__ float un_fwd(int op, float x, float p) {
    switch (op) {
        case RT_SCALE: return x * p;
        case RT_OFFSET: return x + p;
        case RT_NEG: return x * -1.0f;
        case RT_SQUARE: return x * x;
        case RT_SQRT: return sqrtf(x);
        case RT_EXP: return expf(x);
        case RT_LN: return logf(fmaxf(x, 1e-12f));
        case RT_RELU: return fmaxf(x, 0.0f);
        case RT_LEAKY_RELU: return x > 0.0f ? x : p * x;
        case RT_SIGMOID: return 1.0f / (1.0f + expf(-x));
        case RT_TANH: return tanhf(x);
    }
    return 0.0f;
}

// Adjoint contribution g * f'(.), written with the input x or the output y
// exactly as the reference's closures do.
__device__ __forceinline__ float un_bwd(int op, float g, float x, float y, float p) {
    switch (op) {
        case RT_SCALE: return g * p;
        case RT_OFFSET: return g;
        case RT_NEG: return g * -1.0f;
        case RT_SQUARE: return (g * x) * 2.0f;
        case RT_SQRT: return g / (y * 2.0f);
        case RT_EXP: return g * y;
        case RT_LN: return g / x;
        case RT_RELU: return g * (x > 0.0f ? 1.0f : 0.0f);
        case RT_LEAKY_RELU: return g * (x > 0.0f ? 1.0f : p);
        case RT_SIGMOID: return g * (y * (1.0f - y));
        case RT_TANH: return g * (1.0f - y * y);
    }
    return 0.0f;
}

__global__ void unary_fwd_kernel(int op, const float* x, int64_t ldx, float* y, int64_t ldy, int64_t rows,
                                 int64_t cols, float p) {
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        y[i * ldy + j] = un_fwd(op, x[i * ldx + j], p);
    }
}

__global__ void unary_bwd_kernel(int op, const float* g, int64_t ldg, const float* x, int64_t ldx, const float* y,
                                 int64_t ldy, float* gx, int64_t ldgx, int64_t rows, int64_t cols, float p) {
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        gx[i * ldgx + j] = un_bwd(op, g[i * ldg + j], x[i * ldx + j], y[i * ldy + j], p);
    }
}

// ------------------------------------------------------ broadcasting binary
enum Bcast : int { kFull = 0, kRow = 1, kCol = 2, kScalar = 3 };

struct Opnd {
    const float* p;
    int64_t ld;
    int mode;
};

__device__ __forceinline__ float at(const Opnd& o, int64_t i, int64_t j) {
    switch (o.mode) {
        case kRow: return o.p[j];
        case kCol: return o.p[i * o.ld];
        case kScalar: return o.p[0];
    }
    return o.p[i * o.ld + j];
}

__device__ __forceinline__ float bin_fwd(int op, float a, float b) {
    switch (op) {
        case RT_ADD: return a + b;
        case RT_SUB: return a - b;
        case RT_MUL: return a * b;
        case RT_DIV: return a / b;
    }
    return 0.0f;
}

__global__ void binary_fwd_kernel(int op, Opnd a, Opnd b, float* c, int64_t ldc, int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        c[i * ldc + j] = bin_fwd(op, at(a, i, j), at(b, i, j));
    }
}

// The full-shape adjoint contribution of operand `which` (0 = a, 1 = b),
// before the reduction to its shape (ops.rs:49-121):
//   add: g, g    sub: g, -g    mul: g*b, g*a    div: g/b, -((g*a)/(b*b))
__global__ void binary_bwd_kernel(int op, int which, const float* g, int64_t ldg, Opnd a, Opnd b, float* out,
                                  int64_t ldo, int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        const float gv = g[i * ldg + j];
        float v = 0.0f;
        switch (op) {
            case RT_ADD: v = gv; break;
            case RT_SUB: v = which == 0 ? gv : -gv; break;
            case RT_MUL: v = which == 0 ? gv * at(b, i, j) : gv * at(a, i, j); break;
            case RT_DIV: {
                const float bv = at(b, i, j);
                v = which == 0 ? gv / bv : -((gv * at(a, i, j)) / (bv * bv));
                break;
            }
        }
        out[i * ldo + j] = v;
    }
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Block sum in a fixed order (warp trees, then warp 0 over the warp sums).
__device__ float block_sum(float v) {
    __shared__ float ws[kThreads / 32];
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) ws[w] = v;
    __syncthreads();
    float s = 0.0f;
    if (w == 0) {
        s = lane < kThreads / 32 ? ws[lane] : 0.0f;
        s = warp_sum(s);
    }
    return s;  // valid in thread 0
}

// Row sums: dst[i * ldd] = sum_j src[i, j] (the [m, n] -> [m, 1] reduce_to).
__global__ void row_sums_kernel(const float* src, int64_t lds, int64_t rows, int64_t cols, float* dst, int64_t ldd) {
    const int lane = threadIdx.x & 31;
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < rows;
         i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        float s = 0.0f;
        for (int64_t j = lane; j < cols; j += 32) s += src[i * lds + j];
        s = warp_sum(s);
        if (lane == 0) dst[i * ldd] = s;
    }
}

// Column sums: dst[j] = sum_i src[i, j] (the [m, n] -> [1, n] reduce_to):
// thread j walks its column in row order.
__global__ void col_sums_kernel(const float* src, int64_t lds, int64_t rows, int64_t cols, float* dst) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < cols; j += (int64_t)gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (int64_t i = 0; i < rows; ++i) s += src[i * lds + j];
        dst[j] = s;
    }
}

// Total sum, stage 1: partial[b] = sum of block b's grid-strided elements
// (the grid size is fixed per call, so the order is too).
__global__ void sum_partial_kernel(const float* src, int64_t lds, int64_t rows, int64_t cols, float* partial) {
    const int64_t n = rows * cols;
    float s = 0.0f;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        s += src[i * lds + j];
    }
    s = block_sum(s);
    if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

// Stage 2: out[0] = (sum of the partials) / div, times sign.
__global__ void sum_final_kernel(const float* partial, int count, float div, float sign, float* out) {
    float s = 0.0f;
    for (int b = threadIdx.x; b < count; b += blockDim.x) s += partial[b];
    s = block_sum(s);
    if (threadIdx.x == 0) out[0] = sign * s / div;
}

// dst = g[0] / div everywhere (adjoint of sum and mean, ops.rs:239-255).
__global__ void fill_kernel(float* dst, int64_t ldd, int64_t rows, int64_t cols, const float* g, float div) {
    const float v = g[0] / div;
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        dst[i * ldd + j] = v;
    }
}

// ------------------------------------------------------------ row softmax
// Warp per row (tensor.rs:455-472): max, exp(z - max) and their sum, divide.
__global__ void softmax_fwd_kernel(const float* z, int64_t ldz, float* s, int64_t lds, int64_t rows, int64_t cols) {
    const int lane = threadIdx.x & 31;
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < rows;
         i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const float* zr = z + i * ldz;
        float mx = -INFINITY;
        for (int64_t j = lane; j < cols; j += 32) mx = fmaxf(mx, zr[j]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        float sum = 0.0f;
        for (int64_t j = lane; j < cols; j += 32) {
            const float e = expf(zr[j] - mx);
            s[i * lds + j] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        for (int64_t j = lane; j < cols; j += 32) s[i * lds + j] = s[i * lds + j] / sum;
    }
}

// Adjoint (ops.rs:288-309): per row dot = g . s, then s * (g - dot).
__global__ void softmax_bwd_kernel(const float* g, int64_t ldg, const float* s, int64_t lds, float* gz, int64_t ldz,
                                   int64_t rows, int64_t cols) {
    const int lane = threadIdx.x & 31;
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < rows;
         i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        float dot = 0.0f;
        for (int64_t j = lane; j < cols; j += 32) dot += g[i * ldg + j] * s[i * lds + j];
        dot = warp_sum(dot);
        for (int64_t j = lane; j < cols; j += 32) gz[i * ldz + j] = s[i * lds + j] * (g[i * ldg + j] - dot);
    }
}

// ------------------------------------------------------------------ losses
// mae (losses.rs:46-55): |d| for the mean, and the adjoint sign(d) * (g / n)
// with sign(0) = +1.
__global__ void abs_kernel(const float* d, int64_t ldd, float* out, int64_t ldo, int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        out[i * ldo + j] = fabsf(d[i * ldd + j]);
    }
}

__global__ void mae_bwd_kernel(const float* d, int64_t ldd, const float* g, float count, float* out, int64_t ldo,
                               int64_t rows, int64_t cols) {
    const float k = g[0] / count;
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        out[i * ldo + j] = (d[i * ldd + j] >= 0.0f ? 1.0f : -1.0f) * k;
    }
}

// binary cross-entropy (losses.rs:143-160) on c = clamp(p, 1e-7, 1 - 1e-7):
// term = y ln c + (1 - y) ln(1 - c) (the loss is -sum / N), adjoint
// (c - y) / (c (1 - c)) * (g / N).
__device__ __forceinline__ float bce_clamp(float p) { return fminf(fmaxf(p, 1e-7f), 1.0f - 1e-7f); }

__global__ void bce_term_kernel(const float* p, int64_t ldp, const float* y, int64_t ldy, float* out, int64_t ldo,
                                int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        const float c = bce_clamp(p[i * ldp + j]), yv = y[i * ldy + j];
        out[i * ldo + j] = yv * logf(c) + (1.0f - yv) * logf(1.0f - c);
    }
}

__global__ void bce_bwd_kernel(const float* p, int64_t ldp, const float* y, int64_t ldy, const float* g, float count,
                               float* out, int64_t ldo, int64_t rows, int64_t cols) {
    const float k = g[0] / count;
    const int64_t n = rows * cols;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / cols, j = t - i * cols;
        const float c = bce_clamp(p[i * ldp + j]), yv = y[i * ldy + j];
        out[i * ldo + j] = ((c - yv) / (c * (1.0f - c))) * k;
    }
}

// accuracy (losses.rs:181-185): rows whose first arg-max equals the label.
__global__ void accuracy_kernel(const float* z, int64_t ldz, int64_t rows, int64_t cols, const uint32_t* labels,
                                unsigned long long* hits) {
    const int lane = threadIdx.x & 31;
    unsigned long long mine = 0;
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < rows;
         i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        float best = -INFINITY;
        int64_t arg = cols;  // none yet; NaN rows never win
        for (int64_t j = lane; j < cols; j += 32) {
            const float v = z[i * ldz + j];
            if (v > best || (arg == cols && v == best)) best = v, arg = j;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int64_t oa = __shfl_xor_sync(0xffffffffu, arg, off);
            if (ob > best || (ob == best && oa < arg)) best = ob, arg = oa;
        }
        // argmax_rows (tensor.rs:476-492) takes element 0 first, so a NaN
        // there is the row's answer; later NaNs never win
        if (lane == 0 && (isnan(z[i * ldz]) ? 0 : arg) == (int64_t)labels[i]) ++mine;
    }
    if (lane == 0 && mine) atomicAdd(hits, mine);
}

// -------------------------------------------------------------- SGD momentum
// v = v * mu + g * lr ; theta -= v (optim.rs:97-112), each op rounded alone.
__global__ void sgd_momentum_kernel(float* theta, const float* g, float* v, int64_t n, float lr, float mu) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const float vi = __fadd_rn(__fmul_rn(v[t], mu), __fmul_rn(g[t], lr));
        v[t] = vi;
        theta[t] = __fsub_rn(theta[t], vi);
    }
}

// ----------------------------------------------------------------- helpers
int launched(rt_ctx* ctx) {
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}

Opnd opnd(const Buf& b, int mode) { return Opnd{b.p, b.ld, mode}; }

// Broadcast mode of an operand of shape [r, c] against [rows, cols].
int mode_of(const Buf& b, int64_t rows, int64_t cols) {
    if (b.rows == rows && b.cols == cols) return kFull;
    if (b.rows == 1 && b.cols == 1) return kScalar;
    if (b.rows == 1 && b.cols == cols) return kRow;
    if (b.cols == 1 && b.rows == rows) return kCol;
    return -1;
}

// dst (shape [1,1]) = sum of all of src, / div, * sign; deterministic.
int sum_all(rt_tape* t, const Buf& src, float div, float sign, const Buf& dst) {
    const int64_t n = src.rows * src.cols;
    int blocks = (int)((n + kThreads * 16 - 1) / (kThreads * 16));
    if (blocks > 512) blocks = 512;
    if (blocks < 1) blocks = 1;
    Buf partial;
    RT_TRY(t->alloc(partial, 1, blocks));
    sum_partial_kernel<<<blocks, kThreads, 0, t->ctx->stream>>>(src.p, src.ld, src.rows, src.cols, partial.p);
    RT_TRY(launched(t->ctx));
    sum_final_kernel<<<1, kThreads, 0, t->ctx->stream>>>(partial.p, blocks, div, sign, dst.p);
    return launched(t->ctx);
}

// Adds the full-shape contribution `full` to operand `idx` (shape `shape`),
// reducing the broadcast axes first (tensor.rs:399-438).
int reduce_into(rt_tape* t, int idx, const Buf& shape, int mode, const Buf& full) {
    if (mode == kFull) return t->accumulate(idx, full);
    Buf r;
    RT_TRY(t->alloc(r, shape.rows, shape.cols));
    cudaStream_t st = t->ctx->stream;
    if (mode == kScalar) {
        RT_TRY(sum_all(t, full, 1.0f, 1.0f, r));
    } else if (mode == kRow) {
        col_sums_kernel<<<(unsigned)grid_for(full.cols, t->ctx), kThreads, 0, st>>>(full.p, full.ld, full.rows,
                                                                                 full.cols, r.p);
        RT_TRY(launched(t->ctx));
    } else {
        const int64_t warps_needed = full.rows;
        int64_t blocks = (warps_needed * 32 + kThreads - 1) / kThreads;
        if (blocks > (int64_t)t->ctx->sm_count * 16) blocks = (int64_t)t->ctx->sm_count * 16;
        row_sums_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), kThreads, 0, st>>>(full.p, full.ld, full.rows,
                                                                                  full.cols, r.p, r.ld);
        RT_TRY(launched(t->ctx));
    }
    return t->accumulate(idx, r);
}

int64_t warp_blocks(int64_t rows, const rt_ctx* ctx) {
    int64_t b = (rows * 32 + kThreads - 1) / kThreads;
    const int64_t cap = (int64_t)ctx->sm_count * 16;
    if (b > cap) b = cap;
    return b < 1 ? 1 : b;
}

int target_buf(rt_tape* t, const rt_tensor* target, const Buf& like, Buf* out) {
    RT_CHECK(target && target->dtype == RT_F32, "loss target must be an f32 tensor");
    RT_CHECK(target->ctx == t->ctx, "loss target belongs to another context");
    RT_CHECK(target->rows == like.rows && target->cols == like.cols,
             "loss target shape [%lld,%lld] differs from the prediction's [%lld,%lld]", (long long)target->rows,
             (long long)target->cols, (long long)like.rows, (long long)like.cols);
    out->p = static_cast<float*>(target->ptr);
    out->rows = target->rows;
    out->cols = target->cols;
    out->ld = target->ld;
    return RT_OK;
}

}  // namespace

extern "C" {

int rt_var_unary(rt_var* a, rt_unary_op op, float param, rt_var** out) {
    RT_TRY(check_var(a));
    RT_CHECK(out && op >= RT_SCALE && op <= RT_TANH, "rt_var_unary: bad arguments");
    rt_tape* t = a->tape;
    const Buf X = t->nodes[a->idx].value;
    Buf Y;
    RT_TRY(t->alloc(Y, X.rows, X.cols));
    const int64_t n = X.rows * X.cols;
    if (n > 0) {
        unary_fwd_kernel<<<(unsigned)grid_for(n, t->ctx), kThreads, 0, t->ctx->stream>>>(op, X.p, X.ld, Y.p, Y.ld,
                                                                                      X.rows, X.cols, param);
        RT_TRY(launched(t->ctx));
    }
    const int ia = a->idx;
    *out = t->push({ia},
                   [t, X, Y, ia, op, param](const Buf& g) -> int {
                       Buf gx;
                       RT_TRY(t->alloc(gx, X.rows, X.cols));
                       const int64_t n = X.rows * X.cols;
                       if (n > 0) {
                           unary_bwd_kernel<<<(unsigned)grid_for(n, t->ctx), kThreads, 0, t->ctx->stream>>>(
                               op, g.p, g.ld, X.p, X.ld, Y.p, Y.ld, gx.p, gx.ld, X.rows, X.cols, param);
                           RT_TRY(launched(t->ctx));
                       }
                       return t->accumulate(ia, gx);
                   },
                   Y);
    return RT_OK;
}

int rt_var_binary(rt_var* a, rt_var* b, rt_binary_op op, rt_var** out) {
    RT_TRY(check_var(a));
    RT_TRY(check_var(b));
    RT_CHECK(out && a->tape == b->tape, "operands belong to different tapes");
    RT_CHECK(op >= RT_ADD && op <= RT_DIV, "rt_var_binary: unknown op %d", (int)op);
    rt_tape* t = a->tape;
    const Buf A = t->nodes[a->idx].value, B = t->nodes[b->idx].value;
    // broadcast_shapes for rank 2: per axis equal sizes, or one of them 1
    auto axis = [](int64_t x, int64_t y, int64_t* r) {
        if (x == y || y == 1) {
            *r = x;
            return true;
        }
        if (x == 1) {
            *r = y;
            return true;
        }
        return false;
    };
    int64_t rows = 0, cols = 0;
    const bool ok = axis(A.rows, B.rows, &rows) && axis(A.cols, B.cols, &cols);
    const int ma = ok ? mode_of(A, rows, cols) : -1, mb = ok ? mode_of(B, rows, cols) : -1;
    RT_CHECK(ok && ma >= 0 && mb >= 0, "shapes [%lld,%lld] and [%lld,%lld] do not broadcast", (long long)A.rows,
             (long long)A.cols, (long long)B.rows, (long long)B.cols);
    Buf C;
    RT_TRY(t->alloc(C, rows, cols));
    const int64_t n = rows * cols;
    if (n > 0) {
        binary_fwd_kernel<<<(unsigned)grid_for(n, t->ctx), kThreads, 0, t->ctx->stream>>>(op, opnd(A, ma), opnd(B, mb),
                                                                                       C.p, C.ld, rows, cols);
        RT_TRY(launched(t->ctx));
    }
    const int ia = a->idx, ib = b->idx;
    *out = t->push({ia, ib},
                   [t, A, B, ma, mb, ia, ib, op, rows, cols](const Buf& g) -> int {
                       const int64_t n = rows * cols;
                       for (int which = 0; which < 2; ++which) {
                           Buf full;
                           RT_TRY(t->alloc(full, rows, cols));
                           if (n > 0) {
                               binary_bwd_kernel<<<(unsigned)grid_for(n, t->ctx), kThreads, 0, t->ctx->stream>>>(
                                   op, which, g.p, g.ld, opnd(A, ma), opnd(B, mb), full.p, full.ld, rows, cols);
                               RT_TRY(launched(t->ctx));
                           }
                           RT_TRY(reduce_into(t, which == 0 ? ia : ib, which == 0 ? A : B, which == 0 ? ma : mb, full));
                       }
                       return RT_OK;
                   },
                   C);
    return RT_OK;
}

// Var::sum / Var::mean (ops.rs:239-255): scalar [1, 1] of the total (or the
// total / N); the adjoint is that scalar's adjoint (/ N) everywhere.
static int sum_or_mean(rt_var* a, bool mean, rt_var** out) {
    RT_TRY(check_var(a));
    RT_CHECK(out, "bad arguments");
    rt_tape* t = a->tape;
    const Buf X = t->nodes[a->idx].value;
    const float count = (float)(X.rows * X.cols);
    const float div = mean ? count : 1.0f;
    Buf S;
    RT_TRY(t->alloc(S, 1, 1));
    RT_TRY(sum_all(t, X, div, 1.0f, S));
    const int ia = a->idx;
    *out = t->push({ia},
                   [t, X, ia, div](const Buf& g) -> int {
                       Buf gx;
                       RT_TRY(t->alloc(gx, X.rows, X.cols));
                       const int64_t n = X.rows * X.cols;
                       if (n > 0) {
                           fill_kernel<<<(unsigned)grid_for(n, t->ctx), kThreads, 0, t->ctx->stream>>>(
                               gx.p, gx.ld, X.rows, X.cols, g.p, div);
                           RT_TRY(launched(t->ctx));
                       }
                       return t->accumulate(ia, gx);
                   },
                   S);
    return RT_OK;
}

int rt_var_sum(rt_var* a, rt_var** out) { return sum_or_mean(a, false, out); }
int rt_var_mean(rt_var* a, rt_var** out) { return sum_or_mean(a, true, out); }

int rt_var_softmax(rt_var* a, rt_var** out) {
    RT_TRY(check_var(a));
    RT_CHECK(out, "bad arguments");
    rt_tape* t = a->tape;
    const Buf Z = t->nodes[a->idx].value;
    Buf S;
    RT_TRY(t->alloc(S, Z.rows, Z.cols));
    if (Z.rows * Z.cols > 0) {
        softmax_fwd_kernel<<<(unsigned)warp_blocks(Z.rows, t->ctx), kThreads, 0, t->ctx->stream>>>(Z.p, Z.ld, S.p, S.ld,
                                                                                                Z.rows, Z.cols);
        RT_TRY(launched(t->ctx));
    }
    const int ia = a->idx;
    *out = t->push({ia},
                   [t, S, ia](const Buf& g) -> int {
                       Buf gz;
                       RT_TRY(t->alloc(gz, S.rows, S.cols));
                       if (S.rows * S.cols > 0) {
                           softmax_bwd_kernel<<<(unsigned)warp_blocks(S.rows, t->ctx), kThreads, 0, t->ctx->stream>>>(
                               g.p, g.ld, S.p, S.ld, gz.p, gz.ld, S.rows, S.cols);
                           RT_TRY(launched(t->ctx));
                       }
                       return t->accumulate(ia, gz);
                   },
                   S);
    return RT_OK;
}

// losses::mse (losses.rs:31-34): (pred - target).square().mean(), three nodes
// after a constant leaf for the target, as composed in the reference.
int rt_loss_mse(rt_var* pred, const rt_tensor* target, rt_var** out) {
    RT_TRY(check_var(pred));
    RT_CHECK(out, "bad arguments");
    rt_tape* t = pred->tape;
    Buf T;
    RT_TRY(target_buf(t, target, t->nodes[pred->idx].value, &T));
    rt_var *c, *d, *sq;
    RT_TRY(rt_tape_constant(t, target, &c));
    RT_TRY(rt_var_binary(pred, c, RT_SUB, &d));
    RT_TRY(rt_var_unary(d, RT_SQUARE, 0.0f, &sq));
    return rt_var_mean(sq, out);
}

// losses::mae (losses.rs:46-55): d = pred - target (a node), then one node
// for mean |d| whose adjoint is sign(d) * (g / N).
int rt_loss_mae(rt_var* pred, const rt_tensor* target, rt_var** out) {
    RT_TRY(check_var(pred));
    RT_CHECK(out, "bad arguments");
    rt_tape* t = pred->tape;
    Buf T;
    RT_TRY(target_buf(t, target, t->nodes[pred->idx].value, &T));
    rt_var *c, *d;
    RT_TRY(rt_tape_constant(t, target, &c));
    RT_TRY(rt_var_binary(pred, c, RT_SUB, &d));
    const Buf D = t->nodes[d->idx].value;
    const float count = (float)(D.rows * D.cols);
    Buf absd, L;
    RT_TRY(t->alloc(absd, D.rows, D.cols));
    RT_TRY(t->alloc(L, 1, 1));
    if (D.rows * D.cols > 0) {
        abs_kernel<<<(unsigned)grid_for(D.rows * D.cols, t->ctx), kThreads, 0, t->ctx->stream>>>(
            D.p, D.ld, absd.p, absd.ld, D.rows, D.cols);
        RT_TRY(launched(t->ctx));
    }
    RT_TRY(sum_all(t, absd, count, 1.0f, L));
    const int id = d->idx;
    *out = t->push({id},
                   [t, D, id, count](const Buf& g) -> int {
                       Buf gd;
                       RT_TRY(t->alloc(gd, D.rows, D.cols));
                       if (D.rows * D.cols > 0) {
                           mae_bwd_kernel<<<(unsigned)grid_for(D.rows * D.cols, t->ctx), kThreads, 0, t->ctx->stream>>>(
                               D.p, D.ld, g.p, count, gd.p, gd.ld, D.rows, D.cols);
                           RT_TRY(launched(t->ctx));
                       }
                       return t->accumulate(id, gd);
                   },
                   L);
    return RT_OK;
}

// losses::binary_cross_entropy (losses.rs:143-160) from probabilities.
int rt_loss_bce(rt_var* probs, const rt_tensor* target, rt_var** out) {
    RT_TRY(check_var(probs));
    RT_CHECK(out, "bad arguments");
    rt_tape* t = probs->tape;
    const Buf P = t->nodes[probs->idx].value;
    Buf Yt;
    RT_TRY(target_buf(t, target, P, &Yt));
    // the tape keeps its own copy of the target, like the reference's clone
    Buf Y;
    RT_TRY(t->alloc(Y, P.rows, P.cols));
    if (P.rows * P.cols > 0)
        RT_CUDA(cudaMemcpy2DAsync(Y.p, Y.ld * 4, Yt.p, Yt.ld * 4, Yt.cols * 4, Yt.rows, cudaMemcpyDeviceToDevice,
                                  t->ctx->stream));
    const float count = (float)(P.rows * P.cols);
    Buf term, L;
    RT_TRY(t->alloc(term, P.rows, P.cols));
    RT_TRY(t->alloc(L, 1, 1));
    if (P.rows * P.cols > 0) {
        bce_term_kernel<<<(unsigned)grid_for(P.rows * P.cols, t->ctx), kThreads, 0, t->ctx->stream>>>(
            P.p, P.ld, Y.p, Y.ld, term.p, term.ld, P.rows, P.cols);
        RT_TRY(launched(t->ctx));
    }
    RT_TRY(sum_all(t, term, count, -1.0f, L));
    const int ip = probs->idx;
    *out = t->push({ip},
                   [t, P, Y, ip, count](const Buf& g) -> int {
                       Buf gp;
                       RT_TRY(t->alloc(gp, P.rows, P.cols));
                       if (P.rows * P.cols > 0) {
                           bce_bwd_kernel<<<(unsigned)grid_for(P.rows * P.cols, t->ctx), kThreads, 0, t->ctx->stream>>>(
                               P.p, P.ld, Y.p, Y.ld, g.p, count, gp.p, gp.ld, P.rows, P.cols);
                           RT_TRY(launched(t->ctx));
                       }
                       return t->accumulate(ip, gp);
                   },
                   L);
    return RT_OK;
}

int rt_accuracy(rt_ctx* ctx, const rt_tensor* logits, const rt_tensor* labels, float* out) {
    RT_CHECK(ctx && logits && labels && out, "rt_accuracy: bad arguments");
    RT_CHECK(logits->dtype == RT_F32 && labels->dtype == RT_U32 && labels->rows * labels->cols == logits->rows,
             "rt_accuracy: f32 logits [n, c] and u32 labels [n] expected");
    if (logits->rows == 0) {
        *out = std::nanf("");  // 0 / 0, as the reference's mean over no rows
        return RT_OK;
    }
    unsigned long long* hits = nullptr;
    RT_CUDA(cudaMallocAsync((void**)&hits, sizeof(*hits), ctx->stream));
    RT_CUDA(cudaMemsetAsync(hits, 0, sizeof(*hits), ctx->stream));
    accuracy_kernel<<<(unsigned)warp_blocks(logits->rows, ctx), kThreads, 0, ctx->stream>>>(
        static_cast<const float*>(logits->ptr), logits->ld, logits->rows, logits->cols,
        static_cast<const uint32_t*>(labels->ptr), hits);
    RT_TRY(launched(ctx));
    unsigned long long h = 0;
    RT_CUDA(cudaMemcpyAsync(&h, hits, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream));
    RT_CUDA(cudaFreeAsync(hits, ctx->stream));
    RT_CUDA(cudaStreamSynchronize(ctx->stream));
    *out = (float)h / (float)logits->rows;
    return RT_OK;
}

}  // extern "C"

// ------------------------------------------------------------ SGD momentum
struct rt_sgd_state {
    rt_ctx* ctx = nullptr;
    float lr = 0, momentum = 0;
    std::unordered_map<uint64_t, float*> velocity;
};

extern "C" {

int rt_sgd_create(rt_ctx* ctx, float lr, float momentum, rt_sgd_state** out) {
    RT_CHECK(ctx && out, "rt_sgd_create: bad arguments");
    rt_sgd_state* s = new rt_sgd_state;
    s->ctx = ctx;
    s->lr = lr;
    s->momentum = momentum;
    *out = s;
    return RT_OK;
}

int rt_sgd_destroy(rt_sgd_state* s) {
    if (!s) return RT_OK;
    cudaStreamSynchronize(s->ctx->stream);
    for (auto& kv : s->velocity) cudaFree(kv.second);
    delete s;
    return RT_OK;
}

// Sgd::step (optim.rs:81-114): without momentum theta -= g * lr; with it the
// velocity (created zeroed per parameter) v = v * mu + g * lr, theta -= v.
int rt_sgd_state_step(rt_sgd_state* s, int n, rt_param* const* params, rt_tape* grads) {
    RT_CHECK(s && (n == 0 || params) && grads && grads->backward_done, "rt_sgd_state_step: bad arguments");
    if (s->momentum == 0.0f) return rt_sgd_step(s->ctx, n, params, grads, s->lr);
    rt_ctx* ctx = s->ctx;
    for (int i = 0; i < n; ++i) {
        rt_param* p = params[i];
        auto it = grads->param_nodes.find(p->id);
        if (it == grads->param_nodes.end() || !grads->grads[it->second].p) continue;
        const Buf& g = grads->grads[it->second];
        RT_CHECK(g.ld == p->value.ld && g.rows == p->value.rows, "gradient/parameter layout mismatch");
        const int64_t count = p->value.rows * p->value.ld;
        float*& v = s->velocity[p->id];
        if (!v) {
            RT_CUDA(cudaMalloc((void**)&v, (size_t)(count > 0 ? count : 1) * 4));
            RT_CUDA(cudaMemsetAsync(v, 0, (size_t)(count > 0 ? count : 1) * 4, ctx->stream));
        }
        if (count > 0) {
            sgd_momentum_kernel<<<(unsigned)grid_for(count, ctx), kThreads, 0, ctx->stream>>>(p->value.p, g.p, v, count,
                                                                                          s->lr, s->momentum);
            RT_TRY(launched(ctx));
        }
    }
    return RT_OK;
}

}  // extern "C"
