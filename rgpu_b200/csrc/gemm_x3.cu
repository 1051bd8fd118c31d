// f32 GEMM on the tensor cores: three tf32 tcgen05 products ("3xTF32").
//
// rtensor's f32 GEMMs (crates/rtensor/src/gpu/gemm.rs MM_FAST, splitk.rs
// MM_SPLITK) compute in full f32 and the f32 parity bar is 1e-4 relative L2
// per gradient, which a single tf32 product (10 explicit mantissa bits) does
// not meet.  Each operand x is split into
//     hi = x rounded to the nearest tf32 value        (ties to even)
//     lo = x - hi rounded to the nearest tf32 value   (x - hi is exact in f32)
// and C = lo(A) hi(B) + hi(A) lo(B) + hi(A) hi(B), all three accumulated in
// one TMEM accumulator.  |x - hi| <= 2^-11 |x| and the part of x that lo
// drops is <= 2^-22 |x|, so the dropped lo*lo term and lo's rounding are
// about 2^-22 of each product, and with both roundings to nearest their
// errors carry no sign bias that would add up along k (clearing low bits
// instead gives every product an error of the product's own sign, which
// accumulates coherently on data whose sums cancel).  The tensor-core
// accumulation adds its own rounding, which grows with k as in the bf16 path.
//
// The split runs as one pass that writes both operands' hi/lo planes into a
// workspace, K-major for both ([m][k] for A, [n][k] for B): tcgen05 reads
// MN-major tf32 operands only in the 32-byte-atom 128-byte swizzle, so an
// operand stored MN-major ([k][m] for A in dW = X^T dY, [k][n] for B in
// Y = X W) is transposed on the way, through a 64 x 64 shared-memory tile
// that keeps both the reads and the writes coalesced.  The GEMM is the
// one-CTA tcgen05 kernel of gemm_tc.cu in its X3 form (both operands
// K-major): 3-D TMA maps whose third coordinate picks the plane, and a k loop
// of three segments.
#include "internal.h"

namespace rt {
namespace {

constexpr int64_t kPlaneAlign = 32;  // plane row stride: a multiple of 32 floats (128 bytes)

int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// One operand: `mn` x `k` logical, stored either K-major ([mn][ld_src],
// transpose = 0) or MN-major ([k][ld_src], transpose = 1); its planes are
// [2][mn][ldw] with ldw = round_up(k, 32).
struct Operand {
    const float* src;
    int64_t ld_src, mn, k;
    int transpose;
    float* dst;
    int64_t ldw;
};

Operand operand_a(const GemmDesc& g) {
    Operand o{};
    o.src = static_cast<const float*>(g.a);
    o.ld_src = g.lda;
    o.mn = g.m;
    o.k = g.k;
    o.transpose = g.layout == RT_TN;  // A stored [k][m]
    o.ldw = round_up(g.k, kPlaneAlign);
    return o;
}

Operand operand_b(const GemmDesc& g) {
    Operand o{};
    o.src = static_cast<const float*>(g.b);
    o.ld_src = g.ldb;
    o.mn = g.n;
    o.k = g.k;
    o.transpose = g.layout != RT_NT;  // B stored [k][n]; NT stores it [n][k]
    o.ldw = round_up(g.k, kPlaneAlign);
    return o;
}

size_t plane_floats(const Operand& o) { return (size_t)o.mn * (size_t)o.ldw; }

// Rounds a finite f32 to the nearest tf32 value (10 explicit mantissa bits),
// ties to even: add just under half a tf32 ulp plus the lowest kept bit, then
// clear the 13 dropped bits (a carry out of the mantissa steps the exponent,
// which is the correctly rounded result).
__device__ __forceinline__ float tf32_round(float x) {
    uint32_t u = __float_as_uint(x);
    u = (u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
    return __uint_as_float(u);
}

// Non-finite values go whole into the hi plane (a NaN keeps its payload);
// the GEMM then yields a non-finite output row, NaN where the hi(A) lo(B)
// product meets inf * 0.  A finite x within half a tf32 ulp of FLT_MAX, which
// would round to inf, keeps its truncated hi.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    if (isfinite(x)) {
        hi = tf32_round(x);
        if (!isfinite(hi)) hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
        lo = tf32_round(x - hi);  // x - hi is exact: x and hi share all but the low bits
    } else {
        hi = x;
        lo = 0.0f;
    }
}

constexpr int kSplitThreads = 256;
constexpr int kT = 64;  // transposing tile: 64 k x 64 mn

// blockIdx.y selects the operand (uniform per block, so the barriers of the
// transposing form are reached by every thread of the block).
__global__ void __launch_bounds__(kSplitThreads) split_planes_kernel(Operand a, Operand b) {
    pdl_wait();  // programmatic dependent launch: the kernel before this one is done
    pdl_launch_dependents();
    __shared__ float tile[kT][kT + 1];
    const Operand& o = blockIdx.y == 0 ? a : b;
    float* hi_plane = o.dst;
    float* lo_plane = o.dst + (size_t)o.mn * o.ldw;
    const int tid = threadIdx.x;
    if (!o.transpose) {
        const int64_t stride = (int64_t)gridDim.x * kSplitThreads;
        const bool vec = (o.k % 4 == 0) && (o.ld_src % 4 == 0) && ((reinterpret_cast<uintptr_t>(o.src) & 15) == 0);
        if (vec) {
            const int64_t q = o.k / 4;
            const int64_t total = o.mn * q;
            for (int64_t i = (int64_t)blockIdx.x * kSplitThreads + tid; i < total; i += stride) {
                const int64_t r = i / q, c = (i - r * q) * 4;
                float4 x = __ldg(reinterpret_cast<const float4*>(o.src + r * o.ld_src + c));
                float4 h, l;
                split_tf32(x.x, h.x, l.x);
                split_tf32(x.y, h.y, l.y);
                split_tf32(x.z, h.z, l.z);
                split_tf32(x.w, h.w, l.w);
                *reinterpret_cast<float4*>(hi_plane + r * o.ldw + c) = h;
                *reinterpret_cast<float4*>(lo_plane + r * o.ldw + c) = l;
            }
        } else {
            const int64_t total = o.mn * o.k;
            for (int64_t i = (int64_t)blockIdx.x * kSplitThreads + tid; i < total; i += stride) {
                const int64_t r = i / o.k, c = i - r * o.k;
                float h, l;
                split_tf32(__ldg(o.src + r * o.ld_src + c), h, l);
                hi_plane[r * o.ldw + c] = h;
                lo_plane[r * o.ldw + c] = l;
            }
        }
        return;
    }
    // transposing form: source [k][mn] -> planes [mn][k], one 64 x 64 tile at a
    // time.  Reads: 16 threads cover a 256-byte source row segment (float4);
    // writes: 16 threads cover a 256-byte plane row segment (float4).
    const int64_t tiles_mn = (o.mn + kT - 1) / kT, tiles_k = (o.k + kT - 1) / kT;
    const int quad = tid % 16, rsub = tid / 16;  // 16 quads x 16 rows per pass, 4 passes
    const bool src_vec = (o.ld_src % 4 == 0) && ((reinterpret_cast<uintptr_t>(o.src) & 15) == 0);
    for (int64_t t = blockIdx.x; t < tiles_mn * tiles_k; t += gridDim.x) {
        const int64_t mn0 = (t % tiles_mn) * kT, k0 = (t / tiles_mn) * kT;
        const bool full_mn = mn0 + kT <= o.mn;
#pragma unroll
        for (int pass = 0; pass < 4; ++pass) {
            const int r = rsub + 16 * pass;  // k row within the tile
            const int64_t kk = k0 + r, c = mn0 + 4 * quad;
            float v[4];
            if (kk < o.k && full_mn && src_vec) {
                const float4 x = __ldg(reinterpret_cast<const float4*>(o.src + kk * o.ld_src + c));
                v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) v[e] = (kk < o.k && c + e < o.mn) ? __ldg(o.src + kk * o.ld_src + c + e) : 0.0f;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) tile[r][4 * quad + e] = v[e];
        }
        __syncthreads();
        const bool full_k = k0 + kT <= o.k;
#pragma unroll
        for (int pass = 0; pass < 4; ++pass) {
            const int r = rsub + 16 * pass;  // mn row within the tile
            const int64_t row = mn0 + r, c = k0 + 4 * quad;
            if (row < o.mn) {
                float h[4], l[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) split_tf32(tile[4 * quad + e][r], h[e], l[e]);
                if (full_k) {
                    *reinterpret_cast<float4*>(hi_plane + row * o.ldw + c) = make_float4(h[0], h[1], h[2], h[3]);
                    *reinterpret_cast<float4*>(lo_plane + row * o.ldw + c) = make_float4(l[0], l[1], l[2], l[3]);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (c + e < o.k) {
                            hi_plane[row * o.ldw + c + e] = h[e];
                            lo_plane[row * o.ldw + c + e] = l[e];
                        }
                }
            }
        }
        __syncthreads();
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool gemm_x3_supported(const rt_ctx* ctx, const GemmDesc& g) {
    if (ctx->cc_major != 10 || !ctx->f32_tensor) return false;
    if (g.in_dtype != RT_F32) return false;
    if (g.m < 1 || g.n < 1 || g.k < 1) return false;
    if (g.m >= (1ll << 31) || g.n >= (1ll << 31) || g.k >= (1ll << 31)) return false;
    // The operands are copied into aligned planes; only the output side has
    // alignment rules (vector stores, vector mask loads).
    const int64_t os = g.out_dtype == RT_BF16 ? 2 : 4;
    if (!aligned16(g.c) || (g.ldc * os) % 16) return false;
    if (g.epi == RT_EPI_RELU_MASK && (!aligned16(g.mask) || (g.ldmask * 4) % 16)) return false;
    return true;
}

size_t gemm_x3_workspace_bytes(const GemmDesc& g) {
    Operand a = operand_a(g), b = operand_b(g);
    const size_t fa = round_up((int64_t)(2 * plane_floats(a)), 64);  // keep B's planes 256-byte aligned
    return (fa + 2 * plane_floats(b)) * sizeof(float);
}

int launch_gemm_x3(rt_ctx* ctx, const GemmDesc& g, float* ws, size_t ws_bytes, cudaStream_t st) {
    RT_CHECK(gemm_x3_supported(ctx, g), "operands not eligible for the 3xTF32 GEMM");
    const size_t need = gemm_x3_workspace_bytes(g);
    RT_CHECK(ws && ws_bytes >= need && aligned16(ws), "3xTF32 workspace too small or misaligned: %zu < %zu bytes",
             ws_bytes, need);
    Operand a = operand_a(g), b = operand_b(g);
    a.dst = ws;
    b.dst = ws + round_up((int64_t)(2 * plane_floats(a)), 64);
    // enough blocks for the larger operand: 4096 elements per block and pass
    const int64_t work = a.mn * a.k > b.mn * b.k ? a.mn * a.k : b.mn * b.k;
    int64_t blocks = (work + 4095) / 4096;
    const int64_t cap = (int64_t)ctx->sm_count * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    RT_CUDA(launch_k(ctx->plan_pdl, split_planes_kernel, dim3((unsigned)blocks, 2), dim3(kSplitThreads), 0, st, a, b));
    count_launch(ctx);
    X3Planes x3{a.dst, a.ldw, (int64_t)plane_floats(a), b.dst, b.ldw, (int64_t)plane_floats(b)};
    return launch_gemm_tc_x3(ctx, g, x3, st);
}

int gemm_x3_init(rt_ctx* ctx) {
    (void)ctx;
    return gemm_tc_x3_init();
}

}  // namespace rt
