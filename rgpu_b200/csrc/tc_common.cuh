// Shared pieces of the tcgen05 GEMM kernels (one-CTA and two-CTA forms): PTX
// wrappers for mbarriers, TMA, tcgen05 MMA/TMEM, the shared-memory and
// instruction descriptors, the tile scheduler, the fused epilogue and the
// host-side tensor-map encoder.
#pragma once

#include <cuda.h>

#include <mutex>

#include "internal.h"

namespace rt {
namespace tc {

constexpr int kThreads = 256;
constexpr int BM = 128;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait.  Returns false when the limit expired or another role
// aborted; the caller then leaves its loop.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > kWaitLimitNs) return false;
        }
    }
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// 3-D box load (x, y, plane): the 3xTF32 GEMM reads its hi and lo operand
// planes through one map whose third dimension selects the plane.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

// TMA store of a shared-memory box to global memory (bulk-group completion);
// the box is clipped at the tensor's bounds.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int32_t x, int32_t y, int32_t z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the shared-memory sources of this thread's bulk stores are read.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// ... all but the `pending` most recent bulk groups of this thread (0, 1, 3 or
// 7: the staging rings below hold 1, 2, 4 or 8 slots).
__device__ __forceinline__ void bulk_wait_read_upto(int pending) {
    switch (pending) {
        case 1: asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); break;
        case 3: asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory"); break;
        case 7: asm volatile("cp.async.bulk.wait_group.read 7;" ::: "memory"); break;
        default: asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); break;
    }
}
// Wait until this thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Make this thread's generic-proxy shared-memory writes visible to the async proxy (TMA).
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

template <bool kTF32>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    if constexpr (kTF32) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// 32 lanes x 32 columns of 32-bit accumulator: thread i of the warp receives
// row (lane base + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (tcgen05 "version 1" layout): start address,
// leading/stride byte offsets (16-byte units) and the 128-byte swizzle mode.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for tcgen05
    d |= (uint64_t)2 << 61;  // 128-byte swizzle
    return d;
}

// Instruction descriptor for kind::f16 (bf16 x bf16) or kind::tf32, f32 accumulate.
__host__ __device__ constexpr uint32_t make_idesc(bool tf32, bool a_mn, bool b_mn, int n, int m) {
    return (1u << 4)                              // D format: f32
           | ((tf32 ? 2u : 1u) << 7)              // A format: bf16 = 1, tf32 = 2
           | ((tf32 ? 2u : 1u) << 10)             // B format
           | ((a_mn ? 1u : 0u) << 15)             // A major-ness (1 = MN-major)
           | ((b_mn ? 1u : 0u) << 16)             // B major-ness
           | ((uint32_t)(n >> 3) << 17)           // N / 8
           | ((uint32_t)(m >> 4) << 24);          // M / 16
}

struct TcParams {
    int64_t m, n, k;
    int tiles_m, tiles_n, splits, kblocks, kb_per_split, group;
    void* c;
    int64_t ldc;
    float* ws;
    const float* bias;
    const void* mask;
    int64_t ldmask;
    int epi;
    int out_bf16;
    int* err;
    OptFuse opt;
    int kb_seg;  // 3xTF32: k blocks per product segment (the k loop runs 3 * kb_seg blocks); 0 otherwise
    int tma_store;  // epilogue: 1 = C and 2 = split-K partials through shared-memory staging and TMA stores,
                    // 3 = fused optimiser through the staging boxes (opt_chunk), 4 = rows scattered to
                    // their owners' receive buffers over peer memory (p2p_chunk), 0 = direct stores
    P2PScatter p2p;
    // Split bf16 A (a_lo) outside the pair kernel's SPLIT_A form: the k loop runs twice the
    // k blocks, alternating A's low-order plane (tmap_a2) and A itself at each k block; B is
    // the same for both.
    int split_a;
    void* c_lo;  // bf16 output's low-order plane (same ldc): bf16(v - bf16(v)); null = none
    int pdl;  // PDL_* (internal.h): how this launch waits for the kernel before it
    int* tile_ctr;  // pair kernel: zeroed tile counter of this launch (dynamic schedule); null = static
};

// Epilogue staging: one 32 x 32 output chunk per epilogue warp (4 KB), the
// layout of a 128-byte (f32) or 64-byte (bf16) swizzled TMA box.
constexpr int kStageBytes = 32 * 32 * 4;

// Stage geometry shared by host and device.
template <typename TIn, int BN>
struct Geo {
    static constexpr int ES = sizeof(TIn);
    static constexpr int BK = 128 / ES;        // one 128-byte swizzle row of k
    static constexpr int CHUNK = 128 / ES;     // MN elements per 128-byte row (MN-major boxes)
    static constexpr int UK = 32 / ES;         // k per tcgen05.mma
    static constexpr int A_BYTES = BM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
    static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr int EPI_BYTES = 4 * kStageBytes;  // 4 epilogue warps
    static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ void tile_coords(const TcParams& p, int t, int& split, int& mb, int& nb) {
    int per = p.tiles_m * p.tiles_n;
    split = t / per;
    int r = t % per;
    int gsz = p.group * p.tiles_n;
    int g = r / gsz;
    int first = g * p.group;
    int rows = min(p.tiles_m - first, p.group);
    int in = r % gsz;
    mb = first + in % rows;
    nb = in / rows;
}

__device__ __forceinline__ void record_error(int* err, int code, int detail) {
    if (atomicCAS(err, 0, code) == 0) err[1] = detail;
}

template <typename TOut>
__device__ __forceinline__ float load_mask_elem(const void* mask, int64_t idx);
template <>
__device__ __forceinline__ float load_mask_elem<float>(const void* mask, int64_t idx) {
    return static_cast<const float*>(mask)[idx];
}
template <>
__device__ __forceinline__ float load_mask_elem<__nv_bfloat16>(const void* mask, int64_t idx) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(mask)[idx]);
}

// Epilogue arithmetic for 32 consecutive columns of one row (row < m).
template <typename TOut>
__device__ __forceinline__ void epilogue_math(const TcParams& p, int64_t row, int64_t col0, float (&v)[32]) {
    const int64_t n = p.n;
    const bool full = col0 + 32 <= n;
    if (p.epi == RT_EPI_BIAS || p.epi == RT_EPI_BIAS_RELU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = v[j] + (col0 + j < n ? __ldg(p.bias + col0 + j) : 0.0f);
        if (p.epi == RT_EPI_BIAS_RELU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
        }
    } else if (p.epi == RT_EPI_RELU_MASK) {
        const int64_t base = row * p.ldmask + col0;
        if (full && sizeof(TOut) == 2) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.mask) + base);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 u = src[q];
                const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[q * 8 + j] = v[q * 8 + j] * (__bfloat162float(h[j]) > 0.0f ? 1.0f : 0.0f);
            }
        } else if (full) {
            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.mask) + base);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4 u = src[q];
                v[q * 4 + 0] = v[q * 4 + 0] * (u.x > 0.0f ? 1.0f : 0.0f);
                v[q * 4 + 1] = v[q * 4 + 1] * (u.y > 0.0f ? 1.0f : 0.0f);
                v[q * 4 + 2] = v[q * 4 + 2] * (u.z > 0.0f ? 1.0f : 0.0f);
                v[q * 4 + 3] = v[q * 4 + 3] * (u.w > 0.0f ? 1.0f : 0.0f);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < n) v[j] = v[j] * (load_mask_elem<TOut>(p.mask, base + j) > 0.0f ? 1.0f : 0.0f);
        }
    }
}

// Low-order part of an epilogue result: v - bf16(v), exact in f32 (v and its
// bf16 rounding share the exponent range), rounded to bf16 where it is stored.
__device__ __forceinline__ float lo_part(float v) { return v - __bfloat162float(__float2bfloat16_rn(v)); }

// Direct stores of one row's 32 columns (the thread's own row) to `base`
// (row stride ldc); LO stores the low-order parts of the bf16 rounding.
template <typename TOut, bool LO = false>
__device__ __forceinline__ void store_chunk_to(void* base, int64_t ldc, int64_t n, int64_t row, int64_t col0,
                                               const float (&v)[32]) {
    const bool full = col0 + 32 <= n;
    if constexpr (sizeof(TOut) == 2) {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(base) + row * ldc + col0;
        auto val = [&](int j) { return LO ? lo_part(v[j]) : v[j]; };
        if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 u;
                __nv_bfloat162 h0 = __floats2bfloat162_rn(val(q * 8 + 0), val(q * 8 + 1));
                __nv_bfloat162 h1 = __floats2bfloat162_rn(val(q * 8 + 2), val(q * 8 + 3));
                __nv_bfloat162 h2 = __floats2bfloat162_rn(val(q * 8 + 4), val(q * 8 + 5));
                __nv_bfloat162 h3 = __floats2bfloat162_rn(val(q * 8 + 6), val(q * 8 + 7));
                u.x = *reinterpret_cast<uint32_t*>(&h0);
                u.y = *reinterpret_cast<uint32_t*>(&h1);
                u.z = *reinterpret_cast<uint32_t*>(&h2);
                u.w = *reinterpret_cast<uint32_t*>(&h3);
                reinterpret_cast<uint4*>(dst)[q] = u;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < n) dst[j] = __float2bfloat16_rn(val(j));
        }
    } else {
        float* dst = static_cast<float*>(base) + row * ldc + col0;
        if (full) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
                reinterpret_cast<float4*>(dst)[q] = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < n) dst[j] = v[j];
        }
    }
}

// SPLIT_C: the kernel instantiation that also stores the low-order plane c_lo.
template <typename TOut, bool SPLIT_C = false>
__device__ __forceinline__ void epilogue_chunk(const TcParams& p, int64_t row, int64_t col0, float (&v)[32]) {
    epilogue_math<TOut>(p, row, col0, v);
    store_chunk_to<TOut>(p.c, p.ldc, p.n, row, col0, v);
    if constexpr (SPLIT_C && sizeof(TOut) == 2) store_chunk_to<TOut, true>(p.c_lo, p.ldc, p.n, row, col0, v);
}

// Writes lane `lane`'s row of a 32 x 32 chunk into the warp's staging box,
// swizzled as the C tensor map expects: f32 rows are 128 bytes (16-byte
// unit q of row r at q ^ (r & 7)), bf16 rows 64 bytes (unit q at
// q ^ ((r >> 1) & 3)).  Each 8-lane phase of a 16-byte store then covers all
// 32 banks once.
template <typename TOut, bool LO = false>
__device__ __forceinline__ void stage_row(uint8_t* box, int lane, const float (&v)[32]) {
    if constexpr (sizeof(TOut) == 2) {
        uint8_t* row = box + lane * 64;
        auto val = [&](int j) { return LO ? lo_part(v[j]) : v[j]; };
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 u;
            __nv_bfloat162 h0 = __floats2bfloat162_rn(val(q * 8 + 0), val(q * 8 + 1));
            __nv_bfloat162 h1 = __floats2bfloat162_rn(val(q * 8 + 2), val(q * 8 + 3));
            __nv_bfloat162 h2 = __floats2bfloat162_rn(val(q * 8 + 4), val(q * 8 + 5));
            __nv_bfloat162 h3 = __floats2bfloat162_rn(val(q * 8 + 6), val(q * 8 + 7));
            u.x = *reinterpret_cast<uint32_t*>(&h0);
            u.y = *reinterpret_cast<uint32_t*>(&h1);
            u.z = *reinterpret_cast<uint32_t*>(&h2);
            u.w = *reinterpret_cast<uint32_t*>(&h3);
            *reinterpret_cast<uint4*>(row + ((q ^ ((lane >> 1) & 3)) << 4)) = u;
        }
    } else {
        uint8_t* row = box + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(row + ((q ^ (lane & 7)) << 4)) =
                make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
    }
}

// Staged store of a warp's 32 x 32 chunk at (row0, col0): wait until the
// box's previous TMA store has read it, fill it, hand it to the async proxy
// and issue the store from lane 0.  Rows >= m and columns >= n are clipped
// by the TMA unit.
template <typename TOut>
__device__ __forceinline__ void stage_and_store(const CUtensorMap* tmap_c, uint8_t* box, int lane, int64_t row0,
                                                int64_t col0, const float (&v)[32], int split = -1) {
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
    stage_row<TOut>(box, lane, v);
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
        if (split < 0)
            tma_store_2d(tmap_c, smem_u32(box), (int32_t)col0, (int32_t)row0);
        else
            tma_store_3d(tmap_c, smem_u32(box), (int32_t)col0, (int32_t)row0, split);
        bulk_commit();
    }
}

// A warp's staging box(es) as a ring of slots: a 32 x 32 chunk takes 4 KB as
// f32 and 2 KB as bf16, so each 4 KB box holds one f32 or two bf16 slots.
// seq counts the warp's chunks; a chunk waits only until the store that last
// used its slot (nslots chunks back) has read it, so consecutive bf16 chunks
// alternate halves of the box.  split >= 0 stores into slice `split` of the
// split-K workspace (3-D map).
template <typename TOut>
__device__ __forceinline__ void stage_and_store_ring(const CUtensorMap* tmap_c, uint8_t* boxes, int nboxes, int lane,
                                                     int64_t row0, int64_t col0, const float (&v)[32],
                                                     uint32_t& seq, int split = -1) {
    constexpr int slot_bytes = 32 * 32 * (int)sizeof(TOut);
    const int nslots = nboxes * (kStageBytes / slot_bytes);
    uint8_t* box = boxes + (int)(seq % (uint32_t)nslots) * slot_bytes;
    if (lane == 0) bulk_wait_read_upto(nslots - 1);
    __syncwarp();
    stage_row<TOut>(box, lane, v);
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
        if (split < 0)
            tma_store_2d(tmap_c, smem_u32(box), (int32_t)col0, (int32_t)row0);
        else
            tma_store_3d(tmap_c, smem_u32(box), (int32_t)col0, (int32_t)row0, split);
        bulk_commit();
    }
    ++seq;
}

// ReLU mask of one row's 32 bf16 columns, loaded ahead of the accumulator
// (the caller issues these loads before its TMEM load, so both latencies
// overlap), then applied: v *= 1[mask > 0].
__device__ __forceinline__ void load_mask_bf16(const TcParams& p, int64_t row, int64_t col0, uint4 (&mk)[4]) {
    const uint4* src =
        reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.mask) + row * p.ldmask + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) mk[q] = src[q];
}
__device__ __forceinline__ void apply_mask_bf16(float (&v)[32], const uint4 (&mk)[4]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&mk[q]);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[q * 8 + j] = v[q * 8 + j] * (__bfloat162float(h[j]) > 0.0f ? 1.0f : 0.0f);
    }
}

// The same for a bf16 chunk with a low-order plane: the warp's 4 KB box holds
// the chunk's bf16(v) in its first 2 KB and bf16(v - bf16(v)) in its second,
// stored through the C map and the c_lo map in one bulk group.
__device__ __forceinline__ void stage_and_store_split(const CUtensorMap* tmap_hi, const CUtensorMap* tmap_lo,
                                                      uint8_t* box, int lane, int64_t row0, int64_t col0,
                                                      const float (&v)[32]) {
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
    stage_row<__nv_bfloat16>(box, lane, v);
    stage_row<__nv_bfloat16, true>(box + kStageBytes / 2, lane, v);
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(tmap_hi, smem_u32(box), (int32_t)col0, (int32_t)row0);
        tma_store_2d(tmap_lo, smem_u32(box + kStageBytes / 2), (int32_t)col0, (int32_t)row0);
        bulk_commit();
    }
}

// Fused optimiser epilogue (tma_store == 3) for one warp's 32 x 32 chunk of a
// dW tile: lane = row row0 + lane, v = its gradients in columns col0..col0+31.
// The chunk is transposed through the warp's 4 KB box (element (r, c) at
// r * 32 + (c ^ r), conflict-free for the row-per-lane writes and for the
// reads below); then one warp instruction covers four 128-byte rows (lane l:
// row 4 i + (l >> 3), columns 4 (l & 7) .. + 3), so the optimiser's reads of
// theta / m / v and its writes of them, of the bf16 shadow and of the
// gradient itself (C) are whole-line accesses.  Four rows' loads are issued
// before the first store.  Rounding as the stand-alone kernels (adam_one /
// sgd_one), so the update is bit-identical to theirs.
__device__ __forceinline__ void opt_chunk(const TcParams& p, float* box, int lane, int64_t row0, int64_t col0,
                                          const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 32; ++c) box[lane * 32 + (c ^ lane)] = v[c];
    __syncwarp();
    const OptFuse& o = p.opt;
    const bool adam = o.kind == 2;
    const int cq = (lane & 7) * 4;
    const int64_t col = col0 + cq;
    float* C = static_cast<float*>(p.c);
    const uintptr_t al = reinterpret_cast<uintptr_t>(o.theta) | reinterpret_cast<uintptr_t>(C) |
                         (adam ? reinterpret_cast<uintptr_t>(o.m) | reinterpret_cast<uintptr_t>(o.v) : 0);
    const bool fast = row0 + 32 <= p.m && col0 + 32 <= p.n && (p.ldc & 3) == 0 && (al & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(o.shadow) & 7) == 0;
    if (fast) {
        const float b1 = o.beta1, b2 = o.beta2;
        const float omb1 = __fsub_rn(1.0f, b1), omb2 = __fsub_rn(1.0f, b2);
        const float ic1 = adam ? o.sc->inv_c1 : 0.0f, ic2 = adam ? o.sc->inv_c2 : 0.0f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float g[4][4];
            float4 th[4], mm[4], vv[4];
            int64_t idx[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int rr = (h * 4 + u) * 4 + (lane >> 3);
                idx[u] = (row0 + rr) * p.ldc + col;
#pragma unroll
                for (int j = 0; j < 4; ++j) g[u][j] = box[rr * 32 + ((cq + j) ^ rr)];
                th[u] = *reinterpret_cast<const float4*>(o.theta + idx[u]);
                mm[u] = adam ? *reinterpret_cast<const float4*>(o.m + idx[u]) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                vv[u] = adam ? *reinterpret_cast<const float4*>(o.v + idx[u]) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float t4[4] = {th[u].x, th[u].y, th[u].z, th[u].w};
                float m4[4] = {mm[u].x, mm[u].y, mm[u].z, mm[u].w};
                float v4[4] = {vv[u].x, vv[u].y, vv[u].z, vv[u].w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    t4[j] = adam ? adam_one(t4[j], g[u][j], m4[j], v4[j], b1, b2, omb1, omb2, ic1, ic2, o.eps, o.lr)
                                 : sgd_one(t4[j], g[u][j], o.lr);
                *reinterpret_cast<float4*>(o.theta + idx[u]) = make_float4(t4[0], t4[1], t4[2], t4[3]);
                if (adam) {
                    *reinterpret_cast<float4*>(o.m + idx[u]) = make_float4(m4[0], m4[1], m4[2], m4[3]);
                    *reinterpret_cast<float4*>(o.v + idx[u]) = make_float4(v4[0], v4[1], v4[2], v4[3]);
                }
                if (o.shadow) {
                    __nv_bfloat162 lo = __floats2bfloat162_rn(t4[0], t4[1]);
                    __nv_bfloat162 hi = __floats2bfloat162_rn(t4[2], t4[3]);
                    uint2 pk;
                    pk.x = *reinterpret_cast<uint32_t*>(&lo);
                    pk.y = *reinterpret_cast<uint32_t*>(&hi);
                    *reinterpret_cast<uint2*>(o.shadow + idx[u]) = pk;
                }
                *reinterpret_cast<float4*>(C + idx[u]) = make_float4(g[u][0], g[u][1], g[u][2], g[u][3]);
            }
        }
    } else {
        // ragged edge of the output, or unaligned buffers: element by element
#pragma unroll 1
        for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3);
            const int64_t row = row0 + rr;
            if (row >= p.m) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (col + j >= p.n) break;
                float g = box[rr * 32 + ((cq + j) ^ rr)];
                const int64_t i = row * p.ldc + col + j;
                opt_apply_row<1>(o, i, &g, 1);
                C[i] = g;
            }
        }
    }
    __syncwarp();  // the box is rewritten by the next chunk
}

// Peer-scatter epilogue (tma_store == 4) for one warp's 32 x 32 chunk of a dW
// tile, lane = row row0 + lane: transposed through the warp's box as in
// opt_chunk, then each lane stores four consecutive columns of one row, four
// rows per warp instruction, to the row's owner (a peer's receive buffer, or
// this rank's own) or, past owned_end, to C.  The caller ends the kernel's
// epilogue with a system-scope fence, so every store is in place before the
// rank's barrier after the GEMM.
__device__ __forceinline__ void p2p_chunk(const TcParams& p, float* box, int lane, int64_t row0, int64_t col0,
                                          const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 32; ++c) box[lane * 32 + (c ^ lane)] = v[c];
    __syncwarp();
    const P2PScatter& s = p.p2p;
    const int cq = (lane & 7) * 4;
    const int64_t col = col0 + cq;
    float* C = static_cast<float*>(p.c);
#pragma unroll 2
    for (int it = 0; it < 8; ++it) {
        const int rr = it * 4 + (lane >> 3);
        const int64_t i = row0 + rr;
        if (i >= p.m) continue;
        float* dst;
        if (i < s.owned_end) {
            const int64_t o = i / s.rows_owned;
            dst = s.peer[o] + (int64_t)s.rank * s.q_stride + (s.base_row + i - o * s.rows_owned) * s.ld;
        } else {
            dst = C + i * p.ldc;
        }
        float g[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) g[j] = box[rr * 32 + ((cq + j) ^ rr)];
        if (col + 4 <= p.n && (reinterpret_cast<uintptr_t>(dst + col) & 15) == 0) {
            *reinterpret_cast<float4*>(dst + col) = make_float4(g[0], g[1], g[2], g[3]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (col + j < p.n) dst[col + j] = g[j];
        }
    }
    __syncwarp();
}

// ------------------------------------------------------------------ host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D row-major tensor: `inner` contiguous elements per row, `outer` rows,
// row stride `ld` elements; box (box_inner x box_outer), 128-byte swizzle.
inline int make_tmap(CUtensorMap* map, const void* base, bool bf16, int64_t inner, int64_t outer, int64_t ld,
              int box_inner, int box_outer, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(RT_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
    const int es = bf16 ? 2 : 4;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(RT_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): inner %lld outer %lld ld %lld box %dx%d",
                    (int)r, (long long)inner, (long long)outer, (long long)ld, box_inner, box_outer);
    return RT_OK;
}

// Output map for the staged epilogue: [m, n] row-major, row stride ldc, box
// 32 x 32 (128-byte swizzle for f32 rows, 64-byte for bf16 rows).
inline int make_tmap_out(CUtensorMap* map, void* c, bool bf16, int64_t m, int64_t n, int64_t ldc) {
    return make_tmap(map, c, bf16, n, m, ldc, 32, 32, bf16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
}

// 3-D f32 tensor of `planes` [outer, inner] planes, row stride `ld`, plane
// stride `plane` elements; box (box_inner x box_outer x 1), 128-byte swizzle.
inline int make_tmap_planes(CUtensorMap* map, const float* base, int64_t inner, int64_t outer, int64_t ld,
                            int64_t plane, int planes, int box_inner, int box_outer) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(RT_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)(ld * 4), (cuuint64_t)(plane * 4)};
    cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(RT_ERR_INVALID,
                    "cuTensorMapEncodeTiled (planes) failed (%d): inner %lld outer %lld ld %lld plane %lld box %dx%d",
                    (int)r, (long long)inner, (long long)outer, (long long)ld, (long long)plane, box_inner, box_outer);
    return RT_OK;
}

// Split-K partials [splits][m][n] f32 (row stride n) for the staged epilogue:
// box 32 x 32 x 1, 128-byte swizzle.  n * 4 must be a multiple of 16.
inline int make_tmap_ws(CUtensorMap* map, float* ws, int64_t m, int64_t n, int splits) {
    return make_tmap_planes(map, ws, n, m, n, m * n, splits, 32, 32);
}

}  // namespace tc
}  // namespace rt
