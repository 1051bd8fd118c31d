// Tensor-core GEMM for sm_100a: tcgen05.mma with TMEM accumulators, operands
// staged by TMA into 128B-swizzled shared memory, a persistent tile loop with
// L2-grouped rasterisation, and fused epilogues.
//
// It replaces rtensor's scalar GEMMs (crates/rtensor/src/gpu/gemm.rs MM_FAST
// mm / mm_atb / mm_abt and MM_EPILOGO mm_bias, splitk.rs MM_SPLITK) and its
// packed-f16 mixed-precision GEMM (mista.rs:58-323) with bf16 operands and f32
// accumulation:
//   RT_NN  Y  = X W        A K-major,  B MN-major
//   RT_NT  dX = dY W^T     A K-major,  B K-major
//   RT_TN  dW = X^T dY     A MN-major, B MN-major  (split-K for small tile counts)
//
// CTA = 256 threads, one CTA per SM (about 192 KB of shared memory):
//   warp 0      TMA producer (one lane)
//   warp 1      MMA issuer (one lane): tcgen05.mma cta_group::1, M = 128
//   warp 2      TMEM allocator
//   warps 4..7  epilogue: tcgen05.ld -> bias / ReLU / ReLU-mask -> global
// Two TMEM accumulators (2 x BN f32 columns) let the epilogue of one tile
// overlap the main loop of the next.
//
// Every mbarrier wait is bounded: if a wait exceeds kWaitLimitNs the role
// records an error in the context's device error word, raises a shared abort
// flag and leaves its loop; in-flight TMA loads and MMAs are drained (with
// bounded waits) and TMEM is freed before the CTA returns.  The host reports
// RT_ERR_DEVICE_TIMEOUT at the next rt_ctx_sync.  No trap, no unbounded spin.
//
// No TMA load here uses the cluster-wide broadcast form: every CTA loads its
// own operand tiles, so the kernel is safe to run on every GPU of a
// data-parallel job.
#include <cuda.h>

#include <mutex>

#include "internal.h"

namespace rt {
namespace {

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
};

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
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
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

// Epilogue for 32 consecutive columns of one row.
template <typename TOut>
__device__ __forceinline__ void epilogue_chunk(const TcParams& p, int64_t row, int64_t col0, float (&v)[32]) {
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
    if constexpr (sizeof(TOut) == 2) {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.c) + row * p.ldc + col0;
        if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 u;
                __nv_bfloat162 h0 = __floats2bfloat162_rn(v[q * 8 + 0], v[q * 8 + 1]);
                __nv_bfloat162 h1 = __floats2bfloat162_rn(v[q * 8 + 2], v[q * 8 + 3]);
                __nv_bfloat162 h2 = __floats2bfloat162_rn(v[q * 8 + 4], v[q * 8 + 5]);
                __nv_bfloat162 h3 = __floats2bfloat162_rn(v[q * 8 + 6], v[q * 8 + 7]);
                u.x = *reinterpret_cast<uint32_t*>(&h0);
                u.y = *reinterpret_cast<uint32_t*>(&h1);
                u.z = *reinterpret_cast<uint32_t*>(&h2);
                u.w = *reinterpret_cast<uint32_t*>(&h3);
                reinterpret_cast<uint4*>(dst)[q] = u;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < n) dst[j] = __float2bfloat16_rn(v[j]);
        }
    } else {
        float* dst = static_cast<float*>(p.c) + row * p.ldc + col0;
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

template <typename TIn, bool A_MN, bool B_MN, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   TcParams p) {
    using G = Geo<TIn, BN>;
    constexpr bool kTF32 = sizeof(TIn) == 4;
    constexpr int STAGES = G::STAGES;
    constexpr uint32_t IDESC = make_idesc(kTF32, A_MN, B_MN, BN, BM);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + STAGES * G::A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * G::STAGE_BYTES);
    // bars: full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2], drain
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = bars + 2 * STAGES + 2;
    uint64_t* drain = bars + 2 * STAGES + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint32_t* last_phase = tmem_slot + 2;  // [STAGES]: 0 = never issued, else parity + 1

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
            last_phase[s] = 0;
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&tfull[s]), 1);
            mbar_init(smem_u32(&tempty[s]), 4);
        }
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(G::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int total_tiles = p.tiles_m * p.tiles_n * p.splits;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
            int split, mb, nb;
            tile_coords(p, t, split, mb, nb);
            int kb0 = split * p.kb_per_split;
            int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            const int m0 = mb * BM, n0 = nb * BN;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                const uint32_t fb = smem_u32(&full[stage]);
                mbar_expect_tx(fb, G::STAGE_BYTES);
                last_phase[stage] = phase + 1;
                const int k0 = kb * G::BK;
                const uint32_t sa = smem_u32(smem_a + stage * G::A_BYTES);
                const uint32_t sb = smem_u32(smem_b + stage * G::B_BYTES);
                if (A_MN) {
#pragma unroll
                    for (int c = 0; c < BM / G::CHUNK; ++c)
                        tma_load_2d(sa + c * (G::BK * 128), &tmap_a, m0 + c * G::CHUNK, k0, fb);
                } else {
                    tma_load_2d(sa, &tmap_a, k0, m0, fb);
                }
                if (B_MN) {
#pragma unroll
                    for (int c = 0; c < BN / G::CHUNK; ++c)
                        tma_load_2d(sb + c * (G::BK * 128), &tmap_b, n0 + c * G::CHUNK, k0, fb);
                } else {
                    tma_load_2d(sb, &tmap_b, k0, n0, fb);
                }
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        if (!ok) {
            record_error(p.err, DEV_TIMEOUT_PRODUCER, blockIdx.x);
            *abort_flag = 1;
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------ MMA issuer
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        // Byte offsets inside a stage buffer between consecutive MMAs along k.
        constexpr uint32_t A_KSTEP = A_MN ? G::UK * 128 : 32;
        constexpr uint32_t B_KSTEP = B_MN ? G::UK * 128 : 32;
        constexpr uint32_t A_LBO = A_MN ? G::BK * 128 : 16;
        constexpr uint32_t B_LBO = B_MN ? G::BK * 128 : 16;
        for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
            int split, mb, nb;
            tile_coords(p, t, split, mb, nb);
            int kb0 = split * p.kb_per_split;
            int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem_a + stage * G::A_BYTES);
                const uint32_t sb = smem_u32(smem_b + stage * G::B_BYTES);
#pragma unroll
                for (int kk = 0; kk < G::BK / G::UK; ++kk) {
                    uint64_t ad = smem_desc(sa + kk * A_KSTEP, A_LBO, 1024);
                    uint64_t bd = smem_desc(sb + kk * B_KSTEP, B_LBO, 1024);
                    tc_mma<kTF32>(d_tmem, ad, bd, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(smem_u32(&empty[stage]));
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
            tc_commit(smem_u32(&tfull[acc]));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (!ok) {
            record_error(p.err, DEV_TIMEOUT_MMA, blockIdx.x);
            *abort_flag = 1;
        }
        // Drain: wait until every MMA this thread issued has completed.
        tc_commit(smem_u32(drain));
        mbar_wait(smem_u32(drain), 0, abort_flag);
    } else if (warp >= 4) {
        // ------------------------------------------------ epilogue
        const int ew = warp - 4;  // TMEM lanes [32 ew, 32 ew + 32)
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
            int split, mb, nb;
            tile_coords(p, t, split, mb, nb);
            bool got = mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int64_t row = (int64_t)mb * BM + ew * 32 + lane;
            const uint32_t tbase = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                const int64_t col0 = (int64_t)nb * BN + c;
                if (col0 >= p.n) break;  // uniform across the warp
                float v[32];
                tmem_ld_32x32(tbase + (uint32_t)c, v);
                if (row < p.m) {
                    if (p.ws) {
                        float* dst = p.ws + (int64_t)split * p.m * p.n + row * p.n + col0;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < p.n) dst[j] = v[j];
                    } else {
                        if (p.opt.kind) {
                            // optimiser step on theta[row, col0 .. col0+31] with this gradient chunk
                            int64_t rem = p.n - col0;
                            int cnt = rem < 32 ? (int)rem : 32;
                            opt_apply_row<32>(p.opt, row * p.ldc + col0, v, cnt);
                        }
                        if (p.out_bf16)
                            epilogue_chunk<__nv_bfloat16>(p, row, col0, v);
                        else
                            epilogue_chunk<float>(p, row, col0, v);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (!ok && lane == 0) {
            record_error(p.err, DEV_TIMEOUT_EPILOGUE, blockIdx.x);
            *abort_flag = 1;
        }
    }

    __syncwarp();  // reconverge the role warps before the block-wide barrier
    __syncthreads();
    if (*abort_flag && threadIdx.x == 0) {
        // Let TMA loads still in flight land before the CTA's shared memory is released.
        for (int s = 0; s < STAGES; ++s)
            if (last_phase[s]) {
                volatile int never = 0;
                mbar_wait(smem_u32(&full[s]), last_phase[s] - 1, &never);
            }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(G::TMEM_COLS)
                     : "memory");
    }
}

// ------------------------------------------------------------------ host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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
int make_tmap(CUtensorMap* map, const void* base, bool bf16, int64_t inner, int64_t outer, int64_t ld,
              int box_inner, int box_outer) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(RT_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
    const int es = bf16 ? 2 : 4;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(RT_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): inner %lld outer %lld ld %lld box %dx%d",
                    (int)r, (long long)inner, (long long)outer, (long long)ld, box_inner, box_outer);
    return RT_OK;
}

template <typename TIn, bool A_MN, bool B_MN, int BN>
int launch_variant(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    using G = Geo<TIn, BN>;
    const bool bf16 = sizeof(TIn) == 2;
    CUtensorMap ta, tb;
    // A: logical [m,k].  K-major storage [m][lda]; MN-major storage [k][lda].
    if (A_MN)
        RT_TRY(make_tmap(&ta, g.a, bf16, g.m, g.k, g.lda, G::CHUNK, G::BK));
    else
        RT_TRY(make_tmap(&ta, g.a, bf16, g.k, g.m, g.lda, G::BK, BM));
    // B: logical [k,n].  K-major storage [n][ldb]; MN-major storage [k][ldb].
    if (B_MN)
        RT_TRY(make_tmap(&tb, g.b, bf16, g.n, g.k, g.ldb, G::CHUNK, G::BK));
    else
        RT_TRY(make_tmap(&tb, g.b, bf16, g.k, g.n, g.ldb, G::BK, BN));

    TcParams p{};
    GemmDesc gr = g;  // descriptor for the split-K reduction (effective split count)
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.tiles_m = (int)((g.m + BM - 1) / BM);
    p.tiles_n = (int)((g.n + BN - 1) / BN);
    p.kblocks = (int)((g.k + G::BK - 1) / G::BK);
    int splits = g.split_k > 1 ? g.split_k : 1;
    if (splits > p.kblocks) splits = p.kblocks;
    p.kb_per_split = (p.kblocks + splits - 1) / splits;
    splits = (p.kblocks + p.kb_per_split - 1) / p.kb_per_split;  // no empty slice
    p.splits = splits;
    gr.split_k = splits;
    p.group = ctx->l2_group;
    p.c = g.c;
    p.ldc = g.ldc;
    p.ws = splits > 1 ? g.workspace : nullptr;
    p.bias = g.bias;
    p.mask = g.mask;
    p.ldmask = g.ldmask;
    p.epi = g.epi;
    p.out_bf16 = g.out_dtype == RT_BF16;
    p.err = ctx->dev_err;
    p.opt = g.opt;

    int64_t tiles = (int64_t)p.tiles_m * p.tiles_n * p.splits;
    int grid = (int)(tiles < ctx->sm_count ? tiles : ctx->sm_count);
    gemm_tc_kernel<TIn, A_MN, B_MN, BN><<<grid, kThreads, G::SMEM, st>>>(ta, tb, p);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    if (splits > 1) return launch_splitk_reduce(ctx, gr, st);
    return RT_OK;
}

template <typename TIn, bool A_MN, bool B_MN, int BN>
int set_smem_attr() {
    RT_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<TIn, A_MN, B_MN, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Geo<TIn, BN>::SMEM));
    return RT_OK;
}

template <typename TIn, int BN>
int set_smem_attrs_bn() {
    RT_TRY((set_smem_attr<TIn, false, true, BN>()));
    RT_TRY((set_smem_attr<TIn, false, false, BN>()));
    RT_TRY((set_smem_attr<TIn, true, true, BN>()));
    return RT_OK;
}

template <typename TIn, int BN>
int launch_layout(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    switch (g.layout) {
        case RT_NN: return launch_variant<TIn, false, true, BN>(ctx, g, st);
        case RT_NT: return launch_variant<TIn, false, false, BN>(ctx, g, st);
        case RT_TN: return launch_variant<TIn, true, true, BN>(ctx, g, st);
    }
    return fail(RT_ERR_INVALID, "unknown layout");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// Raises the dynamic shared-memory limit of every kernel instantiation once
// per device, outside any stream capture.
int gemm_tc_init(rt_ctx* ctx) {
    (void)ctx;
    RT_TRY((set_smem_attrs_bn<__nv_bfloat16, 64>()));
    RT_TRY((set_smem_attrs_bn<__nv_bfloat16, 128>()));
    RT_TRY((set_smem_attrs_bn<__nv_bfloat16, 256>()));
    return RT_OK;
}

bool gemm_tc_supported(const rt_ctx* ctx, const GemmDesc& g) {
    if (ctx->cc_major != 10) return false;
    if (g.in_dtype != RT_BF16) return false;  // f32 operands keep the exact SIMT path
    if (g.m < 1 || g.n < 1 || g.k < 1) return false;
    if (g.m >= (1ll << 31) || g.n >= (1ll << 31) || g.k >= (1ll << 31)) return false;
    const int64_t es = 2, os = g.out_dtype == RT_BF16 ? 2 : 4;
    if (!aligned16(g.a) || !aligned16(g.b) || !aligned16(g.c)) return false;
    if ((g.lda * es) % 16 || (g.ldb * es) % 16 || (g.ldc * os) % 16) return false;
    if (g.epi == RT_EPI_RELU_MASK && (!aligned16(g.mask) || (g.ldmask * os) % 16)) return false;
    return true;
}

int launch_gemm_tc(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    if (!gemm_tc_supported(ctx, g)) return fail(RT_ERR_UNSUPPORTED, "operands not eligible for the tensor-core GEMM");
    if (g.n <= 64) return launch_layout<__nv_bfloat16, 64>(ctx, g, st);
    if (g.n <= 128) return launch_layout<__nv_bfloat16, 128>(ctx, g, st);
    return launch_layout<__nv_bfloat16, 256>(ctx, g, st);
}

}  // namespace rt
