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
#include "tc_common.cuh"

namespace rt {
namespace {
using namespace tc;
// X3 (f32 only, both operands K-major): the operands are [2][mn][k] hi/lo
// planes read through 3-D maps, and the k loop runs three product segments
// over the same k range: lo(A) hi(B), hi(A) lo(B), then hi(A) hi(B) (the
// small terms first).
// Split bf16 A (p.split_a): twice the k blocks, alternating A's low-order
// plane (tmap_a2) and A at each k block, both against the same B tile.
// A bf16 output with a low-order plane (p.c_lo) is stored through tmap_c and
// tmap_c2.
template <typename TIn, bool A_MN, bool B_MN, int BN, bool X3 = false, bool SPLIT_C = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_c, const __grid_constant__ CUtensorMap tmap_a2,
                   const __grid_constant__ CUtensorMap tmap_c2, TcParams p) {
    static_assert(!X3 || (sizeof(TIn) == 4 && !A_MN && !B_MN), "3xTF32 planes are f32 and K-major");
    using G = Geo<TIn, BN>;
    constexpr bool kTF32 = sizeof(TIn) == 4;
    constexpr int STAGES = G::STAGES;
    constexpr uint32_t IDESC = make_idesc(kTF32, A_MN, B_MN, BN, BM);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_a = smem;
    uint8_t* smem_b = smem + STAGES * G::A_BYTES;
    uint8_t* smem_epi = smem + STAGES * G::STAGE_BYTES;  // [4 epilogue warps][32 x 32] output staging
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + G::EPI_BYTES);
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
        if (p.tma_store) prefetch_tmap(&tmap_c);
        if (p.split_a) prefetch_tmap(&tmap_a2);
        if (SPLIT_C && p.tma_store) prefetch_tmap(&tmap_c2);
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
                int k0 = kb * G::BK;
                int plane_a = 0, plane_b = 0;
                const CUtensorMap* map_a = &tmap_a;
                if constexpr (X3) {
                    const int seg = kb / p.kb_seg;
                    k0 = (kb - seg * p.kb_seg) * G::BK;
                    plane_a = seg == 0;
                    plane_b = seg == 1;
                } else {
                    if (p.split_a) {
                        // k blocks alternate: A's low-order plane at k block kb / 2, then A at
                        // the same k block, so the second load of each B tile hits L2
                        k0 = (kb >> 1) * G::BK;
                        if ((kb & 1) == 0) map_a = &tmap_a2;
                    }
                }
                const uint32_t sa = smem_u32(smem_a + stage * G::A_BYTES);
                const uint32_t sb = smem_u32(smem_b + stage * G::B_BYTES);
                if constexpr (X3) {
                    tma_load_3d(sa, &tmap_a, k0, m0, plane_a, fb);
                    tma_load_3d(sb, &tmap_b, k0, n0, plane_b, fb);
                } else {
                    if (A_MN) {
#pragma unroll
                        for (int c = 0; c < BM / G::CHUNK; ++c)
                            tma_load_2d(sa + c * (G::BK * 128), map_a, m0 + c * G::CHUNK, k0, fb);
                    } else {
                        tma_load_2d(sa, map_a, k0, m0, fb);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int c = 0; c < BN / G::CHUNK; ++c)
                            tma_load_2d(sb + c * (G::BK * 128), &tmap_b, n0 + c * G::CHUNK, k0, fb);
                    } else {
                        tma_load_2d(sb, &tmap_b, k0, n0, fb);
                    }
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
            const int64_t row0 = (int64_t)mb * BM + ew * 32;
            const int64_t row = row0 + lane;
            const uint32_t tbase = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                const int64_t col0 = (int64_t)nb * BN + c;
                if (col0 >= p.n) break;  // uniform across the warp
                float v[32];
                tmem_ld_32x32(tbase + (uint32_t)c, v);
                if (p.tma_store == 2) {
                    // staged split-K partials: slice `split` of the [splits][m][n] workspace
                    stage_and_store<float>(&tmap_c, smem_epi + ew * kStageBytes, lane, row0, col0, v, split);
                } else if (p.tma_store == 1) {
                    // staged: coalesced TMA stores of the warp's 32 x 32 chunk
                    uint8_t* box = smem_epi + ew * kStageBytes;
                    if (p.out_bf16) {
                        if (row < p.m) epilogue_math<__nv_bfloat16>(p, row, col0, v);
                        if constexpr (SPLIT_C)
                            stage_and_store_split(&tmap_c, &tmap_c2, box, lane, row0, col0, v);
                        else
                            stage_and_store<__nv_bfloat16>(&tmap_c, box, lane, row0, col0, v);
                    } else {
                        if (row < p.m) epilogue_math<float>(p, row, col0, v);
                        stage_and_store<float>(&tmap_c, box, lane, row0, col0, v);
                    }
                } else if (p.tma_store == 4) {
                    // rows scattered to their owners' receive buffers (peer memory)
                    p2p_chunk(p, reinterpret_cast<float*>(smem_epi + ew * kStageBytes), lane, row0, col0, v);
                } else if (p.tma_store == 3) {
                    // fused optimiser: the chunk updates theta / m / v / shadow and is stored as C
                    opt_chunk(p, reinterpret_cast<float*>(smem_epi + ew * kStageBytes), lane, row0, col0, v);
                } else if (row < p.m) {
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
                            epilogue_chunk<__nv_bfloat16, SPLIT_C>(p, row, col0, v);
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
        if ((p.tma_store == 1 || p.tma_store == 2) && lane == 0) bulk_wait_all();  // this warp's output stores are complete
        if (p.tma_store == 4) __threadfence_system();  // peer-memory stores in place before the kernel ends
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

template <typename TIn, bool A_MN, bool B_MN, int BN, bool X3, bool SPLIT_C = false>
int launch_variant(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st, const X3Planes* x3) {
    using G = Geo<TIn, BN>;
    const bool bf16 = sizeof(TIn) == 2;
    CUtensorMap ta, tb, tc, ta2, tc2;
    if constexpr (X3) {
        // hi/lo planes of the operands, both K-major: A [2][m][k], B [2][n][k]
        RT_TRY(make_tmap_planes(&ta, x3->a, g.k, g.m, x3->lda, x3->a_plane, 2, G::BK, BM));
        RT_TRY(make_tmap_planes(&tb, x3->b, g.k, g.n, x3->ldb, x3->b_plane, 2, G::BK, BN));
        ta2 = ta;
    } else {
        // A: logical [m,k].  K-major storage [m][lda]; MN-major storage [k][lda].
        if (A_MN)
            RT_TRY(make_tmap(&ta, g.a, bf16, g.m, g.k, g.lda, G::CHUNK, G::BK));
        else
            RT_TRY(make_tmap(&ta, g.a, bf16, g.k, g.m, g.lda, G::BK, BM));
        ta2 = ta;
        if (g.a_lo) {  // A's low-order plane: the same geometry
            if (A_MN)
                RT_TRY(make_tmap(&ta2, g.a_lo, bf16, g.m, g.k, g.lda, G::CHUNK, G::BK));
            else
                RT_TRY(make_tmap(&ta2, g.a_lo, bf16, g.k, g.m, g.lda, G::BK, BM));
        }
        // B: logical [k,n].  K-major storage [n][ldb]; MN-major storage [k][ldb].
        if (B_MN)
            RT_TRY(make_tmap(&tb, g.b, bf16, g.n, g.k, g.ldb, G::CHUNK, G::BK));
        else
            RT_TRY(make_tmap(&tb, g.b, bf16, g.k, g.n, g.ldb, G::BK, BN));
    }

    TcParams p{};
    GemmDesc gr = g;  // descriptor for the split-K reduction (effective split count)
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.tiles_m = (int)((g.m + BM - 1) / BM);
    p.tiles_n = (int)((g.n + BN - 1) / BN);
    p.kblocks = (int)((g.k + G::BK - 1) / G::BK);
    p.kb_seg = 0;
    if constexpr (X3) {
        p.kb_seg = p.kblocks;
        p.kblocks *= 3;
    } else {
        if (g.a_lo) {
            p.split_a = 1;
            p.kblocks *= 2;  // each k block twice: A's low-order plane, then A
        }
    }
    p.c_lo = g.c_lo;
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
    p.tma_store = 0;
    p.p2p = g.p2p;
    tc = ta;  // unused unless a staged store is chosen
    tc2 = ta;
    if (g.p2p.world > 0) {
        // scattered over peer memory: one k slice, f32 gradient, no fused update
        if (splits != 1 || p.out_bf16 || g.opt.kind)
            return fail(RT_ERR_UNSUPPORTED, "peer-scatter GEMM needs one k slice, f32 output and no fused update");
        p.tma_store = 4;
    } else if (ctx->tma_store && splits == 1 && !g.opt.kind) {
        p.tma_store = 1;
        RT_TRY(make_tmap_out(&tc, g.c, p.out_bf16 != 0, g.m, g.n, g.ldc));
        if (g.c_lo) RT_TRY(make_tmap_out(&tc2, g.c_lo, true, g.m, g.n, g.ldc));
    } else if (ctx->tma_store && splits == 1 && !p.out_bf16) {
        p.tma_store = 3;  // fused optimiser through the epilogue boxes
    } else if (ctx->tma_store && splits > 1 && g.n % 4 == 0 && (reinterpret_cast<uintptr_t>(g.workspace) & 15) == 0) {
        p.tma_store = 2;
        RT_TRY(make_tmap_ws(&tc, g.workspace, g.m, g.n, splits));
    }

    int64_t tiles = (int64_t)p.tiles_m * p.tiles_n * p.splits;
    int sms = g.max_sms > 0 && g.max_sms < ctx->sm_count ? g.max_sms : ctx->sm_count;
    int grid = (int)(tiles < sms ? tiles : sms);
    gemm_tc_kernel<TIn, A_MN, B_MN, BN, X3, SPLIT_C><<<grid, kThreads, G::SMEM, st>>>(ta, tb, tc, ta2, tc2, p);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    if (splits > 1) return launch_splitk_reduce(ctx, gr, st);
    return RT_OK;
}

template <typename TIn, bool A_MN, bool B_MN, int BN, bool X3, bool SPLIT_C = false>
int set_smem_attr() {
    RT_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<TIn, A_MN, B_MN, BN, X3, SPLIT_C>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Geo<TIn, BN>::SMEM));
    return RT_OK;
}

template <typename TIn, int BN, bool X3 = false>
int set_smem_attrs_bn() {
    RT_TRY((set_smem_attr<TIn, false, true, BN, X3>()));
    RT_TRY((set_smem_attr<TIn, false, false, BN, X3>()));
    RT_TRY((set_smem_attr<TIn, true, true, BN, X3>()));
    if constexpr (!X3) RT_TRY((set_smem_attr<TIn, false, true, BN, X3, true>()));  // forward with c_lo
    return RT_OK;
}

// The forward (NN) layout with a low-order output plane has its own
// instantiation (SPLIT_C), so the other kernels carry none of its epilogue.
template <typename TIn, int BN, bool X3 = false>
int launch_layout(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st, const X3Planes* x3 = nullptr) {
    if constexpr (!X3) {
        if (g.c_lo) {
            if (g.layout != RT_NN) return fail(RT_ERR_UNSUPPORTED, "c_lo is supported for the NN layout only");
            return launch_variant<TIn, false, true, BN, X3, true>(ctx, g, st, x3);
        }
    }
    switch (g.layout) {
        case RT_NN: return launch_variant<TIn, false, true, BN, X3>(ctx, g, st, x3);
        case RT_NT: return launch_variant<TIn, false, false, BN, X3>(ctx, g, st, x3);
        case RT_TN: return launch_variant<TIn, true, true, BN, X3>(ctx, g, st, x3);
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
    if ((g.a_lo && !aligned16(g.a_lo)) || (g.c_lo && !aligned16(g.c_lo))) return false;
    if ((g.lda * es) % 16 || (g.ldb * es) % 16 || (g.ldc * os) % 16) return false;
    if (g.epi == RT_EPI_RELU_MASK && (!aligned16(g.mask) || (g.ldmask * os) % 16)) return false;
    return true;
}

// f32 GEMM from split operand planes (gemm_x3.cu prepares them).
// Both planes are K-major whatever g.layout is (tcgen05 takes MN-major tf32
// operands only in the 32-byte-atom swizzle, so the split transposes instead).
int gemm_tc_x3_init() {
    RT_TRY((set_smem_attr<float, false, false, 64, true>()));
    RT_TRY((set_smem_attr<float, false, false, 128, true>()));
    RT_TRY((set_smem_attr<float, false, false, 256, true>()));
    return RT_OK;
}

// Few output tiles: when even 128 x 128 tiles leave more than half of the SMs
// without one, the GEMM is bound by how fast its busy SMs stream operands and
// write C, so 128 x 64 one-CTA tiles (twice the CTAs) go first.
static bool few_tiles(const rt_ctx* ctx, const GemmDesc& g) {
    const int64_t splits = g.split_k > 1 ? g.split_k : 1;
    return ((g.m + 127) / 128) * ((g.n + 127) / 128) * splits * 2 < ctx->sm_count && g.n > 64;
}

int launch_gemm_tc_x3(rt_ctx* ctx, const GemmDesc& g, const X3Planes& x3, cudaStream_t st) {
    if (few_tiles(ctx, g)) return launch_variant<float, false, false, 64, true>(ctx, g, st, &x3);
    if (gemm_tc2_x3_wanted(ctx, g)) return launch_gemm_tc2_x3(ctx, g, x3, st);
    if (g.n <= 64) return launch_variant<float, false, false, 64, true>(ctx, g, st, &x3);
    if (g.n <= 128) return launch_variant<float, false, false, 128, true>(ctx, g, st, &x3);
    return launch_variant<float, false, false, 256, true>(ctx, g, st, &x3);
}

int launch_gemm_tc(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    if (!gemm_tc_supported(ctx, g)) return fail(RT_ERR_UNSUPPORTED, "operands not eligible for the tensor-core GEMM");
    if (few_tiles(ctx, g)) return launch_layout<__nv_bfloat16, 64>(ctx, g, st);
    if (gemm_tc2_wanted(ctx, g)) return launch_gemm_tc2(ctx, g, st);
    if (g.n <= 64) return launch_layout<__nv_bfloat16, 64>(ctx, g, st);
    if (g.n <= 128) return launch_layout<__nv_bfloat16, 128>(ctx, g, st);
    return launch_layout<__nv_bfloat16, 256>(ctx, g, st);
}

}  // namespace rt
