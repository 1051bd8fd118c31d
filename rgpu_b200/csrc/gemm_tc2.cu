// Two-CTA tensor-core GEMM (tcgen05 cta_group::2): a cluster of two CTAs on a
// pair of SMs computes a 256 x BN tile with one MMA stream.
//
// Same operands, layouts, epilogues and bounded-wait rules as the one-CTA
// kernel in gemm_tc.cu; what changes is how a tile's operands are split:
//   - CTA rank r of the pair loads A rows [128 r, 128 r + 128) of the tile and
//     B columns [BN/2 r, BN/2 (r + 1)), each into its own shared memory at the
//     same offsets; per 64-deep k block that is 32 KB per CTA instead of the
//     48 KB a one-CTA 128 x 256 tile needs, which leaves room for 6 stages;
//   - the leader (rank 0) issues tcgen05.mma.cta_group::2 (M = 256); the
//     tensor cores read both CTAs' halves and each CTA's TMEM receives its own
//     128 accumulator rows;
//   - both CTAs' TMA loads complete on the leader's full barrier (the
//     .cta_group::2 form of the load names the leader's barrier), and only the
//     leader posts the expected byte count of the pair;
//   - the leader's MMA thread releases stages and publishes finished
//     accumulators with one tcgen05.commit per CTA (its own barrier and the
//     peer's, addressed through mapa); the peer's epilogue warps arrive
//     remotely on the leader's TMEM-empty barrier.
// Every CTA loads its own tiles: no load is shared between CTAs.
//
// X3 form (f32 operands, both K-major hi/lo planes from gemm_x3.cu): tf32
// MMAs over three k segments, as in the one-CTA kernel; per 32-deep k block a
// CTA loads 16 KB of A and 16 KB of B for 2 x 128 x 256 x 32 MMA work, half
// the L2-to-SM bytes per FLOP of the one-CTA 128 x 256 tile.
#include "tc_common.cuh"

namespace rt {
namespace {
using namespace tc;

constexpr int BM2 = 256;  // rows per CTA pair
// 12 warps: 0 TMA producer, 1 MMA issuer (leader), 2 TMEM allocator, 3 idle,
// 4..11 epilogue (two warps per TMEM lane quadrant, each taking half of the
// tile's columns, so short-k tiles do not wait on the epilogue).
constexpr int kThreads2 = 384;
constexpr int kEpiWarps = 8;

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// Orders this thread's accesses at cluster scope (here: a ring slot's tile
// id, written by the pair leader, read after the slot's barrier completed).
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }

// Dynamic tile schedule (TcParams::tile_ctr set): the pair leader's producer
// claims each next tile with an atomic add and publishes its id in a ring of
// kRing slots held by both CTAs; the producer of the other CTA, the MMA issuer
// and the epilogue warps of both CTAs read the ids in order and release each
// slot on the leader's barrier.  A pair that starts late (its SMs still busy
// with other kernels) then simply takes fewer tiles.
constexpr int kRing = 12;
constexpr int kRingConsumers = 2 * kEpiWarps + 2;  // epilogue warps of both CTAs, MMA issuer, peer producer

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA load whose completion is counted on the pair leader's barrier.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                                 uint32_t leader_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(leader_bar)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                                                 int32_t z, uint32_t leader_bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(leader_bar)
        : "memory");
}

__device__ __forceinline__ void tc_commit_pair(uint32_t cluster_bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
                 : "memory");
}

template <bool kTF32>
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    if constexpr (kTF32) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

template <typename TIn, int BN, bool SPLIT_A = false>
struct Geo2 {
    static constexpr int ES = sizeof(TIn);
    static constexpr int BK = 128 / ES;
    static constexpr int CHUNK = 128 / ES;
    static constexpr int UK = 32 / ES;
    static constexpr int BNH = BN / 2;  // B rows (n) held by each CTA
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = BNH * 128;
    static constexpr int A_PLANES = SPLIT_A ? 2 : 1;  // SPLIT_A: A and its low-order plane share a stage
    static constexpr int STAGE_BYTES = A_PLANES * A_BYTES + B_BYTES;
    static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int EPI_BYTES = kEpiWarps * kStageBytes;
    static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 512 /*barriers, tile ring*/;
    static_assert(STAGES >= 3, "the operand ring needs at least three stages to overlap loads and MMAs");
    static_assert(SMEM <= 227 * 1024, "dynamic shared memory above the per-CTA limit");
};

// Split bf16 A (A + a_lo, through tmap_a2) and a bf16 output's low-order
// plane (p.c_lo, through tmap_c2).  SPLIT_A (the NN forward GEMM of a layer
// fed by split activations): each stage holds A's low-order plane, A and the
// B tile, and the MMAs run the lo products, then A's, on that one B tile, so
// B crosses L2 -> SMEM once per k block (4 stages of 48 KB instead of 6 of
// 32 KB).  Other layouts given a_lo keep the interleaved form (p.split_a: the
// k loop alternates a lo and a hi k block, loading B twice).
template <typename TIn, bool A_MN, bool B_MN, int BN, bool X3 = false, bool SPLIT_C = false, bool SPLIT_A = false>
__global__ void __launch_bounds__(kThreads2, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_c, const __grid_constant__ CUtensorMap tmap_a2,
                    const __grid_constant__ CUtensorMap tmap_c2, TcParams p) {
    static_assert(!X3 || (sizeof(TIn) == 4 && !A_MN && !B_MN), "3xTF32 planes are f32 and K-major");
    static_assert(!SPLIT_A || (sizeof(TIn) == 2 && !A_MN && !X3), "split A planes are bf16 and K-major");
    using G = Geo2<TIn, BN, SPLIT_A>;
    constexpr bool kTF32 = sizeof(TIn) == 4;
    constexpr int STAGES = G::STAGES;
    constexpr uint32_t IDESC = make_idesc(kTF32, A_MN, B_MN, BN, BM2);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* smem_a = smem;
    uint8_t* smem_alo = smem + STAGES * G::A_BYTES;  // SPLIT_A: A's low-order plane of each stage
    uint8_t* smem_b = smem + STAGES * G::A_PLANES * G::A_BYTES;
    uint8_t* smem_epi = smem + STAGES * G::STAGE_BYTES;  // [8 epilogue warps][32 x 32] output staging
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + G::EPI_BYTES);
    uint64_t* full = bars;                     // leader: both CTAs' bytes of a stage
    uint64_t* empty = bars + STAGES;           // each CTA: stage released by the MMAs
    uint64_t* tfull = bars + 2 * STAGES;       // each CTA: accumulator ready
    uint64_t* tempty = bars + 2 * STAGES + 2;  // leader: accumulator drained by both epilogues
    uint64_t* drain = bars + 2 * STAGES + 4;
    uint64_t* rfull = bars + 2 * STAGES + 5;            // each CTA: ring slot holds the next tile id
    uint64_t* rempty = bars + 2 * STAGES + 5 + kRing;   // leader: ring slot read by every consumer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5 + 2 * kRing);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint32_t* last_phase = tmem_slot + 2;
    int* ring_tile = reinterpret_cast<int*>(last_phase + STAGES);
    static_assert((2 * STAGES + 5 + 2 * kRing) * 8 + (2 + STAGES + kRing) * 4 <= 512, "barrier area");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const int cluster_id = blockIdx.x >> 1;
    const int num_clusters = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
            last_phase[s] = 0;
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&tfull[s]), 1);
            mbar_init(smem_u32(&tempty[s]), 2 * kEpiWarps);  // epilogue warps of both CTAs
        }
        mbar_init(smem_u32(drain), 1);
        for (int r = 0; r < kRing; ++r) {
            mbar_init(smem_u32(&rfull[r]), 1);
            mbar_init(smem_u32(&rempty[r]), kRingConsumers);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_b);
        if (p.tma_store) prefetch_tmap(&tmap_c);
        if (SPLIT_A || p.split_a) prefetch_tmap(&tmap_a2);
        if (SPLIT_C && p.tma_store) prefetch_tmap(&tmap_c2);
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(G::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // barrier initialisation and the TMEM address are now visible to the pair
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t peer_abort = mapa_shared(smem_u32((const void*)abort_flag), peer);
    auto raise_abort = [&]() {
        *abort_flag = 1;
        st_cluster_u32(peer_abort, 1u);
    };

    const int total_tiles = p.tiles_m * p.tiles_n * p.splits;
    const bool dyn = p.tile_ctr != nullptr;

    // A consumer's next tile id from its CTA's ring (-1: no tiles left).  All
    // lanes of a calling warp wait; one arrival per consumer releases the
    // slot on the leader's barrier.  False if the wait gave up.
    auto ring_next = [&](uint32_t& slot, uint32_t& ph, bool arrive, int& t) -> bool {
        if (!mbar_wait(smem_u32(&rfull[slot]), ph, abort_flag)) return false;
        fence_acq_rel_cluster();
        t = reinterpret_cast<volatile int*>(ring_tile)[slot];
        __syncwarp(__activemask());
        if (arrive) mbar_arrive_cluster(mapa_shared(smem_u32(&rempty[slot]), 0));
        if (++slot == kRing) {
            slot = 0;
            ph ^= 1;
        }
        return true;
    };

    // Programmatic dependent launch (PDL_* in internal.h).  The set-up above
    // touched no global memory.  Dependents may launch once this CTA is past
    // its own wait: right away unless the epilogue waits, then from the
    // epilogue warps after their wait (and from every other thread at its end).
    if (p.pdl == PDL_WAIT_START) pdl_wait();
    if (p.pdl != PDL_WAIT_EPILOGUE) pdl_launch_dependents();

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer (both CTAs)
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        uint32_t rs = 0, rph = 0;
        // the leader claims one tile ahead, so the atomic's latency overlaps the current tile's loads
        int claimed = dyn && rank == 0 ? atomicAdd(p.tile_ctr, 1) : 0;
        for (int ts = cluster_id; ok; ts += num_clusters) {
            int t = ts;
            if (dyn && rank == 0) {
                // publish the claimed tile's id to both CTAs' rings, then claim the next
                if (!mbar_wait(smem_u32(&rempty[rs]), rph ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                t = claimed < total_tiles ? claimed : -1;
                if (t >= 0) claimed = atomicAdd(p.tile_ctr, 1);
                ring_tile[rs] = t;
                st_cluster_u32(mapa_shared(smem_u32(&ring_tile[rs]), 1), (uint32_t)t);
                mbar_arrive_cluster(mapa_shared(smem_u32(&rfull[rs]), 0));
                mbar_arrive_cluster(mapa_shared(smem_u32(&rfull[rs]), 1));
                if (++rs == kRing) {
                    rs = 0;
                    rph ^= 1;
                }
            } else if (dyn) {
                if (!ring_next(rs, rph, true, t)) {
                    ok = false;
                    break;
                }
            }
            if (t < 0 || t >= total_tiles) break;
            int split, mb, nb;
            tile_coords(p, t, split, mb, nb);
            int kb0 = split * p.kb_per_split;
            int kb1 = min(p.kblocks, kb0 + p.kb_per_split);
            const int m0 = mb * BM2 + (int)rank * 128;
            const int n0 = nb * BN + (int)rank * G::BNH;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                const uint32_t leader_full = mapa_shared(smem_u32(&full[stage]), 0);
                if (rank == 0) mbar_expect_tx(smem_u32(&full[stage]), 2 * G::STAGE_BYTES);
                last_phase[stage] = phase + 1;
                const uint32_t sa = smem_u32(smem_a + stage * G::A_BYTES);
                const uint32_t sb = smem_u32(smem_b + stage * G::B_BYTES);
                if constexpr (X3) {
                    // segments: lo(A) hi(B), hi(A) lo(B), hi(A) hi(B)
                    const int seg = kb / p.kb_seg;
                    const int k0 = (kb - seg * p.kb_seg) * G::BK;
                    tma_load_3d_pair(sa, &tmap_a, k0, m0, seg == 0 ? 1 : 0, leader_full);
                    tma_load_3d_pair(sb, &tmap_b, k0, n0, seg == 1 ? 1 : 0, leader_full);
                } else {
                    int k0 = kb * G::BK;
                    const CUtensorMap* map_a = &tmap_a;
                    if constexpr (SPLIT_A) {
                        // A's low-order plane of this k block into the stage's second A slot
                        tma_load_2d_pair(smem_u32(smem_alo + stage * G::A_BYTES), &tmap_a2, k0, m0, leader_full);
                    } else if (p.split_a) {
                        // k blocks alternate: A's low-order plane at k block kb / 2, then A at
                        // the same k block, so the second load of each B tile hits L2
                        k0 = (kb >> 1) * G::BK;
                        if ((kb & 1) == 0) map_a = &tmap_a2;
                    }
                    if (A_MN) {
#pragma unroll
                        for (int c = 0; c < 128 / G::CHUNK; ++c)
                            tma_load_2d_pair(sa + c * (G::BK * 128), map_a, m0 + c * G::CHUNK, k0, leader_full);
                    } else {
                        tma_load_2d_pair(sa, map_a, k0, m0, leader_full);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int c = 0; c < G::BNH / G::CHUNK; ++c)
                            tma_load_2d_pair(sb + c * (G::BK * 128), &tmap_b, n0 + c * G::CHUNK, k0, leader_full);
                    } else {
                        tma_load_2d_pair(sb, &tmap_b, k0, n0, leader_full);
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
            raise_abort();
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ------------------------------------------------ MMA issuer (pair leader)
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        constexpr uint32_t A_KSTEP = A_MN ? G::UK * 128 : 32;
        constexpr uint32_t B_KSTEP = B_MN ? G::UK * 128 : 32;
        constexpr uint32_t A_LBO = A_MN ? G::BK * 128 : 16;
        constexpr uint32_t B_LBO = B_MN ? G::BK * 128 : 16;
        uint32_t rs = 0, rph = 0;
        for (int ts = cluster_id; ok; ts += num_clusters) {
            int t = ts;
            if (dyn && !ring_next(rs, rph, true, t)) {
                ok = false;
                break;
            }
            if (t < 0 || t >= total_tiles) break;
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
                if constexpr (SPLIT_A) {
                    // the low-order products first (small terms), then A's, on the same B
                    const uint32_t sl = smem_u32(smem_alo + stage * G::A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < G::BK / G::UK; ++kk) {
                        uint64_t ad = smem_desc(sl + kk * A_KSTEP, A_LBO, 1024);
                        uint64_t bd = smem_desc(sb + kk * B_KSTEP, B_LBO, 1024);
                        tc_mma_pair<kTF32>(d_tmem, ad, bd, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
                    }
                }
#pragma unroll
                for (int kk = 0; kk < G::BK / G::UK; ++kk) {
                    uint64_t ad = smem_desc(sa + kk * A_KSTEP, A_LBO, 1024);
                    uint64_t bd = smem_desc(sb + kk * B_KSTEP, B_LBO, 1024);
                    tc_mma_pair<kTF32>(d_tmem, ad, bd, IDESC, (SPLIT_A || kb > kb0 || kk > 0) ? 1u : 0u);
                }
                // release the stage in both CTAs once these MMAs have read it
                tc_commit_pair(smem_u32(&empty[stage]));
                tc_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
            tc_commit_pair(smem_u32(&tfull[acc]));
            tc_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (!ok) {
            record_error(p.err, DEV_TIMEOUT_MMA, blockIdx.x);
            raise_abort();
        }
        tc_commit_pair(smem_u32(drain));
        mbar_wait(smem_u32(drain), 0, abort_flag);
    } else if (warp >= 4) {
        // ------------------------------------------------ epilogue (both CTAs)
        if (p.pdl == PDL_WAIT_EPILOGUE) {
            pdl_wait();  // the kernel before this one has finished reading what the epilogue writes
            pdl_launch_dependents();
        }
        const int ew = (warp - 4) & 3;        // TMEM lane quadrant
        const int half = (warp - 4) >> 2;     // column half of the tile
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t store_seq = 0;  // chunks this warp has staged (its slot ring position)
        bool ok = true;
        uint32_t rs = 0, rph = 0;
        for (int ts = cluster_id;; ts += num_clusters) {
            int t = ts;
            if (dyn) {
                bool got_tile = ring_next(rs, rph, lane == 0, t);
                if (!__all_sync(0xffffffffu, got_tile)) {
                    ok = false;
                    break;
                }
            }
            if (t < 0 || t >= total_tiles) break;
            int split, mb, nb;
            tile_coords(p, t, split, mb, nb);
            bool got = mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int64_t row0 = (int64_t)mb * BM2 + (int64_t)rank * 128 + ew * 32;
            const int64_t row = row0 + lane;
            const uint32_t tbase = tmem_base + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
            for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
                const int64_t col0 = (int64_t)nb * BN + c;
                if (col0 >= p.n) break;
                float v[32];
                // bf16 ReLU-mask epilogue: the mask's loads go out before the TMEM load
                const bool pre_mask = p.tma_store == 1 && p.out_bf16 && p.epi == RT_EPI_RELU_MASK && row < p.m &&
                                      col0 + 32 <= p.n;
                uint4 mk[4];
                if (pre_mask) load_mask_bf16(p, row, col0, mk);
                tmem_ld_32x32(tbase + (uint32_t)c, v);
                uint8_t* box = smem_epi + (warp - 4) * kStageBytes;  // this warp's staging box
                if (p.tma_store == 2) {
                    // staged split-K partials: slice `split` of the [splits][m][n] workspace
                    stage_and_store_ring<float>(&tmap_c, box, 1, lane, row0, col0, v, store_seq, split);
                } else if (p.tma_store == 1) {
                    // staged: coalesced TMA stores of the warp's 32 x 32 chunk
                    if (p.out_bf16) {
                        if (pre_mask)
                            apply_mask_bf16(v, mk);
                        else if (row < p.m)
                            epilogue_math<__nv_bfloat16>(p, row, col0, v);
                        if constexpr (SPLIT_C)
                            stage_and_store_split(&tmap_c, &tmap_c2, box, lane, row0, col0, v);
                        else
                            stage_and_store_ring<__nv_bfloat16>(&tmap_c, box, 1, lane, row0, col0, v, store_seq);
                    } else {
                        if (row < p.m) epilogue_math<float>(p, row, col0, v);
                        stage_and_store_ring<float>(&tmap_c, box, 1, lane, row0, col0, v, store_seq);
                    }
                } else if (p.tma_store == 4) {
                    // rows scattered to their owners' receive buffers (peer memory)
                    p2p_chunk(p, reinterpret_cast<float*>(box), lane, row0, col0, v);
                } else if (p.tma_store == 3) {
                    // fused optimiser: the chunk updates theta / m / v / shadow and is stored as C
                    opt_chunk(p, reinterpret_cast<float*>(box), lane, row0, col0, v);
                } else if (row < p.m) {
                    if (p.ws) {
                        float* dst = p.ws + (int64_t)split * p.m * p.n + row * p.n + col0;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < p.n) dst[j] = v[j];
                    } else {
                        if (p.opt.kind) {
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
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        if (!ok && lane == 0) {
            record_error(p.err, DEV_TIMEOUT_EPILOGUE, blockIdx.x);
            raise_abort();
        }
        if ((p.tma_store == 1 || p.tma_store == 2) && lane == 0) bulk_wait_all();  // this warp's output stores are complete
        if (p.tma_store == 4) __threadfence_system();  // peer-memory stores in place before the kernel ends
    }

    __syncwarp();
    if (p.pdl == PDL_WAIT_EPILOGUE && warp < 4) {
        pdl_wait();
        pdl_launch_dependents();
    }
    __syncthreads();
    if (*abort_flag && rank == 0 && threadIdx.x == 0) {
        // Both CTAs' TMA loads complete on the leader's barriers: wait for the
        // last phase issued into each stage before either CTA can exit.
        for (int s = 0; s < STAGES; ++s)
            if (last_phase[s]) {
                volatile int never = 0;
                mbar_wait(smem_u32(&full[s]), last_phase[s] - 1, &never);
            }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no remote arrive or load is outstanding past this point
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(G::TMEM_COLS)
                     : "memory");
    }
}

template <typename TIn, bool A_MN, bool B_MN, int BN, bool X3 = false, bool SPLIT_C = false, bool SPLIT_A = false>
int launch_pair_variant(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st, const X3Planes* x3 = nullptr) {
    using G = Geo2<TIn, BN, SPLIT_A>;
    const bool bf16 = sizeof(TIn) == 2;
    CUtensorMap ta, tb, tc, ta2, tc2;
    if constexpr (X3) {
        RT_TRY(make_tmap_planes(&ta, x3->a, g.k, g.m, x3->lda, x3->a_plane, 2, G::BK, 128));
        RT_TRY(make_tmap_planes(&tb, x3->b, g.k, g.n, x3->ldb, x3->b_plane, 2, G::BK, G::BNH));
        ta2 = ta;
    } else {
        if (A_MN)
            RT_TRY(make_tmap(&ta, g.a, bf16, g.m, g.k, g.lda, G::CHUNK, G::BK));
        else
            RT_TRY(make_tmap(&ta, g.a, bf16, g.k, g.m, g.lda, G::BK, 128));
        ta2 = ta;
        if (g.a_lo) {  // A's low-order plane: the same geometry
            if (A_MN)
                RT_TRY(make_tmap(&ta2, g.a_lo, bf16, g.m, g.k, g.lda, G::CHUNK, G::BK));
            else
                RT_TRY(make_tmap(&ta2, g.a_lo, bf16, g.k, g.m, g.lda, G::BK, 128));
        }
        if (B_MN)
            RT_TRY(make_tmap(&tb, g.b, bf16, g.n, g.k, g.ldb, G::CHUNK, G::BK));
        else
            RT_TRY(make_tmap(&tb, g.b, bf16, g.k, g.n, g.ldb, G::BK, G::BNH));
    }

    TcParams p{};
    GemmDesc gr = g;
    p.m = g.m;
    p.n = g.n;
    p.k = g.k;
    p.tiles_m = (int)((g.m + BM2 - 1) / BM2);
    p.tiles_n = (int)((g.n + BN - 1) / BN);
    p.kblocks = (int)((g.k + G::BK - 1) / G::BK);
    p.kb_seg = 0;
    if constexpr (X3) {
        p.kb_seg = p.kblocks;
        p.kblocks *= 3;
    } else {
        if (g.a_lo && !SPLIT_A) {
            p.split_a = 1;
            p.kblocks *= 2;  // each k block twice: A's low-order plane, then A
        }
    }
    p.c_lo = g.c_lo;
    int splits = g.split_k > 1 ? g.split_k : 1;
    if (splits > p.kblocks) splits = p.kblocks;
    p.kb_per_split = (p.kblocks + splits - 1) / splits;
    splits = (p.kblocks + p.kb_per_split - 1) / p.kb_per_split;
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
    // the 3xTF32 planes come from the split kernel launched just before
    p.pdl = X3 && g.pdl != PDL_NONE ? PDL_WAIT_START : g.pdl;
    p.tile_ctr = ctx->dyn_tiles != 0 ? g.tile_ctr : nullptr;
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
    int64_t clusters = sms / 2;
    if (tiles < clusters) clusters = tiles;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
    cfg.blockDim = dim3(kThreads2, 1, 1);
    cfg.dynamicSmemBytes = G::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.pdl != PDL_NONE && ctx->pdl) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 2;
    } else {
        p.pdl = PDL_NONE;  // an ordinary launch: nothing to wait for
    }
    RT_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<TIn, A_MN, B_MN, BN, X3, SPLIT_C, SPLIT_A>, ta, tb, tc, ta2, tc2, p));
    count_launch(ctx);
    if (splits > 1) return launch_splitk_reduce(ctx, gr, st);
    return RT_OK;
}

// The forward (NN) layout with a low-order output plane has its own
// instantiation (SPLIT_C), so the other kernels carry none of its epilogue.
template <int BN>
int launch_pair_layout(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    if (g.c_lo) {
        if (g.layout != RT_NN) return fail(RT_ERR_UNSUPPORTED, "c_lo is supported for the NN layout only");
        if (g.a_lo) return launch_pair_variant<__nv_bfloat16, false, true, BN, false, true, true>(ctx, g, st);
        return launch_pair_variant<__nv_bfloat16, false, true, BN, false, true>(ctx, g, st);
    }
    if (g.a_lo && g.layout == RT_NN) return launch_pair_variant<__nv_bfloat16, false, true, BN, false, false, true>(ctx, g, st);
    switch (g.layout) {
        case RT_NN: return launch_pair_variant<__nv_bfloat16, false, true, BN>(ctx, g, st);
        case RT_NT: return launch_pair_variant<__nv_bfloat16, false, false, BN>(ctx, g, st);
        case RT_TN: return launch_pair_variant<__nv_bfloat16, true, true, BN>(ctx, g, st);
    }
    return fail(RT_ERR_INVALID, "unknown layout");
}


template <bool A_MN, bool B_MN, int BN, typename TIn = __nv_bfloat16, bool X3 = false, bool SPLIT_C = false,
          bool SPLIT_A = false>
int set_attr_pair() {
    RT_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<TIn, A_MN, B_MN, BN, X3, SPLIT_C, SPLIT_A>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Geo2<TIn, BN, SPLIT_A>::SMEM));
    return RT_OK;
}

}  // namespace

int gemm_tc2_init(rt_ctx* ctx) {
    (void)ctx;
    RT_TRY((set_attr_pair<false, true, 128>()));
    RT_TRY((set_attr_pair<false, false, 128>()));
    RT_TRY((set_attr_pair<true, true, 128>()));
    RT_TRY((set_attr_pair<false, true, 256>()));
    RT_TRY((set_attr_pair<false, false, 256>()));
    RT_TRY((set_attr_pair<true, true, 256>()));
    RT_TRY((set_attr_pair<false, false, 128, float, true>()));
    RT_TRY((set_attr_pair<false, false, 256, float, true>()));
    RT_TRY((set_attr_pair<false, true, 128, __nv_bfloat16, false, true>()));  // forward with c_lo
    RT_TRY((set_attr_pair<false, true, 256, __nv_bfloat16, false, true>()));
    RT_TRY((set_attr_pair<false, true, 128, __nv_bfloat16, false, true, true>()));  // split A (+ c_lo)
    RT_TRY((set_attr_pair<false, true, 256, __nv_bfloat16, false, true, true>()));
    RT_TRY((set_attr_pair<false, true, 128, __nv_bfloat16, false, false, true>()));
    RT_TRY((set_attr_pair<false, true, 256, __nv_bfloat16, false, false, true>()));
    return RT_OK;
}

// Pair tiles pay off when the output has at least one full 256-row tile and
// a 128-wide column tile; smaller problems keep the one-CTA kernel.
bool gemm_tc2_wanted(const rt_ctx* ctx, const GemmDesc& g) {
    return ctx->pair_gemm && g.in_dtype == RT_BF16 && g.m >= 256 && g.n > 64;
}

// 256-wide column tiles unless they leave more than half of the SM pairs
// idle, then 128-wide ones (as the 3xTF32 form below).
int launch_gemm_tc2(rt_ctx* ctx, const GemmDesc& g, cudaStream_t st) {
    const int64_t tiles256 = ((g.m + BM2 - 1) / BM2) * ((g.n + 255) / 256) * (g.split_k > 1 ? g.split_k : 1);
    if (g.n <= 128 || tiles256 * 4 < ctx->sm_count) return launch_pair_layout<128>(ctx, g, st);
    return launch_pair_layout<256>(ctx, g, st);
}

bool gemm_tc2_x3_wanted(const rt_ctx* ctx, const GemmDesc& g) {
    return ctx->pair_gemm && g.m >= 256 && g.n > 64;
}

// 3xTF32 from K-major hi/lo planes.  256-wide column tiles unless they leave
// more than half of the SM pairs idle, then 128-wide ones.
int launch_gemm_tc2_x3(rt_ctx* ctx, const GemmDesc& g, const X3Planes& x3, cudaStream_t st) {
    const int64_t tiles256 = ((g.m + BM2 - 1) / BM2) * ((g.n + 255) / 256) * (g.split_k > 1 ? g.split_k : 1);
    if (g.n <= 128 || tiles256 * 4 < ctx->sm_count)
        return launch_pair_variant<float, false, false, 128, true>(ctx, g, st, &x3);
    return launch_pair_variant<float, false, false, 256, true>(ctx, g, st, &x3);
}

}  // namespace rt
