// The whole-step plan: counterpart of rtensor's GpuMlp
// (crates/rtensor/src/gpu/mod.rs:1289-1562).  The plan is built once
// (buffers, GEMM descriptors, split-K choices), the step is captured into a
// CUDA graph, and every step replays it: no host round-trip between the
// forward GEMMs, softmax-CE, the backward GEMMs with their fused epilogues,
// the optional NCCL allreduce of dW/db and the optimiser.
//
// Backward recurrence (gpu/mod.rs:35-46):
//   delta_L = (P - Y) / n_global
//   delta_{l-1} = (delta_l W_l^T) * 1[A_{l-1} > 0]     (l > 0)
//   [dW_l; db_l] = [A_{l-1}, 1]^T delta_l
//
// Layout choices that remove kernels from the step:
//   - every layer input (x and each hidden A_l) carries one extra column of
//     ones, so the dW GEMM over [A, 1] produces db as its last row and no
//     separate column reduction runs;
//   - W_l and b_l share one [d_l + 1, ld] block (b in the last row), and so do
//     their gradients and Adam moments, so one optimiser launch updates both;
//   - on one device with SGD or Adam, per layer the dX GEMM (the last reader
//     of W_l) runs first and the dW GEMM second, with the update fused into
//     its epilogue (backward_fused);
//   - otherwise (data parallelism, no optimiser, RTGPU_FUSED_OPT=0) the dW
//     GEMM runs first, in row chunks whose gradient sums (allreduce, or the
//     sharded optimiser's reduce-scatter by NCCL or copy engines) start on the
//     comm stream while the next chunk computes; the dX GEMM second; each
//     chunk's update on the optimiser stream once the dX GEMM is done and the
//     chunk is summed (backward_and_update).  The first layer's dW is chunked
//     there too: it is the last GEMM of the step, so its update then trails
//     it by one chunk only;
//   - bf16 plans keep hidden activations that feed another hidden layer as
//     hi + lo bf16 planes (the next forward GEMM's second k segment);
//   - the pair-kernel GEMMs launch as programmatic dependents of the kernel
//     before them (GemmDesc::pdl), and under data parallelism take their tiles
//     from per-GEMM counters that the pass zeroes at its start;
//   - two input slots: a host step copies the next batch on a copy stream
//     while the previous step computes.
#include <cstdlib>
#include <cstring>
#include <vector>

#include "internal.h"

namespace rt {
int run_gemm(rt_ctx* ctx, GemmDesc g, cudaStream_t stream, size_t ws_bytes);
int comm_allreduce(rt_comm* comm, float* buf, int64_t count, cudaStream_t st);
int comm_allreduce_bf16(rt_comm* comm, __nv_bfloat16* buf, int64_t count, cudaStream_t st);
int comm_reduce_scatter(rt_comm* comm, float* buf, int64_t count, cudaStream_t st);
int comm_all_gather(rt_comm* comm, void* buf, int64_t count, int elem_bytes, cudaStream_t st, bool second = false);
bool comm_open_second(rt_comm* comm, int* status);
int comm_rank(const rt_comm* comm);
int comm_world(const rt_comm* comm);
}  // namespace rt

using namespace rt;

namespace {

int64_t round8(int64_t x) { return (x + 7) / 8 * 8; }
// Row strides of GEMM operands are kept at multiples of 64 elements so every
// 128-byte TMA row segment starts on a 128-byte line.
int64_t round64(int64_t x) { return (x + 63) / 64 * 64; }
// Leading dimension (elements) of a layer's [d+1, u] blocks: 64-element
// multiples (128-byte TMA row segments), 8 below 64 units.
int64_t plan_ld(int64_t u) { return u >= 64 ? round64(u) : round8(u); }

// Start row of chunk c of `rows` rows cut into the plan's first-layer chunks
// (boundaries on 256-row tile edges; the last chunk takes the remainder).
int64_t chunk_row_of(int64_t rows, int chunks, int c) {
    if (c >= chunks) return rows;
    return rows * c / chunks / 256 * 256;
}

struct PlanLayer {
    int64_t d = 0, u = 0;
    int64_t ld = 0;      // row stride of the [d+1, ld] parameter blocks and of delta_l
    int64_t ld_act = 0;  // row stride of A_l (u + 1 columns: activations and the ones column)
    float* w32 = nullptr;            // [d+1, ld] f32: W rows 0..d-1, bias row d
    float* b = nullptr;              // = w32 + d*ld
    __nv_bfloat16* w16 = nullptr;    // bf16 shadow of w32 (bf16 plans)
    float *m = nullptr, *v = nullptr;  // Adam moments [d+1, ld]
    float* g = nullptr;              // gradient [d+1, ld]: dW rows 0..d-1, db row d
    float* db = nullptr;             // = g + d*ld
    void* act = nullptr;    // hidden: A_l [n, ld_act] (operand dtype); last: logits f32 [n, ld]
    void* act_lo = nullptr; // split-activation bf16 plans, layers feeding a hidden layer: A_l's low-order plane
    void* delta = nullptr;  // delta_l [n, ld] (operand dtype)
    int split_dw = 1;
    float* ws = nullptr;    // split-K partials for the dW GEMM
    size_t ws_bytes = 0;
    __nv_bfloat16* g16 = nullptr;  // bf16 copy of g for a bf16 gradient allreduce
    // The dW GEMM in `chunks` row chunks of [dW; db], each with its events:
    // computed (ready), allreduced (comm), updated (opt); dx: the dX GEMM done.
    int chunks = 1;
    std::vector<cudaEvent_t> ev_ready, ev_comm, ev_opt, ev_ag;
    cudaEvent_t ev_dx = nullptr;
    // Peer-memory reduce-scatter (sharded optimiser, RTGPU_P2P_RS=1): the dW
    // GEMM's epilogue stores each weight row to its owner's receive buffer
    // `recv` ([world][d / world][ld] f32: one region per source rank), mapped
    // into this process for every rank at peers[q].
    bool p2p = false;
    float* recv = nullptr;
    void* peers[kMaxPeers] = {};
    // Copy-engine exchange (sharded optimiser, the default where every rank
    // maps every other rank's buffers): each rank copies owner q's flat piece
    // of a finished dW chunk into ce_recv of rank q, region `this rank`, at
    // ce_off[chunk]; ce_recv is [world][d * ld / world] f32 (per source rank,
    // this rank's pieces of every chunk in chunk order; a rank's own region is
    // unused, it sums its own partial in place).  After its update a
    // rank's piece of the bf16 weights is pulled by every other rank from its
    // w16 (w16_peers[q] maps rank q's shadow).  No SM moves these bytes.
    bool ce = false;
    float* ce_recv = nullptr;
    void* ce_peers[kMaxPeers] = {};
    void* w16_peers[kMaxPeers] = {};
    std::vector<int64_t> ce_off;
};

struct Slot {
    void* x = nullptr;          // [n, ldx] operand dtype, ones column at d0
    uint32_t* labels = nullptr;
    void* stage = nullptr;      // host-dtype staging when it differs from the plan's
    size_t stage_bytes = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool timed = false;
    // the forward pass alone (inference), captured on first use
    cudaGraph_t fwd_graph = nullptr;
    cudaGraphExec_t fwd_exec = nullptr;
    cudaEvent_t ready = nullptr, free_ = nullptr;
};

struct OpRecord {
    const char* label;
    double flops;
};

}  // namespace

struct rt_mlp {
    rt_ctx* ctx = nullptr;
    rt_mlp_config cfg{};
    std::vector<int64_t> dims;
    std::vector<PlanLayer> L;
    rt_dtype adt = RT_F32;
    // bf16 plans with RT_ACT_SPLIT: every hidden activation that feeds another
    // hidden layer is stored as the pair hi = bf16(a) (act) and lo =
    // bf16(a - hi) (act_lo); that layer's forward GEMM reads both, the dW
    // GEMMs and the ReLU masks read hi.  The output layer's input needs no lo
    // plane: its rounding moves the logits by ~1e-3 of their spread and flips
    // no ReLU mask.
    bool split_act = false;
    int64_t n = 0, ldx = 0;
    Slot slot[2];
    int next_slot = 0;
    int last_slot = 0;
    float* loss_rows = nullptr;
    float* loss_all = nullptr;  // [world * batch] per-row losses of every rank (rt_mlp_global_loss)
    OptScalars* opt = nullptr;
    // f32 plans: hi/lo operand planes of the 3xTF32 GEMMs, sized for the
    // largest GEMM of the step (the GEMMs run one after another on one stream)
    float* x3_ws = nullptr;
    size_t x3_ws_bytes = 0;
    std::vector<void*> allocs;
    cudaStream_t copy_stream = nullptr;

    bool timing = false;
    std::vector<cudaEvent_t> events;
    std::vector<OpRecord> ops;
    int kernels_per_step = 0;
    int kernels_per_forward = 0;

    rt_comm* comm = nullptr;
    int comm_sm_reserve = 0;  // SMs the backward GEMMs leave to NCCL while gradients are reduced
    cudaStream_t comm_stream = nullptr;
    bool comm_bf16 = false;  // allreduce the gradients in bf16 (bf16 plans, RTGPU_GRAD_COMM=bf16)
    // Fused update (one device, SGD or Adam; RTGPU_FUSED_OPT=0 turns it off):
    // each dW GEMM applies the optimiser to its output tile in the epilogue,
    // so the update rides inside the GEMM instead of running after it.
    bool fuse_opt = false;
    // Sharded optimiser (bf16 plans with an optimiser under data parallelism):
    // each gradient chunk is reduce-scattered, every rank updates its 1/world
    // slice of the f32 masters and moments, and the bf16 weights are
    // all-gathered; the f32 masters, moments and reduced gradients outside a
    // rank's slices are gathered only when read (rt_mlp_weights / grads /
    // save_state, then collective).
    bool sharded = false;
    int rank = 0, world = 1;
    // the weight all-gathers' own stream and NCCL communicator (when NCCL can
    // split one off); otherwise they share the comm stream
    cudaStream_t ag_stream = nullptr;
    float* scratch = nullptr;  // one word for barriers and agreement collectives
    // One tile counter per pair-kernel GEMM of a captured pass (dynamic tile
    // schedule), zeroed by the pass's first node.
    static constexpr int kTileCtrs = 64;
    int* tile_ctrs = nullptr;
    // per-layer optimiser on a side stream, overlapping the remaining backward GEMMs
    cudaStream_t opt_stream = nullptr;
    // Copy-engine exchange: one stream per peer for the gradient scatter and
    // one per peer for the weight pulls, so that the copies to (or from)
    // different ranks run on different copy engines at once; fork/join
    // events tie them to the comm and all-gather streams.
    cudaStream_t ce_scatter[kMaxPeers] = {}, ce_pull[kMaxPeers] = {};
    cudaEvent_t ce_fork = nullptr, ce_fork2 = nullptr;
    cudaEvent_t ce_join[kMaxPeers] = {}, ce_join2[kMaxPeers] = {};
};

namespace {

// Every plan buffer is zeroed on the context stream, and every later set-up
// copy and kernel goes to that stream too, so they are ordered (the context
// stream does not synchronise with the legacy default stream).
int dalloc(rt_mlp* m, void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail(RT_ERR_OOM, "plan allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
    m->allocs.push_back(*p);
    e = cudaMemsetAsync(*p, 0, bytes ? bytes : 16, m->ctx->stream);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, "cudaMemsetAsync failed: %s", cudaGetErrorString(e));
    return RT_OK;
}

template <typename T>
int dalloc_t(rt_mlp* m, T** p, size_t count) {
    return dalloc(m, reinterpret_cast<void**>(p), count * sizeof(T));
}

void drop_graphs(rt_mlp* m) {
    for (auto& s : m->slot) {
        if (s.exec) cudaGraphExecDestroy(s.exec);
        if (s.graph) cudaGraphDestroy(s.graph);
        if (s.fwd_exec) cudaGraphExecDestroy(s.fwd_exec);
        if (s.fwd_graph) cudaGraphDestroy(s.fwd_graph);
        s.exec = nullptr;
        s.graph = nullptr;
        s.fwd_exec = nullptr;
        s.fwd_graph = nullptr;
    }
}

// Unmaps the peers' buffers of every peer-scatter and copy-engine layer.
void teardown_p2p(rt_mlp* m) {
    for (PlanLayer& P : m->L) {
        if (P.p2p) {
            comm_unshare_buffer(m->comm, P.peers);
            P.p2p = false;
        }
        if (P.ce) {
            comm_unshare_buffer(m->comm, P.ce_peers);
            comm_unshare_buffer(m->comm, P.w16_peers);
            P.ce = false;
        }
    }
}

void free_all(rt_mlp* m) {
    drop_graphs(m);
    teardown_p2p(m);
    for (auto& s : m->slot) {
        if (s.ready) cudaEventDestroy(s.ready);
        if (s.free_) cudaEventDestroy(s.free_);
        if (s.stage) cudaFree(s.stage);
    }
    for (auto e : m->events) cudaEventDestroy(e);
    for (auto& P : m->L) {
        for (auto e : P.ev_ready) cudaEventDestroy(e);
        for (auto e : P.ev_comm) cudaEventDestroy(e);
        for (auto e : P.ev_opt) cudaEventDestroy(e);
        for (auto e : P.ev_ag) cudaEventDestroy(e);
        if (P.ev_dx) cudaEventDestroy(P.ev_dx);
    }
    for (int q = 0; q < kMaxPeers; ++q) {
        if (m->ce_scatter[q]) cudaStreamDestroy(m->ce_scatter[q]);
        if (m->ce_pull[q]) cudaStreamDestroy(m->ce_pull[q]);
        if (m->ce_join[q]) cudaEventDestroy(m->ce_join[q]);
        if (m->ce_join2[q]) cudaEventDestroy(m->ce_join2[q]);
    }
    if (m->ce_fork) cudaEventDestroy(m->ce_fork);
    if (m->ce_fork2) cudaEventDestroy(m->ce_fork2);
    if (m->comm_stream) cudaStreamDestroy(m->comm_stream);
    if (m->ag_stream) cudaStreamDestroy(m->ag_stream);
    if (m->opt_stream) cudaStreamDestroy(m->opt_stream);
    if (m->copy_stream) cudaStreamDestroy(m->copy_stream);
    for (void* p : m->allocs) cudaFree(p);
    m->allocs.clear();
}

// Enqueues the optimiser update of the flat elements [o, o + n) of layer P's
// [d+1, ld] parameter block on st.
int enqueue_update_flat(rt_mlp* m, PlanLayer& P, int64_t o, int64_t n, cudaStream_t st) {
    OptTensor t{P.w32 + o, P.g + o, P.m ? P.m + o : nullptr, P.v ? P.v + o : nullptr, P.w16 ? P.w16 + o : nullptr,
                P.ld, P.ld, n};
    if (m->cfg.optimizer == RT_OPT_ADAM)
        return launch_adam(m->ctx, &t, 1, m->opt, m->cfg.lr, m->cfg.beta1, m->cfg.beta2, m->cfg.eps, st);
    if (m->cfg.optimizer == RT_OPT_SGD) return launch_sgd(m->ctx, &t, 1, m->cfg.lr, st);
    return RT_OK;
}

// Under the sharded optimiser the weight rows [r0, min(r1, d)) of a chunk are
// split into world equal flat slices; the bias row d, which the forward
// epilogue reads in f32, stays replicated (allreduced, updated on every rank).
int64_t shard_end(const PlanLayer& P, int64_t r1) { return r1 < P.d ? r1 : P.d; }

// This rank's flat slice of the weight rows of chunk [r0, r1) of a [d+1, ld]
// parameter block: its length (0 when the chunk holds only the bias row) and,
// in *off, its first element.
int64_t shard_slice(int64_t d, int64_t ld, int64_t r0, int64_t r1, int world, int rank, int64_t* off) {
    const int64_t e = r1 < d ? r1 : d;
    if (e <= r0 || world < 1) {
        *off = r0 * ld;
        return 0;
    }
    const int64_t piece = (e - r0) * ld / world;
    *off = r0 * ld + (int64_t)rank * piece;
    return piece;
}

// Rows [r0, r1) of the parameter block: the whole range, or under the sharded
// optimiser this rank's slice of the weight rows plus the bias row.
int enqueue_update_rows(rt_mlp* m, PlanLayer& P, int64_t r0, int64_t r1, cudaStream_t st) {
    if (!m->sharded) return enqueue_update_flat(m, P, r0 * P.ld, (r1 - r0) * P.ld, st);
    int64_t off = 0;
    const int64_t piece = shard_slice(P.d, P.ld, r0, r1, m->world, m->rank, &off);
    if (piece > 0) RT_TRY(enqueue_update_flat(m, P, off, piece, st));
    if (r1 > P.d) RT_TRY(enqueue_update_flat(m, P, P.d * P.ld, P.ld, st));
    return RT_OK;
}

// ---------------------------------------------------------------- step body
struct Enqueuer {
    rt_mlp* m;
    cudaStream_t st;
    int s;  // input slot
    bool forward_only;
    int op_index = 0;
    int ctr_used = 0;

    // This GEMM's own tile counter (the pass zeroes them all at its start), or
    // null for the round-robin schedule: by default on one device, where
    // nothing else holds SMs when a GEMM starts, and once the counters run out.
    int* next_ctr() {
        const int policy = m->ctx->dyn_tiles;  // 1 always, 0 never, -1 under data parallelism
        if (policy == 0 || (policy < 0 && !m->comm)) return nullptr;
        return m->tile_ctrs && ctr_used < rt_mlp::kTileCtrs ? m->tile_ctrs + ctr_used++ : nullptr;
    }

    int mark(const char* label, double flops) {
        if (m->timing && !forward_only) {
            if ((size_t)op_index + 1 >= m->events.size()) return fail(RT_ERR_INVALID, "timing event overflow");
            RT_CUDA(cudaEventRecordWithFlags(m->events[op_index + 1], st, cudaEventRecordExternal));
            if ((size_t)op_index >= m->ops.size()) m->ops.push_back({label, flops});
        }
        ++op_index;
        return RT_OK;
    }

    int begin() {
        if (m->timing && !forward_only) RT_CUDA(cudaEventRecordWithFlags(m->events[0], st, cudaEventRecordExternal));
        return RT_OK;
    }

    const void* input_of(int l) const { return l == 0 ? m->slot[s].x : m->L[l - 1].act; }

    int64_t ld_in(int l) const { return l == 0 ? m->ldx : m->L[l - 1].ld_act; }
    int backward_sms() const {
        return m->comm && m->comm_sm_reserve > 0 ? m->ctx->sm_count - m->comm_sm_reserve : 0;
    }
    const void* weights(const PlanLayer& P) const {
        return m->adt == RT_BF16 ? (const void*)P.w16 : (const void*)P.w32;
    }

    int forward() {
        const int nl = (int)m->L.size();
        if (m->tile_ctrs) RT_CUDA(cudaMemsetAsync(m->tile_ctrs, 0, rt_mlp::kTileCtrs * sizeof(int), st));
        for (int l = 0; l < nl; ++l) {
            PlanLayer& P = m->L[l];
            bool last = l == nl - 1;
            GemmDesc g{};
            g.layout = RT_NN;
            g.in_dtype = m->adt;
            g.out_dtype = last ? RT_F32 : m->adt;
            g.m = m->n;
            g.n = P.u;
            g.k = P.d;
            g.a = input_of(l);
            g.lda = ld_in(l);
            g.b = weights(P);
            g.ldb = P.ld;
            g.c = P.act;
            g.ldc = last ? P.ld : P.ld_act;
            g.epi = last ? RT_EPI_BIAS : RT_EPI_BIAS_RELU;
            g.bias = P.b;
            g.split_k = 1;
            if (m->split_act) {
                if (l > 0 && !last) g.a_lo = m->L[l - 1].act_lo;  // hidden layer: (A_hi + A_lo) W
                if (l + 2 < nl) g.c_lo = P.act_lo;                // A_l feeds a hidden layer: hi and lo planes
            }
            g.x3_ws = m->x3_ws;
            g.x3_ws_bytes = m->x3_ws_bytes;
            g.pdl = PDL_WAIT_START;  // reads the previous layer's activations
            g.tile_ctr = next_ctr();
            RT_TRY(run_gemm(m->ctx, g, st, 0));
            // FLOPs are the algorithmic 2 n d u; a split-A GEMM runs twice that on the tensor cores
            const char* label = last ? "fwd_gemm_bias" : g.a_lo ? "fwd_gemm_bias_relu_split" : "fwd_gemm_bias_relu";
            RT_TRY(mark(label, 2.0 * m->n * P.d * P.u));
        }
        return RT_OK;
    }

    // [dW_l; db_l] rows [r0, r1) = ([A_{l-1}, 1] columns r0..r1)^T delta_l (TN, K = batch), f32.
    int dw_gemm_rows(PlanLayer& P, int l, int64_t r0, int64_t r1, int pdl) {
        const int64_t rows = P.d + 1;
        GemmDesc g = dw_desc(P, l, r0, r1);
        g.pdl = pdl;
        g.tile_ctr = next_ctr();
        if (P.p2p) {
            // weight rows go to their owners' receive buffers, the bias row to g
            const int64_t e = shard_end(P, r1);
            RT_CHECK(e > r0 && (e - r0) % m->world == 0 && m->world <= kMaxPeers, "peer-scatter chunk [%lld, %lld)",
                     (long long)r0, (long long)e);
            for (int q = 0; q < m->world; ++q) {
                RT_CHECK(P.peers[q] != nullptr, "peer-scatter layer without rank %d's buffer", q);
                g.p2p.peer[q] = static_cast<float*>(P.peers[q]);
            }
            g.p2p.rank = m->rank;
            g.p2p.world = m->world;
            g.p2p.rows_owned = (e - r0) / m->world;
            g.p2p.owned_end = e - r0;
            g.p2p.base_row = r0 / m->world;
            g.p2p.q_stride = P.d / m->world * P.ld;
            g.p2p.ld = P.ld;
        }
        RT_TRY(run_gemm(m->ctx, g, st, P.ws_bytes));
        // FLOPs of the weight rows (the bias row is not counted, as everywhere)
        const char* label = !m->fuse_opt ? "dw_gemm"
                            : m->cfg.optimizer == RT_OPT_ADAM ? "dw_gemm_adam"
                                                              : "dw_gemm_sgd";
        return mark(label, 2.0 * m->n * (double)(r1 - r0 - (r1 == rows ? 1 : 0)) * P.u);
    }

    // The [dW; db] rows [r0, r1) GEMM of layer l, as dw_gemm_rows launches it.
    GemmDesc dw_desc(PlanLayer& P, int l, int64_t r0, int64_t r1) const {
        GemmDesc g{};
        g.layout = RT_TN;
        g.in_dtype = m->adt;
        g.out_dtype = RT_F32;
        g.m = r1 - r0;
        g.n = P.u;
        g.k = m->n;
        g.a = static_cast<const uint8_t*>(input_of(l)) + r0 * dtype_size(m->adt);  // A columns r0..r1
        g.lda = ld_in(l);
        g.b = P.delta;
        g.ldb = P.ld;
        g.c = P.g + r0 * P.ld;
        g.ldc = P.ld;
        g.epi = RT_EPI_NONE;
        g.split_k = P.split_dw;
        g.workspace = P.ws;
        g.max_sms = backward_sms();
        g.x3_ws = m->x3_ws;
        g.x3_ws_bytes = m->x3_ws_bytes;
        if (m->fuse_opt) {
            // the epilogue applies the update to rows [r0, r1) of theta (and m, v, shadow)
            const int64_t o = r0 * P.ld;
            g.opt.kind = m->cfg.optimizer == RT_OPT_ADAM ? 2 : 1;
            g.opt.theta = P.w32 + o;
            g.opt.m = P.m ? P.m + o : nullptr;
            g.opt.v = P.v ? P.v + o : nullptr;
            g.opt.shadow = P.w16 ? P.w16 + o : nullptr;
            g.opt.sc = m->opt;
            g.opt.lr = m->cfg.lr;
            g.opt.beta1 = m->cfg.beta1;
            g.opt.beta2 = m->cfg.beta2;
            g.opt.eps = m->cfg.eps;
        }
        return g;
    }

    // Sums gradient rows [r0, r1) (chunk c) over the ranks on the comm stream
    // (in bf16 when the plan reduces in bf16: cast, allreduce, cast back into g).
    int allreduce_rows(PlanLayer& P, int c, int64_t r0, int64_t r1) {
        cudaStream_t cs = m->comm_stream;
        const int64_t count = (r1 - r0) * P.ld;
        if (P.ce) {
            // copy-engine reduce-scatter: this rank's partial of every owner's
            // piece goes to that owner's receive region for this rank; once
            // every rank has passed the barrier, the owner sums the world
            // partials, source rank by source rank, into its piece of g
            const int64_t e = shard_end(P, r1);
            if (e > r0) {
                const int64_t piece = (e - r0) * P.ld / m->world, region = P.d * P.ld / m->world;
                RT_CUDA(cudaEventRecord(m->ce_fork, cs));
                for (int q = 0; q < m->world; ++q) {
                    if (q == m->rank) continue;  // the owner reads its own partial in place
                    cudaStream_t sq = m->ce_scatter[q];
                    RT_CUDA(cudaStreamWaitEvent(sq, m->ce_fork, 0));
                    float* dst = static_cast<float*>(P.ce_peers[q]) + (int64_t)m->rank * region + P.ce_off[c];
                    RT_CUDA(cudaMemcpyAsync(dst, P.g + r0 * P.ld + (int64_t)q * piece, (size_t)piece * 4,
                                            cudaMemcpyDeviceToDevice, sq));
                    RT_CUDA(cudaEventRecord(m->ce_join[q], sq));
                    RT_CUDA(cudaStreamWaitEvent(cs, m->ce_join[q], 0));
                }
                RT_TRY(comm_barrier(m->comm, m->scratch, cs));
                float* own = P.g + r0 * P.ld + (int64_t)m->rank * piece;
                RT_TRY(launch_sum_partials_own(m->ctx, own, own, P.ce_recv + P.ce_off[c], region, m->world, m->rank,
                                               piece, cs));
            }
            if (r1 > P.d) RT_TRY(comm_allreduce(m->comm, P.db, P.ld, cs));
            return RT_OK;
        }
        if (P.p2p) {
            // Every rank's GEMM has stored its partials of this chunk into the
            // owners' receive buffers once all ranks pass the barrier; the
            // owner then sums them, source rank by source rank, into its
            // slice of g.
            const int64_t e = shard_end(P, r1), h = (e - r0) / m->world;
            RT_TRY(comm_barrier(m->comm, m->scratch, cs));
            if (e > r0)
                RT_TRY(launch_sum_partials(m->ctx, P.g + (r0 + (int64_t)m->rank * h) * P.ld,
                                           P.recv + r0 / m->world * P.ld, P.d / m->world * P.ld, m->world, h * P.ld, cs));
            if (r1 > P.d) RT_TRY(comm_allreduce(m->comm, P.db, P.ld, cs));
            return RT_OK;
        }
        if (m->sharded) {
            const int64_t e = shard_end(P, r1);
            if (e > r0) RT_TRY(comm_reduce_scatter(m->comm, P.g + r0 * P.ld, (e - r0) * P.ld / m->world, cs));
            if (r1 > P.d) RT_TRY(comm_allreduce(m->comm, P.db, P.ld, cs));
            return RT_OK;
        }
        if (!m->comm_bf16) return comm_allreduce(m->comm, P.g + r0 * P.ld, count, cs);
        __nv_bfloat16* h = P.g16 + r0 * P.ld;
        RT_TRY(launch_cast(m->ctx, P.g + r0 * P.ld, RT_F32, P.ld, h, RT_BF16, P.ld, r1 - r0, P.ld, cs));
        RT_TRY(comm_allreduce_bf16(m->comm, h, count, cs));
        return launch_cast(m->ctx, h, RT_BF16, P.ld, P.g + r0 * P.ld, RT_F32, P.ld, r1 - r0, P.ld, cs);
    }

    // Sharded optimiser: the all-gathers of every chunk of layer P (l > 0),
    // each after this rank's update of its slice of the chunk.
    int gather_layer(PlanLayer& P) {
        if (!m->sharded || m->cfg.optimizer == RT_OPT_NONE) return RT_OK;
        for (int c = 0; c < P.chunks; ++c)
            RT_TRY(gather_weights(P, c, chunk_row_of(P.d + 1, P.chunks, c), chunk_row_of(P.d + 1, P.chunks, c + 1)));
        return RT_OK;
    }

    // Sharded optimiser: once this rank has updated its slice of chunk c, the
    // chunk's bf16 weights are all-gathered on the comm stream.
    int gather_weights(PlanLayer& P, int c, int64_t r0, int64_t r1) {
        if (!m->sharded) return RT_OK;
        if (P.ce) {
            // once every rank has updated its piece of chunk c (the barrier on
            // the second communicator), pull the other ranks' pieces of the
            // bf16 weights into this rank's shadow
            cudaStream_t as = m->ag_stream;
            RT_CUDA(cudaStreamWaitEvent(as, P.ev_opt[c], 0));
            const int64_t e = shard_end(P, r1);
            if (e > r0) {
                RT_TRY(comm_barrier(m->comm, m->scratch + 1, as, true));
                const int64_t piece = (e - r0) * P.ld / m->world;
                RT_CUDA(cudaEventRecord(m->ce_fork2, as));
                for (int q = 0; q < m->world; ++q) {
                    if (q == m->rank) continue;
                    cudaStream_t sq = m->ce_pull[q];
                    RT_CUDA(cudaStreamWaitEvent(sq, m->ce_fork2, 0));
                    const int64_t o = r0 * P.ld + (int64_t)q * piece;
                    RT_CUDA(cudaMemcpyAsync(P.w16 + o, static_cast<const __nv_bfloat16*>(P.w16_peers[q]) + o,
                                            (size_t)piece * 2, cudaMemcpyDeviceToDevice, sq));
                    RT_CUDA(cudaEventRecord(m->ce_join2[q], sq));
                    RT_CUDA(cudaStreamWaitEvent(as, m->ce_join2[q], 0));
                }
            }
            RT_CUDA(cudaEventRecord(P.ev_ag[c], as));
            return RT_OK;
        }
        if (!m->ag_stream) RT_CUDA(cudaStreamWaitEvent(m->comm_stream, P.ev_opt[c], 0));
        cudaStream_t as = m->ag_stream ? m->ag_stream : m->comm_stream;
        if (m->ag_stream) RT_CUDA(cudaStreamWaitEvent(as, P.ev_opt[c], 0));
        const int64_t e = shard_end(P, r1);
        if (e > r0) RT_TRY(comm_all_gather(m->comm, P.w16 + r0 * P.ld, (e - r0) * P.ld / m->world, 2, as, m->ag_stream != nullptr));
        RT_CUDA(cudaEventRecord(P.ev_ag[c], as));
        return RT_OK;
    }

    // delta_{l-1} = (delta_l W_l^T) * 1[A_{l-1} > 0]  (NT, fused mask)
    int dx_gemm(int l, int pdl) {
        PlanLayer& P = m->L[l];
        PlanLayer& Q = m->L[l - 1];
        GemmDesc h{};
        h.pdl = pdl;
        h.tile_ctr = next_ctr();
        h.layout = RT_NT;
        h.in_dtype = m->adt;
        h.out_dtype = m->adt;
        h.m = m->n;
        h.n = P.d;
        h.k = P.u;
        h.a = P.delta;
        h.lda = P.ld;
        h.b = weights(P);
        h.ldb = P.ld;
        h.c = Q.delta;
        h.ldc = Q.ld;
        h.epi = RT_EPI_RELU_MASK;
        h.mask = Q.act;
        h.ldmask = Q.ld_act;
        h.split_k = 1;
        h.max_sms = backward_sms();
        h.x3_ws = m->x3_ws;
        h.x3_ws_bytes = m->x3_ws_bytes;
        RT_TRY(run_gemm(m->ctx, h, st, 0));
        return mark("dx_gemm_relu_mask", 2.0 * m->n * P.d * P.u);
    }

    // Backward with the update fused into the dW GEMMs (one device): per
    // layer, top down, the dX GEMM first (the last reader of W_l), then the
    // dW GEMM, whose epilogue updates W_l, b_l and their moments in place.
    int backward_fused() {
        const int nl = (int)m->L.size();
        PlanLayer& Last = m->L[nl - 1];
        double gb = (double)(m->cfg.global_batch > 0 ? m->cfg.global_batch : m->n);
        if (m->cfg.optimizer == RT_OPT_ADAM) {
            RT_TRY(launch_opt_step_begin(m->ctx, m->opt, m->cfg.beta1, m->cfg.beta2, st));
            RT_TRY(mark("adam_scalars", 0));
        }
        RT_TRY(launch_xent(m->ctx, (const float*)Last.act, Last.ld, m->slot[s].labels, m->n, Last.u,
                           (float)(1.0 / gb), Last.delta, m->adt, Last.ld, m->loss_rows, st));
        RT_TRY(mark("softmax_xent", 0));
        // Launch order per layer, top down: dX_l, then dW_l.  dX_l reads delta_l
        // (complete once the dW GEMM before it has passed its epilogue wait; after
        // softmax-CE it waits at its start) and W_l, which no running GEMM
        // writes.  dW_l's epilogue overwrites W_l, which dX_l reads: its k loop
        // starts at once, its epilogue waits for dX_l (the first layer's dW has
        // no dX before it and overwrites nothing the GEMM before it reads).
        for (int l = nl - 1; l >= 0; --l) {
            PlanLayer& P = m->L[l];
            if (l > 0) RT_TRY(dx_gemm(l, l == nl - 1 ? PDL_WAIT_START : PDL_NO_WAIT));
            for (int c = 0; c < P.chunks; ++c)
                RT_TRY(dw_gemm_rows(P, l, chunk_row_of(P.d + 1, P.chunks, c), chunk_row_of(P.d + 1, P.chunks, c + 1),
                                    c == 0 && l > 0 ? PDL_WAIT_EPILOGUE
                                    : c == 0 && l == nl - 1 ? PDL_WAIT_START
                                                            : PDL_NO_WAIT));
        }
        return RT_OK;
    }

    // Backward and update with separate update kernels (data parallelism, no
    // optimiser, or RTGPU_FUSED_OPT=0).  Per layer, top down: the dW GEMM (in
    // row chunks of [dW; db], contiguous rows of the parameter block), each
    // chunk handed to the comm stream for its gradient sum as soon as it is
    // computed (allreduce; or, sharded, a reduce-scatter or the peer-scatter
    // barrier and owner sum); then the dX GEMM, the last reader of W_l in the
    // step; then, on the optimiser stream, each chunk's update (of this rank's
    // slice, when sharded) once dX is done and the chunk is summed, and the
    // sharded weight all-gathers.  The first layer has no dX GEMM, so its chunk
    // updates follow the chunk GEMMs directly: its dW GEMM is the last GEMM of
    // the step, and chunking it keeps the trailing exchange to one chunk.
    int backward_and_update() {
        if (m->fuse_opt) return backward_fused();
        const int nl = (int)m->L.size();
        const bool update = m->cfg.optimizer != RT_OPT_NONE;
        PlanLayer& Last = m->L[nl - 1];
        double gb = (double)(m->cfg.global_batch > 0 ? m->cfg.global_batch : m->n);
        if (m->cfg.optimizer == RT_OPT_ADAM) {
            RT_TRY(launch_opt_step_begin(m->ctx, m->opt, m->cfg.beta1, m->cfg.beta2, st));
            RT_TRY(mark("adam_scalars", 0));
        }
        RT_TRY(launch_xent(m->ctx, (const float*)Last.act, Last.ld, m->slot[s].labels, m->n, Last.u,
                           (float)(1.0 / gb), Last.delta, m->adt, Last.ld, m->loss_rows, st));
        RT_TRY(mark("softmax_xent", 0));
        for (int l = nl - 1; l >= 0; --l) {
            PlanLayer& P = m->L[l];
            const int64_t rows = P.d + 1;
            for (int c = 0; c < P.chunks; ++c) {
                const int64_t r0 = chunk_row_of(rows, P.chunks, c), r1 = chunk_row_of(rows, P.chunks, c + 1);
                // chunk 0 reads delta_l, which the GEMM launched just before it
                // (dX_{l+1}, or softmax-CE) writes; the other chunks read only
                // what was complete when chunk 0 passed its wait
                RT_TRY(dw_gemm_rows(P, l, r0, r1, c == 0 ? PDL_WAIT_START : PDL_NO_WAIT));
                RT_CUDA(cudaEventRecord(P.ev_ready[c], st));
                if (m->comm) {
                    RT_CUDA(cudaStreamWaitEvent(m->comm_stream, P.ev_ready[c], 0));
                    RT_TRY(allreduce_rows(P, c, r0, r1));
                    RT_CUDA(cudaEventRecord(P.ev_comm[c], m->comm_stream));
                }
                if (update && l == 0) {
                    RT_CUDA(cudaStreamWaitEvent(m->opt_stream, P.ev_ready[c], 0));
                    if (m->comm) RT_CUDA(cudaStreamWaitEvent(m->opt_stream, P.ev_comm[c], 0));
                    RT_TRY(enqueue_update_rows(m, P, r0, r1, m->opt_stream));
                    RT_CUDA(cudaEventRecord(P.ev_opt[c], m->opt_stream));
                    RT_TRY(gather_weights(P, c, r0, r1));
                }
            }
            // Sharded optimiser: the previous layer's weight all-gathers go on
            // the comm stream only now, behind this layer's reduce-scatters.
            // Enqueued earlier, they would hold this layer's gradient sums
            // until the previous layer's dX GEMM and updates were done.
            if (l + 1 < nl && !m->ag_stream) RT_TRY(gather_layer(m->L[l + 1]));
            if (l > 0) {
                // delta_l was complete when this layer's chunk 0 passed its wait,
                // and no running GEMM writes W_l or the mask
                RT_TRY(dx_gemm(l, PDL_NO_WAIT));
                if (update) {
                    RT_CUDA(cudaEventRecord(P.ev_dx, st));
                    RT_CUDA(cudaStreamWaitEvent(m->opt_stream, P.ev_dx, 0));
                    for (int c = 0; c < P.chunks; ++c) {
                        const int64_t r0 = chunk_row_of(rows, P.chunks, c), r1 = chunk_row_of(rows, P.chunks, c + 1);
                        if (m->comm) RT_CUDA(cudaStreamWaitEvent(m->opt_stream, P.ev_comm[c], 0));
                        RT_TRY(enqueue_update_rows(m, P, r0, r1, m->opt_stream));
                        RT_CUDA(cudaEventRecord(P.ev_opt[c], m->opt_stream));
                    }
                    if (m->ag_stream) RT_TRY(gather_layer(P));  // own queue: right away
                }
            }
        }
        for (PlanLayer& P : m->L)
            for (int c = 0; c < P.chunks; ++c) {
                if (m->sharded)
                    RT_CUDA(cudaStreamWaitEvent(st, P.ev_ag[c], 0));
                else if (update)
                    RT_CUDA(cudaStreamWaitEvent(st, P.ev_opt[c], 0));
                else if (m->comm)
                    RT_CUDA(cudaStreamWaitEvent(st, P.ev_comm[c], 0));
            }
        if (update) RT_TRY(mark(m->cfg.optimizer == RT_OPT_ADAM ? "adam_tail" : "sgd_tail", 0));
        return RT_OK;
    }
};

void set_fuse_opt(rt_mlp* m) {
    const char* e = getenv("RTGPU_FUSED_OPT");
    m->fuse_opt = !m->comm && m->cfg.optimizer != RT_OPT_NONE && !(e && e[0] == '0');
}

// Peer-memory reduce-scatter for the sharded optimiser (RTGPU_P2P_RS=1):
// every layer whose dW chunks take the one-slice tensor-core GEMM and split
// into equal row ranges per rank gets a receive buffer, mapped into every
// rank's process; its dW GEMM then scatters rows to their owners itself and
// the layer's NCCL reduce-scatters become a barrier plus the owner's sum.
// Collective: every rank takes the same decisions in the same order, and a
// layer whose buffers some rank could not map stays on NCCL everywhere.
int setup_p2p(rt_mlp* m) {
    const char* e = getenv("RTGPU_P2P_RS");
    if (!m->sharded || !(e && e[0] == '1') || m->world > kMaxPeers) return RT_OK;
    Enqueuer q{m, m->ctx->stream, 0, false};
    for (size_t l = 0; l < m->L.size(); ++l) {
        PlanLayer& P = m->L[l];
        bool ok = P.d % m->world == 0;
        for (int c = 0; ok && c < P.chunks; ++c) {
            const int64_t r0 = chunk_row_of(P.d + 1, P.chunks, c), r1 = chunk_row_of(P.d + 1, P.chunks, c + 1);
            const int64_t end = shard_end(P, r1);
            ok = end > r0 && (end - r0) % m->world == 0 && gemm_p2p_capable(m->ctx, q.dw_desc(P, (int)l, r0, r1));
        }
        if (!ok) continue;
        if (!P.recv) RT_TRY(dalloc_t(m, &P.recv, (size_t)P.d * P.ld));
        const int shared = comm_share_buffer(m->comm, P.recv, P.peers);
        int st = RT_OK;
        const bool everywhere = comm_all_true(m->comm, shared == RT_OK, m->scratch, &st);
        RT_TRY(st);
        if (!everywhere) {
            if (shared == RT_OK) comm_unshare_buffer(m->comm, P.peers);
            continue;
        }
        P.p2p = true;
    }
    return RT_OK;
}

// Copy-engine exchange for the sharded optimiser (the default; RTGPU_CE_EXCHANGE=0
// keeps NCCL's reduce-scatter and all-gather): every layer whose chunks split
// into equal flat pieces per rank gets a receive buffer, and that buffer and
// the layer's bf16 shadow are mapped into every rank's process.  Collective:
// every rank takes the same decisions in the same order, and a layer that
// some rank could not map stays on NCCL everywhere.
int setup_ce(rt_mlp* m) {
    const char* e = getenv("RTGPU_CE_EXCHANGE");
    // RTGPU_CE_MAX_WORLD (default 2): the largest world that uses copy engines.  Each chunk costs world - 1
    // copies each way plus two barriers; on 2 B200s that beat NCCL's reduce-scatter (8.20 against 8.48 ms
    // per step), on 4 and 8 the queued copies trailed the last GEMM by 1.2 and 2.1 ms.
    const char* w = getenv("RTGPU_CE_MAX_WORLD");
    const int max_world = w && w[0] ? atoi(w) : 2;
    if (!m->sharded || !m->ag_stream || (e && e[0] == '0') || m->world > kMaxPeers || m->world > max_world)
        return RT_OK;
    for (PlanLayer& P : m->L) {
        if (P.p2p || !P.w16) continue;
        bool ok = (P.d * P.ld) % m->world == 0;
        P.ce_off.assign(P.chunks, 0);
        int64_t off = 0;
        for (int c = 0; ok && c < P.chunks; ++c) {
            const int64_t r0 = chunk_row_of(P.d + 1, P.chunks, c), end = shard_end(P, chunk_row_of(P.d + 1, P.chunks, c + 1));
            if (end <= r0) continue;
            ok = ((end - r0) * P.ld) % m->world == 0;
            P.ce_off[c] = off;
            off += (end - r0) * P.ld / m->world;
        }
        if (!ok) continue;
        if (!P.ce_recv) RT_TRY(dalloc_t(m, &P.ce_recv, (size_t)P.d * P.ld));
        const int a = comm_share_buffer(m->comm, P.ce_recv, P.ce_peers);
        const int b = comm_share_buffer(m->comm, P.w16, P.w16_peers);
        int st = RT_OK;
        const bool everywhere = comm_all_true(m->comm, a == RT_OK && b == RT_OK, m->scratch, &st);
        RT_TRY(st);
        if (!everywhere) {
            if (a == RT_OK) comm_unshare_buffer(m->comm, P.ce_peers);
            if (b == RT_OK) comm_unshare_buffer(m->comm, P.w16_peers);
            continue;
        }
        P.ce = true;
    }
    bool any = false;
    for (const PlanLayer& P : m->L) any = any || P.ce;
    if (any && !m->ce_fork) {
        RT_CUDA(cudaEventCreateWithFlags(&m->ce_fork, cudaEventDisableTiming));
        RT_CUDA(cudaEventCreateWithFlags(&m->ce_fork2, cudaEventDisableTiming));
        for (int q = 0; q < m->world; ++q) {
            RT_CUDA(cudaStreamCreateWithFlags(&m->ce_scatter[q], cudaStreamNonBlocking));
            RT_CUDA(cudaStreamCreateWithFlags(&m->ce_pull[q], cudaStreamNonBlocking));
            RT_CUDA(cudaEventCreateWithFlags(&m->ce_join[q], cudaEventDisableTiming));
            RT_CUDA(cudaEventCreateWithFlags(&m->ce_join2[q], cudaEventDisableTiming));
        }
    }
    return RT_OK;
}

// Chunks of each layer's dW GEMM: the first layer always (its update would
// otherwise trail the step), and under data parallelism every layer with at
// least 128 MB of gradients (its sum starts a chunk after the GEMM does;
// smaller layers lose more to the narrower GEMMs than the overlap gains); 4
// chunks for >= 4096 rows, 2 for >= 2048.  RTGPU_FIRST_LAYER_CHUNKS /
// RTGPU_DW_CHUNKS override.
int dw_chunks(size_t layer, int64_t d, int64_t ld, bool data_parallel, bool fused_update) {
    auto rule = [](int64_t rows) { return rows >= 4096 ? 4 : rows >= 2048 ? 2 : 1; };
    const char* env0 = getenv("RTGPU_FIRST_LAYER_CHUNKS");
    const char* envd = getenv("RTGPU_DW_CHUNKS");
    const int64_t rows = d + 1;
    int ch = 1;
    if (layer == 0 && !fused_update) ch = env0 && env0[0] ? atoi(env0) : rule(rows);
    else if (data_parallel) ch = envd && envd[0] ? atoi(envd) : rows * ld * 4 >= (128ll << 20) ? rule(rows) : 1;
    if (ch < 1) ch = 1;
    if (ch > 8) ch = 8;
    while (ch > 1 && chunk_row_of(rows, ch, 1) == 0) --ch;  // every chunk non-empty
    return ch;
}

int prepare_chunks(rt_mlp* m) {
    for (size_t l = 0; l < m->L.size(); ++l) {
        PlanLayer& P = m->L[l];
        const int ch = dw_chunks(l, P.d, P.ld, m->comm != nullptr, m->fuse_opt);
        if (ch == P.chunks && !P.ev_ready.empty()) continue;
        for (auto e : P.ev_ready) cudaEventDestroy(e);
        for (auto e : P.ev_comm) cudaEventDestroy(e);
        for (auto e : P.ev_opt) cudaEventDestroy(e);
        for (auto e : P.ev_ag) cudaEventDestroy(e);
        P.chunks = ch;
        P.ev_ready.assign(ch, nullptr);
        P.ev_comm.assign(ch, nullptr);
        P.ev_opt.assign(ch, nullptr);
        P.ev_ag.assign(ch, nullptr);
        for (int c = 0; c < ch; ++c)
            if (cudaEventCreateWithFlags(&P.ev_ready[c], cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&P.ev_comm[c], cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&P.ev_opt[c], cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&P.ev_ag[c], cudaEventDisableTiming) != cudaSuccess)
                return fail(RT_ERR_CUDA, "event creation failed");
        if (!P.ev_dx && cudaEventCreateWithFlags(&P.ev_dx, cudaEventDisableTiming) != cudaSuccess)
            return fail(RT_ERR_CUDA, "event creation failed");
    }
    return RT_OK;
}

int capture_step(rt_mlp* m, int s) {
    cudaStream_t st = m->ctx->stream;
    Slot& S = m->slot[s];
    if (S.exec) {
        cudaGraphExecDestroy(S.exec);
        S.exec = nullptr;
    }
    if (S.graph) {
        cudaGraphDestroy(S.graph);
        S.graph = nullptr;
    }
    uint64_t before = m->ctx->launches;
    RT_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    m->ctx->plan_pdl = m->ctx->pdl;
    Enqueuer q{m, st, s, false};
    int rc = q.begin();
    if (rc == RT_OK) rc = q.forward();
    if (rc == RT_OK) rc = q.backward_and_update();
    m->ctx->plan_pdl = false;
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (rc != RT_OK) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, "step capture failed: %s", cudaGetErrorString(e));
    S.graph = graph;
    RT_CUDA(cudaGraphInstantiate(&S.exec, graph, cudaGraphInstantiateFlagUseNodePriority));
    m->kernels_per_step = (int)(m->ctx->launches - before);
    S.timed = m->timing;
    return RT_OK;
}

int launch_slot(rt_mlp* m, int s) {
    Slot& S = m->slot[s];
    if (!S.exec || S.timed != m->timing) RT_TRY(capture_step(m, s));
    RT_CUDA(cudaGraphLaunch(S.exec, m->ctx->stream));
    RT_CUDA(cudaEventRecord(S.free_, m->ctx->stream));
    m->ctx->launches += (uint64_t)m->kernels_per_step;
    m->last_slot = s;
    return RT_OK;
}

// The forward pass of slot s as a CUDA graph (captured on first use).
int launch_forward(rt_mlp* m, int s) {
    Slot& S = m->slot[s];
    cudaStream_t st = m->ctx->stream;
    if (!S.fwd_exec) {
        uint64_t before = m->ctx->launches;
        RT_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        m->ctx->plan_pdl = m->ctx->pdl;
        Enqueuer q{m, st, s, true};
        int rc = q.forward();
        m->ctx->plan_pdl = false;
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (rc != RT_OK) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (e != cudaSuccess) return fail(RT_ERR_CUDA, "forward capture failed: %s", cudaGetErrorString(e));
        S.fwd_graph = graph;
        RT_CUDA(cudaGraphInstantiate(&S.fwd_exec, graph, 0));
        m->kernels_per_forward = (int)(m->ctx->launches - before);
    }
    RT_CUDA(cudaGraphLaunch(S.fwd_exec, st));
    RT_CUDA(cudaEventRecord(S.free_, st));
    m->ctx->launches += (uint64_t)m->kernels_per_forward;
    m->last_slot = s;
    return RT_OK;
}

// Copies one batch into slot s on stream st (x columns 0..d0-1; the ones
// column stays).
int fill_slot(rt_mlp* m, int s, const void* x, rt_dtype xdt, const uint32_t* labels, cudaMemcpyKind kind,
              cudaStream_t st) {
    Slot& S = m->slot[s];
    const int64_t d0 = m->dims[0];
    RT_CHECK(xdt == RT_F32 || xdt == RT_BF16, "x dtype must be RT_F32 or RT_BF16");
    if (xdt == m->adt) {
        size_t es = dtype_size(xdt);
        RT_CUDA(cudaMemcpy2DAsync(S.x, m->ldx * es, x, d0 * es, d0 * es, m->n, kind, st));
    } else {
        const void* src = x;
        if (kind == cudaMemcpyHostToDevice) {
            size_t bytes = (size_t)m->n * d0 * dtype_size(xdt);
            if (S.stage_bytes < bytes) {
                if (S.stage) cudaFree(S.stage);
                S.stage = nullptr;
                S.stage_bytes = 0;
                RT_CUDA(cudaMalloc(&S.stage, bytes));
                S.stage_bytes = bytes;
            }
            RT_CUDA(cudaMemcpyAsync(S.stage, x, bytes, kind, st));
            src = S.stage;
        }
        RT_TRY(launch_cast(m->ctx, src, xdt, d0, S.x, m->adt, m->ldx, m->n, d0, st));
    }
    RT_CUDA(cudaMemcpyAsync(S.labels, labels, (size_t)m->n * 4, kind, st));
    return RT_OK;
}

int read_packed(rt_mlp* m, const void* src, rt_dtype dt, int64_t rows, int64_t cols, int64_t ld, float* host) {
    cudaStream_t st = m->ctx->stream;
    if (dt == RT_F32) {
        RT_CUDA(cudaMemcpy2DAsync(host, cols * 4, src, ld * 4, cols * 4, rows, cudaMemcpyDeviceToHost, st));
    } else {
        float* tmp = nullptr;
        RT_CUDA(cudaMallocAsync((void**)&tmp, (size_t)rows * cols * 4, st));
        RT_TRY(launch_cast(m->ctx, src, dt, ld, tmp, RT_F32, cols, rows, cols, st));
        RT_CUDA(cudaMemcpyAsync(host, tmp, (size_t)rows * cols * 4, cudaMemcpyDeviceToHost, st));
        RT_CUDA(cudaFreeAsync(tmp, st));
    }
    RT_CUDA(cudaStreamSynchronize(st));
    return RT_OK;
}

// Sharded optimiser: completes a [d+1, ld] f32 buffer of layer P (masters,
// moments or reduced gradients, of which each rank holds its slices) by an
// in-place all-gather of every chunk's weight rows.  Collective: every rank
// calls it, in the same order.
int gather_block(rt_mlp* m, PlanLayer& P, float* buf) {
    if (!m->sharded || !buf) return RT_OK;
    cudaStream_t st = m->ctx->stream;
    for (int c = 0; c < P.chunks; ++c) {
        const int64_t r0 = chunk_row_of(P.d + 1, P.chunks, c);
        const int64_t e = shard_end(P, chunk_row_of(P.d + 1, P.chunks, c + 1));
        if (e > r0) RT_TRY(comm_all_gather(m->comm, buf + r0 * P.ld, (e - r0) * P.ld / m->world, 4, st));
    }
    return RT_OK;
}

int refresh_shadow(rt_mlp* m, PlanLayer& P, cudaStream_t st) {
    if (m->adt != RT_BF16) return RT_OK;
    return launch_cast(m->ctx, P.w32, RT_F32, P.ld, P.w16, RT_BF16, P.ld, P.d + 1, P.ld, st);
}

}  // namespace

extern "C" {

int64_t rt_plan_ld(int64_t units) { return units < 1 ? 0 : plan_ld(units); }

int rt_plan_dw_chunks(int layer, int64_t d, int64_t units, int data_parallel, int fused_update) {
    if (layer < 0 || d < 1 || units < 1) return 0;
    return dw_chunks((size_t)layer, d, plan_ld(units), data_parallel != 0, fused_update != 0);
}

int64_t rt_plan_chunk_row(int64_t rows, int chunks, int c) {
    if (rows < 0 || chunks < 1 || c < 0) return -1;
    return chunk_row_of(rows, chunks, c);
}

int64_t rt_plan_shard_slice(int64_t d, int64_t units, int64_t r0, int64_t r1, int world, int rank, int64_t* offset) {
    if (!offset || d < 1 || units < 1 || world < 1 || rank < 0 || rank >= world || r0 < 0 || r1 < r0) return -1;
    return shard_slice(d, plan_ld(units), r0, r1, world, rank, offset);
}

int rt_mlp_create(rt_ctx* ctx, const rt_mlp_config* cfg, const float* const* weights, const float* const* biases,
                  rt_mlp** out) {
    RT_CHECK(ctx && cfg && out && weights, "rt_mlp_create: bad arguments");
    RT_CHECK(cfg->n_layers >= 1 && cfg->dims, "rt_mlp_create: model without layers");
    RT_CHECK(cfg->batch >= 1, "rt_mlp_create: batch must be >= 1");
    RT_CHECK(cfg->dtype == RT_F32 || cfg->dtype == RT_BF16, "rt_mlp_create: dtype must be RT_F32 or RT_BF16");
    RT_CHECK(cfg->optimizer >= RT_OPT_NONE && cfg->optimizer <= RT_OPT_ADAM, "rt_mlp_create: unknown optimizer");
    RT_CHECK(cfg->activations == RT_ACT_SPLIT || cfg->activations == RT_ACT_BF16,
             "rt_mlp_create: unknown activations mode %d", (int)cfg->activations);
    for (int l = 0; l <= cfg->n_layers; ++l) RT_CHECK(cfg->dims[l] >= 1, "rt_mlp_create: dims[%d] < 1", l);
    for (int l = 0; l < cfg->n_layers; ++l) RT_CHECK(weights[l] != nullptr, "rt_mlp_create: weights[%d] is NULL", l);
    RT_CUDA(cudaSetDevice(ctx->device));
    rt_mlp* m = new rt_mlp;
    m->ctx = ctx;
    m->cfg = *cfg;
    m->dims.assign(cfg->dims, cfg->dims + cfg->n_layers + 1);
    m->cfg.dims = m->dims.data();
    m->adt = cfg->dtype;
    m->split_act = m->adt == RT_BF16 && cfg->activations == RT_ACT_SPLIT;
    m->n = cfg->batch;
    const size_t es = dtype_size(m->adt);
    const int nl = cfg->n_layers;
    int s = RT_OK;
    auto bail = [&](int code) {
        free_all(m);
        delete m;
        return code;
    };

    m->ldx = round64(m->dims[0] + 1);
    for (auto& S : m->slot) {
        if ((s = dalloc(m, &S.x, (size_t)m->n * m->ldx * es))) return bail(s);
        if ((s = dalloc_t(m, &S.labels, (size_t)m->n))) return bail(s);
        if ((s = launch_fill_column(ctx, S.x, m->adt, m->n, m->ldx, m->dims[0], 1.0f, ctx->stream)))
            return bail(s);
        if (cudaEventCreateWithFlags(&S.ready, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&S.free_, cudaEventDisableTiming) != cudaSuccess)
            return bail(fail(RT_ERR_CUDA, "event creation failed"));
    }
    if (cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&m->opt_stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(RT_ERR_CUDA, "stream creation failed"));
    if ((s = dalloc_t(m, &m->loss_rows, (size_t)m->n))) return bail(s);
    if ((s = dalloc_t(m, &m->opt, 1))) return bail(s);
    if ((s = dalloc_t(m, &m->tile_ctrs, rt_mlp::kTileCtrs))) return bail(s);
    m->L.resize(nl);
    for (int l = 0; l < nl; ++l) {
        PlanLayer& P = m->L[l];
        P.d = m->dims[l];
        P.u = m->dims[l + 1];
        P.ld = plan_ld(P.u);
        bool last = l == nl - 1;
        P.ld_act = last ? P.ld : round64(P.u + 1);
        size_t pn = (size_t)(P.d + 1) * P.ld;
        if ((s = dalloc_t(m, &P.w32, pn))) return bail(s);
        if ((s = dalloc_t(m, &P.g, pn))) return bail(s);
        P.b = P.w32 + P.d * P.ld;
        P.db = P.g + P.d * P.ld;
        if (cfg->optimizer == RT_OPT_ADAM) {
            if ((s = dalloc_t(m, &P.m, pn))) return bail(s);
            if ((s = dalloc_t(m, &P.v, pn))) return bail(s);
        }
        if (m->adt == RT_BF16 && (s = dalloc_t(m, &P.w16, pn))) return bail(s);
        if ((s = dalloc(m, &P.act, (size_t)m->n * P.ld_act * (last ? 4 : es)))) return bail(s);
        if (l + 2 < nl && m->split_act && (s = dalloc(m, &P.act_lo, (size_t)m->n * P.ld_act * es)))
            return bail(s);
        if (!last && (s = launch_fill_column(ctx, P.act, m->adt, m->n, P.ld_act, P.u, 1.0f, ctx->stream)))
            return bail(s);
        if ((s = dalloc(m, &P.delta, (size_t)m->n * P.ld * es))) return bail(s);
        if (cudaMemcpy2DAsync(P.w32, P.ld * 4, weights[l], P.u * 4, P.u * 4, P.d, cudaMemcpyHostToDevice,
                              ctx->stream) != cudaSuccess)
            return bail(fail(RT_ERR_CUDA, "weight upload failed"));
        if (biases && biases[l] &&
            cudaMemcpyAsync(P.b, biases[l], (size_t)P.u * 4, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess)
            return bail(fail(RT_ERR_CUDA, "bias upload failed"));
        if ((s = refresh_shadow(m, P, ctx->stream))) return bail(s);
        // split-K for the dW GEMM when its output tiles cannot fill the GPU
        // (the library's rule; the output layer's narrow-N dW slices the same way)
        int split = choose_split_k(ctx, P.d + 1, P.u, m->n, m->adt);
        if (P.u <= kSkinnyMax) {
            // the skinny dW kernel: up to 64 k slices of >= 32 rows (its threads are latency bound)
            int64_t sp = m->n / 32;
            split = (int)(sp < 1 ? 1 : sp > 64 ? 64 : sp);
        }
        P.split_dw = split;
        if (split > 1) {
            P.ws_bytes = (size_t)split * (P.d + 1) * P.u * 4;
            if ((s = dalloc(m, (void**)&P.ws, P.ws_bytes))) return bail(s);
        }
    }
    if (m->adt == RT_F32 && ctx->fast_gemm && ctx->f32_tensor) {
        size_t need = 0;
        for (int l = 0; l < nl; ++l) {
            const PlanLayer& P = m->L[l];
            GemmDesc f{}, w{}, x{};
            f.layout = RT_NN, f.m = m->n, f.n = P.u, f.k = P.d;      // forward
            w.layout = RT_TN, w.m = P.d + 1, w.n = P.u, w.k = m->n;  // [dW; db]
            x.layout = RT_NT, x.m = m->n, x.n = P.d, x.k = P.u;      // dX
            for (const GemmDesc* g : {&f, &w, &x}) {
                size_t b = gemm_x3_workspace_bytes(*g);
                if (b > need) need = b;
            }
        }
        if ((s = dalloc(m, (void**)&m->x3_ws, need))) return bail(s);
        m->x3_ws_bytes = need;
    }
    set_fuse_opt(m);
    if ((s = prepare_chunks(m))) return bail(s);
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return bail(fail(RT_ERR_CUDA, "plan setup sync failed"));
    *out = m;
    return RT_OK;
}

int rt_mlp_destroy(rt_mlp* m) {
    if (!m) return RT_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->copy_stream) cudaStreamSynchronize(m->copy_stream);
    free_all(m);
    delete m;
    return RT_OK;
}

int rt_mlp_step(rt_mlp* m, const void* x_dev, rt_dtype x_dtype, const uint32_t* labels_dev) {
    RT_CHECK(m && x_dev && labels_dev, "rt_mlp_step: bad arguments");
    int s = m->next_slot;
    m->next_slot ^= 1;
    // device inputs: copy on the compute stream (GpuMlp::carregar, gpu/mod.rs:1486-1495)
    RT_TRY(fill_slot(m, s, x_dev, x_dtype, labels_dev, cudaMemcpyDeviceToDevice, m->ctx->stream));
    return launch_slot(m, s);
}

int rt_mlp_step_host(rt_mlp* m, const void* x_host, rt_dtype x_dtype, const uint32_t* labels_host,
                     float* loss_rows_host) {
    RT_CHECK(m && x_host && labels_host, "rt_mlp_step_host: bad arguments");
    int s = m->next_slot;
    m->next_slot ^= 1;
    Slot& S = m->slot[s];
    // The copy stream refills slot s once the step that last read it is done,
    // overlapping the step that is running on the other slot.
    RT_CUDA(cudaStreamWaitEvent(m->copy_stream, S.free_, 0));
    RT_TRY(fill_slot(m, s, x_host, x_dtype, labels_host, cudaMemcpyHostToDevice, m->copy_stream));
    RT_CUDA(cudaEventRecord(S.ready, m->copy_stream));
    RT_CUDA(cudaStreamWaitEvent(m->ctx->stream, S.ready, 0));
    RT_TRY(launch_slot(m, s));
    if (loss_rows_host)
        RT_CUDA(cudaMemcpyAsync(loss_rows_host, m->loss_rows, (size_t)m->n * 4, cudaMemcpyDeviceToHost,
                                m->ctx->stream));
    return RT_OK;
}

int rt_mlp_forward_only(rt_mlp* m, const void* x_dev, rt_dtype x_dtype) {
    RT_CHECK(m && x_dev, "rt_mlp_forward_only: bad arguments");
    RT_CHECK(x_dtype == RT_F32 || x_dtype == RT_BF16, "x dtype must be RT_F32 or RT_BF16");
    const int64_t d0 = m->dims[0];
    cudaStream_t st = m->ctx->stream;
    int s = m->next_slot;
    m->next_slot ^= 1;
    Slot& S = m->slot[s];
    if (x_dtype == m->adt) {
        size_t es = dtype_size(x_dtype);
        RT_CUDA(cudaMemcpy2DAsync(S.x, m->ldx * es, x_dev, d0 * es, d0 * es, m->n, cudaMemcpyDeviceToDevice, st));
    } else {
        RT_TRY(launch_cast(m->ctx, x_dev, x_dtype, d0, S.x, m->adt, m->ldx, m->n, d0, st));
    }
    return launch_forward(m, s);
}

int rt_mlp_forward_host(rt_mlp* m, const void* x_host, rt_dtype x_dtype, float* logits_host) {
    RT_CHECK(m && x_host, "rt_mlp_forward_host: bad arguments");
    RT_CHECK(x_dtype == RT_F32 || x_dtype == RT_BF16, "x dtype must be RT_F32 or RT_BF16");
    int s = m->next_slot;
    m->next_slot ^= 1;
    Slot& S = m->slot[s];
    const int64_t d0 = m->dims[0];
    // the copy stream refills slot s once the work that last read it is done
    RT_CUDA(cudaStreamWaitEvent(m->copy_stream, S.free_, 0));
    if (x_dtype == m->adt) {
        size_t es = dtype_size(x_dtype);
        RT_CUDA(cudaMemcpy2DAsync(S.x, m->ldx * es, x_host, d0 * es, d0 * es, m->n, cudaMemcpyHostToDevice,
                                  m->copy_stream));
    } else {
        size_t bytes = (size_t)m->n * d0 * dtype_size(x_dtype);
        if (S.stage_bytes < bytes) {
            RT_CUDA(cudaStreamSynchronize(m->copy_stream));
            if (S.stage) cudaFree(S.stage);
            S.stage = nullptr;
            S.stage_bytes = 0;
            RT_CUDA(cudaMalloc(&S.stage, bytes));
            S.stage_bytes = bytes;
        }
        RT_CUDA(cudaMemcpyAsync(S.stage, x_host, bytes, cudaMemcpyHostToDevice, m->copy_stream));
        RT_TRY(launch_cast(m->ctx, S.stage, x_dtype, d0, S.x, m->adt, m->ldx, m->n, d0, m->copy_stream));
    }
    RT_CUDA(cudaEventRecord(S.ready, m->copy_stream));
    RT_CUDA(cudaStreamWaitEvent(m->ctx->stream, S.ready, 0));
    RT_TRY(launch_forward(m, s));
    if (logits_host) {
        const PlanLayer& P = m->L.back();
        RT_CUDA(cudaMemcpy2DAsync(logits_host, P.u * 4, P.act, P.ld * 4, P.u * 4, m->n, cudaMemcpyDeviceToHost,
                                  m->ctx->stream));
    }
    return RT_OK;
}

int rt_mlp_logits(rt_mlp* m, float* host) {
    RT_CHECK(m && host, "bad arguments");
    PlanLayer& P = m->L.back();
    return read_packed(m, P.act, RT_F32, m->n, P.u, P.ld, host);
}

int rt_mlp_last_loss(rt_mlp* m, float* out) {
    RT_CHECK(m && out, "bad arguments");
    std::vector<float> rows((size_t)m->n);
    RT_TRY(read_packed(m, m->loss_rows, RT_F32, 1, m->n, m->n, rows.data()));
    // mean_all (tensor.rs:279-286): sequential f32 sum, then / len.
    float sum = 0.0f;
    for (float v : rows) sum += v;
    *out = sum / (float)m->n;
    return rt_ctx_sync(m->ctx);
}

int rt_mlp_global_loss(rt_mlp* m, float* out) {
    RT_CHECK(m && out, "bad arguments");
    if (!m->comm || m->world == 1) return rt_mlp_last_loss(m, out);
    // All-gather the ranks' per-row losses (rank r holds rows [r*n, (r+1)*n)
    // of the global batch), then mean_all's sequential f32 sum over the
    // global batch in row order: the single-device loss, bit for bit.
    cudaStream_t st = m->ctx->stream;
    const int64_t n = m->n, total = n * m->world;
    if (!m->loss_all) RT_TRY(dalloc_t(m, &m->loss_all, (size_t)total));
    RT_CUDA(cudaMemcpyAsync(m->loss_all + (int64_t)m->rank * n, m->loss_rows, (size_t)n * 4,
                            cudaMemcpyDeviceToDevice, st));
    RT_TRY(comm_all_gather(m->comm, m->loss_all, n, 4, st));
    std::vector<float> rows((size_t)total);
    RT_TRY(read_packed(m, m->loss_all, RT_F32, 1, total, total, rows.data()));
    float sum = 0.0f;
    for (float v : rows) sum += v;
    *out = sum / (float)total;
    return RT_OK;
}

int rt_mlp_weights(rt_mlp* m, int layer, float* w, float* b) {
    RT_CHECK(m && layer >= 0 && layer < (int)m->L.size(), "bad layer index");
    PlanLayer& P = m->L[layer];
    if (w) RT_TRY(gather_block(m, P, P.w32));
    if (w) RT_TRY(read_packed(m, P.w32, RT_F32, P.d, P.u, P.ld, w));
    if (b) RT_TRY(read_packed(m, P.b, RT_F32, 1, P.u, P.u, b));
    return RT_OK;
}

int rt_mlp_grads(rt_mlp* m, int layer, float* dw, float* db) {
    RT_CHECK(m && layer >= 0 && layer < (int)m->L.size(), "bad layer index");
    PlanLayer& P = m->L[layer];
    if (dw) RT_TRY(gather_block(m, P, P.g));
    if (dw) RT_TRY(read_packed(m, P.g, RT_F32, P.d, P.u, P.ld, dw));
    if (db) RT_TRY(read_packed(m, P.db, RT_F32, 1, P.u, P.u, db));
    return rt_ctx_sync(m->ctx);
}

int rt_mlp_set_weights(rt_mlp* m, int layer, const float* w, const float* b) {
    RT_CHECK(m && layer >= 0 && layer < (int)m->L.size(), "bad layer index");
    PlanLayer& P = m->L[layer];
    cudaStream_t st = m->ctx->stream;
    if (w) RT_CUDA(cudaMemcpy2DAsync(P.w32, P.ld * 4, w, P.u * 4, P.u * 4, P.d, cudaMemcpyHostToDevice, st));
    if (b) RT_CUDA(cudaMemcpyAsync(P.b, b, (size_t)P.u * 4, cudaMemcpyHostToDevice, st));
    RT_TRY(refresh_shadow(m, P, st));
    RT_CUDA(cudaStreamSynchronize(st));
    return RT_OK;
}

}  // extern "C"

namespace {

// Byte size of the state buffer and, when `blocks` is non-null, each layer's
// block sizes in floats.
size_t state_bytes(const rt_mlp* m) {
    size_t b = sizeof(rt_mlp_state_header) + sizeof(int64_t) * m->dims.size();
    const size_t per = m->cfg.optimizer == RT_OPT_ADAM ? 3 : 1;
    for (const PlanLayer& P : m->L) b += per * (size_t)(P.d + 1) * P.u * sizeof(float);
    return b;
}

// Copies the [d+1, u] block of a [d+1, ld] device buffer to or from packed host memory.
int copy_block(rt_mlp* m, const PlanLayer& P, float* dev, uint8_t* host, bool to_host) {
    cudaStream_t st = m->ctx->stream;
    if (to_host)
        RT_CUDA(cudaMemcpy2DAsync(host, P.u * 4, dev, P.ld * 4, P.u * 4, P.d + 1, cudaMemcpyDeviceToHost, st));
    else
        RT_CUDA(cudaMemcpy2DAsync(dev, P.ld * 4, host, P.u * 4, P.u * 4, P.d + 1, cudaMemcpyHostToDevice, st));
    return RT_OK;
}

}  // namespace

extern "C" {

int rt_mlp_state_size(rt_mlp* m, size_t* bytes) {
    RT_CHECK(m && bytes, "rt_mlp_state_size: bad arguments");
    *bytes = state_bytes(m);
    return RT_OK;
}

int rt_mlp_save_state(rt_mlp* m, void* host, size_t bytes) {
    RT_CHECK(m && host, "rt_mlp_save_state: bad arguments");
    RT_CHECK(bytes >= state_bytes(m), "rt_mlp_save_state: buffer of %zu bytes, state needs %zu", bytes,
             state_bytes(m));
    cudaStream_t st = m->ctx->stream;
    RT_CUDA(cudaStreamSynchronize(st));  // the last step (and its side-stream updates) are done
    OptScalars sc{};
    RT_CUDA(cudaMemcpy(&sc, m->opt, sizeof(sc), cudaMemcpyDeviceToHost));
    uint8_t* p = static_cast<uint8_t*>(host);
    rt_mlp_state_header h{};
    h.magic = RT_MLP_STATE_MAGIC;
    h.version = 1;
    h.n_layers = (int32_t)m->L.size();
    h.optimizer = m->cfg.optimizer;
    h.adam_step = sc.t;
    std::memcpy(p, &h, sizeof(h));
    p += sizeof(h);
    std::memcpy(p, m->dims.data(), sizeof(int64_t) * m->dims.size());
    p += sizeof(int64_t) * m->dims.size();
    for (PlanLayer& P : m->L) {
        RT_TRY(gather_block(m, P, P.w32));
        RT_TRY(gather_block(m, P, P.m));
        RT_TRY(gather_block(m, P, P.v));
    }
    for (PlanLayer& P : m->L) {
        const size_t blk = (size_t)(P.d + 1) * P.u * 4;
        RT_TRY(copy_block(m, P, P.w32, p, true));
        p += blk;
        if (m->cfg.optimizer == RT_OPT_ADAM) {
            RT_TRY(copy_block(m, P, P.m, p, true));
            p += blk;
            RT_TRY(copy_block(m, P, P.v, p, true));
            p += blk;
        }
    }
    RT_CUDA(cudaStreamSynchronize(st));
    return RT_OK;
}

int rt_mlp_load_state(rt_mlp* m, const void* host, size_t bytes) {
    RT_CHECK(m && host, "rt_mlp_load_state: bad arguments");
    RT_CHECK(bytes >= sizeof(rt_mlp_state_header), "rt_mlp_load_state: buffer too small for a header");
    const uint8_t* p = static_cast<const uint8_t*>(host);
    rt_mlp_state_header h;
    std::memcpy(&h, p, sizeof(h));
    RT_CHECK(h.magic == RT_MLP_STATE_MAGIC && h.version == 1, "rt_mlp_load_state: not a version-1 plan state");
    RT_CHECK(h.n_layers == (int32_t)m->L.size(), "rt_mlp_load_state: state has %d layers, plan %d", h.n_layers,
             (int)m->L.size());
    RT_CHECK(h.optimizer == m->cfg.optimizer, "rt_mlp_load_state: state optimiser %d, plan %d", h.optimizer,
             (int)m->cfg.optimizer);
    RT_CHECK(bytes >= state_bytes(m), "rt_mlp_load_state: buffer of %zu bytes, state needs %zu", bytes,
             state_bytes(m));
    p += sizeof(h);
    for (size_t l = 0; l < m->dims.size(); ++l) {
        int64_t d;
        std::memcpy(&d, p + l * sizeof(int64_t), sizeof(d));
        RT_CHECK(d == m->dims[l], "rt_mlp_load_state: dims[%zu] is %lld in the state, %lld in the plan", l,
                 (long long)d, (long long)m->dims[l]);
    }
    p += sizeof(int64_t) * m->dims.size();
    cudaStream_t st = m->ctx->stream;
    RT_CUDA(cudaStreamSynchronize(st));
    for (PlanLayer& P : m->L) {
        const size_t blk = (size_t)(P.d + 1) * P.u * 4;
        RT_TRY(copy_block(m, P, P.w32, const_cast<uint8_t*>(p), false));
        p += blk;
        if (m->cfg.optimizer == RT_OPT_ADAM) {
            RT_TRY(copy_block(m, P, P.m, const_cast<uint8_t*>(p), false));
            p += blk;
            RT_TRY(copy_block(m, P, P.v, const_cast<uint8_t*>(p), false));
            p += blk;
        }
        RT_TRY(refresh_shadow(m, P, st));
    }
    OptScalars sc{};
    sc.t = (int)h.adam_step;  // the next step recomputes the bias corrections from t + 1
    RT_CUDA(cudaMemcpyAsync(m->opt, &sc, sizeof(sc), cudaMemcpyHostToDevice, st));
    RT_CUDA(cudaStreamSynchronize(st));
    return RT_OK;
}

int rt_mlp_dispatches_per_step(rt_mlp* m, int* out) {
    RT_CHECK(m && out, "bad arguments");
    if (!m->slot[0].exec) RT_TRY(capture_step(m, 0));
    *out = m->kernels_per_step;
    return RT_OK;
}

int rt_mlp_enable_timing(rt_mlp* m, int on) {
    RT_CHECK(m, "bad arguments");
    m->timing = on != 0;
    if (m->timing && m->events.empty()) {
        m->events.resize(64);
        for (auto& e : m->events) RT_CUDA(cudaEventCreate(&e));
    }
    return RT_OK;
}

int rt_mlp_op_count(rt_mlp* m, int* count) {
    RT_CHECK(m && count, "bad arguments");
    *count = m->timing ? (int)m->ops.size() : 0;
    return RT_OK;
}

int rt_mlp_op_time(rt_mlp* m, int i, const char** label, double* flops, float* ms) {
    RT_CHECK(m && m->timing && i >= 0 && i < (int)m->ops.size(), "op index out of range (timing off?)");
    if (label) *label = m->ops[i].label;
    if (flops) *flops = m->ops[i].flops;
    if (ms) RT_CUDA(cudaEventElapsedTime(ms, m->events[i], m->events[i + 1]));
    return RT_OK;
}

int rt_mlp_comm_mode(rt_mlp* m, int* mode) {
    RT_CHECK(m && mode, "bad arguments");
    bool p2p = false, ce = false;
    for (const PlanLayer& P : m->L) p2p = p2p || P.p2p, ce = ce || P.ce;
    *mode = !m->comm ? RT_COMM_NONE
            : p2p ? RT_COMM_SHARDED_P2P
            : ce ? RT_COMM_SHARDED_CE
            : m->sharded ? RT_COMM_SHARDED_OPT
            : m->comm_bf16 ? RT_COMM_ALLREDUCE_BF16
                           : RT_COMM_ALLREDUCE;
    return RT_OK;
}

int rt_mlp_set_comm(rt_mlp* m, rt_comm* comm) {
    RT_CHECK(m, "bad arguments");
    RT_CUDA(cudaStreamSynchronize(m->ctx->stream));  // no step still uses the old exchange
    teardown_p2p(m);
    m->comm = comm;
    // RTGPU_COMM_SM_RESERVE=<n>: backward GEMMs run on sm_count - n SMs so the
    // gradient allreduce has SMs of its own (an even count keeps CTA pairs whole).
    // Default 16: measured on 8 B200s, +3 % step throughput over 0.
    const char* r = getenv("RTGPU_COMM_SM_RESERVE");
    m->comm_sm_reserve = r ? (atoi(r) + 1) / 2 * 2 : 16;
    if (m->comm_sm_reserve < 0 || m->comm_sm_reserve >= m->ctx->sm_count) m->comm_sm_reserve = 0;
    if (comm && !m->comm_stream) {
        // The collectives get the highest stream priority: when SMs free up
        // during backward, NCCL's blocks are dispatched before the update
        // kernels' (the step graph keeps per-node priorities).
        int least = 0, greatest = 0;
        RT_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
        RT_CUDA(cudaStreamCreateWithPriority(&m->comm_stream, cudaStreamNonBlocking, greatest));
    }
    // RTGPU_GRAD_COMM=bf16: bf16 plans sum their gradients in bf16 (half the
    // NVLink bytes; the parity bar of bf16 plans is 2e-2)
    const char* gc = getenv("RTGPU_GRAD_COMM");
    m->comm_bf16 = comm && m->adt == RT_BF16 && gc && std::strcmp(gc, "bf16") == 0;
    if (m->comm_bf16)
        for (PlanLayer& P : m->L)
            if (!P.g16) {
                void* p = nullptr;
                RT_TRY(dalloc(m, &p, (size_t)(P.d + 1) * P.ld * 2));
                P.g16 = static_cast<__nv_bfloat16*>(p);
            }
    set_fuse_opt(m);
    RT_TRY(prepare_chunks(m));
    // Sharded optimiser: bf16 plans (their GEMMs read only the bf16 weights)
    // with an optimiser, more than one rank, every chunk divisible by the
    // world size; RTGPU_SHARDED_OPT=0 keeps the replicated update.
    m->rank = comm_rank(comm);
    m->world = comm_world(comm);
    const char* so = getenv("RTGPU_SHARDED_OPT");
    bool sharded = comm && m->world > 1 && m->adt == RT_BF16 && m->cfg.optimizer != RT_OPT_NONE &&
                   !m->comm_bf16 && !(so && so[0] == '0');
    for (const PlanLayer& P : m->L)
        for (int c = 0; sharded && c < P.chunks; ++c) {
            const int64_t r0 = chunk_row_of(P.d + 1, P.chunks, c);
            const int64_t e = shard_end(P, chunk_row_of(P.d + 1, P.chunks, c + 1));
            if (e > r0 && ((e - r0) * P.ld) % m->world) sharded = false;
        }
    m->sharded = sharded;
    if (sharded && !m->ag_stream) {
        // Collective: every rank reaches this with the same plan shape.
        int st = RT_OK;
        if (comm_open_second(comm, &st)) {
            int least = 0, greatest = 0;
            RT_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
            RT_CUDA(cudaStreamCreateWithPriority(&m->ag_stream, cudaStreamNonBlocking, greatest));
        }
        RT_TRY(st);
    }
    if (sharded && !m->scratch) RT_TRY(dalloc_t(m, &m->scratch, 4));
    RT_TRY(setup_p2p(m));
    RT_TRY(setup_ce(m));
    // With every layer on the copy-engine exchange, NCCL only runs barriers
    // and the bias rows' allreduces: the backward GEMMs keep every SM.
    bool all_ce = m->sharded;
    for (const PlanLayer& P : m->L) all_ce = all_ce && P.ce;
    if (all_ce && !getenv("RTGPU_COMM_SM_RESERVE")) m->comm_sm_reserve = 0;
    m->ops.clear();
    drop_graphs(m);
    return RT_OK;
}

}  // extern "C"
