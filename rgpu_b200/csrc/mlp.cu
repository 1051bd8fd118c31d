// The whole-step plan: counterpart of rtensor's GpuMlp
// (crates/rtensor/src/gpu/mod.rs:1289-1562).  The plan is built once
// (buffers, GEMM descriptors, split-K choices), the step is captured into a
// CUDA graph, and every step replays it: no host round-trip between the
// forward GEMMs, softmax-CE, the backward GEMMs with their fused epilogues,
// the optional NCCL allreduce of dW/db and the optimiser.
//
// Backward recurrence (gpu/mod.rs:35-46):
//   delta_L = (P - Y) / n_global
//   dW_l = A_{l-1}^T delta_l        db_l = 1^T delta_l
//   delta_{l-1} = (delta_l W_l^T) * 1[A_{l-1} > 0]     (l > 0)
#include <cstring>
#include <vector>

#include "internal.h"

namespace rt {
int run_gemm(rt_ctx* ctx, GemmDesc g, cudaStream_t stream, size_t ws_bytes);
int comm_allreduce(rt_comm* comm, float* buf, int64_t count, cudaStream_t st);
}  // namespace rt

using namespace rt;

namespace {

int64_t round8(int64_t x) { return (x + 7) / 8 * 8; }

struct PlanLayer {
    int64_t d = 0, u = 0, ld = 0;  // W_l is [d, u] with row stride ld
    float* w32 = nullptr;
    __nv_bfloat16* w16 = nullptr;  // bf16 shadow (bf16 plans)
    float* b = nullptr;
    float *mw = nullptr, *vw = nullptr, *mb = nullptr, *vb = nullptr;
    float* dw = nullptr;
    float* db = nullptr;
    void* act = nullptr;    // hidden: A_l [n, u] (operand dtype); last: logits f32
    void* delta = nullptr;  // delta_l [n, u] (operand dtype)
    int split_dw = 1;
    float* ws = nullptr;    // split-K partials for dW_l
    size_t ws_bytes = 0;
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
    rt_dtype adt = RT_F32;  // operand / activation dtype
    int64_t n = 0, ldx = 0;
    void* x = nullptr;
    uint32_t* labels = nullptr;
    float* loss_rows = nullptr;
    float* colsum_ws = nullptr;
    OptScalars* opt = nullptr;
    void* x_stage = nullptr;  // host-path staging when the host dtype differs
    size_t x_stage_bytes = 0;
    std::vector<void*> allocs;

    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool graph_timed = false;
    bool timing = false;
    std::vector<cudaEvent_t> events;
    std::vector<OpRecord> ops;
    std::vector<float> op_ms;
    int kernels_per_step = 0;

    rt_comm* comm = nullptr;
    cudaStream_t comm_stream = nullptr;
    std::vector<cudaEvent_t> comm_ready, comm_done;
};

namespace {

int dalloc(rt_mlp* m, void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail(RT_ERR_OOM, "plan allocation of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
    m->allocs.push_back(*p);
    e = cudaMemset(*p, 0, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, "cudaMemset failed: %s", cudaGetErrorString(e));
    return RT_OK;
}

template <typename T>
int dalloc_t(rt_mlp* m, T** p, size_t count, size_t elem = sizeof(T)) {
    return dalloc(m, reinterpret_cast<void**>(p), count * elem);
}

void free_all(rt_mlp* m) {
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    m->exec = nullptr;
    m->graph = nullptr;
    for (auto e : m->events) cudaEventDestroy(e);
    for (auto e : m->comm_ready) cudaEventDestroy(e);
    for (auto e : m->comm_done) cudaEventDestroy(e);
    if (m->comm_stream) cudaStreamDestroy(m->comm_stream);
    for (void* p : m->allocs) cudaFree(p);
    m->allocs.clear();
}

// ---------------------------------------------------------------- step body
struct Enqueuer {
    rt_mlp* m;
    cudaStream_t st;
    bool forward_only;
    int op_index = 0;

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

    const void* input_of(int l) const { return l == 0 ? m->x : m->L[l - 1].act; }
    int64_t ld_in(int l) const { return l == 0 ? m->ldx : m->L[l - 1].ld; }
    const void* weights(const PlanLayer& P) const {
        return m->adt == RT_BF16 ? (const void*)P.w16 : (const void*)P.w32;
    }

    int forward() {
        const int nl = (int)m->L.size();
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
            g.ldc = P.ld;
            g.epi = last ? RT_EPI_BIAS : RT_EPI_BIAS_RELU;
            g.bias = P.b;
            g.split_k = 1;
            RT_TRY(run_gemm(m->ctx, g, st, 0));
            RT_TRY(mark(last ? "fwd_gemm_bias" : "fwd_gemm_bias_relu", 2.0 * m->n * P.d * P.u));
        }
        return RT_OK;
    }

    int backward_and_update() {
        const int nl = (int)m->L.size();
        PlanLayer& Last = m->L[nl - 1];
        double gb = (double)(m->cfg.global_batch > 0 ? m->cfg.global_batch : m->n);
        RT_TRY(launch_xent(m->ctx, (const float*)Last.act, Last.ld, m->labels, m->n, Last.u, (float)(1.0 / gb),
                           Last.delta, m->adt, Last.ld, m->loss_rows, st));
        RT_TRY(mark("softmax_xent", 0));
        for (int l = nl - 1; l >= 0; --l) {
            PlanLayer& P = m->L[l];
            // dW_l = A_{l-1}^T delta_l  (TN, K = batch), f32 output for the optimiser.
            GemmDesc g{};
            g.layout = RT_TN;
            g.in_dtype = m->adt;
            g.out_dtype = RT_F32;
            g.m = P.d;
            g.n = P.u;
            g.k = m->n;
            g.a = input_of(l);
            g.lda = ld_in(l);
            g.b = P.delta;
            g.ldb = P.ld;
            g.c = P.dw;
            g.ldc = P.ld;
            g.epi = RT_EPI_NONE;
            g.split_k = P.split_dw;
            g.workspace = P.ws;
            RT_TRY(run_gemm(m->ctx, g, st, P.ws_bytes));
            RT_TRY(mark("dw_gemm", 2.0 * m->n * P.d * P.u));
            // db_l = 1^T delta_l
            RT_TRY(launch_colsum(m->ctx, P.delta, m->adt, m->n, P.u, P.ld, m->colsum_ws, P.db, st));
            RT_TRY(mark("db_colsum", 0));
            if (m->comm) {
                RT_CUDA(cudaEventRecord(m->comm_ready[l], st));
                RT_CUDA(cudaStreamWaitEvent(m->comm_stream, m->comm_ready[l], 0));
                RT_TRY(comm_allreduce(m->comm, P.dw, P.d * P.ld, m->comm_stream));
                RT_TRY(comm_allreduce(m->comm, P.db, round8(P.u), m->comm_stream));
                RT_CUDA(cudaEventRecord(m->comm_done[l], m->comm_stream));
            }
            if (l > 0) {
                // delta_{l-1} = (delta_l W_l^T) * 1[A_{l-1} > 0]  (NT, fused mask).
                PlanLayer& Q = m->L[l - 1];
                GemmDesc h{};
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
                h.ldmask = Q.ld;
                h.split_k = 1;
                RT_TRY(run_gemm(m->ctx, h, st, 0));
                RT_TRY(mark("dx_gemm_relu_mask", 2.0 * m->n * P.d * P.u));
            }
        }
        if (m->comm)
            for (int l = 0; l < nl; ++l) RT_CUDA(cudaStreamWaitEvent(st, m->comm_done[l], 0));
        if (m->cfg.optimizer == RT_OPT_NONE) return RT_OK;
        std::vector<OptTensor> ts;
        for (auto& P : m->L) {
            ts.push_back({P.w32, P.dw, P.mw, P.vw, P.w16, P.ld, P.ld, P.d * P.ld});
            ts.push_back({P.b, P.db, P.mb, P.vb, nullptr, 0, round8(P.u), round8(P.u)});
        }
        if (m->cfg.optimizer == RT_OPT_ADAM) {
            RT_TRY(launch_opt_step_begin(m->ctx, m->opt, m->cfg.beta1, m->cfg.beta2, st));
            RT_TRY(mark("adam_scalars", 0));
            RT_TRY(launch_adam(m->ctx, ts.data(), (int)ts.size(), m->opt, m->cfg.lr, m->cfg.beta1, m->cfg.beta2,
                               m->cfg.eps, st));
            RT_TRY(mark("adam", 0));
        } else {
            RT_TRY(launch_sgd(m->ctx, ts.data(), (int)ts.size(), m->cfg.lr, st));
            RT_TRY(mark("sgd", 0));
        }
        return RT_OK;
    }
};

int capture_step(rt_mlp* m) {
    cudaStream_t st = m->ctx->stream;
    if (m->exec) {
        cudaGraphExecDestroy(m->exec);
        m->exec = nullptr;
    }
    if (m->graph) {
        cudaGraphDestroy(m->graph);
        m->graph = nullptr;
    }
    uint64_t before = m->ctx->launches;
    RT_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    Enqueuer q{m, st, false};
    int s = q.begin();
    if (s == RT_OK) s = q.forward();
    if (s == RT_OK) s = q.backward_and_update();
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (s != RT_OK) {
        if (graph) cudaGraphDestroy(graph);
        return s;
    }
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, "step capture failed: %s", cudaGetErrorString(e));
    m->graph = graph;
    RT_CUDA(cudaGraphInstantiate(&m->exec, graph, 0));
    m->kernels_per_step = (int)(m->ctx->launches - before);
    m->graph_timed = m->timing;
    return RT_OK;
}

int copy_input(rt_mlp* m, const void* x, rt_dtype xdt, const uint32_t* labels, cudaMemcpyKind kind) {
    cudaStream_t st = m->ctx->stream;
    const int64_t d0 = m->dims[0];
    RT_CHECK(xdt == RT_F32 || xdt == RT_BF16, "x dtype must be RT_F32 or RT_BF16");
    if (xdt == m->adt) {
        size_t es = dtype_size(xdt);
        RT_CUDA(cudaMemcpy2DAsync(m->x, m->ldx * es, x, d0 * es, d0 * es, m->n, kind, st));
    } else {
        const void* src = x;
        if (kind == cudaMemcpyHostToDevice) {
            size_t bytes = (size_t)m->n * d0 * dtype_size(xdt);
            if (m->x_stage_bytes < bytes) {
                if (m->x_stage) cudaFree(m->x_stage);
                m->x_stage = nullptr;
                m->x_stage_bytes = 0;
                RT_CUDA(cudaMalloc(&m->x_stage, bytes));
                m->x_stage_bytes = bytes;
            }
            RT_CUDA(cudaMemcpyAsync(m->x_stage, x, bytes, kind, st));
            src = m->x_stage;
        }
        RT_TRY(launch_cast(m->ctx, src, xdt, d0, m->x, m->adt, m->ldx, m->n, d0, st));
    }
    RT_CUDA(cudaMemcpyAsync(m->labels, labels, (size_t)m->n * 4, kind, st));
    return RT_OK;
}

int launch_step(rt_mlp* m) {
    if (!m->exec || m->graph_timed != m->timing) RT_TRY(capture_step(m));
    RT_CUDA(cudaGraphLaunch(m->exec, m->ctx->stream));
    m->ctx->launches += (uint64_t)m->kernels_per_step;
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

}  // namespace

extern "C" {

int rt_mlp_create(rt_ctx* ctx, const rt_mlp_config* cfg, const float* const* weights, const float* const* biases,
                  rt_mlp** out) {
    RT_CHECK(ctx && cfg && out && weights, "rt_mlp_create: bad arguments");
    RT_CHECK(cfg->n_layers >= 1 && cfg->dims, "rt_mlp_create: model without layers");
    RT_CHECK(cfg->batch >= 1, "rt_mlp_create: batch must be >= 1");
    RT_CHECK(cfg->dtype == RT_F32 || cfg->dtype == RT_BF16, "rt_mlp_create: dtype must be RT_F32 or RT_BF16");
    RT_CHECK(cfg->optimizer >= RT_OPT_NONE && cfg->optimizer <= RT_OPT_ADAM, "rt_mlp_create: unknown optimizer");
    for (int l = 0; l <= cfg->n_layers; ++l) RT_CHECK(cfg->dims[l] >= 1, "rt_mlp_create: dims[%d] < 1", l);
    RT_CUDA(cudaSetDevice(ctx->device));
    rt_mlp* m = new rt_mlp;
    m->ctx = ctx;
    m->cfg = *cfg;
    m->dims.assign(cfg->dims, cfg->dims + cfg->n_layers + 1);
    m->cfg.dims = m->dims.data();
    m->adt = cfg->dtype;
    m->n = cfg->batch;
    const size_t es = dtype_size(m->adt);
    const int nl = cfg->n_layers;
    int s = RT_OK;
    auto bail = [&](int code) {
        free_all(m);
        delete m;
        return code;
    };

    m->ldx = round8(m->dims[0]);
    if ((s = dalloc(m, &m->x, (size_t)m->n * m->ldx * es))) return bail(s);
    if ((s = dalloc_t(m, &m->labels, (size_t)m->n))) return bail(s);
    if ((s = dalloc_t(m, &m->loss_rows, (size_t)m->n))) return bail(s);
    if ((s = dalloc_t(m, &m->opt, 1))) return bail(s);
    int64_t max_u = 0;
    m->L.resize(nl);
    for (int l = 0; l < nl; ++l) {
        PlanLayer& P = m->L[l];
        P.d = m->dims[l];
        P.u = m->dims[l + 1];
        P.ld = round8(P.u);
        if (P.u > max_u) max_u = P.u;
        size_t wn = (size_t)P.d * P.ld, bn = (size_t)round8(P.u), an = (size_t)m->n * P.ld;
        bool last = l == nl - 1;
        if ((s = dalloc_t(m, &P.w32, wn))) return bail(s);
        if ((s = dalloc_t(m, &P.b, bn))) return bail(s);
        if ((s = dalloc_t(m, &P.dw, wn))) return bail(s);
        if ((s = dalloc_t(m, &P.db, bn))) return bail(s);
        if (cfg->optimizer == RT_OPT_ADAM) {
            if ((s = dalloc_t(m, &P.mw, wn))) return bail(s);
            if ((s = dalloc_t(m, &P.vw, wn))) return bail(s);
            if ((s = dalloc_t(m, &P.mb, bn))) return bail(s);
            if ((s = dalloc_t(m, &P.vb, bn))) return bail(s);
        }
        if (m->adt == RT_BF16 && (s = dalloc_t(m, &P.w16, wn))) return bail(s);
        if ((s = dalloc(m, &P.act, an * (last ? 4 : es)))) return bail(s);
        if ((s = dalloc(m, &P.delta, an * es))) return bail(s);
        // weights in (host f32 packed [d,u] -> padded rows)
        if (cudaMemcpy2D(P.w32, P.ld * 4, weights[l], P.u * 4, P.u * 4, P.d, cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(RT_ERR_CUDA, "weight upload failed"));
        if (biases && biases[l] &&
            cudaMemcpy(P.b, biases[l], (size_t)P.u * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(RT_ERR_CUDA, "bias upload failed"));
        if (m->adt == RT_BF16 &&
            (s = launch_cast(ctx, P.w32, RT_F32, P.ld, P.w16, RT_BF16, P.ld, P.d, P.ld, ctx->stream)))
            return bail(s);
        // split-K for dW_l when its output tiles cannot fill the GPU.
        int64_t tiles = ((P.d + 127) / 128) * ((P.u + 255) / 256);
        int split = 1;
        if (tiles * 4 < (int64_t)ctx->sm_count * 3) {
            int64_t sp = (int64_t)ctx->sm_count / tiles;
            int64_t kb = (m->n + 63) / 64;
            if (sp > kb / 4) sp = kb / 4;
            if (sp > 16) sp = 16;
            split = sp < 1 ? 1 : (int)sp;
        }
        P.split_dw = split;
        if (split > 1) {
            P.ws_bytes = (size_t)split * P.d * P.u * 4;
            if ((s = dalloc(m, (void**)&P.ws, P.ws_bytes))) return bail(s);
        }
    }
    if ((s = dalloc_t(m, &m->colsum_ws, (size_t)colsum_scratch_rows(m->n) * max_u))) return bail(s);
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return bail(fail(RT_ERR_CUDA, "plan setup sync failed"));
    *out = m;
    return RT_OK;
}

int rt_mlp_destroy(rt_mlp* m) {
    if (!m) return RT_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    if (m->x_stage) cudaFree(m->x_stage);
    free_all(m);
    delete m;
    return RT_OK;
}

int rt_mlp_step(rt_mlp* m, const void* x_dev, rt_dtype x_dtype, const uint32_t* labels_dev) {
    RT_CHECK(m && x_dev && labels_dev, "rt_mlp_step: bad arguments");
    RT_TRY(copy_input(m, x_dev, x_dtype, labels_dev, cudaMemcpyDeviceToDevice));
    return launch_step(m);
}

int rt_mlp_step_host(rt_mlp* m, const void* x_host, rt_dtype x_dtype, const uint32_t* labels_host,
                     float* loss_rows_host) {
    RT_CHECK(m && x_host && labels_host, "rt_mlp_step_host: bad arguments");
    RT_TRY(copy_input(m, x_host, x_dtype, labels_host, cudaMemcpyHostToDevice));
    RT_TRY(launch_step(m));
    if (loss_rows_host)
        RT_CUDA(cudaMemcpyAsync(loss_rows_host, m->loss_rows, (size_t)m->n * 4, cudaMemcpyDeviceToHost,
                                m->ctx->stream));
    return RT_OK;
}

int rt_mlp_forward_only(rt_mlp* m, const void* x_dev, rt_dtype x_dtype) {
    RT_CHECK(m && x_dev, "rt_mlp_forward_only: bad arguments");
    const int64_t d0 = m->dims[0];
    cudaStream_t st = m->ctx->stream;
    if (x_dtype == m->adt) {
        size_t es = dtype_size(x_dtype);
        RT_CUDA(cudaMemcpy2DAsync(m->x, m->ldx * es, x_dev, d0 * es, d0 * es, m->n, cudaMemcpyDeviceToDevice, st));
    } else {
        RT_TRY(launch_cast(m->ctx, x_dev, x_dtype, d0, m->x, m->adt, m->ldx, m->n, d0, st));
    }
    Enqueuer q{m, st, true};
    return q.forward();
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

int rt_mlp_weights(rt_mlp* m, int layer, float* w, float* b) {
    RT_CHECK(m && layer >= 0 && layer < (int)m->L.size(), "bad layer index");
    PlanLayer& P = m->L[layer];
    if (w) RT_TRY(read_packed(m, P.w32, RT_F32, P.d, P.u, P.ld, w));
    if (b) RT_TRY(read_packed(m, P.b, RT_F32, 1, P.u, P.u, b));
    return RT_OK;
}

int rt_mlp_grads(rt_mlp* m, int layer, float* dw, float* db) {
    RT_CHECK(m && layer >= 0 && layer < (int)m->L.size(), "bad layer index");
    PlanLayer& P = m->L[layer];
    if (dw) RT_TRY(read_packed(m, P.dw, RT_F32, P.d, P.u, P.ld, dw));
    if (db) RT_TRY(read_packed(m, P.db, RT_F32, 1, P.u, P.u, db));
    return rt_ctx_sync(m->ctx);
}

int rt_mlp_set_weights(rt_mlp* m, int layer, const float* w, const float* b) {
    RT_CHECK(m && layer >= 0 && layer < (int)m->L.size(), "bad layer index");
    PlanLayer& P = m->L[layer];
    cudaStream_t st = m->ctx->stream;
    if (w) {
        RT_CUDA(cudaMemcpy2DAsync(P.w32, P.ld * 4, w, P.u * 4, P.u * 4, P.d, cudaMemcpyHostToDevice, st));
        if (m->adt == RT_BF16) RT_TRY(launch_cast(m->ctx, P.w32, RT_F32, P.ld, P.w16, RT_BF16, P.ld, P.d, P.ld, st));
    }
    if (b) RT_CUDA(cudaMemcpyAsync(P.b, b, (size_t)P.u * 4, cudaMemcpyHostToDevice, st));
    RT_CUDA(cudaStreamSynchronize(st));
    return RT_OK;
}

int rt_mlp_dispatches_per_step(rt_mlp* m, int* out) {
    RT_CHECK(m && out, "bad arguments");
    if (!m->exec) RT_TRY(capture_step(m));
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

int rt_mlp_set_comm(rt_mlp* m, rt_comm* comm) {
    RT_CHECK(m, "bad arguments");
    m->comm = comm;
    if (comm && !m->comm_stream) {
        RT_CUDA(cudaStreamCreateWithFlags(&m->comm_stream, cudaStreamNonBlocking));
        m->comm_ready.resize(m->L.size());
        m->comm_done.resize(m->L.size());
        for (auto& e : m->comm_ready) RT_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        for (auto& e : m->comm_done) RT_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    if (m->exec) {
        cudaGraphExecDestroy(m->exec);
        m->exec = nullptr;
    }
    if (m->graph) {
        cudaGraphDestroy(m->graph);
        m->graph = nullptr;
    }
    return RT_OK;
}

}  // extern "C"
