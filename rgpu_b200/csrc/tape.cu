// Reverse-mode tape on the GPU: the counterpart of rtensor's Tape / Param /
// Var / Grads (crates/rtensor/src/tape.rs:43-249) for the operations a Dense
// network is built from (ops.rs:49-53 add, 125-129 matmul, 190-194 relu) and
// the fused softmax cross-entropy (losses.rs:99-115), plus the optimisers that
// consume Grads (optim.rs:64-198).
//
// Every value and adjoint lives in device memory, allocated stream-ordered
// (cudaMallocAsync on the context stream) and released when the tape is
// destroyed.  Forward ops and the backward sweep only enqueue kernels of this
// library on the context stream: nothing waits for the device until the
// caller reads a value (rt_var_item, rt_param_read).
//
// As in tape.rs, nodes are appended in topological order, the backward is one
// reverse sweep, a node's adjoint is the sum of the contributions of every
// consumer (in-place accumulation, tape.rs:213-224), and Param::watch reuses
// the parameter's leaf node when the same parameter is watched twice on one
// tape (tape.rs:124-131).
#include "tape_internal.h"

using namespace rt;
using rt::tp::Buf;
using rt::tp::check_var;
using rt::tp::ld_for;
using rt::tp::Node;

namespace {

uint64_t next_param_id() {
    static uint64_t id = 0;
    return ++id;
}

}  // namespace

namespace {

GemmDesc f32_gemm(rt_layout layout, int64_t m, int64_t n, int64_t k, const Buf& a, const Buf& b, Buf& c) {
    GemmDesc g{};
    g.layout = layout;
    g.in_dtype = RT_F32;
    g.out_dtype = RT_F32;
    g.m = m;
    g.n = n;
    g.k = k;
    g.a = a.p;
    g.lda = a.ld;
    g.b = b.p;
    g.ldb = b.ld;
    g.c = c.p;
    g.ldc = c.ld;
    g.epi = RT_EPI_NONE;
    g.split_k = 1;
    return g;
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------- Param
int rt_param_create(rt_ctx* ctx, const float* host, int64_t rows, int64_t cols, rt_param** out) {
    RT_CHECK(ctx && out && rows >= 0 && cols >= 0, "rt_param_create: bad arguments");
    rt_param* p = new rt_param;
    p->ctx = ctx;
    p->id = next_param_id();
    p->value.rows = rows;
    p->value.cols = cols;
    p->value.ld = ld_for(cols);
    size_t bytes = (size_t)(rows > 0 ? rows : 1) * (size_t)p->value.ld * 4;
    cudaError_t e = cudaMalloc((void**)&p->value.p, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(p->value.p, 0, bytes, ctx->stream);
    if (e == cudaSuccess && host && rows * cols > 0)
        e = cudaMemcpy2DAsync(p->value.p, p->value.ld * 4, host, cols * 4, cols * 4, rows, cudaMemcpyHostToDevice,
                              ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        if (p->value.p) cudaFree(p->value.p);
        delete p;
        return fail(RT_ERR_CUDA, "rt_param_create: %s", cudaGetErrorString(e));
    }
    *out = p;
    return RT_OK;
}

int rt_param_destroy(rt_param* p) {
    if (!p) return RT_OK;
    cudaStreamSynchronize(p->ctx->stream);
    if (p->value.p) cudaFree(p->value.p);
    delete p;
    return RT_OK;
}

int rt_param_read(rt_param* p, float* host) {
    RT_CHECK(p && host, "rt_param_read: bad arguments");
    const Buf& b = p->value;
    if (b.rows * b.cols == 0) return RT_OK;
    RT_CUDA(cudaMemcpy2DAsync(host, b.cols * 4, b.p, b.ld * 4, b.cols * 4, b.rows, cudaMemcpyDeviceToHost,
                              p->ctx->stream));
    RT_CUDA(cudaStreamSynchronize(p->ctx->stream));
    return RT_OK;
}

int rt_param_write(rt_param* p, const float* host) {
    RT_CHECK(p && host, "rt_param_write: bad arguments");
    const Buf& b = p->value;
    if (b.rows * b.cols == 0) return RT_OK;
    RT_CUDA(cudaMemcpy2DAsync(b.p, b.ld * 4, host, b.cols * 4, b.cols * 4, b.rows, cudaMemcpyHostToDevice,
                              p->ctx->stream));
    RT_CUDA(cudaStreamSynchronize(p->ctx->stream));
    return RT_OK;
}

int rt_param_value(rt_param* p, rt_tensor** view) {
    RT_CHECK(p && view, "rt_param_value: bad arguments");
    int64_t shape[2] = {p->value.rows, p->value.cols};
    return rt_tensor_wrap(p->ctx, p->value.p, RT_F32, 2, shape, p->value.ld, view);
}

// -------------------------------------------------------------------- Tape
int rt_tape_create(rt_ctx* ctx, rt_tape** out) {
    RT_CHECK(ctx && out, "rt_tape_create: bad arguments");
    rt_tape* t = new rt_tape;
    t->ctx = ctx;
    *out = t;
    return RT_OK;
}

int rt_tape_destroy(rt_tape* t) {
    if (!t) return RT_OK;
    for (void* p : t->owned) cudaFreeAsync(p, t->ctx->stream);
    for (rt_var* v : t->vars) delete v;
    delete t;
    return RT_OK;
}

int rt_tape_len(rt_tape* t, int* out) {
    RT_CHECK(t && out, "bad arguments");
    *out = (int)t->nodes.size();
    return RT_OK;
}

int rt_tape_constant(rt_tape* t, const rt_tensor* value, rt_var** out) {
    RT_CHECK(t && value && out, "rt_tape_constant: bad arguments");
    RT_CHECK(value->dtype == RT_F32, "rt_tape_constant: the tape computes in f32");
    Buf b;
    RT_TRY(t->alloc(b, value->rows, value->cols));
    if (value->rows * value->cols > 0)
        RT_CUDA(cudaMemcpy2DAsync(b.p, b.ld * 4, value->ptr, value->ld * 4, value->cols * 4, value->rows,
                                  cudaMemcpyDeviceToDevice, t->ctx->stream));
    *out = t->push({}, nullptr, b);
    return RT_OK;
}

int rt_param_watch(rt_param* p, rt_tape* t, rt_var** out) {
    RT_CHECK(p && t && out, "rt_param_watch: bad arguments");
    RT_CHECK(p->ctx == t->ctx, "parameter and tape belong to different contexts");
    auto it = t->param_nodes.find(p->id);
    if (it != t->param_nodes.end()) {
        rt_var* v = new rt_var;
        v->tape = t;
        v->idx = it->second;
        t->vars.push_back(v);
        *out = v;
        return RT_OK;
    }
    // The leaf reads the parameter's buffer in place: optimisers update it only
    // after the backward sweep, as Optimizer::step runs after Var::backward.
    rt_var* v = t->push({}, nullptr, p->value);
    t->param_nodes[p->id] = v->idx;
    *out = v;
    return RT_OK;
}

// C = A B.  Adjoints (ops.rs:125-129): Abar = g B^T, Bbar = A^T g.
int rt_var_matmul(rt_var* a, rt_var* b, rt_var** out) {
    RT_TRY(check_var(a));
    RT_TRY(check_var(b));
    RT_CHECK(out && a->tape == b->tape, "operands belong to different tapes");
    rt_tape* t = a->tape;
    const Buf A = t->nodes[a->idx].value, B = t->nodes[b->idx].value;
    RT_CHECK(A.cols == B.rows, "matmul: incompatible shapes [%lld,%lld] x [%lld,%lld]", (long long)A.rows,
             (long long)A.cols, (long long)B.rows, (long long)B.cols);
    Buf C;
    RT_TRY(t->alloc(C, A.rows, B.cols));
    RT_TRY(run_gemm(t->ctx, f32_gemm(RT_NN, A.rows, B.cols, A.cols, A, B, C), t->ctx->stream, 0));
    const int ia = a->idx, ib = b->idx;
    *out = t->push({ia, ib},
                   [t, A, B, ia, ib](const Buf& g) -> int {
                       Buf ga, gb;
                       RT_TRY(t->alloc(ga, A.rows, A.cols));
                       RT_TRY(run_gemm(t->ctx, f32_gemm(RT_NT, A.rows, A.cols, B.cols, g, B, ga), t->ctx->stream, 0));
                       RT_TRY(t->alloc(gb, B.rows, B.cols));
                       RT_TRY(run_gemm(t->ctx, f32_gemm(RT_TN, B.rows, B.cols, A.rows, A, g, gb), t->ctx->stream, 0));
                       RT_TRY(t->accumulate(ia, ga));
                       return t->accumulate(ib, gb);
                   },
                   C);
    return RT_OK;
}

// C = A + B; same shapes and the row broadcast of a [1, n] operand (the +1b
// of Dense) run here, the other broadcasts through rt_var_binary.
// Adjoints (ops.rs:49-53): each operand receives g reduced to its shape
// (tensor.rs:399-438: the broadcast axis summed).
int rt_var_add(rt_var* a, rt_var* b, rt_var** out) {
    RT_TRY(check_var(a));
    RT_TRY(check_var(b));
    RT_CHECK(out && a->tape == b->tape, "operands belong to different tapes");
    rt_tape* t = a->tape;
    Buf A = t->nodes[a->idx].value, B = t->nodes[b->idx].value;
    int ia = a->idx, ib = b->idx;
    bool swapped = false;
    if (A.rows == 1 && B.rows != 1 && A.cols == B.cols) {  // [1,n] + [m,n]
        std::swap(A, B);
        std::swap(ia, ib);
        swapped = true;
    }
    (void)swapped;
    const bool same = A.rows == B.rows && A.cols == B.cols;
    const bool row_bcast = B.rows == 1 && B.cols == A.cols;
    // the other broadcasts (a column, a scalar, row against column) take the
    // general elementwise path of tape_ops.cu
    if (!same && !row_bcast) return rt_var_binary(a, b, RT_ADD, out);
    Buf C;
    RT_TRY(t->alloc(C, A.rows, A.cols));
    if (A.rows * A.cols > 0)
        RT_CUDA(cudaMemcpy2DAsync(C.p, C.ld * 4, A.p, A.ld * 4, A.cols * 4, A.rows, cudaMemcpyDeviceToDevice,
                                  t->ctx->stream));
    if (same)
        RT_TRY(launch_axpy_inplace(t->ctx, C.p, C.ld, B.p, B.ld, A.rows, A.cols, t->ctx->stream));
    else
        RT_TRY(launch_bias_add(t->ctx, C.p, RT_F32, A.rows, A.cols, C.ld, B.p, t->ctx->stream));
    *out = t->push({ia, ib},
                   [t, A, same, ia, ib](const Buf& g) -> int {
                       RT_TRY(t->accumulate(ia, g));
                       if (same) return t->accumulate(ib, g);
                       Buf gb, scratch;
                       RT_TRY(t->alloc(gb, 1, A.cols));
                       float* ws = nullptr;
                       if (A.rows > 64) {
                           RT_TRY(t->alloc(scratch, colsum_scratch_rows(A.rows), A.cols));
                           ws = scratch.p;
                       }
                       // scratch rows are packed with stride cols in the colsum kernels
                       RT_TRY(launch_colsum(t->ctx, g.p, RT_F32, g.rows, g.cols, g.ld, ws, gb.p, t->ctx->stream));
                       return t->accumulate(ib, gb);
                   },
                   C);
    return RT_OK;
}

// Y = max(X, 0).  Adjoint (ops.rs:190-194): g * 1[X > 0].
int rt_var_relu(rt_var* a, rt_var** out) {
    RT_TRY(check_var(a));
    RT_CHECK(out, "bad arguments");
    rt_tape* t = a->tape;
    const Buf X = t->nodes[a->idx].value;
    Buf Y;
    RT_TRY(t->alloc(Y, X.rows, X.cols));
    RT_TRY(launch_relu(t->ctx, X.p, Y.p, RT_F32, X.rows, X.cols, X.ld, Y.ld, t->ctx->stream));
    const int ia = a->idx;
    *out = t->push({ia},
                   [t, X, ia](const Buf& g) -> int {
                       Buf gx;
                       RT_TRY(t->alloc(gx, g.rows, g.cols));
                       RT_CUDA(cudaMemcpy2DAsync(gx.p, gx.ld * 4, g.p, g.ld * 4, g.cols * 4, g.rows,
                                                 cudaMemcpyDeviceToDevice, t->ctx->stream));
                       RT_TRY(launch_relu_bwd(t->ctx, X.p, gx.p, RT_F32, X.rows, X.cols, X.ld, gx.ld, t->ctx->stream));
                       return t->accumulate(ia, gx);
                   },
                   Y);
    return RT_OK;
}

// Scalar loss L = -(1/n) sum_i ln max(p_{i,y_i}, 1e-12) of the row softmax of
// the logits (losses.rs:99-115, labels instead of one-hot rows).  The loss
// is the root of the graph: its adjoint into the logits is (P - Y) / n.
int rt_softmax_cross_entropy(rt_var* logits, const rt_tensor* labels, rt_var** out) {
    RT_TRY(check_var(logits));
    RT_CHECK(labels && out, "bad arguments");
    rt_tape* t = logits->tape;
    const Buf Z = t->nodes[logits->idx].value;
    RT_CHECK(labels->dtype == RT_U32 && labels->rows * labels->cols == Z.rows,
             "softmax_cross_entropy: labels must be u32 [rows]");
    Buf delta, rows, loss;
    RT_TRY(t->alloc(delta, Z.rows, Z.cols));
    RT_TRY(t->alloc(rows, 1, Z.rows));
    RT_TRY(t->alloc(loss, 1, 1));
    const float scale = Z.rows > 0 ? 1.0f / (float)Z.rows : 0.0f;
    RT_TRY(launch_xent(t->ctx, Z.p, Z.ld, (const uint32_t*)labels->ptr, Z.rows, Z.cols, scale, delta.p, RT_F32,
                       delta.ld, rows.p, t->ctx->stream));
    RT_TRY(launch_mean_rows(t->ctx, rows.p, Z.rows, loss.p, t->ctx->stream));
    const int iz = logits->idx;
    *out = t->push({iz}, [t, delta, iz](const Buf&) -> int { return t->accumulate(iz, delta); }, loss);
    return RT_OK;
}

int rt_var_value(rt_var* v, rt_tensor** view) {
    RT_TRY(check_var(v));
    RT_CHECK(view, "bad arguments");
    const Buf& b = v->tape->nodes[v->idx].value;
    int64_t shape[2] = {b.rows, b.cols};
    return rt_tensor_wrap(v->tape->ctx, b.p, RT_F32, 2, shape, b.ld, view);
}

int rt_var_item(rt_var* v, float* out) {
    RT_TRY(check_var(v));
    RT_CHECK(out, "bad arguments");
    const Buf& b = v->tape->nodes[v->idx].value;
    RT_CHECK(b.rows * b.cols == 1, "item() needs a one-element value, shape [%lld,%lld]", (long long)b.rows,
             (long long)b.cols);
    RT_CUDA(cudaMemcpyAsync(out, b.p, 4, cudaMemcpyDeviceToHost, v->tape->ctx->stream));
    RT_CUDA(cudaStreamSynchronize(v->tape->ctx->stream));
    return RT_OK;
}

// Var::backward (tape.rs:187-229): one reverse sweep from the scalar root.
int rt_var_backward(rt_var* root) {
    RT_TRY(check_var(root));
    rt_tape* t = root->tape;
    const Buf& rv = t->nodes[root->idx].value;
    RT_CHECK(rv.rows * rv.cols == 1, "backward() must start from a scalar, shape [%lld,%lld]", (long long)rv.rows,
             (long long)rv.cols);
    RT_CHECK(!t->backward_done, "backward() already ran on this tape");
    t->grads.assign(t->nodes.size(), Buf{});
    Buf seed;
    RT_TRY(t->alloc(seed, 1, 1));
    const float one = 1.0f;
    RT_CUDA(cudaMemcpyAsync(seed.p, &one, 4, cudaMemcpyHostToDevice, t->ctx->stream));
    RT_CUDA(cudaStreamSynchronize(t->ctx->stream));  // `one` lives on this frame
    t->grads[root->idx] = seed;
    for (int i = root->idx; i >= 0; --i) {
        Node& n = t->nodes[i];
        if (!n.backward || !t->grads[i].p) continue;
        RT_TRY(n.backward(t->grads[i]));
    }
    t->backward_done = true;
    return RT_OK;
}

// Grads::of (tape.rs:238-243): *view = NULL when the parameter took no part.
int rt_grads_of(rt_tape* t, rt_param* p, rt_tensor** view) {
    RT_CHECK(t && p && view, "bad arguments");
    *view = nullptr;
    RT_CHECK(t->backward_done, "rt_grads_of: backward() has not run on this tape");
    auto it = t->param_nodes.find(p->id);
    if (it == t->param_nodes.end() || !t->grads[it->second].p) return RT_OK;
    const Buf& g = t->grads[it->second];
    int64_t shape[2] = {g.rows, g.cols};
    return rt_tensor_wrap(t->ctx, g.p, RT_F32, 2, shape, g.ld, view);
}

}  // extern "C"

// --------------------------------------------------------------- optimisers
struct rt_adam_state {
    rt_ctx* ctx = nullptr;
    float lr = 0, beta1 = 0, beta2 = 0, eps = 0;
    OptScalars* sc = nullptr;
    struct State {
        float* m = nullptr;
        float* v = nullptr;
    };
    std::unordered_map<uint64_t, State> state;
};

namespace {

const Buf* grad_of(rt_tape* t, rt_param* p) {
    auto it = t->param_nodes.find(p->id);
    if (it == t->param_nodes.end() || !t->grads[it->second].p) return nullptr;
    return &t->grads[it->second];
}

}  // namespace

extern "C" {

// Sgd::step without momentum (optim.rs:80-95): theta -= g * lr for every
// parameter that has a gradient.
int rt_sgd_step(rt_ctx* ctx, int n, rt_param* const* params, rt_tape* grads, float lr) {
    RT_CHECK(ctx && (n == 0 || params) && grads && grads->backward_done, "rt_sgd_step: bad arguments");
    for (int i = 0; i < n; ++i) {
        const Buf* g = grad_of(grads, params[i]);
        if (!g) continue;
        rt_param* p = params[i];
        RT_CHECK(g->ld == p->value.ld && g->rows == p->value.rows, "gradient/parameter layout mismatch");
        OptTensor tt{p->value.p, g->p, nullptr, nullptr, nullptr, 0, p->value.ld, p->value.rows * p->value.ld};
        RT_TRY(launch_sgd(ctx, &tt, 1, lr, ctx->stream));
    }
    return RT_OK;
}

// Adam::new / Adam::with_betas (optim.rs:150-158), eps 1e-8 unless given.
int rt_adam_create(rt_ctx* ctx, float lr, float beta1, float beta2, float eps, rt_adam_state** out) {
    RT_CHECK(ctx && out, "rt_adam_create: bad arguments");
    rt_adam_state* a = new rt_adam_state;
    a->ctx = ctx;
    a->lr = lr;
    a->beta1 = beta1;
    a->beta2 = beta2;
    a->eps = eps;
    cudaError_t e = cudaMalloc((void**)&a->sc, sizeof(OptScalars));
    if (e == cudaSuccess) e = cudaMemsetAsync(a->sc, 0, sizeof(OptScalars), ctx->stream);
    if (e != cudaSuccess) {
        delete a;
        return fail(RT_ERR_CUDA, "rt_adam_create: %s", cudaGetErrorString(e));
    }
    *out = a;
    return RT_OK;
}

int rt_adam_destroy(rt_adam_state* a) {
    if (!a) return RT_OK;
    cudaStreamSynchronize(a->ctx->stream);
    for (auto& kv : a->state) {
        cudaFree(kv.second.m);
        cudaFree(kv.second.v);
    }
    cudaFree(a->sc);
    delete a;
    return RT_OK;
}

// Adam::step (optim.rs:162-198): t += 1 on the device, then one fused pass
// per parameter with a gradient; moments are created zeroed on first use.
int rt_adam_step(rt_adam_state* a, int n, rt_param* const* params, rt_tape* grads) {
    RT_CHECK(a && (n == 0 || params) && grads && grads->backward_done, "rt_adam_step: bad arguments");
    rt_ctx* ctx = a->ctx;
    RT_TRY(launch_opt_step_begin(ctx, a->sc, a->beta1, a->beta2, ctx->stream));
    for (int i = 0; i < n; ++i) {
        const Buf* g = grad_of(grads, params[i]);
        if (!g) continue;
        rt_param* p = params[i];
        RT_CHECK(g->ld == p->value.ld && g->rows == p->value.rows, "gradient/parameter layout mismatch");
        size_t bytes = (size_t)(p->value.rows > 0 ? p->value.rows : 1) * (size_t)p->value.ld * 4;
        auto& st = a->state[p->id];
        if (!st.m) {
            RT_CUDA(cudaMalloc((void**)&st.m, bytes));
            RT_CUDA(cudaMalloc((void**)&st.v, bytes));
            RT_CUDA(cudaMemsetAsync(st.m, 0, bytes, ctx->stream));
            RT_CUDA(cudaMemsetAsync(st.v, 0, bytes, ctx->stream));
        }
        OptTensor tt{p->value.p, g->p, st.m, st.v, nullptr, 0, p->value.ld, p->value.rows * p->value.ld};
        RT_TRY(launch_adam(ctx, &tt, 1, a->sc, a->lr, a->beta1, a->beta2, a->eps, ctx->stream));
    }
    return RT_OK;
}

}  // extern "C"
