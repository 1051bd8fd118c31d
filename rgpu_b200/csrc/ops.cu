// Op-level entry points: the counterparts of rtensor's op builders and
// immediate helpers (crates/rtensor/src/gpu/mod.rs:685-953, 1079-1229).
// Each call validates shapes (where the reference panics, this returns
// RT_ERR_INVALID) and enqueues kernels on the context stream.
#include "internal.h"

namespace rt {

static int check_gemm(const GemmDesc& g) {
    RT_CHECK(g.in_dtype == RT_F32 || g.in_dtype == RT_BF16, "GEMM operands must be f32 or bf16");
    RT_CHECK(g.out_dtype == RT_F32 || g.out_dtype == RT_BF16, "GEMM output must be f32 or bf16");
    RT_CHECK(g.m >= 0 && g.n >= 0 && g.k >= 0, "negative GEMM extent");
    RT_CHECK(g.layout == RT_NN || g.layout == RT_NT || g.layout == RT_TN, "unknown GEMM layout %d", (int)g.layout);
    RT_CHECK(g.epi >= RT_EPI_NONE && g.epi <= RT_EPI_RELU_MASK, "unknown epilogue %d", (int)g.epi);
    if (g.m == 0 || g.n == 0) return RT_OK;
    RT_CHECK(g.c != nullptr, "GEMM output pointer is NULL");
    RT_CHECK(g.ldc >= g.n, "ldc %lld < n %lld", (long long)g.ldc, (long long)g.n);
    if (g.k > 0) {
        RT_CHECK(g.a && g.b, "GEMM operand pointer is NULL");
        int64_t a_cols = g.layout == RT_TN ? g.m : g.k;
        int64_t b_cols = g.layout == RT_NT ? g.k : g.n;
        RT_CHECK(g.lda >= a_cols, "lda %lld too small (need >= %lld)", (long long)g.lda, (long long)a_cols);
        RT_CHECK(g.ldb >= b_cols, "ldb %lld too small (need >= %lld)", (long long)g.ldb, (long long)b_cols);
    }
    if (g.epi == RT_EPI_BIAS || g.epi == RT_EPI_BIAS_RELU) RT_CHECK(g.bias, "bias epilogue without a bias vector");
    if (g.epi == RT_EPI_RELU_MASK) {
        RT_CHECK(g.mask, "relu-mask epilogue without a mask");
        RT_CHECK(g.ldmask >= g.n, "ldmask too small");
    }
    if (g.a_lo) RT_CHECK(g.in_dtype == RT_BF16, "a_lo (low-order plane of A) needs bf16 operands");
    if (g.c_lo) {
        RT_CHECK(g.out_dtype == RT_BF16, "c_lo (low-order plane of C) needs a bf16 output");
        RT_CHECK(g.split_k <= 1 && !g.opt.kind && g.p2p.world == 0,
                 "c_lo needs one k slice and no fused update or peer scatter");
    }
    return RT_OK;
}

// Slices for the tensor-core kernel: split only when the output tiles cannot
// fill the GPU and the reduction is deep (the dW = X^T dY case at large
// batch, gpu/mod.rs:1351-1358).  Each slice keeps at least 8 k blocks (512
// deep for bf16) and nothing splits below 24 k blocks: a shallower split
// saves less MMA time than the partial-sum round trip and the reduction
// launch cost.
int choose_split_k(const rt_ctx* ctx, int64_t m, int64_t n, int64_t k, rt_dtype in_dtype) {
    int64_t tiles = ((m + 127) / 128) * ((n + 255) / 256);
    if (tiles <= 0) return 1;
    if (tiles * 4 >= (int64_t)ctx->sm_count * 3) return 1;
    // k blocks of the tensor-core loop: 64 deep for bf16, three 32-deep
    // segments for the 3xTF32 f32 path
    int64_t kblocks = in_dtype == RT_F32 ? 3 * ((k + 31) / 32) : (k + 63) / 64;
    if (kblocks < 24) return 1;
    int64_t s = (int64_t)ctx->sm_count / tiles;
    if (s > kblocks / 8) s = kblocks / 8;
    if (s > 16) s = 16;
    return s < 1 ? 1 : (int)s;
}

static int choose_split(const rt_ctx* ctx, const GemmDesc& g) {
    return choose_split_k(ctx, g.m, g.n, g.k, g.in_dtype);
}

// The context's 3xTF32 operand workspace, grown to `need` bytes unless
// `stream` is being captured (cudaMalloc is not allowed there); the caller
// takes the SIMT kernel when what exists is too small.
static int x3_context_scratch(rt_ctx* ctx, cudaStream_t stream, size_t need, float** ws, size_t* have) {
    if (ctx->x3_scratch_bytes < need) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        RT_CUDA(cudaStreamIsCapturing(stream, &cs));
        if (cs == cudaStreamCaptureStatusNone) {
            const size_t unit = size_t(64) << 20;
            const size_t bytes = (need + unit - 1) / unit * unit;
            void* p = nullptr;
            RT_CUDA(cudaMalloc(&p, bytes));
            if (ctx->x3_scratch) ctx->x3_retired.push_back(ctx->x3_scratch);
            ctx->x3_scratch = static_cast<float*>(p);
            ctx->x3_scratch_bytes = bytes;
        }
    }
    *ws = ctx->x3_scratch;
    *have = ctx->x3_scratch_bytes;
    return RT_OK;
}

// A narrow-K GEMM (k <= 16 < n) is one write of its output; the tensor-core
// kernels (one k-block, zero-filled past k) write it faster than the CUDA-core
// narrow-K kernel.  Measured on B200 with L2 flushed (dW sweep shapes, TN):
// bf16 at k = 1 / 8 / 16 and 8192 x 8192 outputs, 60 / 60 / 60 us against
// 70 / 108 / 168 us, and never slower at smaller outputs.  f32 operands pay
// the 3xTF32 split and three products: ahead from k = 8 at 8192 x 8192
// (83 against 100 us) and from k = 16 at 4096 x 4096 (36 against 51 us),
// behind below that (k = 1: 167 against 69 us).
bool narrow_k_on_tensor_cores(const rt_ctx* ctx, const GemmDesc& g) {
    if (g.n <= kSkinnyMax || g.k > kSkinnyMax) return false;
    if (ctx->skinny_k_max >= 0 && g.k <= ctx->skinny_k_max) return false;
    if (gemm_tc_supported(ctx, g)) return true;
    if (g.no_alloc || !gemm_x3_supported(ctx, g)) return false;
    return ctx->skinny_k_max >= 0 || (g.k >= 8 && (double)g.k * g.m * g.n >= (double)(1 << 28));
}

// Whether run_gemm takes the tensor-core path in one k slice for g, the path
// whose epilogue can scatter rows to their owners over peer memory.
bool gemm_p2p_capable(const rt_ctx* ctx, const GemmDesc& g) {
    if (!ctx->fast_gemm || g.m < 1 || g.n < 1 || g.k < 1 || g.opt.kind || g.out_dtype != RT_F32) return false;
    if (gemm_skinny_wanted(g) && !narrow_k_on_tensor_cores(ctx, g)) return false;
    if (!gemm_tc_supported(ctx, g)) return false;
    return g.split_k == 1;
}

int run_gemm(rt_ctx* ctx, GemmDesc g, cudaStream_t stream, size_t ws_bytes) {
    RT_TRY(check_gemm(g));
    if (g.m == 0 || g.n == 0) return RT_OK;
    if (g.p2p.world > 0) {
        RT_CHECK(gemm_p2p_capable(ctx, g), "peer-scatter GEMM %lldx%lldx%lld is not on the one-slice tensor-core path",
                 (long long)g.m, (long long)g.n, (long long)g.k);
        return launch_gemm_tc(ctx, g, stream);
    }
    if (g.split_k <= 0) {
        g.split_k = g.c_lo ? 1 : choose_split(ctx, g);
        if ((size_t)g.split_k * g.m * g.n * 4 > ws_bytes || !g.workspace) g.split_k = 1;
    }
    if (g.k == 0) g.split_k = 1;
    if (g.split_k > 1) {
        RT_CHECK(g.workspace, "split-K GEMM needs a workspace");
        RT_CHECK((size_t)g.split_k * g.m * g.n * 4 <= ws_bytes, "split-K workspace too small: %zu < %zu bytes",
                 ws_bytes, (size_t)g.split_k * g.m * g.n * 4);
    }
    if (ctx->fast_gemm && gemm_skinny_wanted(g) && !narrow_k_on_tensor_cores(ctx, g))
        return launch_gemm_skinny(ctx, g, stream);
    if (ctx->fast_gemm && gemm_tc_supported(ctx, g)) return launch_gemm_tc(ctx, g, stream);
    if (ctx->fast_gemm && !g.no_alloc && gemm_x3_supported(ctx, g)) {
        const size_t need = gemm_x3_workspace_bytes(g);
        float* ws = g.x3_ws;
        size_t have = g.x3_ws_bytes;
        if (!ws) RT_TRY(x3_context_scratch(ctx, stream, need, &ws, &have));
        if (ws && have >= need) return launch_gemm_x3(ctx, g, ws, have, stream);
        // no workspace could be had (a capture in progress): the SIMT kernel
    }
    return launch_gemm_simt(ctx, g, stream);
}

static GemmDesc desc_from(rt_layout layout, const rt_tensor* a, const rt_tensor* b, rt_tensor* c, int64_t m,
                          int64_t n, int64_t k) {
    GemmDesc g{};
    g.layout = layout;
    g.in_dtype = a->dtype;
    g.out_dtype = c->dtype;
    g.m = m;
    g.n = n;
    g.k = k;
    g.a = a->ptr;
    g.lda = a->ld;
    g.b = b->ptr;
    g.ldb = b->ld;
    g.c = c->ptr;
    g.ldc = c->ld;
    g.epi = RT_EPI_NONE;
    g.split_k = 1;
    return g;
}

static int same_ctx(const rt_ctx* ctx, std::initializer_list<const rt_tensor*> ts) {
    for (const rt_tensor* t : ts) {
        RT_CHECK(t != nullptr, "tensor argument is NULL");
        RT_CHECK(t->ctx == ctx, "tensor belongs to another context");
    }
    return RT_OK;
}

}  // namespace rt

using namespace rt;

extern "C" {

int rt_gemm(rt_ctx* ctx, const rt_gemm_args* a) {
    RT_CHECK(ctx && a, "rt_gemm: bad arguments");
    GemmDesc g{};
    g.layout = a->layout;
    g.in_dtype = a->in_dtype;
    g.out_dtype = a->out_dtype;
    g.m = a->m;
    g.n = a->n;
    g.k = a->k;
    g.a = a->a;
    g.lda = a->lda;
    g.b = a->b;
    g.ldb = a->ldb;
    g.c = a->c;
    g.ldc = a->ldc;
    g.epi = a->epilogue;
    g.bias = a->bias;
    g.mask = a->mask;
    g.ldmask = a->ldmask;
    g.split_k = a->split_k;
    g.workspace = (float*)a->workspace;
    g.a_lo = a->a_lo;
    g.c_lo = a->c_lo;
    return run_gemm(ctx, g, ctx->stream, a->workspace ? a->workspace_bytes : 0);
}

size_t rt_gemm_workspace_size(rt_ctx* ctx, const rt_gemm_args* a) {
    if (!ctx || !a) return 0;
    GemmDesc g{};
    g.in_dtype = a->in_dtype;
    g.m = a->m;
    g.n = a->n;
    g.k = a->k;
    int s = a->split_k > 0 ? a->split_k : a->c_lo ? 1 : choose_split(ctx, g);
    return s > 1 ? (size_t)s * (size_t)a->m * (size_t)a->n * 4 : 0;
}

int rt_matmul(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c) {
    RT_TRY(same_ctx(ctx, {a, b, c}));
    RT_CHECK(a->cols == b->rows && c->rows == a->rows && c->cols == b->cols,
             "matmul: incompatible shapes [%lld,%lld] x [%lld,%lld] -> [%lld,%lld]", (long long)a->rows,
             (long long)a->cols, (long long)b->rows, (long long)b->cols, (long long)c->rows, (long long)c->cols);
    RT_CHECK(a->dtype == b->dtype, "matmul: operand dtypes differ");
    return run_gemm(ctx, desc_from(RT_NN, a, b, c, a->rows, b->cols, a->cols), ctx->stream, 0);
}

int rt_matmul_at_b(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c) {
    RT_TRY(same_ctx(ctx, {a, b, c}));
    RT_CHECK(a->rows == b->rows && c->rows == a->cols && c->cols == b->cols, "matmul_at_b: incompatible shapes");
    RT_CHECK(a->dtype == b->dtype, "matmul_at_b: operand dtypes differ");
    return run_gemm(ctx, desc_from(RT_TN, a, b, c, a->cols, b->cols, a->rows), ctx->stream, 0);
}

int rt_matmul_a_bt(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c) {
    RT_TRY(same_ctx(ctx, {a, b, c}));
    RT_CHECK(a->cols == b->cols && c->rows == a->rows && c->cols == b->rows, "matmul_a_bt: incompatible shapes");
    RT_CHECK(a->dtype == b->dtype, "matmul_a_bt: operand dtypes differ");
    return run_gemm(ctx, desc_from(RT_NT, a, b, c, a->rows, b->rows, a->cols), ctx->stream, 0);
}

int rt_matmul_bias(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c, const rt_tensor* bias,
                   int relu) {
    RT_TRY(same_ctx(ctx, {a, b, c, bias}));
    RT_CHECK(a->cols == b->rows && c->rows == a->rows && c->cols == b->cols, "matmul_bias: incompatible shapes");
    RT_CHECK(a->dtype == b->dtype, "matmul_bias: operand dtypes differ");
    RT_CHECK(bias->dtype == RT_F32 && bias->rows * bias->cols == b->cols, "matmul_bias: bias must be f32 [1,n]");
    GemmDesc g = desc_from(RT_NN, a, b, c, a->rows, b->cols, a->cols);
    g.epi = relu ? RT_EPI_BIAS_RELU : RT_EPI_BIAS;
    g.bias = (const float*)bias->ptr;
    return run_gemm(ctx, g, ctx->stream, 0);
}

int rt_split_k_suggest(int64_t m, int64_t n, int64_t k) {
    // Gpu::fatias_sugeridas (gpu/mod.rs:1079-1088).
    const int64_t target = 64;
    int64_t blocks = ((m + 63) / 64) * ((n + 63) / 64);
    int64_t tiles_k = (k + 15) / 16;
    if (blocks >= target || tiles_k < 8) return 1;
    int64_t s = target / blocks;
    if (s > tiles_k / 4) s = tiles_k / 4;
    return s < 1 ? 1 : (int)s;
}

int64_t rt_split_k_workspace(int64_t m, int64_t n, int slices) { return (int64_t)slices * m * n; }

int rt_matmul_split_k(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c, rt_tensor* partials,
                      int slices, int transposed) {
    RT_TRY(same_ctx(ctx, {a, b, c, partials}));
    RT_CHECK(slices >= 1, "slices must be >= 1");
    int64_t m = transposed ? a->cols : a->rows;
    int64_t k = transposed ? a->rows : a->cols;
    RT_CHECK(b->rows == k && c->rows == m && c->cols == b->cols, "split_k: incompatible shapes");
    RT_CHECK(a->dtype == b->dtype, "split_k: operand dtypes differ");
    RT_CHECK(partials->dtype == RT_F32, "split_k: partials must be f32");
    size_t cap = (size_t)partials->rows * (size_t)partials->ld * 4;
    GemmDesc g = desc_from(transposed ? RT_TN : RT_NN, a, b, c, m, b->cols, k);
    g.split_k = slices;
    g.workspace = (float*)partials->ptr;
    if (slices == 1) return run_gemm(ctx, g, ctx->stream, cap);
    return run_gemm(ctx, g, ctx->stream, cap);
}

int rt_bias_add(rt_ctx* ctx, rt_tensor* z, const rt_tensor* b) {
    RT_TRY(same_ctx(ctx, {z, b}));
    RT_CHECK(b->dtype == RT_F32 && b->rows * b->cols == z->cols, "bias_add: bias must be f32 [1,cols]");
    return launch_bias_add(ctx, z->ptr, z->dtype, z->rows, z->cols, z->ld, (const float*)b->ptr, ctx->stream);
}

int rt_relu(rt_ctx* ctx, const rt_tensor* x, rt_tensor* y) {
    RT_TRY(same_ctx(ctx, {x, y}));
    RT_CHECK(x->rows == y->rows && x->cols == y->cols && x->dtype == y->dtype, "relu: shape/dtype mismatch");
    return launch_relu(ctx, x->ptr, y->ptr, x->dtype, x->rows, x->cols, x->ld, y->ld, ctx->stream);
}

int rt_relu_bwd(rt_ctx* ctx, const rt_tensor* a, rt_tensor* dz) {
    RT_TRY(same_ctx(ctx, {a, dz}));
    RT_CHECK(a->rows == dz->rows && a->cols == dz->cols && a->dtype == dz->dtype, "relu_bwd: shape/dtype mismatch");
    return launch_relu_bwd(ctx, a->ptr, dz->ptr, a->dtype, a->rows, a->cols, a->ld, dz->ld, ctx->stream);
}

int rt_softmax_xent(rt_ctx* ctx, const rt_tensor* logits, const rt_tensor* labels, rt_tensor* delta, rt_tensor* loss,
                    float scale) {
    RT_TRY(same_ctx(ctx, {logits, labels, delta, loss}));
    RT_CHECK(logits->dtype == RT_F32, "softmax_xent: logits must be f32");
    RT_CHECK(labels->dtype == RT_U32 && labels->rows * labels->cols == logits->rows,
             "softmax_xent: labels must be u32 [rows]");
    RT_CHECK(delta->rows == logits->rows && delta->cols == logits->cols, "softmax_xent: delta shape mismatch");
    RT_CHECK(loss->dtype == RT_F32 && loss->rows * loss->cols == logits->rows && loss->ld >= loss->cols,
             "softmax_xent: loss must be f32 [rows]");
    return launch_xent(ctx, (const float*)logits->ptr, logits->ld, (const uint32_t*)labels->ptr, logits->rows,
                       logits->cols, scale, delta->ptr, delta->dtype, delta->ld, (float*)loss->ptr, ctx->stream);
}

int rt_colsum(rt_ctx* ctx, const rt_tensor* src, rt_tensor* dst, rt_tensor* scratch) {
    RT_TRY(same_ctx(ctx, {src, dst}));
    RT_CHECK(dst->dtype == RT_F32 && dst->rows * dst->cols == src->cols, "colsum: dst must be f32 [1,cols]");
    float* ws = nullptr;
    if (src->rows > 64) {
        RT_CHECK(scratch && scratch->ctx == ctx && scratch->dtype == RT_F32, "colsum: needs an f32 scratch tensor");
        size_t need = (size_t)colsum_scratch_rows(src->rows) * (size_t)src->cols;
        RT_CHECK((size_t)scratch->rows * (size_t)scratch->ld >= need, "colsum: scratch too small (need %zu floats)",
                 need);
        ws = (float*)scratch->ptr;
    }
    return launch_colsum(ctx, src->ptr, src->dtype, src->rows, src->cols, src->ld, ws, (float*)dst->ptr, ctx->stream);
}

static int flat_ok(const rt_tensor* a, const rt_tensor* b) {
    return a->rows == b->rows && a->cols == b->cols && a->ld == b->ld;
}

int rt_adam(rt_ctx* ctx, rt_tensor* theta, rt_tensor* m, rt_tensor* v, const rt_tensor* g, float lr, float beta1,
            float beta2, float eps, int t) {
    RT_TRY(same_ctx(ctx, {theta, m, v, g}));
    RT_CHECK(theta->dtype == RT_F32 && m->dtype == RT_F32 && v->dtype == RT_F32 && g->dtype == RT_F32,
             "adam: all buffers must be f32");
    RT_CHECK(flat_ok(theta, m) && flat_ok(theta, v) && flat_ok(theta, g), "adam: buffer layouts differ");
    RT_CHECK(t >= 1, "adam: step t must be >= 1");
    // Scalars for the explicit t in the context's slot (stream-ordered, so
    // consecutive calls on the context stream do not overlap); no host wait.
    RT_TRY(launch_opt_scalars_at(ctx, ctx->op_scalars, t, beta1, beta2, ctx->stream));
    OptTensor T{(float*)theta->ptr, (const float*)g->ptr, (float*)m->ptr, (float*)v->ptr, nullptr, 0, theta->ld,
                theta->rows * theta->ld};
    return launch_adam(ctx, &T, 1, ctx->op_scalars, lr, beta1, beta2, eps, ctx->stream);
}

int rt_sgd(rt_ctx* ctx, rt_tensor* theta, const rt_tensor* g, float lr) {
    RT_TRY(same_ctx(ctx, {theta, g}));
    RT_CHECK(theta->dtype == RT_F32 && g->dtype == RT_F32 && flat_ok(theta, g), "sgd: f32 buffers of equal layout");
    OptTensor T{(float*)theta->ptr, (const float*)g->ptr, nullptr, nullptr, nullptr, 0, theta->ld,
                theta->rows * theta->ld};
    return launch_sgd(ctx, &T, 1, lr, ctx->stream);
}

int rt_cast(rt_ctx* ctx, const rt_tensor* src, rt_tensor* dst) {
    RT_TRY(same_ctx(ctx, {src, dst}));
    RT_CHECK(src->rows == dst->rows && src->cols == dst->cols, "cast: shape mismatch");
    return launch_cast(ctx, src->ptr, src->dtype, src->ld, dst->ptr, dst->dtype, dst->ld, src->rows, src->cols,
                       ctx->stream);
}

}  // extern "C"
