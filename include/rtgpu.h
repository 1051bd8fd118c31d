/*
 * rtgpu.h -- C ABI of the B200 (sm_100a) backend for rtensor's training hot
 * path: Dense-layer GEMMs (Y = XW, dX = dY W^T, dW = X^T dY), fused bias/ReLU
 * and ReLU-mask epilogues, softmax cross-entropy, SGD/Adam, and the whole-step
 * plan (GpuMlp) with optional NCCL data parallelism.
 *
 * Every entry point replaces one item of rtensor's wgpu backend
 * (MMMejias39/RGPU, crates/rtensor/src/gpu/mod.rs) or of its CPU optimiser
 * API; the cited file:line is the interface it stands in for.  Conventions:
 *   - every call returns an rt_status (0 = RT_OK); where the reference panics
 *     on misuse (shape mismatch, batch mismatch) this ABI returns
 *     RT_ERR_INVALID and rt_last_error() describes the problem;
 *   - all work is enqueued asynchronously on the context's CUDA stream; only
 *     the *_download / *_weights / *_grads / *_logits / *_last_loss readers
 *     and rt_ctx_sync block, as Gpu::download / GpuMlp::last_loss do
 *     (gpu/mod.rs:530-566, 1529);
 *   - tensors are row-major with an explicit leading dimension (elements);
 *   - there is no CPU fallback: every compute call runs a CUDA kernel of this
 *     library or fails.
 */
#ifndef RTGPU_H
#define RTGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RTGPU_ABI_VERSION 2

typedef enum {
    RT_OK = 0,
    RT_ERR_INVALID = 1,        /* bad argument or shape (reference: panic!/assert!) */
    RT_ERR_CUDA = 2,           /* CUDA runtime/driver error */
    RT_ERR_NCCL = 3,           /* NCCL error */
    RT_ERR_OOM = 4,            /* device allocation failed */
    RT_ERR_DEVICE_TIMEOUT = 5, /* a bounded device-side wait expired */
    RT_ERR_UNSUPPORTED = 6     /* no device, wrong architecture, feature off */
} rt_status;

typedef enum { RT_F32 = 0, RT_BF16 = 1, RT_U32 = 2 } rt_dtype;

typedef struct rt_ctx rt_ctx;       /* gpu::Gpu        (gpu/mod.rs:224-247) */
typedef struct rt_tensor rt_tensor; /* gpu::GpuTensor  (gpu/mod.rs:191-195) */
typedef struct rt_mlp rt_mlp;       /* gpu::GpuMlp     (gpu/mod.rs:1319-1336) */
typedef struct rt_comm rt_comm;     /* NCCL communicator (no reference counterpart:
                                       data parallelism is absent, crates/rtensor/README.md:123) */

/* ---------------------------------------------------------------- errors */
/* Message of the last failing call on this thread (Result<_, String> Err payload,
 * gpu/mod.rs:263-277). */
const char* rt_last_error(void);
int rt_abi_version(void);

/* --------------------------------------------------------------- context */
/* Gpu::new / Gpu::com_adaptador (gpu/mod.rs:263-298): bind CUDA device
 * `device`, create the context stream, check for sm_100. */
int rt_ctx_create(int device, rt_ctx** out);
int rt_ctx_destroy(rt_ctx* ctx);
/* Gpu::info (gpu/mod.rs:411-413). */
int rt_ctx_info(const rt_ctx* ctx, char* buf, size_t len);
/* Gpu::sync (gpu/mod.rs:564-566); also reports RT_ERR_DEVICE_TIMEOUT when a
 * kernel's bounded wait expired since the last sync. */
int rt_ctx_sync(rt_ctx* ctx);
/* No counterpart in the reference.  Exercises the device-timeout path without
 * a fault: enqueues a kernel whose one thread waits on a barrier that nothing
 * signals, with the GEMMs' bounded wait (2 s), and records a timeout when it
 * gives up.  The next rt_ctx_sync returns RT_ERR_DEVICE_TIMEOUT; the context
 * stays usable. */
int rt_ctx_selftest_timeout(rt_ctx* ctx);
/* The cudaStream_t work is enqueued on (Gpu::queue, gpu/mod.rs:422-424). */
void* rt_ctx_stream(rt_ctx* ctx);
/* Use a caller-owned cudaStream_t instead (NULL restores the context's own).
 * No counterpart in the reference: wgpu owns its one queue. */
int rt_ctx_set_stream(rt_ctx* ctx, void* stream);
/* Gpu::set_fast_gemm (gpu/mod.rs:442-448): 1 = tcgen05/TMA tensor-core GEMM
 * where the operands allow it (default), 0 = tiled SIMT GEMM everywhere. */
int rt_ctx_set_fast_gemm(rt_ctx* ctx, int on);
/* f32 GEMMs under set_fast_gemm(1): 1 = tensor cores as three tf32 products
 * (3xTF32, about f32 accuracy; default), 0 = the SIMT f32 kernel.  Same
 * switch family as Gpu::set_fast_gemm (gpu/mod.rs:442-448); the reference's
 * f32 GEMMs have no tensor-core form.  RTGPU_F32_TENSOR=0 sets the default. */
int rt_ctx_set_f32_tensor(rt_ctx* ctx, int on);
/* Gpu::set_grupo_l2 (gpu/mod.rs:452-458): tile rows per L2 raster group. */
int rt_ctx_set_l2_group(rt_ctx* ctx, int group);
/* Number of kernels this context has launched so far (evidence counter).  No
 * counterpart in the reference. */
int rt_ctx_launch_count(const rt_ctx* ctx, uint64_t* out);

/* Page-locked host memory for asynchronous copies.  No counterpart in the
 * reference (wgpu stages host data itself); used with rt_mlp_step_host. */
int rt_host_alloc(size_t bytes, void** out);
int rt_host_free(void* p);

/* --------------------------------------------------------------- tensors */
/* Gpu::zeros (gpu/mod.rs:501-506): rank 1 or 2, leading dimension padded so
 * that every row starts 16-byte aligned. */
int rt_tensor_zeros(rt_ctx* ctx, rt_dtype dtype, int rank, const int64_t* shape, rt_tensor** out);
/* Gpu::upload (gpu/mod.rs:509-516): host f32 -> device tensor of `dtype`
 * (RT_BF16 rounds to nearest even on the device). */
int rt_tensor_upload(rt_ctx* ctx, rt_dtype dtype, const float* host, int rank, const int64_t* shape,
                     rt_tensor** out);
/* upload_labels (gpu/mod.rs:1671-1675). */
int rt_upload_labels(rt_ctx* ctx, const uint32_t* labels, int64_t n, rt_tensor** out);
/* Gpu::download (gpu/mod.rs:530-545): blocking; bf16 widens to f32.  `host`
 * holds rows*cols floats, packed (no padding). */
int rt_tensor_download(rt_ctx* ctx, const rt_tensor* t, float* host);
/* Non-owning view of caller memory (cudarc-style raw handle).  `ld` in
 * elements; 0 means packed.  The reference's GpuTensor always owns its buffer
 * (gpu/mod.rs:191-195); rt_tensor_free releases what rt_tensor_zeros,
 * rt_tensor_upload and rt_upload_labels allocated, and only the handle of a
 * view. */
int rt_tensor_wrap(rt_ctx* ctx, void* device_ptr, rt_dtype dtype, int rank, const int64_t* shape,
                   int64_t ld, rt_tensor** out);
int rt_tensor_free(rt_tensor* t);
void* rt_tensor_ptr(const rt_tensor* t);
/* GpuTensor's shape fields (gpu/mod.rs:191-195): rows, cols, ld (rank-1
 * tensors report rows = 1). */
int rt_tensor_dims(const rt_tensor* t, int64_t* rows, int64_t* cols, int64_t* ld);

/* ------------------------------------------------------------------- ops */
/* All ops enqueue on the context stream.  GEMM operands are f32 or bf16 (both
 * operands of one GEMM share a type); outputs are f32 or bf16; accumulation is
 * always f32. */

/* Gpu::op_matmul (gpu/mod.rs:685-688): C[m,n] = A[m,k] B[k,n]. */
int rt_matmul(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c);
/* Gpu::op_matmul_at_b (gpu/mod.rs:691-694): C = A^T B with A stored [k,m] (dW = X^T dY). */
int rt_matmul_at_b(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c);
/* Gpu::op_matmul_a_bt (gpu/mod.rs:697-700): C = A B^T with B stored [n,k] (dX = dY W^T). */
int rt_matmul_a_bt(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c);
/* Gpu::op_matmul_bias (gpu/mod.rs:722-749): C = A B + 1 bias, ReLU if relu != 0. */
int rt_matmul_bias(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c,
                   const rt_tensor* bias, int relu);
/* Gpu::ops_split_k (gpu/mod.rs:1095-1146): C = A B (transposed = 0) or A^T B
 * (transposed = 1) with k split in `slices`; `partials` holds >= slices*m*n
 * f32 (rt_split_k_workspace).  The slices are summed in a fixed order. */
int rt_matmul_split_k(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c,
                      rt_tensor* partials, int slices, int transposed);
/* Gpu::fatias_sugeridas (gpu/mod.rs:1079-1088), same rule: 64-block target,
 * 64x64 blocks, at least 4 16-deep k tiles per slice. */
int rt_split_k_suggest(int64_t m, int64_t n, int64_t k);
int64_t rt_split_k_workspace(int64_t m, int64_t n, int slices);
/* No counterpart in the reference.  The same split-K GEMM as
 * rt_matmul_split_k, for callers that cannot allocate device memory when they
 * call (a host runtime whose own allocator owns the device memory, a loop
 * that forbids allocation after start-up): the partial sums live in a fixed
 * 16 MiB array built into the library (rt_split_k_static_capacity() floats
 * per device, held until the process exits).  Calls needing slices*m*n above
 * that capacity fail with RT_ERR_INVALID.  All calls on a device share the
 * array, so calls whose kernels overlap on the GPU race and must be
 * serialised.  The first call on a context looks up the array's device
 * address (cudaGetSymbolAddress) and keeps it in the context; make that first
 * call before any stream capture begins. */
int rt_matmul_split_k_noalloc(rt_ctx* ctx, const rt_tensor* a, const rt_tensor* b, rt_tensor* c,
                              int slices, int transposed);
int64_t rt_split_k_static_capacity(void);

/* Full-control GEMM used by the plan (and by Rust callers that manage their
 * own buffers).  It folds the reference's GEMM builders into one call:
 * op_matmul / op_matmul_at_b / op_matmul_a_bt (gpu/mod.rs:685-700) by layout,
 * op_matmul_bias (722-749) and op_relu_bwd (778-788) by epilogue, ops_split_k
 * (1095-1146) by split_k.  Logical A is [m,k], logical B is [k,n]:
 *   RT_NN: A stored [m,k] (lda), B stored [k,n] (ldb)      Y  = X W
 *   RT_NT: A stored [m,k],       B stored [n,k]            dX = dY W^T
 *   RT_TN: A stored [k,m],       B stored [k,n]            dW = X^T dY
 * Epilogues (gemm.rs:372-494 MM_EPILOGO and kernels.rs:119-131 RELU_BWD):
 *   RT_EPI_NONE       C = acc
 *   RT_EPI_BIAS       C = acc + bias[j]
 *   RT_EPI_BIAS_RELU  C = max(acc + bias[j], 0)
 *   RT_EPI_RELU_MASK  C = acc * 1[mask[i,j] > 0]   (mask has the output dtype)
 * split_k: 0 = choose, 1 = none, >1 = that many k slices (needs workspace of
 * rt_gemm_workspace_size bytes).
 * Split bf16 planes (NULL = off; bf16 only, same layout and leading dimension
 * as the plane they pair with, no counterpart in the reference):
 *   a_lo  low-order plane of A: the GEMM computes (A + a_lo) B, two bf16
 *         products into one f32 accumulator, so an f32 operand stored as the
 *         pair hi = bf16(x), lo = bf16(x - hi) keeps ~16 significant bits;
 *   c_lo  low-order plane of C: C receives bf16(v) and c_lo receives
 *         bf16(v - bf16(v)) of every epilogue result v (split_k must be 1). */
typedef enum { RT_NN = 0, RT_NT = 1, RT_TN = 2 } rt_layout;
typedef enum { RT_EPI_NONE = 0, RT_EPI_BIAS = 1, RT_EPI_BIAS_RELU = 2, RT_EPI_RELU_MASK = 3 } rt_epilogue;
typedef struct {
    rt_layout layout;
    rt_dtype in_dtype;  /* RT_F32 or RT_BF16 */
    rt_dtype out_dtype; /* RT_F32 or RT_BF16 */
    int64_t m, n, k;
    const void* a; int64_t lda;
    const void* b; int64_t ldb;
    void* c; int64_t ldc;
    rt_epilogue epilogue;
    const float* bias;
    const void* mask; int64_t ldmask;
    int split_k;
    void* workspace; size_t workspace_bytes;
    const void* a_lo;
    void* c_lo;
} rt_gemm_args;
int rt_gemm(rt_ctx* ctx, const rt_gemm_args* args);
size_t rt_gemm_workspace_size(rt_ctx* ctx, const rt_gemm_args* args);

/* Gpu::op_bias_add (gpu/mod.rs:752-762): Z += 1 b. */
int rt_bias_add(rt_ctx* ctx, rt_tensor* z, const rt_tensor* b);
/* Gpu::op_relu (gpu/mod.rs:765-775): Y = max(X, 0). */
int rt_relu(rt_ctx* ctx, const rt_tensor* x, rt_tensor* y);
/* Gpu::op_relu_bwd (gpu/mod.rs:778-788): dz *= 1[a > 0], in place. */
int rt_relu_bwd(rt_ctx* ctx, const rt_tensor* a, rt_tensor* dz);
/* Gpu::op_softmax_xent (gpu/mod.rs:791-808): per-row loss
 * -ln(max(p_y, 1e-12)) and delta = (P - Y) * scale (scale = 1/n for the
 * losses.rs:99-115 adjoint; pass 1/n_global under data parallelism). */
int rt_softmax_xent(rt_ctx* ctx, const rt_tensor* logits, const rt_tensor* labels, rt_tensor* delta,
                    rt_tensor* loss, float scale);
/* Gpu::ops_colsum (gpu/mod.rs:838-855): dst[1,m] = 1^T src, two fixed-order
 * stages through `scratch` (>= ceil(rows/64) x cols f32). */
int rt_colsum(rt_ctx* ctx, const rt_tensor* src, rt_tensor* dst, rt_tensor* scratch);
/* Gpu::op_adam + atualizar_adam (gpu/mod.rs:859-907) with the CPU optimiser's
 * arithmetic (optim.rs:163-198: pre-inverted bias corrections for step t). */
int rt_adam(rt_ctx* ctx, rt_tensor* theta, rt_tensor* m, rt_tensor* v, const rt_tensor* g,
            float lr, float beta1, float beta2, float eps, int t);
/* Sgd::step without momentum (optim.rs:80-95): theta -= g * lr.  The
 * reference has no GPU kernel for it. */
int rt_sgd(rt_ctx* ctx, rt_tensor* theta, const rt_tensor* g, float lr);
/* Gpu::op_empacota_f16 (gpu/mod.rs:1165-1176), bf16 instead of f16:
 * dst (bf16) = round-to-nearest-even(src (f32)). */
int rt_cast(rt_ctx* ctx, const rt_tensor* src, rt_tensor* dst);

/* ------------------------------------------------------------ MLP plan */
typedef enum { RT_OPT_NONE = 0, RT_OPT_SGD = 1, RT_OPT_ADAM = 2 } rt_optimizer;
/* How a bf16 plan stores its hidden activations (f32 plans ignore it):
 *   RT_ACT_SPLIT  (default) each activation that feeds another hidden layer
 *                 as the bf16 pair hi + lo; that layer's forward GEMM reads
 *                 both planes (two bf16 products), the dW GEMM, the ReLU
 *                 mask and the output layer read hi.  Gradients stay within
 *                 the 2e-2 relative-L2 bar of the f32 CPU backend.
 *   RT_ACT_BF16   one bf16 rounding per activation: the forward GEMMs of the
 *                 hidden layers do half the tensor work, but the rounding
 *                 moves pre-activations by ~1e-3 of their spread, which flips
 *                 ReLU masks near zero and puts hidden-layer gradients
 *                 2e-2 .. 8e-2 away from the f32 CPU backend. */
typedef enum { RT_ACT_SPLIT = 0, RT_ACT_BF16 = 1 } rt_activations;
typedef struct {
    int n_layers;          /* Dense layers; dims has n_layers + 1 entries */
    const int64_t* dims;   /* d_0 (inputs) .. d_L (classes) */
    int64_t batch;         /* rows per step on this device */
    int64_t global_batch;  /* rows per step over all ranks (0 = batch) */
    rt_dtype dtype;        /* RT_F32, or RT_BF16: bf16 operands and activations
                              (see rt_activations), f32 accumulate, f32 master
                              weights + bf16 shadow */
    rt_optimizer optimizer;
    float lr, beta1, beta2, eps;
    rt_activations activations; /* bf16 plans: RT_ACT_SPLIT (0, default) or RT_ACT_BF16 */
} rt_mlp_config;

/* GpuMlp::from_params (gpu/mod.rs:1341-1482): hidden layers ReLU, output
 * linear + softmax-CE.  weights[l] is W_l [d_l, d_{l+1}] row-major f32,
 * biases[l] is b_l [d_{l+1}] (NULL = zeros).  The step is captured into a
 * CUDA graph on first use. */
int rt_mlp_create(rt_ctx* ctx, const rt_mlp_config* cfg, const float* const* weights,
                  const float* const* biases, rt_mlp** out);
int rt_mlp_destroy(rt_mlp* mlp);
/* GpuMlp::step (gpu/mod.rs:1499-1511): x [batch, d_0] and labels [batch]
 * already on the device (copied into the plan's input buffers, as
 * GpuMlp::carregar does, gpu/mod.rs:1486-1495), then forward, backward,
 * (allreduce,) update.  x_dtype is RT_F32 or RT_BF16. */
int rt_mlp_step(rt_mlp* mlp, const void* x_dev, rt_dtype x_dtype, const uint32_t* labels_dev);
/* No counterpart in the reference (GpuMlp::step takes device buffers, and
 * carregar copies them device to device).  The same step from page-locked or
 * pageable HOST buffers: the host->device
 * copies and, when loss_rows_host != NULL, the device->host copy of the
 * per-row losses ([batch] f32) are enqueued with the step.  Returns once
 * enqueued; the loss buffer is valid after rt_ctx_sync. */
int rt_mlp_step_host(rt_mlp* mlp, const void* x_host, rt_dtype x_dtype, const uint32_t* labels_host,
                     float* loss_rows_host);
/* GpuMlp::forward_only (gpu/mod.rs:1514-1521): the input is copied into the
 * plan and the forward GEMMs run as a CUDA graph captured on first use. */
int rt_mlp_forward_only(rt_mlp* mlp, const void* x_dev, rt_dtype x_dtype);
/* GpuMlp::forward_only followed by GpuMlp::logits (gpu/mod.rs:1514-1526) from
 * page-locked or pageable HOST memory: the host->device copy of x (on a copy
 * stream, overlapping the previous call's forward), the captured forward and,
 * when logits_host != NULL, the device->host copy of the [batch, classes] f32
 * logits are enqueued.  Returns once enqueued; logits are valid after
 * rt_ctx_sync. */
int rt_mlp_forward_host(rt_mlp* mlp, const void* x_host, rt_dtype x_dtype, float* logits_host);
/* GpuMlp::logits (gpu/mod.rs:1524-1526): [batch, classes] f32, blocking. */
int rt_mlp_logits(rt_mlp* mlp, float* host);
/* GpuMlp::last_loss (gpu/mod.rs:1529-1531): mean row loss, blocking. */
int rt_mlp_last_loss(rt_mlp* mlp, float* out);
/* No counterpart in the reference (GpuMlp is single-device).  The last step's
 * mean loss over the global batch: with a communicator the
 * ranks' per-row losses are all-gathered and summed in global row order
 * (collective: every rank calls it); without one, rt_mlp_last_loss. */
int rt_mlp_global_loss(rt_mlp* mlp, float* out);
/* GpuMlp::weights / grads (gpu/mod.rs:1534-1551) for one layer, blocking,
 * packed f32 (w: d_l*d_{l+1}, b: d_{l+1}); either pointer may be NULL. */
int rt_mlp_weights(rt_mlp* mlp, int layer, float* w, float* b);
int rt_mlp_grads(rt_mlp* mlp, int layer, float* dw, float* db);
/* Param::set (tape.rs:119-121) on the device copy: overwrite W_l / b_l. */
int rt_mlp_set_weights(rt_mlp* mlp, int layer, const float* w, const float* b);
/* Checkpoint / resume of a plan's training state: the f32 masters [W_l; b_l],
 * the Adam moments m_l, v_l and the Adam step count.  The reference keeps no
 * such state format; its nearest pieces are GpuMlp::weights
 * (gpu/mod.rs:1534-1551) and Param::set (tape.rs:119-121), which carry the
 * weights but not the optimiser.  Buffer layout (host byte order):
 *   rt_mlp_state_header, dims[n_layers + 1] (int64),
 *   then per layer l: [d_l + 1, d_{l+1}] f32 row-major ([W_l; b_l], bias last),
 *   and for Adam the m_l and v_l blocks of the same shape.
 * Save waits for the device; load checks the header against the plan (layer
 * dims and optimiser must match), restores the step count and rebuilds the
 * bf16 weight shadow.  Data-parallel ranks hold identical state: save on one
 * rank, load on every rank. */
#define RT_MLP_STATE_MAGIC 0x534D5452u /* "RTMS" */
typedef struct {
    uint32_t magic;
    uint32_t version;  /* 1 */
    int32_t n_layers;
    int32_t optimizer; /* rt_optimizer */
    int64_t adam_step; /* Adam steps taken (bias-correction t) */
} rt_mlp_state_header;
int rt_mlp_state_size(rt_mlp* mlp, size_t* bytes);
int rt_mlp_save_state(rt_mlp* mlp, void* host, size_t bytes);
int rt_mlp_load_state(rt_mlp* mlp, const void* host, size_t bytes);
/* GpuMlp::dispatches_por_passo (gpu/mod.rs:1559-1561): kernels per step. */
int rt_mlp_dispatches_per_step(rt_mlp* mlp, int* out);
/* Gpu::perfilar (gpu/mod.rs:1245-1286): when on, the captured step records a
 * CUDA event around every kernel; rt_mlp_op_times then reports, for the last
 * step, the label, the algorithmic FLOPs (0 for non-GEMM kernels) and the
 * device milliseconds of op i < count. */
int rt_mlp_enable_timing(rt_mlp* mlp, int on);
int rt_mlp_op_count(rt_mlp* mlp, int* count);
int rt_mlp_op_time(rt_mlp* mlp, int i, const char** label, double* flops, float* ms);
/* No counterpart in the reference (GpuMlp is single-device).  Attach a
 * communicator: dW/db are summed over ranks on a second stream,
 * chunk by chunk as backward produces them.  f32 plans, plans without an
 * optimiser and RTGPU_GRAD_COMM=bf16 allreduce the gradients.  bf16 plans with
 * SGD or Adam shard the optimiser (ZeRO stage 1; RTGPU_SHARDED_OPT=0 turns it
 * off): each chunk's weight-row gradients are reduce-scattered, every rank
 * updates its 1/world slice of the f32 masters and moments, and the bf16
 * weights the GEMMs read are all-gathered; bias rows stay replicated.  On a
 * sharded plan rt_mlp_weights, rt_mlp_grads and rt_mlp_save_state first
 * all-gather the f32 state, so every rank must call them together. */
int rt_mlp_set_comm(rt_mlp* mlp, rt_comm* comm);
/* How the attached communicator sums gradients (rt_comm_mode).
 * RT_COMM_SHARDED_P2P: sharded optimiser whose dW GEMMs (some or all layers)
 * scatter their rows to the owning ranks over NVLink peer memory from the
 * GEMM epilogue instead of an NCCL reduce-scatter (RTGPU_P2P_RS=1).
 * RT_COMM_SHARDED_CE: sharded optimiser whose gradient pieces and updated
 * bf16 weights move between the ranks' mapped buffers by copy-engine copies
 * over NVLink (no SM moves them), with one-float NCCL barriers; the default
 * for sharded plans where every rank maps every other rank's buffers
 * (RTGPU_CE_EXCHANGE=0 keeps NCCL's reduce-scatter and all-gather). */
typedef enum {
    RT_COMM_NONE = 0,
    RT_COMM_ALLREDUCE = 1,
    RT_COMM_ALLREDUCE_BF16 = 2,
    RT_COMM_SHARDED_OPT = 3,
    RT_COMM_SHARDED_P2P = 4,
    RT_COMM_SHARDED_CE = 5
} rt_comm_mode;
int rt_mlp_comm_mode(rt_mlp* mlp, int* mode);
/* The plan's data-parallel layout, as host-only queries (no device or plan
 * needed), so that a host runtime sharding the same parameter blocks can agree
 * with the library on where every slice lives.  No counterpart in the
 * reference (GpuMlp is single-device); they describe rt_mlp_set_comm's
 * exchange.  A layer with d inputs and `units` outputs keeps W and b as one
 * [d+1, rt_plan_ld(units)] f32 block (bias last).  Its dW GEMM runs in
 * rt_plan_dw_chunks(...) row chunks (data_parallel: a communicator is
 * attached; fused_update: one device with SGD/Adam, the update inside the dW
 * epilogue; honours RTGPU_FIRST_LAYER_CHUNKS / RTGPU_DW_CHUNKS); chunk c holds
 * rows [rt_plan_chunk_row(d+1, chunks, c), rt_plan_chunk_row(d+1, chunks, c+1)).
 * Under the sharded optimiser rank r of `world` updates the flat elements
 * [*offset, *offset + returned length) of each chunk's weight rows (the bias
 * row stays replicated); -1 on bad arguments. */
int64_t rt_plan_ld(int64_t units);
int rt_plan_dw_chunks(int layer, int64_t d, int64_t units, int data_parallel, int fused_update);
int64_t rt_plan_chunk_row(int64_t rows, int chunks, int c);
int64_t rt_plan_shard_slice(int64_t d, int64_t units, int64_t r0, int64_t r1, int world, int rank,
                            int64_t* offset);

/* ------------------------------------------------------ autodiff tape */
/* Reverse-mode tape on the GPU for the ops a Dense network is made of.  All
 * values and adjoints are f32 device buffers owned by the tape; every op and
 * the backward sweep only enqueue kernels on the context stream. */
typedef struct rt_tape rt_tape;   /* tape::Tape  (tape.rs:43-67) */
typedef struct rt_var rt_var;     /* tape::Var   (tape.rs:136-184); owned by its tape */
typedef struct rt_param rt_param; /* tape::Param (tape.rs:76-132) */
typedef struct rt_adam_state rt_adam_state; /* optim::Adam (optim.rs:142-160) */

/* Param::new (tape.rs:86-92): rows x cols f32 from host (NULL = zeros). */
int rt_param_create(rt_ctx* ctx, const float* host, int64_t rows, int64_t cols, rt_param** out);
int rt_param_destroy(rt_param* p);
/* Param::value (tape.rs:102-104), blocking copy to host. */
int rt_param_read(rt_param* p, float* host);
/* Param::set (tape.rs:119-121). */
int rt_param_write(rt_param* p, const float* host);
/* Param::value (tape.rs:102-104) as a device view (non-owning rt_tensor). */
int rt_param_value(rt_param* p, rt_tensor** view);
/* Tape::new (tape.rs:50-52) / drop. */
int rt_tape_create(rt_ctx* ctx, rt_tape** out);
int rt_tape_destroy(rt_tape* t);
int rt_tape_len(rt_tape* t, int* out);
/* constant (tape.rs:70-73): copies value (f32) into a leaf. */
int rt_tape_constant(rt_tape* t, const rt_tensor* value, rt_var** out);
/* Param::watch (tape.rs:124-131): the leaf of p, reused if already watched. */
int rt_param_watch(rt_param* p, rt_tape* t, rt_var** out);
/* Var::matmul (ops.rs:125-129), Var::add with [1,n] row broadcast
 * (ops.rs:49-53), Var::relu (ops.rs:190-194). */
int rt_var_matmul(rt_var* a, rt_var* b, rt_var** out);
int rt_var_add(rt_var* a, rt_var* b, rt_var** out);
int rt_var_relu(rt_var* a, rt_var** out);
/* losses::softmax_cross_entropy (losses.rs:99-115) with integer labels
 * (u32 [rows]) in place of the one-hot rows; the scalar loss must be the root
 * of the backward sweep. */
int rt_softmax_cross_entropy(rt_var* logits, const rt_tensor* labels, rt_var** out);
/* The remaining differentiable ops of ops.rs on rank-2 values.  Binary ops
 * broadcast a [1,n] row, [m,1] column or [1,1] scalar operand against [m,n]
 * (tensor.rs:183-246) and reduce each operand's adjoint back to its shape
 * (tensor.rs:399-438):
 *   RT_ADD Var::add (ops.rs:49-53)   RT_SUB Var::sub (61-64)
 *   RT_MUL Var::mul (76-82)          RT_DIV Var::div (93-101) */
typedef enum { RT_ADD = 0, RT_SUB = 1, RT_MUL = 2, RT_DIV = 3 } rt_binary_op;
int rt_var_binary(rt_var* a, rt_var* b, rt_binary_op op, rt_var** out);
/* Pointwise ops; `param` is k for scale/offset and the slope for leaky_relu:
 *   RT_SCALE Var::scale (ops.rs:132-135)   RT_OFFSET Var::offset (139-142)
 *   RT_NEG Var::neg (145-147)              RT_SQUARE Var::square (150-154)
 *   RT_SQRT Var::sqrt (158-162)            RT_EXP Var::exp (166-170)
 *   RT_LN Var::ln (176-180)                RT_RELU Var::relu (190-194)
 *   RT_LEAKY_RELU Var::leaky_relu (197-204)
 *   RT_SIGMOID Var::sigmoid (212-216)      RT_TANH Var::tanh (223-227) */
typedef enum {
    RT_SCALE = 0, RT_OFFSET = 1, RT_NEG = 2, RT_SQUARE = 3, RT_SQRT = 4, RT_EXP = 5,
    RT_LN = 6, RT_RELU = 7, RT_LEAKY_RELU = 8, RT_SIGMOID = 9, RT_TANH = 10
} rt_unary_op;
int rt_var_unary(rt_var* a, rt_unary_op op, float param, rt_var** out);
/* Var::sum, Var::mean (ops.rs:239-255): scalar [1,1] results. */
int rt_var_sum(rt_var* a, rt_var** out);
int rt_var_mean(rt_var* a, rt_var** out);
/* Var::softmax (ops.rs:288-309): row softmax with its O(c) adjoint. */
int rt_var_softmax(rt_var* a, rt_var** out);
/* losses::mse (losses.rs:31-34), losses::mae (46-55) and
 * losses::binary_cross_entropy (143-160) against an f32 target of the
 * prediction's shape (copied into the tape). */
int rt_loss_mse(rt_var* pred, const rt_tensor* target, rt_var** out);
int rt_loss_mae(rt_var* pred, const rt_tensor* target, rt_var** out);
int rt_loss_bce(rt_var* probs, const rt_tensor* target, rt_var** out);
/* losses::accuracy (losses.rs:181-185): fraction of rows whose first arg-max
 * equals the label (u32 [rows]); blocking. */
int rt_accuracy(rt_ctx* ctx, const rt_tensor* logits, const rt_tensor* labels, float* out);
/* Var::value (tape.rs:143-145) as a device view; Tensor::item (blocking). */
int rt_var_value(rt_var* v, rt_tensor** view);
int rt_var_item(rt_var* v, float* out);
/* Var::backward (tape.rs:187-229): enqueue the reverse sweep from a scalar. */
int rt_var_backward(rt_var* root);
/* Grads::of (tape.rs:238-243): device view of the parameter's gradient, or
 * *view = NULL when the parameter took no part in the graph. */
int rt_grads_of(rt_tape* t, rt_param* p, rt_tensor** view);
/* Sgd::step without momentum (optim.rs:80-95). */
int rt_sgd_step(rt_ctx* ctx, int n, rt_param* const* params, rt_tape* grads, float lr);
/* Adam::with_betas (optim.rs:157-159) and Adam::step (optim.rs:162-198). */
int rt_adam_create(rt_ctx* ctx, float lr, float beta1, float beta2, float eps, rt_adam_state** out);
int rt_adam_destroy(rt_adam_state* a);
int rt_adam_step(rt_adam_state* a, int n, rt_param* const* params, rt_tape* grads);
/* Sgd::new / Sgd::with_momentum (optim.rs:64-77) and Sgd::step (81-114): the
 * velocity v = v * mu + g * lr is kept per parameter, theta -= v. */
typedef struct rt_sgd_state rt_sgd_state;
int rt_sgd_create(rt_ctx* ctx, float lr, float momentum, rt_sgd_state** out);
int rt_sgd_destroy(rt_sgd_state* s);
int rt_sgd_state_step(rt_sgd_state* s, int n, rt_param* const* params, rt_tape* grads);

/* ------------------------------------------------------------------ NCCL */
/* No counterpart in the reference (single-device).  NCCL communicator over
 * NVLink, one process per GPU.  128-byte ncclUniqueId, created on one rank and
 * shared out of band. */
int rt_comm_unique_id(unsigned char id[128]);
int rt_comm_init(rt_ctx* ctx, int rank, int world, const unsigned char id[128], rt_comm** out);
int rt_comm_destroy(rt_comm* comm);
/* In-place sum over ranks on the context stream. */
int rt_comm_allreduce_f32(rt_comm* comm, float* dev_buf, int64_t count);

#ifdef __cplusplus
}
#endif
#endif /* RTGPU_H */
