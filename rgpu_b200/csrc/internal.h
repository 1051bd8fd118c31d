// Internal declarations shared by the translation units of librtgpu.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "optim_math.cuh"
#include "rtgpu.h"

namespace rt {

// ------------------------------------------------------------------ errors
void set_error(const std::string& msg);
int fail(int code, const char* fmt, ...);

#define RT_CUDA(call)                                                                   \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            return ::rt::fail(RT_ERR_CUDA, "%s failed: %s (%s:%d)", #call,              \
                              cudaGetErrorString(e_), __FILE__, __LINE__);              \
    } while (0)

#define RT_CHECK(cond, ...)                                                             \
    do {                                                                                \
        if (!(cond)) return ::rt::fail(RT_ERR_INVALID, __VA_ARGS__);                    \
    } while (0)

#define RT_TRY(expr)                                                                    \
    do {                                                                                \
        int s_ = (expr);                                                                \
        if (s_ != RT_OK) return s_;                                                     \
    } while (0)

// Device-side error codes written to ctx->dev_err[0] by kernels whose
// bounded waits expire (never a trap: the context stays usable).
enum DevErr : int { DEV_OK = 0, DEV_TIMEOUT_PRODUCER = 1, DEV_TIMEOUT_MMA = 2, DEV_TIMEOUT_EPILOGUE = 3, DEV_TIMEOUT_SELFTEST = 4 };

inline size_t dtype_size(rt_dtype d) { return d == RT_BF16 ? 2 : 4; }

}  // namespace rt

struct rt_ctx {
    int device = 0;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int* dev_err = nullptr;  // [4] ints: first device error code, detail
    rt::OptScalars* op_scalars = nullptr;  // Adam scalars for op-level rt_adam (inside dev_err's allocation)
    bool fast_gemm = true;
    bool pair_gemm = true;  // two-CTA tcgen05 tiles where the problem is large enough
    bool f32_tensor = true;  // f32 GEMMs on the tensor cores (3xTF32) when fast_gemm is on
    bool tma_store = true;   // tensor-core GEMM epilogues store C through shared memory and TMA
    bool pdl = true;  // plan GEMMs may launch as programmatic dependents (GemmDesc::pdl)
    bool plan_pdl = false;  // a plan pass is being captured: its small kernels launch as programmatic dependents
    int dyn_tiles = -1;  // plan GEMMs hand out tiles dynamically (GemmDesc::tile_ctr): 1 always, 0 never,
                         // -1 under data parallelism (where other streams' kernels hold SMs at GEMM starts)
    int skinny_k_max = -1;   // narrow-K GEMMs (n > 16) deeper than this go to the tensor cores; -1: by size
    // Grow-only workspace for the hi/lo operand copies of 3xTF32 GEMMs that
    // bring none of their own.  A replaced buffer is kept until the context
    // is destroyed: graphs captured earlier may still reference it.
    float* x3_scratch = nullptr;
    size_t x3_scratch_bytes = 0;
    std::vector<void*> x3_retired;
    int l2_group = 8;
    // device address of rt_matmul_split_k_noalloc's built-in scratch array
    // (looked up on that entry point's first call on this context)
    float* splitk_static = nullptr;
    uint64_t launches = 0;
    char name[256] = {0};
};

struct rt_tensor {
    rt_ctx* ctx = nullptr;
    void* ptr = nullptr;
    rt_dtype dtype = RT_F32;
    int rank = 2;
    int64_t rows = 0, cols = 0, ld = 0;
    bool owned = false;
};

namespace rt {

// ------------------------------------------------------------- kernels
// GEMM problem in "logical" form: C[m,n] = op(A)[m,k] * op(B)[k,n].
constexpr int kMaxPeers = 8;

// dW GEMM output scattered to its owners over peer memory (the sharded
// optimiser's reduce-scatter done by the GEMM epilogue): launch row i < owned_end
// belongs to rank o = i / rows_owned and is stored, as this rank's partial, at
//   peer[o][rank * q_stride + (base_row + i - o * rows_owned) * ld + column]
// in rank o's receive buffer; rows >= owned_end (the bias row) go to C as usual.
// world == 0: off.
struct P2PScatter {
    float* peer[kMaxPeers];
    int rank, world;
    int64_t rows_owned, owned_end, base_row, q_stride, ld;
};

struct GemmDesc {
    rt_layout layout;
    rt_dtype in_dtype, out_dtype;
    int64_t m, n, k;
    const void* a; int64_t lda;
    const void* b; int64_t ldb;
    void* c; int64_t ldc;
    rt_epilogue epi;
    const float* bias;
    const void* mask; int64_t ldmask;
    int split_k;       // >= 1 after planning
    float* workspace;  // split_k * m * n f32 when split_k > 1
    OptFuse opt;       // optimiser applied to theta[i*ldc + j] with gradient C[i,j] (kind 0 = none)
    int max_sms;       // persistent-grid cap (0 = every SM); leaves SMs to concurrent collectives
    float* x3_ws;      // hi/lo operand copies for the 3xTF32 GEMM (null = context scratch)
    size_t x3_ws_bytes;
    bool no_alloc;     // the call may not allocate device memory (3xTF32 then needs a ready workspace)
    P2PScatter p2p;    // world > 0: the epilogue scatters rows to their owners (tensor-core path, one k slice)
    // Split bf16 planes (bf16 only; same layout and leading dimension as the
    // plane they pair with): C = (A + a_lo) B, and the epilogue result v is
    // stored as bf16(v) in c plus bf16(v - bf16(v)) in c_lo.
    const void* a_lo;
    void* c_lo;
    // Programmatic dependent launch of a pair-kernel GEMM on its stream
    // (PDL_NONE: an ordinary launch).  The plan sets it from what the GEMM
    // reads and writes relative to the kernel launched just before it.
    int pdl;
    // A zeroed int that only this launch uses: the pair kernel then hands out
    // tiles dynamically (an atomic counter) instead of round robin.  Null:
    // round robin.
    int* tile_ctr;
};

// How a GEMM launched as a programmatic dependent of the previous kernel on
// its stream waits for it (griddepcontrol.wait, which returns once that grid
// has completed and its writes are visible):
//   PDL_NONE          ordinary launch
//   PDL_WAIT_START    reads the previous kernel's output: every thread waits
//                     before its first global access
//   PDL_WAIT_EPILOGUE the previous kernel reads what this one writes (a dW
//                     GEMM with the update fused, after the dX GEMM that reads
//                     the same weights): the k loop runs at once, the epilogue
//                     waits before its first global access
//   PDL_NO_WAIT       touches nothing the previous kernel writes or reads
//                     while it runs, and what it reads was complete when that
//                     kernel passed its own wait
// A kernel lets its dependents launch only once it has passed its own wait,
// so "complete before the previous kernel's wait" carries down the chain.
enum { PDL_NONE = 0, PDL_WAIT_START = 1, PDL_WAIT_EPILOGUE = 2, PDL_NO_WAIT = 3 };

// Programmatic dependent launch in device code (PTX griddepcontrol): wait
// until the grid this one depends on has completed and its writes are
// visible; let the grids that depend on this one launch.  Both are no-ops in
// a kernel launched the ordinary way.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The small kernels of a captured plan pass (operand split, skinny and
// few-row GEMMs, split-K reduce, softmax-CE, Adam scalars) start with
// pdl_wait(); pdl_launch_dependents(); and, while rt_ctx::plan_pdl is set,
// launch as programmatic dependents of the kernel before them: their launch
// and set-up overlap that kernel's tail, and each waits for it before it
// touches memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Peer memory of a communicator's ranks (comm.cu).
int comm_share_buffer(rt_comm* comm, void* local, void** peers);
void comm_unshare_buffer(rt_comm* comm, void** peers);
int comm_barrier(rt_comm* comm, float* scratch, cudaStream_t st, bool second = false);
bool comm_all_true(rt_comm* comm, bool mine, float* scratch, int* status);
bool gemm_p2p_capable(const rt_ctx* ctx, const GemmDesc& g);

// Kernel launchers: enqueue on `stream`, return RT_OK or an error code.
int launch_gemm_simt(rt_ctx* ctx, const GemmDesc& g, cudaStream_t stream);
// tcgen05/TMA GEMM; returns RT_ERR_UNSUPPORTED when the operands do not meet
// its alignment rules (caller falls back to the SIMT kernel).
int launch_gemm_tc(rt_ctx* ctx, const GemmDesc& g, cudaStream_t stream);
bool gemm_tc_supported(const rt_ctx* ctx, const GemmDesc& g);
int gemm_tc_init(rt_ctx* ctx);
int gemm_tc2_init(rt_ctx* ctx);
bool gemm_tc2_wanted(const rt_ctx* ctx, const GemmDesc& g);
int launch_gemm_tc2(rt_ctx* ctx, const GemmDesc& g, cudaStream_t stream);
// f32 GEMM as three tf32 tcgen05 products (lo*hi + hi*lo + hi*hi); `ws`
// holds the split operand copies (gemm_x3_workspace_bytes).
bool gemm_x3_supported(const rt_ctx* ctx, const GemmDesc& g);
size_t gemm_x3_workspace_bytes(const GemmDesc& g);
int launch_gemm_x3(rt_ctx* ctx, const GemmDesc& g, float* ws, size_t ws_bytes, cudaStream_t stream);
int gemm_x3_init(rt_ctx* ctx);
// Operand planes of a 3xTF32 GEMM: A as [2][m][lda] and B as [2][n][ldb]
// f32, both K-major (plane 0 = hi, plane 1 = lo).
struct X3Planes {
    const float* a;
    int64_t lda, a_plane;
    const float* b;
    int64_t ldb, b_plane;
};
int gemm_tc_x3_init();
int launch_gemm_tc_x3(rt_ctx* ctx, const GemmDesc& g, const X3Planes& x3, cudaStream_t stream);
bool gemm_tc2_x3_wanted(const rt_ctx* ctx, const GemmDesc& g);
int launch_gemm_tc2_x3(rt_ctx* ctx, const GemmDesc& g, const X3Planes& x3, cudaStream_t stream);
int launch_splitk_reduce(rt_ctx* ctx, const GemmDesc& g, cudaStream_t stream);
// Split-K slice count for a tensor-core GEMM (1 = no split).
int choose_split_k(const rt_ctx* ctx, int64_t m, int64_t n, int64_t k, rt_dtype in_dtype);
// GEMMs with n <= kSkinnyMax or k <= kSkinnyMax (the classes dimension of an
// output layer) on CUDA cores: one pass over the large operand.
constexpr int kSkinnyMax = 16;
bool gemm_skinny_wanted(const GemmDesc& g);
int gemm_skinny_init();
int launch_gemm_skinny(rt_ctx* ctx, const GemmDesc& g, cudaStream_t stream);

int launch_xent(rt_ctx* ctx, const float* logits, int64_t ldz, const uint32_t* labels, int64_t n,
                int64_t classes, float scale, void* delta, rt_dtype delta_dtype, int64_t ldd,
                float* loss_rows, cudaStream_t stream);
int launch_colsum(rt_ctx* ctx, const void* src, rt_dtype dt, int64_t rows, int64_t cols, int64_t ld,
                  float* scratch, float* dst, cudaStream_t stream);
int64_t colsum_scratch_rows(int64_t rows);
int launch_bias_add(rt_ctx* ctx, void* z, rt_dtype dt, int64_t rows, int64_t cols, int64_t ld,
                    const float* b, cudaStream_t stream);
int launch_relu(rt_ctx* ctx, const void* x, void* y, rt_dtype dt, int64_t rows, int64_t cols,
                int64_t ldx, int64_t ldy, cudaStream_t stream);
int launch_relu_bwd(rt_ctx* ctx, const void* a, void* dz, rt_dtype dt, int64_t rows, int64_t cols,
                    int64_t lda, int64_t ldz, cudaStream_t stream);
int launch_cast(rt_ctx* ctx, const void* src, rt_dtype sdt, int64_t lds, void* dst, rt_dtype ddt,
                int64_t ldd, int64_t rows, int64_t cols, cudaStream_t stream);
// out[i] = sum over r < parts, in order, of in[r * q_stride + i], i < n.
int launch_sum_partials(rt_ctx* ctx, float* out, const float* in, int64_t q_stride, int parts, int64_t n,
                        cudaStream_t stream);
// The same with part `own_rank` read from `own` instead of `in` (out may be own).
int launch_sum_partials_own(rt_ctx* ctx, float* out, const float* own, const float* in, int64_t q_stride, int parts,
                            int own_rank, int64_t n, cudaStream_t stream);
// Sets column `col` of a [rows, ld] matrix to `value` (the ones column that
// turns the dW GEMM into a dW + db GEMM).
int launch_fill_column(rt_ctx* ctx, void* p, rt_dtype dt, int64_t rows, int64_t ld, int64_t col, float value,
                       cudaStream_t stream);

// Multi-tensor optimiser.  Each entry updates a packed f32 buffer of n
// elements (theta, g, m, v) and optionally writes a bf16 shadow copy.
struct OptTensor {
    float* theta;
    const float* g;
    float* m;
    float* v;
    __nv_bfloat16* shadow;  // may be null
    int64_t shadow_ld;      // row stride of the shadow (elements)
    int64_t cols;           // row length of theta (for the shadow's stride)
    int64_t n;
};
constexpr int kMaxOptTensors = 16;
int launch_opt_step_begin(rt_ctx* ctx, OptScalars* s, float beta1, float beta2, cudaStream_t stream);
// The scalars of Adam step t (t given by the host, no device read of t).
int launch_opt_scalars_at(rt_ctx* ctx, OptScalars* s, int t, float beta1, float beta2, cudaStream_t stream);
int launch_adam(rt_ctx* ctx, const OptTensor* ts, int count, const OptScalars* s, float lr, float beta1,
                float beta2, float eps, cudaStream_t stream);
int launch_sgd(rt_ctx* ctx, const OptTensor* ts, int count, float lr, cudaStream_t stream);

inline void count_launch(rt_ctx* ctx, int n = 1) { ctx->launches += (uint64_t)n; }

}  // namespace rt
