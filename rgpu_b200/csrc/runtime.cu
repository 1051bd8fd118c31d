// Context, tensors and errors: the part of rtensor's `Gpu` / `GpuTensor`
// (crates/rtensor/src/gpu/mod.rs:180-566) that owns the device, its stream
// and buffers.
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "internal.h"

namespace rt {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

// Reads and clears the device error word; maps it to a status.
static int check_device_error(rt_ctx* ctx) {
    int h[4] = {0, 0, 0, 0};
    RT_CUDA(cudaMemcpy(h, ctx->dev_err, sizeof h, cudaMemcpyDeviceToHost));
    if (h[0] != DEV_OK) {
        int zero[4] = {0, 0, 0, 0};
        RT_CUDA(cudaMemcpy(ctx->dev_err, zero, sizeof zero, cudaMemcpyHostToDevice));
        if (h[0] == DEV_TIMEOUT_SELFTEST)
            return fail(RT_ERR_DEVICE_TIMEOUT, "the self-test wait expired on the device, as it is meant to");
        const char* role = h[0] == DEV_TIMEOUT_PRODUCER ? "TMA producer"
                           : h[0] == DEV_TIMEOUT_MMA    ? "MMA issuer"
                                                        : "epilogue";
        return fail(RT_ERR_DEVICE_TIMEOUT,
                    "a GEMM %s wait expired on the device (detail %d); the kernel returned early "
                    "and its output is invalid",
                    role, h[1]);
    }
    return RT_OK;
}

}  // namespace rt

using namespace rt;

extern "C" {

const char* rt_last_error(void) { return g_last_error.c_str(); }
int rt_abi_version(void) { return RTGPU_ABI_VERSION; }

int rt_ctx_create(int device, rt_ctx** out) {
    RT_CHECK(out != nullptr, "rt_ctx_create: out is NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return fail(RT_ERR_UNSUPPORTED, "no CUDA device available (%s)", cudaGetErrorString(e));
    RT_CHECK(device >= 0 && device < n, "device %d out of range (%d devices)", device, n);
    RT_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    RT_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(RT_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only",
                    device, prop.major, prop.minor);
    rt_ctx* c = new rt_ctx;
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    c->cc_major = prop.major;
    c->cc_minor = prop.minor;
    snprintf(c->name, sizeof c->name, "%s (sm_%d%d, %d SMs, %.1f GB)", prop.name, prop.major, prop.minor,
             prop.multiProcessorCount, prop.totalGlobalMem / 1e9);
    // RTGPU_MAIN_PRIORITY=1 puts the context's stream one level above the
    // lowest priority: under data parallelism the plan's update kernels
    // (lowest, on a side stream) then yield freed SMs to its GEMMs, and the
    // collectives' streams sit above both.  Default: the lowest level.
    int least = 0, greatest = 0;
    cudaDeviceGetStreamPriorityRange(&least, &greatest);
    const char* pr_env = getenv("RTGPU_MAIN_PRIORITY");
    const int prio = (greatest < least && pr_env && pr_env[0] == '1') ? least - 1 : least;
    cudaError_t e1 = cudaStreamCreateWithPriority(&c->own_stream, cudaStreamNonBlocking, prio);
    // one allocation: the device error word (16 bytes) and, 32 bytes in, the
    // Adam scalars of op-level rt_adam calls
    cudaError_t e2 = cudaMalloc(&c->dev_err, 64);
    if (e1 != cudaSuccess || e2 != cudaSuccess) {
        delete c;
        return fail(RT_ERR_CUDA, "context setup failed: %s", cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
    }
    c->stream = c->own_stream;
    cudaMemsetAsync(c->dev_err, 0, 64, c->stream);
    c->op_scalars = reinterpret_cast<rt::OptScalars*>(reinterpret_cast<char*>(c->dev_err) + 32);
    cudaStreamSynchronize(c->stream);
    const char* pair_env = getenv("RTGPU_PAIR_GEMM");
    c->pair_gemm = !(pair_env && pair_env[0] == '0');
    const char* f32_env = getenv("RTGPU_F32_TENSOR");
    c->f32_tensor = !(f32_env && f32_env[0] == '0');
    const char* st_env = getenv("RTGPU_TMA_STORE");
    c->tma_store = !(st_env && st_env[0] == '0');
    const char* pdl_env = getenv("RTGPU_PDL");
    c->pdl = !(pdl_env && pdl_env[0] == '0');
    const char* dyn_env = getenv("RTGPU_DYN_TILES");
    c->dyn_tiles = dyn_env && dyn_env[0] == '0' ? 0 : dyn_env && dyn_env[0] == '1' ? 1 : -1;
    // RTGPU_SKINNY_K_MAX=<k>: narrow-K GEMMs deeper than k go to the tensor
    // cores (default: chosen by dtype and size, see narrow_k_on_tensor_cores)
    const char* sk_env = getenv("RTGPU_SKINNY_K_MAX");
    if (sk_env) c->skinny_k_max = std::max(0, std::min(atoi(sk_env), (int)kSkinnyMax));
    int st = gemm_tc_init(c);
    if (st == RT_OK) st = gemm_tc2_init(c);
    if (st == RT_OK) st = gemm_x3_init(c);
    if (st == RT_OK) st = gemm_skinny_init();
    if (st != RT_OK) {
        cudaFree(c->dev_err);
        cudaStreamDestroy(c->own_stream);
        delete c;
        return st;
    }
    *out = c;
    return RT_OK;
}

int rt_ctx_destroy(rt_ctx* ctx) {
    if (!ctx) return RT_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->x3_scratch) cudaFree(ctx->x3_scratch);
    for (void* p : ctx->x3_retired) cudaFree(p);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return RT_OK;
}

int rt_ctx_info(const rt_ctx* ctx, char* buf, size_t len) {
    RT_CHECK(ctx && buf && len > 0, "rt_ctx_info: bad arguments");
    snprintf(buf, len, "%s", ctx->name);
    return RT_OK;
}

int rt_ctx_sync(rt_ctx* ctx) {
    RT_CHECK(ctx, "rt_ctx_sync: ctx is NULL");
    RT_CUDA(cudaSetDevice(ctx->device));
    RT_CUDA(cudaStreamSynchronize(ctx->stream));
    return check_device_error(ctx);
}

void* rt_ctx_stream(rt_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int rt_ctx_set_stream(rt_ctx* ctx, void* stream) {
    RT_CHECK(ctx, "rt_ctx_set_stream: ctx is NULL");
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
    return RT_OK;
}

int rt_ctx_set_fast_gemm(rt_ctx* ctx, int on) {
    RT_CHECK(ctx, "ctx is NULL");
    ctx->fast_gemm = on != 0;
    return RT_OK;
}

int rt_ctx_set_f32_tensor(rt_ctx* ctx, int on) {
    RT_CHECK(ctx, "ctx is NULL");
    ctx->f32_tensor = on != 0;
    return RT_OK;
}

int rt_ctx_set_l2_group(rt_ctx* ctx, int group) {
    RT_CHECK(ctx, "ctx is NULL");
    ctx->l2_group = group < 1 ? 1 : group;
    return RT_OK;
}

int rt_ctx_launch_count(const rt_ctx* ctx, uint64_t* out) {
    RT_CHECK(ctx && out, "bad arguments");
    *out = ctx->launches;
    return RT_OK;
}

int rt_host_alloc(size_t bytes, void** out) {
    RT_CHECK(out, "out is NULL");
    RT_CUDA(cudaMallocHost(out, bytes ? bytes : 1));
    return RT_OK;
}

int rt_host_free(void* p) {
    if (p) RT_CUDA(cudaFreeHost(p));
    return RT_OK;
}

// ------------------------------------------------------------------ tensors
static int shape_of(int rank, const int64_t* shape, int64_t* rows, int64_t* cols) {
    RT_CHECK(rank == 1 || rank == 2, "rank must be 1 or 2 (got %d)", rank);
    RT_CHECK(shape != nullptr, "shape is NULL");
    if (rank == 1) {
        *rows = 1;
        *cols = shape[0];
    } else {
        *rows = shape[0];
        *cols = shape[1];
    }
    RT_CHECK(*rows >= 0 && *cols >= 0, "negative extent");
    return RT_OK;
}

// Leading dimension rounded so every row starts on a 16-byte boundary (the
// alignment TMA needs for its global strides).
static int64_t padded_ld(int64_t cols, rt_dtype dt) {
    int64_t q = 16 / (int64_t)dtype_size(dt);
    int64_t ld = (cols + q - 1) / q * q;
    return ld < q ? q : ld;
}

int rt_tensor_zeros(rt_ctx* ctx, rt_dtype dtype, int rank, const int64_t* shape, rt_tensor** out) {
    RT_CHECK(ctx && out, "rt_tensor_zeros: bad arguments");
    int64_t rows, cols;
    RT_TRY(shape_of(rank, shape, &rows, &cols));
    rt_tensor* t = new rt_tensor;
    t->ctx = ctx;
    t->dtype = dtype;
    t->rank = rank;
    t->rows = rows;
    t->cols = cols;
    t->ld = padded_ld(cols, dtype);
    t->owned = true;
    size_t bytes = (size_t)(rows > 0 ? rows : 1) * (size_t)t->ld * dtype_size(dtype);
    cudaSetDevice(ctx->device);
    cudaError_t e = cudaMalloc(&t->ptr, bytes);
    if (e != cudaSuccess) {
        delete t;
        return fail(RT_ERR_OOM, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    }
    e = cudaMemsetAsync(t->ptr, 0, bytes, ctx->stream);
    if (e != cudaSuccess) {
        cudaFree(t->ptr);
        delete t;
        return fail(RT_ERR_CUDA, "cudaMemsetAsync failed: %s", cudaGetErrorString(e));
    }
    *out = t;
    return RT_OK;
}

int rt_tensor_wrap(rt_ctx* ctx, void* device_ptr, rt_dtype dtype, int rank, const int64_t* shape,
                   int64_t ld, rt_tensor** out) {
    RT_CHECK(ctx && out && device_ptr, "rt_tensor_wrap: bad arguments");
    int64_t rows, cols;
    RT_TRY(shape_of(rank, shape, &rows, &cols));
    RT_CHECK(ld == 0 || ld >= cols, "ld %lld < cols %lld", (long long)ld, (long long)cols);
    rt_tensor* t = new rt_tensor;
    t->ctx = ctx;
    t->ptr = device_ptr;
    t->dtype = dtype;
    t->rank = rank;
    t->rows = rows;
    t->cols = cols;
    t->ld = ld ? ld : cols;
    t->owned = false;
    *out = t;
    return RT_OK;
}

int rt_tensor_free(rt_tensor* t) {
    if (!t) return RT_OK;
    if (t->owned && t->ptr) {
        cudaSetDevice(t->ctx->device);
        cudaStreamSynchronize(t->ctx->stream);
        cudaFree(t->ptr);
    }
    delete t;
    return RT_OK;
}

void* rt_tensor_ptr(const rt_tensor* t) { return t ? t->ptr : nullptr; }

int rt_tensor_dims(const rt_tensor* t, int64_t* rows, int64_t* cols, int64_t* ld) {
    RT_CHECK(t, "tensor is NULL");
    if (rows) *rows = t->rows;
    if (cols) *cols = t->cols;
    if (ld) *ld = t->ld;
    return RT_OK;
}

int rt_tensor_upload(rt_ctx* ctx, rt_dtype dtype, const float* host, int rank, const int64_t* shape,
                     rt_tensor** out) {
    RT_CHECK(ctx && host && out, "rt_tensor_upload: bad arguments");
    RT_CHECK(dtype == RT_F32 || dtype == RT_BF16, "upload dtype must be RT_F32 or RT_BF16");
    rt_tensor* t = nullptr;
    RT_TRY(rt_tensor_zeros(ctx, dtype, rank, shape, &t));
    size_t rows = (size_t)t->rows, cols = (size_t)t->cols;
    if (rows * cols == 0) {
        *out = t;
        return RT_OK;
    }
    if (dtype == RT_F32) {
        cudaError_t e = cudaMemcpy2DAsync(t->ptr, t->ld * 4, host, cols * 4, cols * 4, rows,
                                          cudaMemcpyHostToDevice, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) {
            rt_tensor_free(t);
            return fail(RT_ERR_CUDA, "upload copy failed: %s", cudaGetErrorString(e));
        }
    } else {
        // Stage as packed f32 on the device, then round to bf16 with the cast kernel.
        float* stage = nullptr;
        cudaError_t e = cudaMalloc(&stage, rows * cols * 4);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(stage, host, rows * cols * 4, cudaMemcpyHostToDevice, ctx->stream);
        int s = RT_OK;
        if (e == cudaSuccess)
            s = launch_cast(ctx, stage, RT_F32, (int64_t)cols, t->ptr, RT_BF16, t->ld, t->rows, t->cols,
                            ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (stage) cudaFree(stage);
        if (e != cudaSuccess || s != RT_OK) {
            rt_tensor_free(t);
            return s != RT_OK ? s : fail(RT_ERR_CUDA, "upload failed: %s", cudaGetErrorString(e));
        }
    }
    *out = t;
    return RT_OK;
}

int rt_upload_labels(rt_ctx* ctx, const uint32_t* labels, int64_t n, rt_tensor** out) {
    RT_CHECK(ctx && labels && out && n >= 0, "rt_upload_labels: bad arguments");
    rt_tensor* t = new rt_tensor;
    t->ctx = ctx;
    t->dtype = RT_U32;
    t->rank = 1;
    t->rows = 1;
    t->cols = n;
    t->ld = n;
    t->owned = true;
    cudaSetDevice(ctx->device);
    cudaError_t e = cudaMalloc(&t->ptr, (size_t)(n > 0 ? n : 1) * 4);
    if (e == cudaSuccess && n > 0) e = cudaMemcpy(t->ptr, labels, (size_t)n * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (t->ptr) cudaFree(t->ptr);
        delete t;
        return fail(RT_ERR_CUDA, "label upload failed: %s", cudaGetErrorString(e));
    }
    *out = t;
    return RT_OK;
}

int rt_tensor_download(rt_ctx* ctx, const rt_tensor* t, float* host) {
    RT_CHECK(ctx && t && host, "rt_tensor_download: bad arguments");
    size_t rows = (size_t)t->rows, cols = (size_t)t->cols;
    if (rows * cols == 0) return RT_OK;
    RT_CUDA(cudaSetDevice(ctx->device));
    if (t->dtype == RT_F32 || t->dtype == RT_U32) {
        RT_CUDA(cudaMemcpy2DAsync(host, cols * 4, t->ptr, t->ld * 4, cols * 4, rows, cudaMemcpyDeviceToHost,
                                  ctx->stream));
        RT_CUDA(cudaStreamSynchronize(ctx->stream));
    } else {
        float* stage = nullptr;
        RT_CUDA(cudaMalloc(&stage, rows * cols * 4));
        int s = launch_cast(ctx, t->ptr, RT_BF16, t->ld, stage, RT_F32, (int64_t)cols, t->rows, t->cols,
                            ctx->stream);
        cudaError_t e = cudaSuccess;
        if (s == RT_OK) e = cudaMemcpyAsync(host, stage, rows * cols * 4, cudaMemcpyDeviceToHost, ctx->stream);
        if (s == RT_OK && e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        cudaFree(stage);
        if (s != RT_OK) return s;
        if (e != cudaSuccess) return fail(RT_ERR_CUDA, "download failed: %s", cudaGetErrorString(e));
    }
    return check_device_error(ctx);
}

}  // extern "C"
