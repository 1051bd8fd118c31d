// Device-timeout self-test: exercises the path by which a GEMM whose barrier
// wait expires reports RT_ERR_DEVICE_TIMEOUT, without faulting anything.  One
// thread waits on a shared-memory mbarrier that nothing arrives on, with the
// same bounded wait (kWaitLimitNs on %globaltimer) the tensor-core GEMMs use;
// when it gives up it records DEV_TIMEOUT_SELFTEST in the context's device
// error word and the kernel returns.  The next rt_ctx_sync reports the
// timeout and clears the word, and the context stays usable.
#include "tc_common.cuh"

namespace rt {
namespace {

__global__ void wait_timeout_kernel(int* err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        tc::mbar_init(tc::smem_u32(&bar), 1);
        abort_flag = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0 && !tc::mbar_wait(tc::smem_u32(&bar), 0, &abort_flag))
        tc::record_error(err, DEV_TIMEOUT_SELFTEST, 0);
}

}  // namespace
}  // namespace rt

using namespace rt;

extern "C" int rt_ctx_selftest_timeout(rt_ctx* ctx) {
    RT_CHECK(ctx, "rt_ctx_selftest_timeout: ctx is NULL");
    RT_CUDA(cudaSetDevice(ctx->device));
    wait_timeout_kernel<<<1, 32, 0, ctx->stream>>>(ctx->dev_err);
    count_launch(ctx);
    RT_CUDA(cudaGetLastError());
    return RT_OK;
}
