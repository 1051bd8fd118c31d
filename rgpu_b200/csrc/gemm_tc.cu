// tcgen05 / TMA tensor-core GEMM (placeholder until the kernel lands).
#include "internal.h"

namespace rt {
bool gemm_tc_supported(const rt_ctx*, const GemmDesc&) { return false; }
int launch_gemm_tc(rt_ctx*, const GemmDesc&, cudaStream_t) {
    return fail(RT_ERR_UNSUPPORTED, "tensor-core GEMM not built");
}
}  // namespace rt
