// gemv_tc.cu -- tensor-core decode GEMV (placeholder until the kernel lands).
#include "common.cuh"
#include "kernels.h"

namespace b200 {
bool gemv_tc_supported(const LinearArgs &) { return false; }
int32_t launch_gemv_tc(const LinearArgs &, cudaStream_t) { return b200_set_error(B200_ERR_UNSUPPORTED, "gemv_tc"); }
}  // namespace b200
