// gemm_sm100.cu -- tcgen05 packed GEMM (placeholder until the kernel lands).
#include "common.cuh"
#include "kernels.h"

namespace b200 {
bool gemm_supported(const LinearArgs &) { return false; }
int32_t launch_gemm(const LinearArgs &, cudaStream_t) { return b200_set_error(B200_ERR_UNSUPPORTED, "gemm"); }
}  // namespace b200
