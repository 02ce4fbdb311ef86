// Busy-expert GEMM path (see gemm.h).
#include "common.cuh"
#include "gemm.h"
#include "internal.h"

namespace dsv41 {

size_t gemm_scratch_bytes(int N, int E, int H, int I) { return 256; }

cudaError_t launch_gemm_gateup(const GemmArgs& a, cudaStream_t st) { return cudaErrorNotSupported; }
cudaError_t launch_gemm_down(const GemmArgs& a, cudaStream_t st) { return cudaErrorNotSupported; }

}  // namespace dsv41
