// tcgen05 GEMM for the projection forward and the matmul gradients (fp32 I/O).
#include "host_launchers.h"

namespace pa {

int launch_gemm_f32(int, const float*, const float*, float*, int, int, int, uint32_t*,
                    cudaStream_t) {
  return PA_ERR_UNSUPPORTED;
}

}  // namespace pa
