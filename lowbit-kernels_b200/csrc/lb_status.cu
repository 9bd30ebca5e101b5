// Device status word: kernels whose waits are bounded (a spin on an mbarrier, a flag or a peer) record an
// error code here when a wait gives up, instead of hanging the GPU; the host reads it with lb_device_error().
#include "lb_common.cuh"
#include "lb_launch.h"

namespace lb {

__device__ int g_device_status;

int device_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  return v;
}

void clear_device_error() {
  int z = 0;
  cudaMemcpyToSymbol(g_device_status, &z, sizeof(int));
}

}  // namespace lb
