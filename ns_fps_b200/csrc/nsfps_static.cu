// nsfps_static.cu -- the fixed scratch array behind nsfps_fps_device_static().
//
// Callers that cannot allocate device memory mid-run (a host that has handed
// all device memory to its own pool, a latency-bound loop where cudaMalloc /
// cudaFree would synchronise the device) use this array instead of the
// growing per-device workspace.  It lives in its own translation unit so that,
// with lazy module loading, its 8 MiB are only reserved on a device once the
// function is first used there.
#include <cuda_runtime.h>

#include "nsfps.h"
#include "nsfps_kernels.h"

namespace nsfps {

namespace {
static __device__ __align__(256) unsigned char g_static_scratch[NSFPS_STATIC_SCRATCH_BYTES];
}  // namespace

// Device address of the array on the current device.
cudaError_t static_scratch_address(void **ptr, size_t *bytes) {
  *ptr = nullptr;
  *bytes = 0;
  cudaError_t e = cudaGetSymbolAddress(ptr, g_static_scratch);
  if (e != cudaSuccess) return e;
  *bytes = sizeof(g_static_scratch);
  return cudaSuccess;
}

}  // namespace nsfps
