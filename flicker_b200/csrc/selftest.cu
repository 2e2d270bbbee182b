// flk_selftest_wait_timeout: exercises the failure path of the bounded in-kernel waits.
//
// One warp waits on an mbarrier that nothing ever arrives at, through the same mbar_wait_warp
// the kernels use. The wait gives up after its time limit (kWaitLimitNs of %globaltimer),
// records FLK_ERR_DEVICE_TIMEOUT in the library's device status word and returns, so the kernel
// ends normally and the CUDA context stays usable: this is the behaviour a protocol bug in a
// kernel would produce, shown without making anything fault or hang.
#include <cuda_runtime.h>

#include <cstdint>

#include "flicker_b200.h"
#include "ptx.cuh"

namespace flk {
int* current_device_status(int* err);

namespace {

__global__ void __launch_bounds__(32) wait_timeout_kernel(int* status, int* result) {
  __shared__ uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none is ever made
    abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const bool ok = mbar_wait_warp(&bar, 0, &abort, status);
  if (threadIdx.x == 0) *result = ok ? 1 : 0;
}

}  // namespace
}  // namespace flk

extern "C" int flk_selftest_wait_timeout(int* result, void* stream) {
  if (result == nullptr) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  int* status = flk::current_device_status(&err);
  if (status == nullptr) return err;
  flk::wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, result);
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}
