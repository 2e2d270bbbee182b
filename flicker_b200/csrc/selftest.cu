// Self-tests of device-side building blocks, each run by a GPU test.
//
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
#include "quotient.cuh"

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

// q_fast[i] = a[i] / b[i] through quotient_rn (one reciprocal per divisor, as the attend
// epilogue uses it per row); q_ref[i] = __fdiv_rn(a[i], b[i]).
__global__ void __launch_bounds__(256) quotient_kernel(const float* a, const float* b, long long n, float* q_fast,
                                                       float* q_ref) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = a[i], y = b[i];
  q_fast[i] = quotient_rn(x, y, __frcp_rn(y));
  q_ref[i] = __fdiv_rn(x, y);
}

// The two ways attend computes 2^x for p = exp(s) (x = s * log2(e)), element by element:
// poly[i] = exp2_poly2 (FMA pipe, degree-4 minimax polynomial), mufu[i] = ex2.approx (SFU).
__global__ void __launch_bounds__(256) exp2_kernel(const float* x, long long n, float* poly, float* mufu) {
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 2;
  if (i >= n) return;
  const bool pair = i + 1 < n;
  const float2 v = make_float2(x[i], pair ? x[i + 1] : 0.0f);
  const float2 e = exp2_poly2(v);
  poly[i] = e.x;
  mufu[i] = ex2_approx(v.x);
  if (pair) {
    poly[i + 1] = e.y;
    mufu[i + 1] = ex2_approx(v.y);
  }
}

}  // namespace

// binaryVersion (major * 10 + minor) of the code the runtime loaded for the attention kernel.
int attend_binary_version(int* version);

}  // namespace flk

extern "C" int flk_selftest_wait_timeout(int* result, void* stream) {
  if (result == nullptr) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  int* status = flk::current_device_status(&err);
  if (status == nullptr) return err;
  flk::wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, result);
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}

// flk_selftest_quotient: the epilogue's reciprocal-and-correction quotient next to __fdiv_rn
// for n operand pairs (device pointers), so a test can compare them bit for bit.
extern "C" int flk_selftest_quotient(const float* a, const float* b, long long n, float* q_fast, float* q_ref,
                                     void* stream) {
  if (n < 0 || (n > 0 && (a == nullptr || b == nullptr || q_fast == nullptr || q_ref == nullptr)))
    return FLK_ERR_INVALID_ARGUMENT;
  if (n == 0) return FLK_OK;
  flk::quotient_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      a, b, n, q_fast, q_ref);
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}

// flk_selftest_exp2: the attend kernel's two exponentials (polynomial and MUFU.EX2) for n device
// floats, so a test can bound their relative error against a float64 reference.
extern "C" int flk_selftest_exp2(const float* x, long long n, float* poly, float* mufu, void* stream) {
  if (n < 0 || (n > 0 && (x == nullptr || poly == nullptr || mufu == nullptr))) return FLK_ERR_INVALID_ARGUMENT;
  if (n == 0) return FLK_OK;
  const long long threads = (n + 1) / 2;
  flk::exp2_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, n, poly, mufu);
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}

// flk_kernel_binary_version: which code the runtime loaded for this library's kernels on the
// current device (100 = sm_100), read from the attention kernel's attributes.
extern "C" int flk_kernel_binary_version(void) {
  int version = 0;
  const int rc = flk::attend_binary_version(&version);
  return rc == FLK_OK ? version : rc;
}
