// C ABI of libflicker_b200 (declared in include/flicker_b200.h).
//
// Validation happens here, on the host, before anything is enqueued: shapes,
// null pointers, 16-byte alignment (vector loads and TMA need it) and the
// device's compute capability. Nothing here allocates device memory,
// synchronises (except flk_device_status) or aborts.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "flicker_b200.h"

namespace flk {
int launch_qk_prep(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos_t,
                   const float* sin_t, float q_gain, int B, int L, int H, uint16_t* q, uint16_t* k, uint16_t* v,
                   cudaStream_t stream);
int launch_attend(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, uint16_t* o,
                  int* status, cudaStream_t stream);
}  // namespace flk

// Device status word: 0, or FLK_ERR_DEVICE_TIMEOUT after a bounded in-kernel wait ran out.
__device__ int g_flk_status = 0;

namespace {

constexpr int kMaxDevices = 64;
constexpr float kExpLimit = 80.0f;  // src/flicker/kernels.py:95

struct DeviceState {
  bool ready = false;
  bool is_sm100 = false;
  int* status = nullptr;  // device address of g_flk_status on this device
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

// Per-device set-up on first use (with that device current): capability check and the
// device address of the status word. Returns nullptr when the device is unusable.
const DeviceState* device_state(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = FLK_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.ready) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
      *err = FLK_ERR_CUDA;
      return nullptr;
    }
    st.is_sm100 = (major == 10 && minor == 0);
    void* addr = nullptr;
    if (st.is_sm100 && cudaGetSymbolAddress(&addr, g_flk_status) != cudaSuccess) {
      *err = FLK_ERR_CUDA;
      return nullptr;
    }
    st.status = static_cast<int*>(addr);
    st.ready = true;
  }
  if (!st.is_sm100) {
    *err = FLK_ERR_NO_DEVICE;
    return nullptr;
  }
  return &st;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int flk_abi_version(void) { return 100; }

const char* flk_error_string(int code) {
  switch (code) {
    case FLK_OK: return "ok";
    case FLK_ERR_INVALID_ARGUMENT: return "invalid argument (shape, null or misaligned pointer)";
    case FLK_ERR_UNSUPPORTED: return "unsupported shape for this build (head_dim must be 128)";
    case FLK_ERR_CUDA: return "CUDA call failed";
    case FLK_ERR_WORKSPACE: return "workspace missing or too small";
    case FLK_ERR_DEVICE_TIMEOUT: return "a bounded in-kernel wait timed out";
    case FLK_ERR_NO_DEVICE: return "current CUDA device is not sm_100 (B200)";
    default: return "unknown flicker_b200 error";
  }
}

int flk_qk_prep(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos,
                const float* sin, float q_gain, int B, int L, int H, int D, uint16_t* q, uint16_t* k, uint16_t* v,
                void* stream) {
  if (B < 0 || L < 0 || H <= 0) return FLK_ERR_INVALID_ARGUMENT;
  if (D != 128) return FLK_ERR_UNSUPPORTED;
  if (!std::isfinite(q_gain)) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(B) * L == 0) return FLK_OK;
  const void* ptrs[] = {qkv, q_scale, k_scale, cos, sin, q, k, v};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  if (!device_state(&err)) return err;
  return flk::launch_qk_prep(qkv, q_scale, k_scale, cos, sin, q_gain, B, L, H, q, k, v,
                             static_cast<cudaStream_t>(stream));
}

size_t flk_attend_workspace_size(int B, int H, int S, int D) {
  (void)B;
  (void)H;
  (void)S;
  (void)D;
  return 0;
}

int flk_attend(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, int D, uint16_t* o,
               void* workspace, size_t ws_bytes, void* stream) {
  (void)workspace;
  (void)ws_bytes;
  if (B < 0 || H <= 0 || S < 0) return FLK_ERR_INVALID_ARGUMENT;
  if (D != 128) return FLK_ERR_UNSUPPORTED;
  if (S % 128 != 0) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(B) * S == 0) return FLK_OK;
  if (static_cast<long long>(B) * H > 65535 || static_cast<long long>(B) * H * S > 0x7FFFFFFFLL)
    return FLK_ERR_UNSUPPORTED;
  const void* ptrs[] = {q, k, v, o};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  const DeviceState* st = device_state(&err);
  if (!st) return err;
  return flk::launch_attend(q, k, v, B, H, S, o, st->status, static_cast<cudaStream_t>(stream));
}

int flk_logit_bound(const float* q_scale, const float* k_scale, int D, float* bound) {
  if (q_scale == nullptr || k_scale == nullptr || bound == nullptr || D <= 0) return FLK_ERR_INVALID_ARGUMENT;
  float mq = 0.f, mk = 0.f;
  for (int i = 0; i < D; ++i) {
    mq = std::fmax(mq, std::fabs(q_scale[i]));
    mk = std::fmax(mk, std::fabs(k_scale[i]));
  }
  *bound = std::sqrt(static_cast<float>(D)) * mq * mk;
  return (*bound < kExpLimit) ? FLK_OK : FLK_ERR_INVALID_ARGUMENT;
}

int flk_device_status(void) {
  int err = FLK_OK;
  if (!device_state(&err)) return err;
  if (cudaDeviceSynchronize() != cudaSuccess) return FLK_ERR_CUDA;
  int value = 0;
  if (cudaMemcpyFromSymbol(&value, g_flk_status, sizeof(int)) != cudaSuccess) return FLK_ERR_CUDA;
  const int zero = 0;
  if (value != 0 && cudaMemcpyToSymbol(g_flk_status, &zero, sizeof(int)) != cudaSuccess) return FLK_ERR_CUDA;
  return value;
}

}  // extern "C"
