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

#include "attend_schedule.cuh"
#include "flicker_b200.h"

namespace flk {
int launch_qk_prep(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos_t,
                   const float* sin_t, float q_gain, int B, int L, int H, int S_out, int row0, uint16_t* q,
                   uint16_t* k, uint16_t* v, cudaStream_t stream);
int launch_attend_layout(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, uint16_t* o,
                         int merged, const AttendSchedule& sch, void* workspace, int* status, cudaStream_t stream);
int launch_attend_gather(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S,
                         uint16_t* const* outs, int n_out, int H_out, int h0, const AttendSchedule& sch,
                         void* workspace, int* status, cudaStream_t stream);
int launch_attend_gather_multicast(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S,
                                   uint16_t* out_mc, int H_out, int h0, const AttendSchedule& sch,
                                   void* workspace, int* status, cudaStream_t stream);
int launch_linear_bf16(const uint16_t* x, const uint16_t* wt, int M, int N, int K, uint16_t* y, int* status, int sms,
                       cudaStream_t stream);
int launch_linear_qk_prep(const uint16_t* x, const uint16_t* wt, int M, int N, int K, int L, int H,
                          const uint16_t* q_scale, const uint16_t* k_scale, const float* cos_t, const float* sin_t,
                          float q_gain, uint16_t* q, uint16_t* k, uint16_t* v, int S_out, int row0, uint16_t* rest,
                          int* status, int sms, cudaStream_t stream);
int launch_w8a8_gemm(const int8_t* xq, const int8_t* wq, const float* x_scale, const float* w_scale, int M, int N,
                     int K, uint16_t* y, int32_t* acc_out, int* status, int sms, cudaStream_t stream);
int launch_quantize_act(const uint16_t* x, const float* inv_s, int M, int K, int8_t* xq, float* x_scale,
                        cudaStream_t stream);
}  // namespace flk

// Device status word: 0, or FLK_ERR_DEVICE_TIMEOUT after a bounded in-kernel wait ran out.
__device__ int g_flk_status = 0;

namespace {

constexpr int kMaxDevices = 64;
constexpr float kExpLimit = 80.0f;  // src/flicker/kernels.py:95

struct DeviceState {
  bool ready = false;
  bool is_sm100 = false;
  int sms = 0;            // streaming multiprocessors
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
    if (cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      *err = FLK_ERR_CUDA;
      return nullptr;
    }
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

bool attend_shape_ok(int B, int H, int S, int D, int* err) {
  if (B < 0 || H <= 0 || S < 0) {
    *err = FLK_ERR_INVALID_ARGUMENT;
    return false;
  }
  if (D != 128) {
    *err = FLK_ERR_UNSUPPORTED;
    return false;
  }
  if (S % 128 != 0) {
    *err = FLK_ERR_INVALID_ARGUMENT;
    return false;
  }
  if (static_cast<long long>(B) * H > 65535 || static_cast<long long>(B) * H * S > 0x7FFFFFFFLL) {
    *err = FLK_ERR_UNSUPPORTED;
    return false;
  }
  return true;
}

}  // namespace

namespace flk {
// Device address of the status word on the current device (set up on first use), or nullptr
// with *err set. Lets other translation units of the library hand it to their kernels.
int* current_device_status(int* err) {
  const DeviceState* st = device_state(err);
  return st ? st->status : nullptr;
}
}  // namespace flk

extern "C" {

int flk_abi_version(void) { return 101; }  // 1.01: flk_attend_schedule added

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

static int qk_prep_entry(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos,
                         const float* sin, float q_gain, int B, int L, int H, int D, uint16_t* q, uint16_t* k,
                         uint16_t* v, int S_out, int row0, void* stream) {
  if (B < 0 || L < 0 || H <= 0) return FLK_ERR_INVALID_ARGUMENT;
  if (row0 < 0 || S_out < 0 || static_cast<long long>(row0) + L > S_out) return FLK_ERR_INVALID_ARGUMENT;
  if (D != 128) return FLK_ERR_UNSUPPORTED;
  if (!std::isfinite(q_gain)) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(B) * L == 0) return FLK_OK;
  const void* ptrs[] = {qkv, q_scale, k_scale, cos, sin, q, k, v};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  if (!device_state(&err)) return err;
  return flk::launch_qk_prep(qkv, q_scale, k_scale, cos, sin, q_gain, B, L, H, S_out, row0, q, k, v,
                             static_cast<cudaStream_t>(stream));
}

int flk_qk_prep(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos,
                const float* sin, float q_gain, int B, int L, int H, int D, uint16_t* q, uint16_t* k, uint16_t* v,
                void* stream) {
  return qk_prep_entry(qkv, q_scale, k_scale, cos, sin, q_gain, B, L, H, D, q, k, v, L, 0, stream);
}

int flk_qk_prep_into(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos,
                     const float* sin, float q_gain, int B, int L, int H, int D, uint16_t* q, uint16_t* k,
                     uint16_t* v, int S_out, int row0, void* stream) {
  return qk_prep_entry(qkv, q_scale, k_scale, cos, sin, q_gain, B, L, H, D, q, k, v, S_out, row0, stream);
}

// The schedule of an attention call: low-occupancy shapes, and shapes whose last wave of work
// items would leave SMs idle, run (partly) split over KV when the caller provides the workspace
// the schedule needs; a caller that passes no workspace (NULL, 0 bytes) gets every item whole.
static int pick_schedule(int B, int H, int S, int sms, void* workspace, size_t ws_bytes,
                         flk::AttendSchedule* sch) {
  *sch = flk::attend_schedule(B, H, S, sms);
  if (!sch->split()) return FLK_OK;
  if (workspace == nullptr && ws_bytes == 0) {
    *sch = flk::attend_unsplit(B, H, S);
    return FLK_OK;
  }
  if (workspace == nullptr || ws_bytes < flk::attend_workspace_bytes(B, H, S, *sch) || !aligned16(workspace))
    return FLK_ERR_WORKSPACE;
  return FLK_OK;
}

size_t flk_attend_workspace_size(int B, int H, int S, int D) {
  int err = FLK_OK;
  if (!attend_shape_ok(B, H, S, D, &err) || static_cast<long long>(B) * S == 0) return 0;
  const DeviceState* st = device_state(&err);
  if (!st) return 0;
  return flk::attend_workspace_bytes(B, H, S, flk::attend_schedule(B, H, S, st->sms));
}

int flk_attend_schedule(int B, int H, int S, int D, int sms, long long* out) {
  int err = FLK_OK;
  if (!attend_shape_ok(B, H, S, D, &err)) return err;
  if (out == nullptr || sms <= 0) return FLK_ERR_INVALID_ARGUMENT;
  const flk::AttendSchedule sch = flk::attend_schedule(B, H, S, sms);
  const long long v[6] = {sch.n_items, sch.n_full, sch.n_a, sch.s_a, sch.s_b, sch.units()};
  for (int i = 0; i < 6; ++i) out[i] = v[i];
  return FLK_OK;
}

static int attend_entry(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, int D,
                        uint16_t* o, int merged, void* workspace, size_t ws_bytes, void* stream) {
  int err = FLK_OK;
  if (!attend_shape_ok(B, H, S, D, &err)) return err;
  if (static_cast<long long>(B) * S == 0) return FLK_OK;
  const void* ptrs[] = {q, k, v, o};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  const DeviceState* st = device_state(&err);
  if (!st) return err;
  flk::AttendSchedule sch;
  if (const int rc = pick_schedule(B, H, S, st->sms, workspace, ws_bytes, &sch); rc != FLK_OK) return rc;
  return flk::launch_attend_layout(q, k, v, B, H, S, o, merged, sch, workspace, st->status,
                                   static_cast<cudaStream_t>(stream));
}

int flk_attend(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, int D, uint16_t* o,
               void* workspace, size_t ws_bytes, void* stream) {
  return attend_entry(q, k, v, B, H, S, D, o, 0, workspace, ws_bytes, stream);
}

int flk_attend_merged(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, int D,
                      uint16_t* o, void* workspace, size_t ws_bytes, void* stream) {
  return attend_entry(q, k, v, B, H, S, D, o, 1, workspace, ws_bytes, stream);
}

int flk_attend_gather(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, int D,
                      uint16_t* const* outs, int n_outs, int H_total, int h0, void* workspace, size_t ws_bytes,
                      void* stream) {
  int err = FLK_OK;
  if (!attend_shape_ok(B, H, S, D, &err)) return err;
  if (outs == nullptr || n_outs < 1 || n_outs > 8) return FLK_ERR_INVALID_ARGUMENT;
  if (h0 < 0 || H_total < 1 || static_cast<long long>(h0) + H > H_total) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(B) * S == 0) return FLK_OK;
  const void* ptrs[] = {q, k, v};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  for (int d = 0; d < n_outs; ++d)
    if (outs[d] == nullptr || !aligned16(outs[d])) return FLK_ERR_INVALID_ARGUMENT;
  const DeviceState* st = device_state(&err);
  if (!st) return err;
  flk::AttendSchedule sch;
  if (const int rc = pick_schedule(B, H, S, st->sms, workspace, ws_bytes, &sch); rc != FLK_OK) return rc;
  return flk::launch_attend_gather(q, k, v, B, H, S, outs, n_outs, H_total, h0, sch, workspace, st->status,
                                   static_cast<cudaStream_t>(stream));
}

int flk_attend_gather_multicast(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S,
                                int D, uint16_t* out_mc, int H_total, int h0, void* workspace, size_t ws_bytes,
                                void* stream) {
  int err = FLK_OK;
  if (!attend_shape_ok(B, H, S, D, &err)) return err;
  if (h0 < 0 || H_total < 1 || static_cast<long long>(h0) + H > H_total) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(B) * S == 0) return FLK_OK;
  const void* ptrs[] = {q, k, v, out_mc};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  const DeviceState* st = device_state(&err);
  if (!st) return err;
  flk::AttendSchedule sch;
  if (const int rc = pick_schedule(B, H, S, st->sms, workspace, ws_bytes, &sch); rc != FLK_OK) return rc;
  return flk::launch_attend_gather_multicast(q, k, v, B, H, S, out_mc, H_total, h0, sch, workspace, st->status,
                                             static_cast<cudaStream_t>(stream));
}

int flk_linear(const uint16_t* x, const uint16_t* wt, int M, int N, int K, uint16_t* y, void* stream) {
  if (M < 0 || N < 0 || K <= 0 || K % 8 != 0) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(M) * N == 0) return FLK_OK;
  const void* ptrs[] = {x, wt, y};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  const DeviceState* st = device_state(&err);
  if (!st) return err;
  return flk::launch_linear_bf16(x, wt, M, N, K, y, st->status, st->sms, static_cast<cudaStream_t>(stream));
}

int flk_linear_qk_prep(const uint16_t* x, const uint16_t* wt, int M, int N, int K, const uint16_t* q_scale,
                       const uint16_t* k_scale, const float* cos, const float* sin, float q_gain, int B, int L, int H,
                       int D, uint16_t* q, uint16_t* k, uint16_t* v, int S_out, int row0, uint16_t* rest,
                       void* stream) {
  if (B < 0 || L < 0 || H <= 0 || K <= 0 || K % 8 != 0 || N < 0) return FLK_ERR_INVALID_ARGUMENT;
  if (D != 128) return FLK_ERR_UNSUPPORTED;
  if (static_cast<long long>(B) * L != M) return FLK_ERR_INVALID_ARGUMENT;
  const long long n_qkv = 3ll * H * D;
  if (N < n_qkv || (N > n_qkv && rest == nullptr)) return FLK_ERR_INVALID_ARGUMENT;
  if (row0 < 0 || S_out < 0 || static_cast<long long>(row0) + L > S_out) return FLK_ERR_INVALID_ARGUMENT;
  if (!std::isfinite(q_gain)) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(B) * L == 0) return FLK_OK;
  const void* ptrs[] = {x, wt, q_scale, k_scale, cos, sin, q, k, v};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  if (rest != nullptr && !aligned16(rest)) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  const DeviceState* st = device_state(&err);
  if (!st) return err;
  return flk::launch_linear_qk_prep(x, wt, M, N, K, L, H, q_scale, k_scale, cos, sin, q_gain, q, k, v, S_out, row0,
                                    rest, st->status, st->sms, static_cast<cudaStream_t>(stream));
}

int flk_w8a8_quantize_act(const uint16_t* x, const float* inv_smooth, int M, int K, int8_t* xq, float* x_scale,
                          void* stream) {
  if (M < 0 || K < 0 || K % 8 != 0) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(M) * K == 0) return FLK_OK;
  if (static_cast<long long>(M) * 32 > 0x7FFFFFFFLL) return FLK_ERR_UNSUPPORTED;
  const void* ptrs[] = {x, inv_smooth, xq, x_scale};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  if (!device_state(&err)) return err;
  return flk::launch_quantize_act(x, inv_smooth, M, K, xq, x_scale, static_cast<cudaStream_t>(stream));
}

static int w8a8_checks(const void* a, const void* b, int M, int N, int K, const void* out) {
  if (M < 0 || N < 0 || K <= 0 || K % 16 != 0) return FLK_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {a, b, out};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return FLK_ERR_INVALID_ARGUMENT;
  return FLK_OK;
}

int flk_w8a8_gemm(const int8_t* xq, const int8_t* wq, const float* x_scale, const float* w_scale, int M, int N, int K,
                  uint16_t* y, void* stream) {
  int err = w8a8_checks(xq, wq, M, N, K, y);
  if (err != FLK_OK) return err;
  if (x_scale == nullptr || w_scale == nullptr) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(M) * N == 0) return FLK_OK;
  const DeviceState* st = device_state(&err);
  if (!st) return err;
  return flk::launch_w8a8_gemm(xq, wq, x_scale, w_scale, M, N, K, y, nullptr, st->status, st->sms,
                               static_cast<cudaStream_t>(stream));
}

int flk_i8_gemm_s32(const int8_t* a, const int8_t* b, int M, int N, int K, int32_t* c, void* stream) {
  int err = w8a8_checks(a, b, M, N, K, c);
  if (err != FLK_OK) return err;
  if (static_cast<long long>(M) * N == 0) return FLK_OK;
  const DeviceState* st = device_state(&err);
  if (!st) return err;
  return flk::launch_w8a8_gemm(a, b, nullptr, nullptr, M, N, K, nullptr, c, st->status, st->sms,
                               static_cast<cudaStream_t>(stream));
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
