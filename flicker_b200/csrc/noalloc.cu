// flk_attend_noalloc: flk_attend for callers that cannot allocate device memory.
//
// Who needs it: a caller that only ever receives its input and output buffers plus a stream,
// and owns no allocator of its own. The typical case is an XLA custom-call handler registered
// without a scratch buffer: the runtime owns all device memory, and calling cudaMalloc from
// inside the handler would synchronise the device in the middle of XLA's asynchronous stream
// work. A serving loop that must never stall on a device-wide allocation is in the same spot.
// flk_attend asks such callers for a workspace when a shape runs (partly) split over KV; this
// entry point instead uses a fixed scratch array compiled into the library, so it allocates
// nothing.
//
// The scratch is a file-scope __device__ array of kScratchBytes (32 MiB). Every GPU that loads
// this library holds it until the process exits, whether or not this entry point is called.
// Shapes whose schedule needs more than that are refused with FLK_ERR_WORKSPACE; shapes that do
// not split (the large, evenly filled ones) never touch it.
//
// Set-up: the first call on a device, with that device current, looks up the array's device
// address with cudaGetSymbolAddress and caches it per device. (A host-side reference to the
// array's name is only a stand-in, not a device address, so it is never passed to a kernel.)
// Make that first call before any stream capture on the device.
//
// Sharing: all calls share the one array, and it keeps whatever the last call wrote. Nothing in
// it has to start at zero: every piece of a split item writes all of its partial rows before the
// combine kernel reads them. Two calls whose kernels overlap on the GPU (e.g. on different streams
// without ordering between them) race on the array; callers must order them.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "attend_schedule.cuh"
#include "flicker_b200.h"

namespace flk {
int launch_attend(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, uint16_t* o,
                  const AttendSchedule& sch, void* workspace, int* status, cudaStream_t stream);
int* current_device_status(int* err);
}  // namespace flk

namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;  // 32 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// Per-device state of this entry point: the scratch's device address and the SM count
// (looked up once, with the device current).
struct NoAllocDevice {
  bool ready = false;
  void* scratch = nullptr;
  int sms = 0;
};

std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kMaxDevices];

}  // namespace

namespace {

const NoAllocDevice* noalloc_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = FLK_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& st = g_noalloc_dev[dev];
  if (!st.ready) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      *err = FLK_ERR_CUDA;
      return nullptr;
    }
    if (major != 10 || minor != 0) {
      *err = FLK_ERR_NO_DEVICE;
      return nullptr;
    }
    void* scratch = nullptr;
    if (cudaGetSymbolAddress(&scratch, g_noalloc_scratch) != cudaSuccess) {
      *err = FLK_ERR_CUDA;
      return nullptr;
    }
    st.scratch = scratch;
    st.ready = true;
  }
  return &st;
}

bool aligned16_noalloc(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int flk_attend_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S,
                                  int D, uint16_t* o, void* stream) {
  if (B < 0 || H <= 0 || S < 0) return FLK_ERR_INVALID_ARGUMENT;
  if (D != 128) return FLK_ERR_UNSUPPORTED;
  if (S % 128 != 0) return FLK_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(B) * H > 65535 || static_cast<long long>(B) * H * S > 0x7FFFFFFFLL)
    return FLK_ERR_UNSUPPORTED;
  if (static_cast<long long>(B) * S == 0) return FLK_OK;
  const void* ptrs[] = {q, k, v, o};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16_noalloc(p)) return FLK_ERR_INVALID_ARGUMENT;
  int err = FLK_OK;
  const NoAllocDevice* st = noalloc_device(&err);
  if (!st) return err;
  const flk::AttendSchedule sch = flk::attend_schedule(B, H, S, st->sms);
  if (flk::attend_workspace_bytes(B, H, S, sch) > kScratchBytes) return FLK_ERR_WORKSPACE;
  int* status = flk::current_device_status(&err);  // the library's device status word
  if (!status) return err;
  return flk::launch_attend(q, k, v, B, H, S, o, sch, sch.split() ? st->scratch : nullptr, status,
                            static_cast<cudaStream_t>(stream));
}
