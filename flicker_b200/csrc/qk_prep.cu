// qk_prep for sm_100a: head split + QK-RMSNorm + lane-pair RoPE (+ q gain) in one HBM pass.
//
// Restates flicker kernels.qk_prep (src/flicker/kernels.py:57-91, body :35-53) as a
// memory-bound CUDA kernel. Work item = one token x a group of 4 consecutive head rows
// of that token's fused QKV row (row r of 3H: r < H -> q head r, r < 2H -> k head r-H,
// else v head r-2H). A half-warp (16 lanes) owns one item; lane j owns columns
// [8j, 8j+8) of every 128-wide head row, so:
//   * every global access is one 16-byte vector per lane and 256 contiguous bytes per
//     half-warp, on both the [B, L, 3HD] read side and the head-major [B, H, L, D]
//     write side (the transpose costs nothing at row granularity);
//   * the RoPE partner of column 2i is column 2i+1 of the same lane (no shuffle);
//   * the cos/sin lane tables and both scale vectors are loaded once per item and reused
//     for its rows (they are L2-resident: 1 KB per token);
//   * the sum of squares is reduced across the 16 lanes with 4 xor-shuffles (q/k rows only;
//     v rows are copied straight through);
//   * all row loads of an item are issued before any math (4 x 16 B in flight per lane).
// Rounding follows the reference body: fp32 norm (rsqrt on the SFU), bf16 round, bf16 x bf16
// scale multiply rounded to bf16, fp32 rotation c*w + s*swap (no FMA contraction), q gain in
// fp32, final bf16 round.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "flicker_b200.h"
#include "qk_math.cuh"

namespace flk {

namespace {

constexpr int kHeadDim = 128;
constexpr int kThreads = 256;

// Division of 32-bit unsigned values by a divisor fixed per launch (Granlund & Montgomery,
// "Division by invariant integers using multiplication", 1994, figure 4.1): with
// l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1, q = (t + ((n - t) >> 1)) >> (l - 1) where
// t = mulhi(m, n), exact for every n < 2^32; d = 1 uses m = 0 and no shifts. The host builds it.
struct FastDiv {
  uint32_t m, s1, s2;
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    const uint32_t t = __umulhi(m, n);
    return (t + ((n - t) >> s1)) >> s2;
  }
};

FastDiv make_fast_div(uint32_t d) {
  if (d <= 1) return FastDiv{0u, 0u, 0u};
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  return FastDiv{static_cast<uint32_t>(m), 1u, l - 1};
}

__device__ __forceinline__ uint4 ld_stream(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <int kRows, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks)
    qk_prep_kernel(const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ q_scale,
                   const uint16_t* __restrict__ k_scale, const float* __restrict__ cos_t,
                   const float* __restrict__ sin_t, float q_gain, int L, int H, int groups, uint32_t n_items,
                   FastDiv div_groups, FastDiv div_L, int S_out, int row0, uint16_t* __restrict__ q_out,
                   uint16_t* __restrict__ k_out, uint16_t* __restrict__ v_out) {
  // 32-bit index math throughout (the host keeps 16 * n_items below 2^31).
  // Let the next kernel in the stream (attend, launched as a programmatic dependent) start its
  // set-up on SMs this grid frees; it waits for this grid's completion before reading q, k, v.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const uint32_t item = (blockIdx.x * kThreads + threadIdx.x) >> 4;
  const int lane16 = threadIdx.x & 15;
  const bool valid = item < n_items;
  const uint32_t it = valid ? item : 0;       // clamped so the index math below stays in range
  const uint32_t token = div_groups.div(it);  // b * L + l
  const int g = static_cast<int>(it - token * groups);
  const uint32_t b32 = div_L.div(token);
  const int l = static_cast<int>(token - b32 * L);
  const int b = static_cast<int>(b32);
  const int rows3 = 3 * H;
  const int col = lane16 * 8;

  // Issue the row loads first (independent of everything else).
  uint4 x[kRows];
  const uint16_t* src = qkv + (static_cast<size_t>(token) * rows3) * kHeadDim + col;
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    const int r = g * kRows + i;
    x[i] = (valid && r < rows3) ? ld_stream(src + static_cast<size_t>(r) * kHeadDim) : make_uint4(0, 0, 0, 0);
  }

  const float4* cp = reinterpret_cast<const float4*>(cos_t + static_cast<size_t>(l) * kHeadDim + col);
  const float4* sp = reinterpret_cast<const float4*>(sin_t + static_cast<size_t>(l) * kHeadDim + col);
  const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
  const float2 cs[4] = {make_float2(c0.x, c0.y), make_float2(c0.z, c0.w), make_float2(c1.x, c1.y),
                        make_float2(c1.z, c1.w)};
  const float2 sn[4] = {make_float2(s0.x, s0.y), make_float2(s0.z, s0.w), make_float2(s1.x, s1.y),
                        make_float2(s1.z, s1.w)};
  const uint4 qsv = __ldg(reinterpret_cast<const uint4*>(q_scale + col));
  const uint4 ksv = __ldg(reinterpret_cast<const uint4*>(k_scale + col));

#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    const int r = g * kRows + i;
    const int kind = r < H ? 0 : (r < 2 * H ? 1 : 2);  // uniform across the half-warp
    const int h = r - kind * H;
    if (!valid || r >= rows3) continue;
    // Token l of this call is row row0 + l of the [B, H, S_out, D] outputs (row0 = 0, S_out = L
    // for a plain call; a text or image stream writes its slice of the joint sequence).
    const size_t dst = ((static_cast<size_t>(b) * H + h) * S_out + row0 + l) * kHeadDim + col;
    if (kind == 2) {  // v rows are copied straight through
      *reinterpret_cast<uint4*>(v_out + dst) = x[i];
      continue;
    }
    // Sum over this half-warp's 16 lanes (the two half-warps of a warp decide independently).
    const unsigned hmask = 0xFFFFu << (threadIdx.x & 16);
    float ss = qk_group_ss(x[i]);
    ss += __shfl_xor_sync(hmask, ss, 8, 16);
    ss += __shfl_xor_sync(hmask, ss, 4, 16);
    ss += __shfl_xor_sync(hmask, ss, 2, 16);
    ss += __shfl_xor_sync(hmask, ss, 1, 16);
    const uint4 o = qk_norm_rope(x[i], ss, kind == 0 ? qsv : ksv, cs, sn, kind == 0 ? q_gain : 1.0f);
    *reinterpret_cast<uint4*>((kind == 0 ? q_out : k_out) + dst) = o;
  }
}

}  // namespace

template <int kRows, int kMinBlocks>
static int launch_rows(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos_t,
                       const float* sin_t, float q_gain, int B, int L, int H, int S_out, int row0, uint16_t* q,
                       uint16_t* k, uint16_t* v, cudaStream_t stream) {
  const int groups = (3 * H + kRows - 1) / kRows;
  const long long n_items = static_cast<long long>(B) * L * groups;
  if (n_items * 16 >= (1ll << 31)) return FLK_ERR_UNSUPPORTED;  // 32-bit thread indices in the kernel
  const long long blocks = (n_items * 16 + kThreads - 1) / kThreads;
  qk_prep_kernel<kRows, kMinBlocks><<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(
      qkv, q_scale, k_scale, cos_t, sin_t, q_gain, L, H, groups, static_cast<uint32_t>(n_items),
      make_fast_div(static_cast<uint32_t>(groups)), make_fast_div(static_cast<uint32_t>(L)), S_out, row0, q, k, v);
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}

int launch_qk_prep(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos_t,
                   const float* sin_t, float q_gain, int B, int L, int H, int S_out, int row0, uint16_t* q,
                   uint16_t* k, uint16_t* v, cudaStream_t stream) {
  // 4 head rows per work item, 4 CTAs of 256 threads per SM (64 registers, no spills): the fastest
  // of the {2, 3, 4, 6, 8} rows x {2..8} CTAs/SM configurations measured at the 1024^2 shape
  // (fewer rows or more CTAs spill; 8 rows x 3 CTAs is 6 % slower).
  return launch_rows<4, 4>(qkv, q_scale, k_scale, cos_t, sin_t, q_gain, B, L, H, S_out, row0, q, k, v, stream);
}

}  // namespace flk
