// qk_prep for sm_100a: head split + QK-RMSNorm + lane-pair RoPE (+ q gain) in one HBM pass.
//
// Restates flicker kernels.qk_prep (src/flicker/kernels.py:57-91, body :35-53) as a
// memory-bound CUDA kernel. Work item = one token x a group of 8 consecutive head rows
// of that token's fused QKV row (row r of 3H: r < H -> q head r, r < 2H -> k head r-H,
// else v head r-2H). A half-warp (16 lanes) owns one item; lane j owns columns
// [8j, 8j+8) of every 128-wide head row, so:
//   * every global access is one 16-byte vector per lane and 256 contiguous bytes per
//     half-warp, on both the [B, L, 3HD] read side and the head-major [B, H, L, D]
//     write side (the transpose costs nothing at row granularity);
//   * the RoPE partner of column 2i is column 2i+1 of the same lane (no shuffle);
//   * the cos/sin lane tables and both scale vectors are loaded once per item and reused
//     for its 8 rows (they are L2-resident: 1 KB per token);
//   * the sum of squares is reduced across the 16 lanes with 4 xor-shuffles;
//   * all 8 row loads of an item are issued before any math (8 x 16 B in flight per lane).
// Rounding follows the reference body exactly: fp32 norm, bf16 round, bf16 x bf16 scale
// multiply rounded to bf16, fp32 rotation c*w + s*swap (no FMA contraction), q gain in
// fp32, final bf16 round.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "flicker_b200.h"

namespace flk {

namespace {

constexpr int kHeadDim = 128;
constexpr int kRowsPerItem = 8;
constexpr int kThreads = 256;

__device__ __forceinline__ uint4 ld_stream(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(kThreads) qk_prep_kernel(const uint16_t* __restrict__ qkv,
                                                           const uint16_t* __restrict__ q_scale,
                                                           const uint16_t* __restrict__ k_scale,
                                                           const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t, float q_gain,
                                                           int L, int H, int groups, long long n_items,
                                                           uint16_t* __restrict__ q_out,
                                                           uint16_t* __restrict__ k_out,
                                                           uint16_t* __restrict__ v_out) {
  const long long item = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 4;
  const int lane16 = threadIdx.x & 15;
  const bool valid = item < n_items;
  const long long it = valid ? item : 0;  // keep every lane in the shuffles below
  const long long token = it / groups;    // b * L + l
  const int g = static_cast<int>(it - token * groups);
  const int l = static_cast<int>(token % L);
  const int b = static_cast<int>(token / L);
  const int rows3 = 3 * H;
  const int col = lane16 * 8;

  // Issue the row loads first (independent of everything else).
  uint4 x[kRowsPerItem];
  const uint16_t* src = qkv + (static_cast<size_t>(token) * rows3) * kHeadDim + col;
#pragma unroll
  for (int i = 0; i < kRowsPerItem; ++i) {
    const int r = g * kRowsPerItem + i;
    x[i] = (valid && r < rows3) ? ld_stream(src + static_cast<size_t>(r) * kHeadDim) : make_uint4(0, 0, 0, 0);
  }

  const float4* cp = reinterpret_cast<const float4*>(cos_t + static_cast<size_t>(l) * kHeadDim + col);
  const float4* sp = reinterpret_cast<const float4*>(sin_t + static_cast<size_t>(l) * kHeadDim + col);
  const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
  const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  const uint4 qsv = __ldg(reinterpret_cast<const uint4*>(q_scale + col));
  const uint4 ksv = __ldg(reinterpret_cast<const uint4*>(k_scale + col));

#pragma unroll
  for (int i = 0; i < kRowsPerItem; ++i) {
    const int r = g * kRowsPerItem + i;
    const int kind = r < H ? 0 : (r < 2 * H ? 1 : 2);  // uniform across the half-warp
    const int h = r - kind * H;
    const uint32_t w[4] = {x[i].x, x[i].y, x[i].z, x[i].w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[2 * j] = bf_lo(w[j]);
      f[2 * j + 1] = bf_hi(w[j]);
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    ss += __shfl_xor_sync(0xffffffffu, ss, 8, 16);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4, 16);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2, 16);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1, 16);
    if (!valid || r >= rows3) continue;

    const size_t dst = ((static_cast<size_t>(b) * H + h) * L + l) * kHeadDim + col;
    if (kind == 2) {
      *reinterpret_cast<uint4*>(v_out + dst) = x[i];
      continue;
    }
    // rsqrt(mean + eps) as 1 / sqrt(.) with IEEE rounding of each step.
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(ss * (1.0f / kHeadDim) + 1e-6f));
    const uint4 sv = kind == 0 ? qsv : ksv;
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
    float n[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      n[2 * j] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(f[2 * j], inv)), bf_lo(sw[j])));
      n[2 * j + 1] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(f[2 * j + 1], inv)), bf_hi(sw[j])));
    }
    const float gain = kind == 0 ? q_gain : 1.0f;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = 2 * j, d = 2 * j + 1;
      float re = __fadd_rn(__fmul_rn(cs[e], n[e]), __fmul_rn(sn[e], n[d]));
      float rd = __fadd_rn(__fmul_rn(cs[d], n[d]), __fmul_rn(sn[d], n[e]));
      if (gain != 1.0f) {
        re = __fmul_rn(gain, re);
        rd = __fmul_rn(gain, rd);
      }
      __nv_bfloat162 pr = __floats2bfloat162_rn(re, rd);
      o[j] = *reinterpret_cast<uint32_t*>(&pr);
    }
    uint16_t* out = kind == 0 ? q_out : k_out;
    *reinterpret_cast<uint4*>(out + dst) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

int launch_qk_prep(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale, const float* cos_t,
                   const float* sin_t, float q_gain, int B, int L, int H, uint16_t* q, uint16_t* k, uint16_t* v,
                   cudaStream_t stream) {
  const int groups = (3 * H + kRowsPerItem - 1) / kRowsPerItem;
  const long long n_items = static_cast<long long>(B) * L * groups;
  const long long threads = n_items * 16;
  const long long blocks = (threads + kThreads - 1) / kThreads;
  if (blocks > 0x7FFFFFFFLL) return FLK_ERR_UNSUPPORTED;
  qk_prep_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(
      qkv, q_scale, k_scale, cos_t, sin_t, q_gain, L, H, groups, n_items, q, k, v);
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}

}  // namespace flk
