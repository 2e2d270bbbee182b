// Per-row arithmetic of flicker's qk_prep body (src/flicker/kernels.py:35-53), shared by the
// standalone qk_prep kernel and the GEMM epilogue that fuses it, so both round identically.
//
// A 128-column head row is handled as 16 groups of 8 columns (4 bf16 pair words, low half =
// even column). Rounding points: fp32 norm (rsqrt on the SFU), bf16 round, bf16 x bf16 scale
// multiply rounded to bf16, fp32 rotation c*w + s*swap (no FMA contraction), q gain in fp32,
// final bf16 round.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

namespace flk {

constexpr int kQkHeadDim = 128;

// bf16 pair word -> the two values as fp32 (exact).
__device__ __forceinline__ float2 qk_unpack(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t qk_pack(float2 v) {
  __nv_bfloat162 b = __float22bfloat162_rn(v);
  return *reinterpret_cast<uint32_t*>(&b);
}

// Sum of squares of one 8-column group (exact squares of bf16 values, fp32 adds in a fixed order).
__device__ __forceinline__ float qk_group_ss(uint4 x) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
  float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = qk_unpack(w[j]);
    s2 = __ffma2_rn(f, f, s2);
  }
  return s2.x + s2.y;
}

// The row's sum of squares from its 16 group sums, added in the order of a 16-lane xor
// butterfly (offsets 8, 4, 2, 1), which is how the standalone kernel reduces across lanes.
__device__ __forceinline__ float qk_row_ss(const float (&p)[16]) {
  float a[8], b[4];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = p[j] + p[j + 8];
#pragma unroll
  for (int j = 0; j < 4; ++j) b[j] = a[j] + a[j + 4];
  return (b[0] + b[2]) + (b[1] + b[3]);
}

// One 8-column group: RMSNorm -> bf16 -> * scale (bf16) -> RoPE in fp32 -> (* gain) -> bf16.
// `ss` is the row's sum of squares over all 128 columns; c / sn are the lane tables of the
// group's 4 pairs (cos repeated, (-sin, +sin)).
__device__ __forceinline__ uint4 qk_norm_rope(uint4 x, float ss, uint4 scale, const float2 (&c)[4],
                                              const float2 (&sn)[4], float gain) {
  // rsqrt(mean + eps) on the SFU (<= 2 ulp; lax.rsqrt's own ulps are not pinned by the reference).
  const float inv = rsqrtf(ss * (1.0f / kQkHeadDim) + 1e-6f);
  const float2 inv2 = make_float2(inv, inv);
  const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
  const uint32_t sw[4] = {scale.x, scale.y, scale.z, scale.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    // bf16(x * inv), then the bf16 x bf16 scale multiply rounded to bf16 (exact product, one rounding).
    __nv_bfloat162 sc = *reinterpret_cast<const __nv_bfloat162*>(&sw[j]);
    const __nv_bfloat162 nb = __hmul2(__float22bfloat162_rn(__fmul2_rn(qk_unpack(xw[j]), inv2)), sc);
    const float2 w = qk_unpack(*reinterpret_cast<const uint32_t*>(&nb));
    // rotation c * w + s * swap(w) with separate roundings (no contraction), as the reference body.
    float2 r = __fadd2_rn(__fmul2_rn(c[j], w), __fmul2_rn(sn[j], make_float2(w.y, w.x)));
    if (gain != 1.0f) r = __fmul2_rn(r, make_float2(gain, gain));
    o[j] = qk_pack(r);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace flk
