// W8A8 SmoothQuant linear for sm_100a: per-token int8 activation quantisation and an int8
// tensor-core GEMM (tcgen05.mma kind::i8, int32 accumulators in TMEM) with the per-token x
// per-channel dequantisation fused into its epilogue.
//
// There is no counterpart in flicker (its linear is a plain bf16 x @ w, src/flicker/nn.py:13-14);
// the arithmetic follows the SmoothQuant method (Xiao et al., 2022) with round-half-even codes:
//   x' = float(x) * inv_smooth[k];  scale_x = max|x'| / 127;  xq = clamp(rint(x' / scale_x), +-127)
//   acc[i, n] = sum_k xq[i, k] * wq[n, k]                      (int32, exact)
//   y[i, n]   = bf16(float(acc) * (scale_x[i] * scale_w[n]))
//
// Batches of at least 256 tokens run on the CTA-pair GEMM of gemm.cu (256 x 256 tiles over two
// SMs, kind::i8, same epilogue arithmetic). Smaller batches use this file's single-CTA kernel
// (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0     TMA producer: per K-block of 128 bytes, one 128x128 box of xq and one 256x128 box
//              of wq (N-major, K contiguous) into a 4-stage ring (48 KB per stage, 128-byte swizzle);
//   warp 1     TMEM allocator + UMMA issuer: 4 MMAs of 128x256x32 per stage into one of two
//              256-column int32 accumulators, so the next tile's MMAs overlap this tile's epilogue;
//   warps 2-5  epilogue: tcgen05.ld the accumulator rows (one TMEM lane per output row), dequantise,
//              round to bf16 and store; rows >= M / columns >= N are masked (TMA zero-fills OOB).
// No TMA multicast.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "flicker_b200.h"
#include "ptx.cuh"

namespace flk {

int launch_gemm_pair_i8(const int8_t* xq, const int8_t* wq, const float* x_scale, const float* w_scale, int M, int N,
                        int K, uint16_t* y, int32_t* acc_out, int* status, int sms, cudaStream_t stream);

namespace {

constexpr int kBM = 128;                  // output rows per tile
constexpr int kBN = 256;                  // output columns per tile
constexpr int kBK = 128;                  // K bytes per stage (one 128-byte swizzle row)
constexpr int kStages = 4;
constexpr int kAStage = kBM * kBK;        // 16 KB
constexpr int kBStage = kBN * kBK;        // 32 KB
constexpr int kGemmThreads = 192;
constexpr uint32_t kTmemCols = 512;

// kind::i8 instruction descriptor: D s32 (2 at bits 4-5), A/B signed int8 (1 at bits 7-9, 10-12),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdescI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((kBN >> 3) << 17) | ((kBM >> 4) << 24);

struct alignas(1024) GemmSmem {
  uint8_t a[kStages][kAStage];
  uint8_t b[kStages][kBStage];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct GemmParams {
  int M, N, K;
  int n_tiles_n;   // ceil(N / kBN)
  int n_tiles;     // ceil(M / kBM) * n_tiles_n
  int k_blocks;    // ceil(K / kBK)
  const float* x_scale;  // [M] (null when writing raw int32)
  const float* w_scale;  // [N]
  uint16_t* y;           // [M, N] bf16, or
  int32_t* acc_out;      // [M, N] int32 (raw accumulators)
  int* status;
};

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %4, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(accumulate), "r"(kIdescI8)
      : "memory");
}

__device__ __forceinline__ uint64_t desc_k(const uint8_t* tile, int kk) {
  return umma_desc_sw128(smem_u32(tile) + kk * 32, 16, 1024);
}

// One epilogue chunk: 32 accumulator columns of one output row -> y (dequantised bf16) or the raw
// int32 accumulators, with row and column masks.
__device__ __forceinline__ void store_chunk(const GemmParams& p, const uint32_t (&r)[32], int row, bool row_ok,
                                           int col0, float sx) {
  if (!row_ok || col0 >= p.N) return;
  const int ncols = min(32, p.N - col0);
  if (p.acc_out) {
    int32_t* dst = p.acc_out + static_cast<size_t>(row) * p.N + col0;
    if (ncols == 32 && (p.N & 3) == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<uint4*>(dst)[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
    } else {
      for (int i = 0; i < ncols; ++i) dst[i] = static_cast<int32_t>(r[i]);
    }
    return;
  }
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int ca = min(col0 + 2 * i, p.N - 1), cb = min(col0 + 2 * i + 1, p.N - 1);
    const float ya = __fmul_rn(__int2float_rn(static_cast<int32_t>(r[2 * i])), __fmul_rn(sx, __ldg(p.w_scale + ca)));
    const float yb = __fmul_rn(__int2float_rn(static_cast<int32_t>(r[2 * i + 1])), __fmul_rn(sx, __ldg(p.w_scale + cb)));
    pk[i] = pack_bf16x2(ya, yb);
  }
  uint16_t* dst = p.y + static_cast<size_t>(row) * p.N + col0;
  if (ncols == 32 && (p.N & 7) == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      reinterpret_cast<uint4*>(dst)[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
  } else {
    for (int i = 0; i < ncols; ++i) dst[i] = static_cast<uint16_t>((pk[i >> 1] >> (16 * (i & 1))) & 0xFFFFu);
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  GemmSmem& sm = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      int n = 0;  // stage fills issued
      int issued[kStages] = {};
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x) {
        const int m0 = (tile / p.n_tiles_n) * kBM, n0 = (tile % p.n_tiles_n) * kBN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++n) {
          const int s = n % kStages, use = n / kStages;
          if (use > 0 && !mbar_wait(&sm.empty[s], (use - 1) & 1, abort, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sm.full[s], kAStage + kBStage);
          tma_load_2d(sm.a[s], &tm_a, kb * kBK, m0, &sm.full[s]);
          tma_load_2d(sm.b[s], &tm_b, kb * kBK, n0, &sm.full[s]);
          issued[s] = use + 1;
        }
      }
      for (int s = 0; s < kStages; ++s)
        if (issued[s] > 0) mbar_drain(&sm.full[s], (issued[s] - 1) & 1, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ UMMA issuer
      int n = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x, ++local) {
        const int buf = local & 1, use = local >> 1;
        if (use > 0 && !mbar_wait(&sm.acc_empty[buf], (use - 1) & 1, abort, p.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kBN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++n) {
          const int s = n % kStages;
          if (!mbar_wait(&sm.full[s], (n / kStages) & 1, abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            umma_i8(d, desc_k(sm.a[s], kk), desc_k(sm.b[s], kk), (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sm.empty[s]);  // the stage is free once these MMAs have read it
        }
        if (ok) tc_commit(&sm.acc_full[buf]);
      }
      tc_commit(&sm.drain);
      mbar_drain(&sm.drain, 0, p.status);
    }
  } else {
    // -------------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    int local = 0;
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1, use = local >> 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.acc_full[buf], use & 1, abort, p.status))) break;
      tc_fence_after();
      const int m0 = (tile / p.n_tiles_n) * kBM, n0 = (tile % p.n_tiles_n) * kBN;
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      const float sx = (row_ok && p.x_scale) ? p.x_scale[row] : 0.f;
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_off + buf * kBN + c * 32, r);
        tmem_wait_ld(r);
        store_chunk(p, r, row, row_ok, n0 + c * 32, sx);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ activation quantisation
// clamp(rint(x' / scale), -127, 127) without a division per element. With inv = rn(1 / scale),
// r = rn(x' * inv) is within 2^-23 relative (|q| <= ~254 even for a subnormal scale: 3e-5
// absolute) of the exact quotient q, and the correctly rounded quotient rn(q) within 1.5e-5 of
// it, so the two round to the same integer unless r lies within 4.5e-5 of a half-integer (or
// rn(q) is a tie). r is rounded to an integer (half to even) by adding 1.5 * 2^23, exact for
// |r| < 2^22; within 2^-14 of a half-integer, or when r is not finite, the correctly rounded
// quotient is computed and converted instead.
__device__ __forceinline__ int quant_code(float xs, float scale, float inv) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23, bit pattern 0x4B400000
  const float r = __fmul_rn(xs, inv);
  const float t = __fadd_rn(r, kRound);
  const float e = fabsf(__fsub_rn(r, __fsub_rn(t, kRound)));  // |r - rint(r)|, exact
  const int q = (e < 0.5f - 6.103515625e-05f) ? __float_as_int(t) - 0x4B400000
                                              : __float2int_rn(__fdiv_rn(xs, scale));
  return max(-127, min(127, q));
}

// quant_code for two values at once, with the same roundings done by packed float2 operations
// (two round-to-nearest results per instruction): r = rn(x' * inv), t = rn(r + 1.5 * 2^23),
// rint(r) = t - 1.5 * 2^23 and r - rint(r) (both exact).
__device__ __forceinline__ void quant_codes2(float2 xs, float scale, float inv, int& q0, int& q1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23, bit pattern 0x4B400000
  constexpr float kLimit = 0.5f - 6.103515625e-05f;
  const float2 r = __fmul2_rn(xs, make_float2(inv, inv));
  const float2 t = __fadd2_rn(r, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 d = __ffma2_rn(n, make_float2(-1.0f, -1.0f), r);
  q0 = fabsf(d.x) < kLimit ? __float_as_int(t.x) - 0x4B400000 : __float2int_rn(__fdiv_rn(xs.x, scale));
  q1 = fabsf(d.y) < kLimit ? __float_as_int(t.y) - 0x4B400000 : __float2int_rn(__fdiv_rn(xs.y, scale));
  q0 = max(-127, min(127, q0));
  q1 = max(-127, min(127, q1));
}

// The low bytes of four codes as one word, code 0 in the lowest byte.
__device__ __forceinline__ uint32_t pack_codes4(int q0, int q1, int q2, int q3) {
  return __byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410);
}

// One warp per row: x' = float(x) * inv_smooth, absmax over the row, scale = absmax / 127,
// q = clamp(rint(x' / scale), -127, 127). K % 8 == 0 (16-byte vectors).
__global__ void __launch_bounds__(256) quantize_act_kernel(const uint16_t* __restrict__ x,
                                                           const float* __restrict__ inv_s, int M, int K,
                                                           int8_t* __restrict__ xq, float* __restrict__ x_scale) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;  // whole warp leaves together
  const uint16_t* xr = x + static_cast<size_t>(row) * K;
  float amax = 0.f;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(inv_s + c));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(inv_s + c + 4));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      amax = fmaxf(amax, fabsf(__fmul_rn(__uint_as_float(w[j] << 16), sv[2 * j])));
      amax = fmaxf(amax, fabsf(__fmul_rn(__uint_as_float(w[j] & 0xFFFF0000u), sv[2 * j + 1])));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  float scale = __fdiv_rn(amax, 127.0f);
  if (!(scale > 0.f)) scale = 1.0f;
  if (lane == 0) x_scale[row] = scale;
  const float inv = __frcp_rn(scale);
  int8_t* qr = xq + static_cast<size_t>(row) * K;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(inv_s + c));
    const float4 s1 = __ldg(reinterpret_cast<const float4*>(inv_s + c + 4));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float xv = (j & 1) ? __uint_as_float(w[j >> 1] & 0xFFFF0000u) : __uint_as_float(w[j >> 1] << 16);
      const int qv = quant_code(__fmul_rn(xv, sv[j]), scale, inv);
      packed[j >> 2] |= (static_cast<uint32_t>(qv) & 0xFFu) << (8 * (j & 3));
    }
    *reinterpret_cast<uint2*>(qr + c) = make_uint2(packed[0], packed[1]);
  }
}

// Same arithmetic with one CTA of 128 threads per row held in registers (K <= 1024 * kIters):
// every load of the row is issued before any math, the absmax is reduced across the CTA, and the
// codes are computed from the registers. Many small CTAs per SM keep the loads of some rows in
// flight while others compute.
constexpr int kRowThreads = 128;
template <int kIters>
__global__ void __launch_bounds__(kRowThreads) quantize_act_row_kernel(const uint16_t* __restrict__ x,
                                                                      const float* __restrict__ inv_s, int K,
                                                                      int8_t* __restrict__ xq,
                                                                      float* __restrict__ x_scale) {
  __shared__ float red[kRowThreads / 32];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const uint16_t* xr = x + static_cast<size_t>(row) * K;
  uint4 v[kIters];
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int c = (it * kRowThreads + tid) * 8;
    v[it] = c < K ? *reinterpret_cast<const uint4*>(xr + c) : make_uint4(0, 0, 0, 0);
  }
  float2 xs[kIters][4];  // x' in pairs: columns (2p, 2p+1) of the thread's 8
  float amax = 0.f;
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int c = (it * kRowThreads + tid) * 8;
    float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
    if (c < K) {
      s0 = __ldg(reinterpret_cast<const float4*>(inv_s + c));
      s1 = __ldg(reinterpret_cast<const float4*>(inv_s + c + 4));
    }
    const uint32_t w[4] = {v[it].x, v[it].y, v[it].z, v[it].w};
    const float2 sv[4] = {make_float2(s0.x, s0.y), make_float2(s0.z, s0.w), make_float2(s1.x, s1.y),
                          make_float2(s1.z, s1.w)};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float2 xv = make_float2(__uint_as_float(w[p] << 16), __uint_as_float(w[p] & 0xFFFF0000u));
      xs[it][p] = __fmul2_rn(xv, sv[p]);
      amax = fmaxf(amax, fmaxf(fabsf(xs[it][p].x), fabsf(xs[it][p].y)));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  float scale = __fdiv_rn(amax, 127.0f);
  if (!(scale > 0.f)) scale = 1.0f;
  if (tid == 0) x_scale[row] = scale;
  const float inv = __frcp_rn(scale);
  int8_t* qr = xq + static_cast<size_t>(row) * K;
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int c = (it * kRowThreads + tid) * 8;
    if (c >= K) break;
    int q[8];
#pragma unroll
    for (int p = 0; p < 4; ++p) quant_codes2(xs[it][p], scale, inv, q[2 * p], q[2 * p + 1]);
    *reinterpret_cast<uint2*>(qr + c) =
        make_uint2(pack_codes4(q[0], q[1], q[2], q[3]), pack_codes4(q[4], q[5], q[6], q[7]));
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [rows, K] int8, K contiguous, boxes of box_rows x 128 bytes with the 128-byte swizzle; OOB reads 0.
bool make_i8_map(CUtensorMap* map, const void* base, long long rows, int K, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

static int launch_w8a8_gemm_single(const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p, int sms,
                                   cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FLK_ERR_CUDA;
  static std::mutex setup_mu;  // first calls from several host threads set up once
  static bool configured[64] = {};
  const size_t smem = sizeof(GemmSmem) + 1024;
  {
    std::lock_guard<std::mutex> lock(setup_mu);
    if (!configured[dev]) {
      if (cudaFuncSetAttribute(w8a8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)) != cudaSuccess)
        return FLK_ERR_CUDA;
      configured[dev] = true;
    }
  }
  const int grid = std::min(p.n_tiles, sms);
  w8a8_gemm_kernel<<<grid, kGemmThreads, smem, stream>>>(ma, mb, p);
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}

int launch_w8a8_gemm(const int8_t* xq, const int8_t* wq, const float* x_scale, const float* w_scale, int M, int N,
                     int K, uint16_t* y, int32_t* acc_out, int* status, int sms, cudaStream_t stream) {
  // Batches of at least 256 tokens run on CTA pairs (256 x 256 tiles); smaller ones on single
  // CTAs (128 x 256 tiles), where half of a pair's tile would be padding.
  if (M >= 256) return launch_gemm_pair_i8(xq, wq, x_scale, w_scale, M, N, K, y, acc_out, status, sms, stream);
  CUtensorMap ma, mb;
  if (!make_i8_map(&ma, xq, M, K, kBM) || !make_i8_map(&mb, wq, N, K, kBN)) return FLK_ERR_CUDA;
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.n_tiles_n = (N + kBN - 1) / kBN;
  p.n_tiles = ((M + kBM - 1) / kBM) * p.n_tiles_n;
  p.k_blocks = (K + kBK - 1) / kBK;
  p.x_scale = x_scale;
  p.w_scale = w_scale;
  p.y = y;
  p.acc_out = acc_out;
  p.status = status;
  return launch_w8a8_gemm_single(ma, mb, p, sms, stream);
}

int launch_quantize_act(const uint16_t* x, const float* inv_s, int M, int K, int8_t* xq, float* x_scale,
                        cudaStream_t stream) {
  // Rows up to 4096 wide: one CTA per row, held in registers; wider rows take the two-pass
  // kernel (one warp per row).
  const unsigned rows = static_cast<unsigned>(M);
  if (K <= 1024)
    quantize_act_row_kernel<1><<<rows, kRowThreads, 0, stream>>>(x, inv_s, K, xq, x_scale);
  else if (K <= 2048)
    quantize_act_row_kernel<2><<<rows, kRowThreads, 0, stream>>>(x, inv_s, K, xq, x_scale);
  else if (K <= 3072)
    quantize_act_row_kernel<3><<<rows, kRowThreads, 0, stream>>>(x, inv_s, K, xq, x_scale);
  else if (K <= 4096)
    quantize_act_row_kernel<4><<<rows, kRowThreads, 0, stream>>>(x, inv_s, K, xq, x_scale);
  else {
    const long long threads = static_cast<long long>(M) * 32;
    quantize_act_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(x, inv_s, M, K, xq,
                                                                                        x_scale);
  }
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}

static_assert(sizeof(GemmSmem) + 1024 <= 232448, "w8a8 shared memory exceeds the 227 KB opt-in limit");

}  // namespace flk
