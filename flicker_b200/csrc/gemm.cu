// CTA-pair tensor-core GEMM for sm_100a: y[M, N] = x[M, K] @ w[K, N] with the weights stored
// N-major (w^T, [N, K], K contiguous), in two operand kinds and three epilogues.
//
//   kind::i8   int8 codes, int32 accumulators  -> epilogue DEQUANT: y = bf16(acc * sx[i] * sw[n])
//                                                  (the W8A8 SmoothQuant linear), or raw int32
//   kind::f16  bf16 operands, fp32 accumulators -> epilogue BF16_OUT: y = bf16(acc), i.e. the
//                                                  reference's linear x @ w (src/flicker/nn.py:13-14)
//                                               -> epilogue QK_PREP: the QKV projection with
//                                                  qk_prep fused into its epilogue (below)
//
// Structure (one CTA per SM, persistent over 256 x 256 output tiles, clusters of two CTAs):
// CTA r of the pair loads rows [128r, 128r + 128) of the tile's x block and rows [128r, 128r+128)
// of its w^T block (128 K bytes per stage, 6 stages of 32 KB, 128-byte swizzle) into its own
// shared memory; the even CTA issues tcgen05.mma.cta_group::2 (256 x 256 x 32 bytes of K) that
// read both CTAs' halves, and CTA r's tensor memory receives output rows [128r, 128r + 128) x all
// 256 columns, double-buffered (2 x 256 of its 512 columns) so one tile's epilogue overlaps the
// next tile's MMAs. Each CTA's loads signal the even CTA's barrier (cta_group::2 TMA, no
// multicast); the even CTA's commits arrive on both CTAs' barriers (commit multicast); both
// CTAs' epilogue warps hand the accumulator back to the even CTA's barrier.
//
// QK_PREP epilogue (the fused form of modules.qkv_prep after linear, modules.py:68-80,127-134,
// 184-190): output columns [0, 3*H*128) are the fused (3, H, D) q, k, v block; each epilogue
// thread owns one token row, and for each 128-column head block of its tile it rounds the
// accumulators to bf16 (the linear's output), then for q and k rows sums the squares in the
// standalone kernel's order, normalises, scales, rotates and (q) applies the gain exactly as
// qk_prep does (qk_math.cuh), and stores the head row to q / k / v [B, H, S_out, D] at row
// row0 + l; columns past the q, k, v block (a single block's mlp part) are stored as bf16 to
// `rest`. The result equals linear followed by qk_prep bit for bit, without the qkv round trip
// through HBM.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "flicker_b200.h"
#include "ptx.cuh"
#include "qk_math.cuh"

namespace flk {

enum class GemmKind { I8, BF16 };
enum class GemmEpi { DEQUANT, BF16_OUT, QK_PREP };

struct PairParams {
  int M, N, K;      // output [M, N]; K in elements
  int k_blocks;     // ceil(K bytes / 128)
  // DEQUANT (kind::i8)
  const float* x_scale;  // [M] (null when writing raw int32)
  const float* w_scale;  // [N]
  int32_t* acc_out;      // [M, N] raw int32 accumulators, or null
  // DEQUANT and BF16_OUT
  uint16_t* y;  // [M, N] bf16
  // QK_PREP
  int L, H, S_out, row0, n_qkv;  // tokens per batch element, heads, output rows, first row, 3*H*128
  const uint16_t* q_scale;
  const uint16_t* k_scale;
  const float* cos_t;
  const float* sin_t;
  float q_gain;
  uint16_t* q;
  uint16_t* k;
  uint16_t* v;
  uint16_t* rest;  // [M, N - n_qkv] bf16, or null when N == n_qkv
  int* status;
};

namespace {

constexpr int kPairBK = 128;                   // K bytes per stage
constexpr int kPairStages = 6;
constexpr int kPairHalf = 128 * kPairBK;       // 16 KB: 128 rows x 128 K bytes
constexpr int kPairStageBytes = 2 * kPairHalf;  // per CTA and stage: x half + w half
constexpr int kPairThreads = 192;
constexpr uint32_t kPairTmemCols = 512;

// Instruction descriptors (M = 256 across the pair, N = 256, both operands K-major):
// D format at bits 4-5 (1 = f32, 2 = s32), A / B formats at 7-9 / 10-12 (bf16 = 1, signed
// int8 = 1), N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdescPairI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((256u >> 4) << 24);
constexpr uint32_t kIdescPairBf16 = (1u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((256u >> 4) << 24);

struct alignas(1024) PairSmem {
  uint8_t a[kPairStages][kPairHalf];
  uint8_t b[kPairStages][kPairHalf];
  uint64_t full[kPairStages];   // even CTA: both halves of the stage have landed (tx bytes of both CTAs)
  uint64_t empty[kPairStages];  // both CTAs: the stage's MMAs are done (multicast commit)
  uint64_t acc_full[2];         // both CTAs: accumulator buffer complete (multicast commit)
  uint64_t acc_empty[2];        // even CTA: the 8 epilogue warps of the pair have read the buffer
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the variable at `p` in the cluster's CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2-D TMA load into this CTA's shared memory whose completion bytes go to the barrier at
// `bar_cluster` (the even CTA's barrier of the pair).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, int c0, int c1, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}
template <GemmKind KD>
__device__ __forceinline__ void umma_pair_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  if constexpr (KD == GemmKind::I8) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %3, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %4, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(accumulate), "r"(kIdescPairI8)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %3, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %4, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(accumulate), "r"(kIdescPairBf16)
        : "memory");
  }
}
// Arrive on the barrier at this offset in both CTAs of the pair once the pair's MMAs issued so
// far have completed.
__device__ __forceinline__ void tc_commit_pair_both_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}\n" ::
          "r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair_own_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
      : "memory");
}
// K-major operand, 128-byte swizzle: the 32-byte K step kk of a 128-row x 128-byte stage half.
__device__ __forceinline__ uint64_t desc_k32(const uint8_t* tile, int kk) {
  return umma_desc_sw128(smem_u32(tile) + kk * 32, 16, 1024);
}

// One DEQUANT epilogue chunk: 32 accumulator columns of one output row -> y (dequantised bf16)
// or the raw int32 accumulators, with row and column masks.
__device__ __forceinline__ void store_dequant_chunk(const PairParams& p, const uint32_t (&r)[32], int row, bool row_ok,
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

// fp32 accumulators of 32 columns -> 16 bf16 pair words (round to nearest even).
__device__ __forceinline__ void round_chunk(const uint32_t (&r)[32], uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
}

// 16 bf16 pair words (32 columns) -> dst[0 .. ncols), 16-byte stores when whole and aligned.
__device__ __forceinline__ void store_bf16_words(uint16_t* dst, const uint32_t (&pk)[16], int ncols, bool vec) {
  if (ncols == 32 && vec) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      reinterpret_cast<uint4*>(dst)[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
  } else {
    for (int i = 0; i < ncols; ++i) dst[i] = static_cast<uint16_t>((pk[i >> 1] >> (16 * (i & 1))) & 0xFFFFu);
  }
}

// One BF16_OUT epilogue chunk: y[row, col0 .. col0 + 32) = bf16(acc), masked.
__device__ __forceinline__ void store_bf16_chunk(const PairParams& p, const uint32_t (&r)[32], int row, bool row_ok,
                                                 int col0) {
  if (!row_ok || col0 >= p.N) return;
  uint32_t pk[16];
  round_chunk(r, pk);
  store_bf16_words(p.y + static_cast<size_t>(row) * p.N + col0, pk, min(32, p.N - col0), (p.N & 7) == 0);
}

// QK_PREP epilogue of one 128-column head block (output columns [c0, c0 + 128)) of this thread's
// token row m. `t_addr` is the TMEM address of the block's first column in this warp's lanes.
// Every lane executes the TMEM loads (they are warp-collective); rows >= M store nothing.
__device__ __forceinline__ void qk_head_block(const PairParams& p, uint32_t t_addr, int m, bool row_ok, int c0) {
  const int hd = p.H * kQkHeadDim;
  if (c0 >= p.n_qkv) {  // past the q, k, v block: plain bf16 into `rest`
    const int width = p.N - p.n_qkv;
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_addr + cc * 32, r);
      tmem_wait_ld(r);
      const int col = c0 - p.n_qkv + cc * 32;
      if (!row_ok || col >= width || p.rest == nullptr) continue;
      uint32_t pk[16];
      round_chunk(r, pk);
      store_bf16_words(p.rest + static_cast<size_t>(m) * width + col, pk, min(32, width - col), (width & 7) == 0);
    }
    return;
  }
  const int part = c0 / hd;  // 0 q, 1 k, 2 v (uniform across the warp)
  const int h = (c0 - part * hd) / kQkHeadDim;
  const int b = m / p.L, l = m - b * p.L;
  uint16_t* base = part == 0 ? p.q : (part == 1 ? p.k : p.v);
  uint16_t* dst = base + ((static_cast<size_t>(b) * p.H + h) * p.S_out + p.row0 + l) * kQkHeadDim;
  if (part == 2) {  // v: the linear's bf16 output, moved to its head-major row
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_addr + cc * 32, r);
      tmem_wait_ld(r);
      if (!row_ok) continue;
      uint32_t pk[16];
      round_chunk(r, pk);
      store_bf16_words(dst + cc * 32, pk, 32, true);
    }
    return;
  }
  // q / k: pass 1 sums the squares of the bf16-rounded row in the standalone kernel's order.
  float part_ss[16];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_addr + cc * 32, r);
    tmem_wait_ld(r);
    uint32_t pk[16];
    round_chunk(r, pk);
#pragma unroll
    for (int g = 0; g < 4; ++g)
      part_ss[cc * 4 + g] = qk_group_ss(make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]));
  }
  const float ss = qk_row_ss(part_ss);
  const uint16_t* scale = part == 0 ? p.q_scale : p.k_scale;
  const float gain = part == 0 ? p.q_gain : 1.0f;
  const float* crow = p.cos_t + static_cast<size_t>(l) * kQkHeadDim;
  const float* srow = p.sin_t + static_cast<size_t>(l) * kQkHeadDim;
  // Pass 2 reloads the accumulators and applies norm, scale, rotation and gain per 8-column group.
#pragma unroll 1
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_addr + cc * 32, r);
    tmem_wait_ld(r);
    if (!row_ok) continue;
    uint32_t pk[16];
    round_chunk(r, pk);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int col = cc * 32 + g * 8;
      const float4 c0v = __ldg(reinterpret_cast<const float4*>(crow + col));
      const float4 c1v = __ldg(reinterpret_cast<const float4*>(crow + col + 4));
      const float4 s0v = __ldg(reinterpret_cast<const float4*>(srow + col));
      const float4 s1v = __ldg(reinterpret_cast<const float4*>(srow + col + 4));
      const float2 cs[4] = {make_float2(c0v.x, c0v.y), make_float2(c0v.z, c0v.w), make_float2(c1v.x, c1v.y),
                            make_float2(c1v.z, c1v.w)};
      const float2 sn[4] = {make_float2(s0v.x, s0v.y), make_float2(s0v.z, s0v.w), make_float2(s1v.x, s1v.y),
                            make_float2(s1v.z, s1v.w)};
      const uint4 sc = __ldg(reinterpret_cast<const uint4*>(scale + col));
      const uint4 o = qk_norm_rope(make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]), ss, sc, cs, sn,
                                   gain);
      *reinterpret_cast<uint4*>(dst + col) = o;
    }
  }
}

template <GemmKind KD, GemmEpi EP>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ PairParams p) {
  extern __shared__ uint8_t smem_raw[];
  PairSmem& sm = *reinterpret_cast<PairSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the pair's MMAs
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 8);  // 4 epilogue warps in each CTA of the pair
    }
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(kPairTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated before any use
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort = &sm.abort;
  const int n_tiles_n = (p.N + 255) / 256;
  const int n_tiles = ((p.M + 255) / 256) * n_tiles_n;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    const bool leader = lane == 0;
    if (leader) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
    }
    // TMA x coordinate of a K block, in elements (128 bytes: 128 int8 or 64 bf16).
    constexpr int kBlockElems = KD == GemmKind::I8 ? kPairBK : kPairBK / 2;
    int n = 0;
    int issued[kPairStages] = {};
    bool ok = true;
    for (int tile = pair; ok && tile < n_tiles; tile += n_pairs) {
      const int m0 = (tile / n_tiles_n) * 256 + 128 * static_cast<int>(rank);
      const int nb0 = (tile % n_tiles_n) * 256 + 128 * static_cast<int>(rank);
      for (int kb = 0; kb < p.k_blocks; ++kb, ++n) {
        const int s = n % kPairStages, use = n / kPairStages;
        if (use > 0 && !mbar_wait_warp(&sm.empty[s], (use - 1) & 1, abort, p.status)) {
          ok = false;
          break;
        }
        if (leader) {
          const uint32_t full0 = mapa_shared(&sm.full[s], 0);
          if (rank == 0) mbar_arrive_expect_tx(&sm.full[s], 2 * kPairStageBytes);
          tma_load_2d_pair(sm.a[s], &tm_a, kb * kBlockElems, m0, full0);
          tma_load_2d_pair(sm.b[s], &tm_b, kb * kBlockElems, nb0, full0);
        }
        issued[s] = use + 1;
        __syncwarp();
      }
    }
    // Never leave with a copy in flight: the even CTA waits (bounded) for the last fill of every
    // stage, which covers both CTAs' copies into it; the odd CTA's copies are covered by the
    // empty[] phases it waited for and by the final cluster barrier, which the even CTA reaches
    // only after its MMAs (the consumers of those copies) have drained.
    if (rank == 0)
      for (int s = 0; s < kPairStages; ++s)
        if (issued[s] > 0) mbar_drain(&sm.full[s], (issued[s] - 1) & 1, p.status);
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------------------------------------------------------- UMMA issuer (even CTA)
      int n = 0, local = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < n_tiles; tile += n_pairs, ++local) {
        const int buf = local & 1, use = local >> 1;
        if (use > 0 && !mbar_wait_warp(&sm.acc_empty[buf], (use - 1) & 1, abort, p.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * 256;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++n) {
          const int s = n % kPairStages;
          if (!mbar_wait_warp(&sm.full[s], (n / kPairStages) & 1, abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kPairBK / 32; ++kk)
            umma_pair_warp<KD>(d, desc_k32(sm.a[s], kk), desc_k32(sm.b[s], kk), (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit_pair_both_warp(&sm.empty[s]);  // the stage is free in both CTAs once read
        }
        if (ok) tc_commit_pair_both_warp(&sm.acc_full[buf]);
      }
      tc_commit_pair_own_warp(&sm.drain);
      mbar_drain(&sm.drain, 0, p.status);
    }
  } else {
    // -------------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp & 3;
    const int row_in_half = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t acc_empty0[2] = {mapa_shared(&sm.acc_empty[0], 0), mapa_shared(&sm.acc_empty[1], 0)};
    int local = 0;
    for (int tile = pair; tile < n_tiles; tile += n_pairs, ++local) {
      const int buf = local & 1, use = local >> 1;
      if (!mbar_wait_warp(&sm.acc_full[buf], use & 1, abort, p.status)) break;
      tc_fence_after();
      const int row = (tile / n_tiles_n) * 256 + 128 * static_cast<int>(rank) + row_in_half;
      const int n0 = (tile % n_tiles_n) * 256;
      const bool row_ok = row < p.M;
      const uint32_t t_base = tmem + lane_off + buf * 256;
      if constexpr (EP == GemmEpi::QK_PREP) {
#pragma unroll 1
        for (int hb = 0; hb < 2; ++hb)
          if (n0 + hb * 128 < p.N) qk_head_block(p, t_base + hb * 128, row, row_ok, n0 + hb * 128);
      } else {
        const float sx = (EP == GemmEpi::DEQUANT && row_ok && p.x_scale) ? p.x_scale[row] : 0.f;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_base + c * 32, r);
          tmem_wait_ld(r);
          if constexpr (EP == GemmEpi::DEQUANT)
            store_dequant_chunk(p, r, row, row_ok, n0 + c * 32, sx);
          else
            store_bf16_chunk(p, r, row, row_ok, n0 + c * 32);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0[buf]);
    }
  }

  tc_fence_before();
  cluster_sync_all();  // the even CTA's MMAs have drained; no CTA reads the other's memory after this
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPairTmemCols) : "memory");
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn gemm_encode_fn() {
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

// [rows, K] row-major operand (K contiguous) through 128-byte x 128-row boxes, 128-byte swizzle.
template <GemmKind KD>
bool make_operand_map(CUtensorMap* map, const void* base, long long rows, int K) {
  EncodeTiledFn enc = gemm_encode_fn();
  if (!enc) return false;
  constexpr int kElem = KD == GemmKind::I8 ? 1 : 2;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * kElem};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kPairBK / kElem), 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType type = KD == GemmKind::I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  return enc(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static_assert(sizeof(PairSmem) + 1024 <= 232448, "pair GEMM shared memory exceeds the 227 KB opt-in limit");

template <GemmKind KD, GemmEpi EP>
int launch_pair(const void* x, const void* wt, PairParams p, int sms, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FLK_ERR_CUDA;
  static std::mutex setup_mu;  // first calls from several host threads set up once
  static bool configured[64] = {};
  const size_t smem = sizeof(PairSmem) + 1024;
  {
    std::lock_guard<std::mutex> lock(setup_mu);
    if (!configured[dev]) {
      if (cudaFuncSetAttribute(gemm_pair_kernel<KD, EP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem)) != cudaSuccess)
        return FLK_ERR_CUDA;
      configured[dev] = true;
    }
  }
  CUtensorMap ma, mb;
  if (!make_operand_map<KD>(&ma, x, p.M, p.K) || !make_operand_map<KD>(&mb, wt, p.N, p.K)) return FLK_ERR_CUDA;
  constexpr int kElem = KD == GemmKind::I8 ? 1 : 2;
  p.k_blocks = static_cast<int>((static_cast<long long>(p.K) * kElem + kPairBK - 1) / kPairBK);
  const int pair_tiles = ((p.M + 255) / 256) * ((p.N + 255) / 256);
  const int pairs = std::max(1, std::min(pair_tiles, sms / 2));
  gemm_pair_kernel<KD, EP><<<2 * pairs, kPairThreads, smem, stream>>>(ma, mb, p);
  return cudaGetLastError() == cudaSuccess ? FLK_OK : FLK_ERR_CUDA;
}

}  // namespace

int launch_gemm_pair_i8(const int8_t* xq, const int8_t* wq, const float* x_scale, const float* w_scale, int M, int N,
                        int K, uint16_t* y, int32_t* acc_out, int* status, int sms, cudaStream_t stream) {
  PairParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.x_scale = x_scale;
  p.w_scale = w_scale;
  p.acc_out = acc_out;
  p.y = y;
  p.status = status;
  return launch_pair<GemmKind::I8, GemmEpi::DEQUANT>(xq, wq, p, sms, stream);
}

int launch_linear_bf16(const uint16_t* x, const uint16_t* wt, int M, int N, int K, uint16_t* y, int* status, int sms,
                       cudaStream_t stream) {
  PairParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.y = y;
  p.status = status;
  return launch_pair<GemmKind::BF16, GemmEpi::BF16_OUT>(x, wt, p, sms, stream);
}

int launch_linear_qk_prep(const uint16_t* x, const uint16_t* wt, int M, int N, int K, int L, int H,
                          const uint16_t* q_scale, const uint16_t* k_scale, const float* cos_t, const float* sin_t,
                          float q_gain, uint16_t* q, uint16_t* k, uint16_t* v, int S_out, int row0, uint16_t* rest,
                          int* status, int sms, cudaStream_t stream) {
  PairParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.L = L;
  p.H = H;
  p.S_out = S_out;
  p.row0 = row0;
  p.n_qkv = 3 * H * kQkHeadDim;
  p.q_scale = q_scale;
  p.k_scale = k_scale;
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.q_gain = q_gain;
  p.q = q;
  p.k = k;
  p.v = v;
  p.rest = rest;
  p.status = status;
  return launch_pair<GemmKind::BF16, GemmEpi::QK_PREP>(x, wt, p, sms, stream);
}

}  // namespace flk
