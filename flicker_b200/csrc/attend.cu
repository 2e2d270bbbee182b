// Bounded (max-free) flash attention for sm_100a: TMA -> shared memory -> tcgen05.mma -> TMEM.
//
// Restates flicker kernels.attend (src/flicker/kernels.py:105-145):
//   s = q k^T (fp32, q already carries 1/sqrt(D)),  p = bf16(exp(s)),
//   l += sum fp32(p),  acc += p v (fp32),  o = bf16(acc / l) once at the end.
// There is no running max and hence no rescaling of acc: the accumulator stays in
// tensor memory for the whole KV loop and is read exactly once, in the epilogue.
//
// A work item is two 128-row query tiles of one (batch, head) and all KV blocks of 128 rows
// (or one KV split of them). attend_persistent_kernel runs one CTA per SM over many items;
// attend_kernel runs one item per CTA (kept for the TMA-staged gathering epilogue, which
// borrows the Q buffers). Warp roles (576 threads, 1 CTA per SM):
//   warp 0       TMA producer: the item's Q tiles, then the K/V ring in stages -- stage j holds
//                V_{j-1} and K_j in a pair of 32 KB slots, two pairs -- so that the issuer waits
//                once per KV block; every fill waits on its buffer's empty barrier (one
//                completion per fill)
//   warp 1       TMEM allocator + UMMA issuer
//   warps 2-17   softmax: 8 warps per query tile, two per TMEM lane quadrant, each owning 64 of
//                the 128 columns of its 32 rows: exp + bf16 round, P written back to TMEM in two
//                32-column chunks (each handed to the issuer with one arrival per warp), row
//                sums; then the epilogue O / l -> bf16 -> global (or fp32 partials for a split).
//                One of them also releases ring stages and Q as it sees the commits (see
//                release_after_s).
// The producer and issuer warps run converged: all 32 lanes walk the loop and wait on the
// barriers with one warp-wide vote per wait; lane 0 issues the TMA loads and elect.sync picks
// the lane that issues each UMMA and commit.
// TMEM (512 columns x 128 lanes, fp32): S_t at columns [128t, 128t+128) for t = 0, 1, with
// P_t (bf16, two per column) written over the first 64 of them; O_t at [256+128t, ...).
// Per KV block the issuer runs, in order:
//   PV_0(j) [needs P_0(j)], S_0(j+1), PV_1(j) [needs P_1(j)], S_1(j+1)
// so one tile's exp overlaps the other tile's two GEMMs (the fixed order keeps the two tiles
// half a period apart). UMMAs from one thread execute in issue order, which is what makes
// writing S_t(j+1) over P_t(j) safe.
// Shared-memory operands use the 128-byte swizzle written by TMA: Q and K are K-major
// (head dim contiguous), V is the MN-major B operand of P.V (head dim contiguous).
// No TMA multicast is used anywhere.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "flicker_b200.h"
#include "attend_schedule.cuh"
#include "ptx.cuh"
#include "quotient.cuh"

namespace flk {

namespace {

constexpr int kTile = 128;                 // query rows per tile, KV rows per block
constexpr int kDim = 128;                  // head dim
constexpr int kSlots = 4;                  // K/V ring slots of 32 KB, in kStages pairs
constexpr int kStages = 2;                 // ring stages: V_{j-1} + K_j each; 2 blocks of lookahead
constexpr int kTileBytes = kTile * kDim * 2;  // 32 KB: one bf16 128 x 128 tile
constexpr int kHalfBytes = kTileBytes / 2;    // one 64-column TMA box (128 B rows)
constexpr int kSoftmaxWarps = 8;           // per query tile: 2 per TMEM lane quadrant
constexpr int kThreads = 32 * (2 + 2 * kSoftmaxWarps);
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

constexpr uint32_t kIdescQK = umma_idesc_bf16_f32(128, 128, false);
constexpr uint32_t kIdescPV = umma_idesc_bf16_f32(128, 128, true);

struct alignas(1024) Smem {
  uint8_t q[2][kTileBytes];
  uint8_t kv[kSlots][kTileBytes];
  uint64_t q_full;
  uint64_t kv_full[kStages];
  // Buffer releases, one arrival (one completion) per fill, so a fill waits for the completion
  // of the fill before it: made by the first softmax warp of the item's last query tile as soon
  // as it has seen the commit that covers the buffer's last readers (see release_after_s).
  uint64_t kv_empty[kStages];
  uint64_t q_empty;  // persistent form: the Q tiles of an item, after its last S
  uint64_t s_full[2];
  uint64_t p_part[2][2];  // [tile][column chunk]: P chunk c of every softmax warp of the tile is in TMEM
  uint64_t o_full[2];
  uint64_t drain;
  // [item parity][tile][column half][row]: row sums of the two column halves. Two copies, so that
  // a persistent CTA's warp writing the next item's sum cannot overtake its partner warp's read
  // of the current one.
  float l_part[2][2][2][kTile];
  uint32_t tmem_base;
  int abort;
};

// Where the bf16 output rows go. Head-major [B, H, S, 128] (kernels.attend), or heads merged into
// [B, S, H_out * 128] rows (merge_heads) with this call's head h at position h0 + h, written
// into each of the n_out buffers: one buffer normally; this GPU's and every peer's output when a
// head-sharded call gathers its heads by storing them straight into the peers' memory. With
// `multicast`, o[0] is an NVLink multicast address bound to every rank's output buffer: each
// 16-byte store is a multimem.st, which the NVSwitch replicates into all of them, so a row
// leaves this GPU once however many ranks receive it.
constexpr int kMaxOuts = 8;
struct OutLayout {
  int merged;
  int H;      // heads of this call
  int H_out;  // heads per merged output row
  int h0;     // first head of this call within a merged row
  int n_out;
  int multicast;
  uint16_t* o[kMaxOuts];
};

// One 16-byte store through a multicast address (every GPU bound to it receives the bytes).
__device__ __forceinline__ void multimem_st16(void* addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

struct Params {
  int S;          // sequence length (multiple of 128)
  int n_tiles;    // S / 128
  int BH;         // batch x heads
  int n_pairs;    // (n_tiles + 1) / 2 query-tile pairs per (batch, head)
  // Work units (AttendSchedule): items [0, n_full) whole, then n_a items split s_a ways over KV,
  // then the remaining items split s_b ways, split index fastest. A whole item's CTA normalises
  // and writes o itself; a piece of a split item writes partials. n_units units in all.
  int n_full, n_a, s_a, s_b;
  int n_units;
  // Partial rows: items split s_a ways own output rows [pa0, pa1), those split s_b ways
  // [pa1, pb1); partial row (slot) of query row r in piece i: tier A (r - pa0) + i (pa1 - pa0),
  // tier B s_a (pa1 - pa0) + (r - pa1) + i (pb1 - pa1).
  long long pa0, pa1, pb1;
  OutLayout out;  // bf16 output
  // When a merged output goes to several buffers (a head-sharded call storing into its peers'
  // outputs) and the CTA writes o itself: one TMA map per buffer over [B*S, H_out*128] bf16,
  // 64-column x 32-row boxes with the 128-byte swizzle, so each warp's block leaves as one tile.
  int tma_out;
  // When a merged output goes through a multicast address and the CTA writes o itself: the
  // 32 x 64 block of each softmax warp is staged in shared memory as for tma_out, then stored by
  // multimem.st in whole 128-byte row pieces (8 lanes per row), which NVLink carries as full lines.
  int stage_mc;
  CUtensorMap out_maps[kMaxOuts];
  float* acc;     // split items: [partial rows, 128] fp32 un-normalised partial P.V
  float* lsum;    // split items: [partial rows] fp32 partial row sums
  int* status;    // device status word
};

// One work unit: query tiles [t0, t0 + nt) of (batch, head) bh against KV blocks [kv0, kv0 + n_kv),
// piece `split` of `splits` (splits == 1: a whole item). A piece's partial row for query row
// `grow` is pbase + grow.
struct Item {
  int bh, t0, nt, split, splits, kv0, n_kv;
  long long pbase;
};

__device__ __forceinline__ Item decode_item(const Params& p, int w) {
  Item it;
  int item;
  if (w < p.n_full) {
    item = w;
    it.split = 0;
    it.splits = 1;
    it.pbase = 0;
  } else if (w - p.n_full < p.n_a * p.s_a) {
    const int u = w - p.n_full;
    item = p.n_full + u / p.s_a;
    it.split = u % p.s_a;
    it.splits = p.s_a;
    it.pbase = it.split * (p.pa1 - p.pa0) - p.pa0;
  } else {
    const int u = w - p.n_full - p.n_a * p.s_a;
    item = p.n_full + p.n_a + u / p.s_b;
    it.split = u % p.s_b;
    it.splits = p.s_b;
    it.pbase = p.s_a * (p.pa1 - p.pa0) + it.split * (p.pb1 - p.pa1) - p.pa1;
  }
  const int pair = item % p.n_pairs;
  it.bh = item / p.n_pairs;
  it.t0 = pair * 2;
  it.nt = min(2, p.n_tiles - it.t0);
  it.kv0 = static_cast<int>(static_cast<long long>(p.n_tiles) * it.split / it.splits);
  it.n_kv = static_cast<int>(static_cast<long long>(p.n_tiles) * (it.split + 1) / it.splits) - it.kv0;
  return it;
}

__device__ __forceinline__ Smem* smem_ptr(uint8_t* raw) {
  const uintptr_t a = (reinterpret_cast<uintptr_t>(raw) + 1023) & ~static_cast<uintptr_t>(1023);
  return reinterpret_cast<Smem*>(a);
}

// exp of one 32-column chunk of a row of S -> 16 packed bf16x2 words of P. One pair in
// kPolyEvery goes through the FMA-pipe polynomial, the rest through MUFU.EX2, so the SFU is
// not the only unit producing exponentials.
constexpr int kPolyEvery = 4;
__device__ __forceinline__ void exp_chunk(const uint32_t (&r)[32], uint32_t (&pk)[16]) {
  const float2 log2e = make_float2(kLog2e, kLog2e);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 x = __fmul2_rn(make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), log2e);
    float2 e;
    if (i % kPolyEvery == kPolyEvery - 1) {
      e = exp2_poly2(x);
    } else {
      e.x = ex2_approx(x.x);
      e.y = ex2_approx(x.y);
    }
    pk[i] = pack_bf16x2(e.x, e.y);
  }
}

// Row sum of the bf16-ROUNDED P values of one chunk (kernels.py:124-125 sums fp32(bf16(exp(s)))),
// done after P is in TMEM and handed to the issuer, i.e. off the softmax -> P.V critical path.
// l += fp32(v) for both bf16 halves of a packed word, one mixed-precision add each (PTX
// add.rn.f32.bf16: the bf16 operand widens exactly, one rounding), i.e. the same arithmetic as
// widening the halves and adding them, in fewer instructions.
__device__ __forceinline__ void add_bf16_halves(uint32_t w, float& lo_acc, float& hi_acc) {
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "add.rn.f32.bf16 %0, lo, %0;\n\tadd.rn.f32.bf16 %1, hi, %1;\n\t}"
      : "+f"(lo_acc), "+f"(hi_acc)
      : "r"(w));
}

__device__ __forceinline__ void row_sum_chunk(const uint32_t (&pk)[16], float2& l0, float2& l1) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i & 1)
      add_bf16_halves(pk[i], l1.x, l1.y);
    else
      add_bf16_halves(pk[i], l0.x, l0.y);
  }
}

// TMEM column (within a tile's S region) of the packed P words for KV rows [16kc, 16kc+16):
// the softmax warp of column half h writes the P of S columns [64h, 64h+64) packed into
// columns [64h, 64h+32), i.e. over S columns it has already read.
__device__ __forceinline__ uint32_t p_col(int kc) { return static_cast<uint32_t>((kc >> 2) * 64 + (kc & 3) * 8); }

// Buffer releases, made by lane 0 of the first softmax warp of the item's last query tile (nt-1)
// once it has seen the commit on s_full[nt-1] that follows S_{nt-1}(j) (right after its own P
// chunk-0 hand-over, which must not wait for them). A commit tracks
// every UMMA issued before it and the issuer runs tile 0's UMMAs of a block before tile 1's, so
// that commit covers every tile's S(j) and every tile's P.V(j-1), issued before S(j). Those are
// the two readers of ring stage `stage` (V of the block before and K_j), which is therefore
// free; when j is the item's last block, so are the Q tiles.
__device__ __forceinline__ void release_after_s(Smem& sm, uint32_t stage, bool last_block) {
  mbar_arrive(&sm.kv_empty[stage % 2]);
  if (last_block) mbar_arrive(&sm.q_empty);
}

// Issues ring stage G (and advances G): V rows `v_row` into the pair's V slot and K rows `k_row`
// into its K slot (a negative row leaves that half out), once the stage's previous fill has been
// released. The whole producer warp calls it; lane 0 (`leader`) issues the copies.
__device__ __forceinline__ bool issue_kv_stage(Smem& sm, const CUtensorMap* tm_k, const CUtensorMap* tm_v, uint32_t& G,
                                               int v_row, int k_row, bool leader, volatile int* abort, int* status) {
  const uint32_t sp = G % kStages, use = G / kStages;
  if (use > 0 && !mbar_wait_warp(&sm.kv_empty[sp], (use - 1) & 1, abort, status)) return false;
  if (leader) {
    mbar_arrive_expect_tx(&sm.kv_full[sp], (v_row >= 0 ? kTileBytes : 0) + (k_row >= 0 ? kTileBytes : 0));
    if (v_row >= 0) {
      tma_load_2d(sm.kv[2 * sp], tm_v, 0, v_row, &sm.kv_full[sp]);
      tma_load_2d(sm.kv[2 * sp] + kHalfBytes, tm_v, 64, v_row, &sm.kv_full[sp]);
    }
    if (k_row >= 0) {
      tma_load_2d(sm.kv[2 * sp + 1], tm_k, 0, k_row, &sm.kv_full[sp]);
      tma_load_2d(sm.kv[2 * sp + 1] + kHalfBytes, tm_k, 64, k_row, &sm.kv_full[sp]);
    }
  }
  __syncwarp();
  ++G;
  return true;
}

// Never leave with a copy in flight: wait (bounded) for the last of the G stage fills on each pair.
__device__ __forceinline__ void drain_kv_stages(Smem& sm, uint32_t G, int* status) {
  for (uint32_t sp = 0; sp < kStages; ++sp) {
    const uint32_t fills = G > sp ? (G - sp + kStages - 1) / kStages : 0;
    if (fills > 0) mbar_drain(&sm.kv_full[sp], (fills - 1) & 1, status);
  }
}

// 128-column output row that holds query row `grow` (= (b * H + h) * S + s): itself in the
// head-major layout; (b * S + s) * H_out + h0 + h when heads are merged (modules.merge_heads,
// src/flicker/modules.py:63-65).
__device__ __forceinline__ size_t out_row(size_t grow, int S, const OutLayout& L) {
  if (!L.merged) return grow;
  const size_t bh = grow / S, s = grow - bh * S;
  const size_t b = bh / L.H, h = bh - b * L.H;
  return (b * S + s) * L.H_out + L.h0 + h;
}

// Stores 16 packed bf16x2 words (32 columns) at element offset `off` of every output buffer.
// A thread that stored into several buffers (peers' among them) ends its epilogue with one
// system-scope fence, so that its stores are visible before whatever synchronisation the
// caller performs after the kernel.
__device__ __forceinline__ void store_out(const OutLayout& L, size_t off, const uint32_t (&pk)[16]) {
  if (L.multicast) {
    uint4* dst = reinterpret_cast<uint4*>(L.o[0] + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) multimem_st16(dst + i, make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]));
    return;
  }
#pragma unroll 1
  for (int d = 0; d < L.n_out; ++d) {
    uint4* dst = reinterpret_cast<uint4*>(L.o[d] + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
  }
}

// Tiled TMA store of a shared-memory box into global memory (async proxy, bulk async-group).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}

// Epilogue of one softmax warp: its 32 rows x 64 columns of O from TMEM, either normalised and
// rounded to bf16 (o = bf16(acc / l), kernels.py:130, the quotient correctly rounded through one
// reciprocal per row) or, for a piece of a split item (splits > 1), the fp32 partials in partial
// row pbase + grow.
// Kept out of line so that this once-per-CTA code sits apart from the KV loop's code. `stage`
// is this warp's 4 KB of shared memory (1024-byte aligned, free once the tile's MMAs are done).
__device__ __noinline__ void store_rows(const Params& p, uint32_t o_addr, size_t grow, int half, int splits,
                                        long long pbase, float l, uint8_t* stage) {
  const float rl = __frcp_rn(l);
  if (splits == 1 && (p.tma_out || p.stage_mc)) {
    // Stage the 32 x 64 block in the 128-byte-swizzled layout the maps expect (16-byte unit j of
    // row r at position j ^ (r & 7): conflict-free), then one lane stores it to every buffer
    // (tma_out) or the warp stores it through the multicast address (stage_mc).
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(o_addr + c * 32, r);
      tmem_wait_ld(r);
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        pk[i] = pack_bf16x2(quotient_rn(__uint_as_float(r[2 * i]), l, rl),
                            quotient_rn(__uint_as_float(r[2 * i + 1]), l, rl));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = c * 4 + i;
        *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
            make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
    }
    if (p.stage_mc) {
      __syncwarp();
      const size_t first = grow - lane;  // the block's first query row
      const int u = lane & 7;
#pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        const int r = i * 4 + (lane >> 3);
        const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128 + ((u ^ (r & 7)) << 4));
        multimem_st16(p.out.o[0] + out_row(first + r, p.S, p.out) * kDim + half * 64 + u * 8, v);
      }
      __threadfence_system();
      __syncwarp();
      return;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {  // grow is the block's first query row here
      const size_t bh = grow / p.S, s0 = grow - bh * p.S;
      const size_t b = bh / p.out.H, h = bh - b * p.out.H;
      const int x = static_cast<int>((p.out.h0 + h) * kDim + half * 64);
      const int y = static_cast<int>(b * p.S + s0);
#pragma unroll 1
      for (int d = 0; d < p.out.n_out; ++d) tma_store_2d(&p.out_maps[d], x, y, stage);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      __threadfence_system();
    }
    __syncwarp();
  } else if (splits == 1) {
    const size_t orow = out_row(grow, p.S, p.out) * kDim + half * 64;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(o_addr + c * 32, r);
      tmem_wait_ld(r);
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        pk[i] = pack_bf16x2(quotient_rn(__uint_as_float(r[2 * i]), l, rl),
                            quotient_rn(__uint_as_float(r[2 * i + 1]), l, rl));
      store_out(p.out, orow + c * 32, pk);
    }
    if (p.out.n_out > 1 || p.out.multicast) __threadfence_system();
  } else {
    // Partial result of this piece: un-normalised fp32 accumulator and row sum.
    const size_t slot = static_cast<size_t>(pbase + static_cast<long long>(grow));
    float* arow = p.acc + slot * kDim + half * 64;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(o_addr + c * 32, r);
      tmem_wait_ld(r);
      uint4* dst = reinterpret_cast<uint4*>(arow + c * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
    }
    if (half == 0) p.lsum[slot] = l;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    attend_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *smem_ptr(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool leader = lane == 0;  // the one lane of a converged warp that issues TMA / UMMA / commits

  // One work unit per CTA (blockIdx.x in the unit order of the schedule): query tiles [t0, t0 + nt)
  // of (batch, head) bh against KV blocks [kv0, kv0 + n_kv). Without a running max the pieces'
  // (acc, l) of a split item simply add.
  const Item it = decode_item(p, blockIdx.x);
  const int bh = it.bh, t0 = it.t0, nt = it.nt, kv0 = it.kv0, n_kv = it.n_kv;
  const int row_base = bh * p.S;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    mbar_init(&sm.q_empty, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_part[t][0], kSoftmaxWarps);  // one arrival per softmax warp
      mbar_init(&sm.p_part[t][1], kSoftmaxWarps);
      mbar_init(&sm.o_full[t], 1);
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
  // Launched as a programmatic dependent of the previous kernel in the stream (normally qk_prep):
  // the set-up above overlaps that kernel's tail, and no thread touches global memory before the
  // previous kernel has completed and its writes are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (whole warp, lane 0 issues)
    if (leader) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&sm.q_full, nt * kTileBytes);
      for (int t = 0; t < nt; ++t) {
        const int row = row_base + (t0 + t) * kTile;
        tma_load_2d(sm.q[t], &tm_q, 0, row, &sm.q_full);
        tma_load_2d(sm.q[t] + kHalfBytes, &tm_q, 64, row, &sm.q_full);
      }
    }
    // The K/V ring runs in stages: stage j holds V_{j-1} and K_j (stage 0 only K_0, stage n_kv only
    // the last V) in slot pair j % 2 (V in slot 2(j % 2), K in slot 2(j % 2) + 1), one full and one
    // empty barrier per pair. Fill f of a pair waits for completion #(f-1) of its kv_empty, which
    // cannot complete again before this fill has landed and been read, so the parity wait always
    // refers to its current or its previous phase, however late this warp runs.
    uint32_t G = 0;
    bool ok = true;
    auto issue_stage = [&](int v_row, int k_row) {
      return issue_kv_stage(sm, &tm_k, &tm_v, G, v_row, k_row, leader, abort, p.status);
    };
    for (int j = 0; ok && j <= n_kv; ++j)
      ok = issue_stage(j > 0 ? row_base + (kv0 + j - 1) * kTile : -1, j < n_kv ? row_base + (kv0 + j) * kTile : -1);
    // Never leave with a copy in flight: wait (bounded) for the last fill of Q and of both pairs.
    mbar_drain(&sm.q_full, 0, p.status);
    drain_kv_stages(sm, G, p.status);
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (whole warp, elect.sync issues)
    auto wait = [&](uint64_t* bar, uint32_t parity) { return mbar_wait_warp(bar, parity, abort, p.status); };
    auto stage_ready = [&](int st) { return wait(&sm.kv_full[st % 2], (st / 2) & 1); };
    // Descriptor low words: Q tile t, K-major ring slot, MN-major (V) ring slot; chunk kc, slot and
    // tile offsets are added to the start field (units of 16 bytes).
    const uint32_t q_lo = umma_desc_lo(smem_u32(sm.q[0]), 16);
    const uint32_t k_lo = umma_desc_lo(smem_u32(sm.kv[0]), 16);
    const uint32_t v_lo = umma_desc_lo(smem_u32(sm.kv[0]), kHalfBytes);
    constexpr uint32_t kTile16 = kTileBytes >> 4;
    auto qk = [&](int t, int slot) {  // S_t = Q_t K^T from ring slot `slot`
#pragma unroll
      for (int kc = 0; kc < 8; ++kc) {
        const uint32_t kcoff = (kc >> 2) * (kHalfBytes >> 4) + (kc & 3) * 2;
        umma_ss_warp_lo(tmem + t * 128, q_lo + t * kTile16 + kcoff, k_lo + slot * kTile16 + kcoff, kIdescQK,
                        kc > 0);
      }
    };
    bool ok = wait(&sm.q_full, 0) && stage_ready(0);
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (t < nt) {
          qk(t, 1);  // S_t(0) = Q_t K_0^T (stage 0, K slot of pair 0)
          tc_commit_warp(&sm.s_full[t]);
        }
      }
    }
    for (int j = 0; ok && j < n_kv; ++j) {
      const int st = j + 1;  // V_j and K_{j+1}
      const bool last = (j == n_kv - 1);
      ok = stage_ready(st);
      if (!ok) break;
      const uint32_t vslot = v_lo + (2 * (st % 2)) * kTile16;
      const int kslot = 2 * (st % 2) + 1;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (t >= nt) break;
        // P.V in two steps: K-chunks {0,1,4,5} (P chunk 0 of both column halves) as soon as every
        // softmax warp has written its first chunk, then {2,3,6,7}.
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          ok = wait(&sm.p_part[t][c], j & 1);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int kc = (i & 1) + 2 * c + 4 * (i >> 1);  // kv rows [16kc, 16kc+16)
            umma_ts_warp_lo(tmem + 256 + t * 128, tmem + t * 128 + p_col(kc), vslot + kc * (2048 >> 4), kIdescPV,
                            (j > 0 || c > 0 || i > 0) ? 1u : 0u);
          }
        }
        if (!ok) break;
        if (last) {
          tc_commit_warp(&sm.o_full[t]);
          continue;
        }
        qk(t, kslot);  // S_t(j+1) = Q_t K_{j+1}^T, written over P_t(j) after the P.V above has read it
        tc_commit_warp(&sm.s_full[t]);
      }
      if (!ok) break;
    }
    // Drain: every UMMA issued above has completed before TMEM is released.
    tc_commit_warp(&sm.drain);
    mbar_drain(&sm.drain, 0, p.status);
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int sw = warp - 2;                  // softmax warp index 0 .. 2*kSoftmaxWarps-1
    const int t = sw / kSoftmaxWarps;         // query tile
    const int half = (sw % kSoftmaxWarps) / 4;  // column half of S / O this warp owns
    const int quad = warp & 3;                // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    if (t < nt) {
      const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
      const uint32_t s_addr = tmem + lane_off + t * 128 + half * 64;
      const bool releaser = t == nt - 1 && sw % kSoftmaxWarps == 0 && lane == 0;
      float2 l0 = make_float2(0.f, 0.f), l1 = make_float2(0.f, 0.f);
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        // Warp-uniform outcome: the tcgen05.ld/st below are .sync.aligned.
        ok = mbar_wait_warp(&sm.s_full[t], j & 1, abort, p.status);
        if (!ok) break;
        tc_fence_after();
        // Two 32-column chunks of this row's half of S; chunk 1 is loading while chunk 0 is
        // exponentiated, and each chunk's P is handed to the issuer as soon as it is in TMEM. The
        // hand-over of chunk 0 waits for nothing else -- not for chunk 1's load (no UMMA touches
        // those columns before chunk 1's own hand-over), nor for the releaser's arrivals, which
        // come after it (a release can be late, never early): the tile's slowest warp sets when
        // the issuer starts P.V, so nothing may sit in front of it (2697-2700 cycles per block
        // against 2765-2770 with the release and the wait ahead of the hand-over).
        uint32_t ra[32], rb[32], pk0[16], pk1[16];
        tmem_ld_32x32b_x32(s_addr, ra);
        tmem_wait_ld(ra);
        tmem_ld_32x32b_x32(s_addr + 32, rb);
        exp_chunk(ra, pk0);
        tmem_st_32x32b_x16(s_addr, pk0);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_part[t][0]);
        if (releaser) release_after_s(sm, j, j == n_kv - 1);
        tmem_wait_ld(rb);
        exp_chunk(rb, pk1);
        tmem_st_32x32b_x16(s_addr + 16, pk1);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_part[t][1]);
        row_sum_chunk(pk0, l0, l1);
        row_sum_chunk(pk1, l0, l1);
      }
      // Row sum over all 128 KV columns: this warp's half plus the other half's partial.
      sm.l_part[0][t][half][row] = (l0.x + l0.y) + (l1.x + l1.y);
      named_barrier_sync(1 + t, 32 * kSoftmaxWarps);
      const float l = sm.l_part[0][t][0][row] + sm.l_part[0][t][1][row];
      if (ok) ok = mbar_wait_warp(&sm.o_full[t], 0, abort, p.status);
      if (ok) {
        tc_fence_after();
        const uint32_t o_addr = tmem + lane_off + 256 + t * 128 + half * 64;
        const size_t grow = static_cast<size_t>(row_base) + (t0 + t) * kTile + row;  // global query row
        store_rows(p, o_addr, grow, half, it.splits, it.pbase, l, sm.q[t] + (sw % kSoftmaxWarps) * 4096);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------
// Persistent form: one CTA per SM walks work units w = blockIdx.x, blockIdx.x + gridDim.x, ...,
// a unit being what one CTA of attend_kernel does (two query tiles of one (batch, head), a whole
// item or one piece of a split one). The barriers keep counting across items, so the next item's Q and K/V loads and its
// first S = Q K^T run while the softmax warps are still in the current item's epilogue, instead
// of after the CTA has exited and a new one has started, allocated TMEM and loaded its tiles.
// Ordering across items, beyond that of attend_kernel:
//   * S_t(0) of item i+1 overwrites tile t's S/P columns after the last P.V of item i, which the
//     issuer issued after every softmax warp of tile t had handed over its last P: safe.
//   * P.V_t(0) of item i+1 overwrites O_t; the softmax warps of tile t hand over P_t(0) of item
//     i+1 only after they have read O_t of item i (tcgen05.ld + wait), so the issuer's wait for
//     that P orders the overwrite after the read.
//   * Q of item i+1 is loaded once S(last) of item i has completed (q_empty, committed right
//     after that S; no later UMMA of item i reads Q).
// The K/V ring stages count blocks over all of the CTA's items: stage G holds V of its block G-1
// and K of its block G, so an item's last V shares a stage with the next item's first K, and the
// release after S(0) of the next item covers both (the last P.V of an item is issued before the
// next item's S(0)). Block j needs exactly V_j and K_{j+1}, one stage, so the issuer waits once
// per block instead of twice (separate K and V slots): 2776-2778 cycles per block against
// 2881-2886 (CTA 0, clock64, bench loop), bit-identical output; with the softmax's chunk-0
// hand-over ahead of the release (see attend_kernel), 2697-2700.
// Used when the CTA itself writes plain (not TMA-staged) output: the TMA-staged epilogue borrows
// the Q buffers, which this form refills early.
__global__ void __launch_bounds__(kThreads, 1)
    attend_persistent_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *smem_ptr(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool leader = lane == 0;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    mbar_init(&sm.q_empty, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_part[t][0], kSoftmaxWarps);
      mbar_init(&sm.p_part[t][1], kSoftmaxWarps);
      mbar_init(&sm.o_full[t], 1);
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
  asm volatile("griddepcontrol.wait;" ::: "memory");
  volatile int* abort = &sm.abort;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (whole warp, lane 0 issues)
    if (leader) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    // Fill f of a buffer (the Q tiles, or a ring stage) waits for completion #(f-1) of its empty
    // barrier; that barrier cannot complete again before fill f has landed and been read, so the
    // parity wait always refers to its current or its previous phase.
    // Stage G of the ring holds V of the CTA's block G-1 and K of its block G (blocks counted
    // over all of the CTA's items, so an item's last V shares a stage with the next item's first K);
    // it fills the slot pair G % 2 (V in slot 2(G % 2), K in slot 2(G % 2) + 1). An item's first
    // stage goes out before the wait for the Q buffers, so that last V never waits behind Q.
    uint32_t G = 0, q_fills = 0;  // stages and Q loads issued
    bool ok = true;
    auto issue_stage = [&](int v_row, int k_row) {
      return issue_kv_stage(sm, &tm_k, &tm_v, G, v_row, k_row, leader, abort, p.status);
    };
    int pending_v = -1;  // row of the previous item's last V, loaded with this item's first K
    for (int w = blockIdx.x; ok && w < p.n_units; w += gridDim.x) {
      const Item it = decode_item(p, w);
      const int row_base = it.bh * p.S;
      ok = issue_stage(pending_v, row_base + it.kv0 * kTile);
      if (!ok) break;
      if (q_fills > 0 && !mbar_wait_warp(&sm.q_empty, (q_fills - 1) & 1, abort, p.status)) {
        ok = false;
        break;
      }
      if (leader) {
        mbar_arrive_expect_tx(&sm.q_full, it.nt * kTileBytes);
        for (int t = 0; t < it.nt; ++t) {
          const int row = row_base + (it.t0 + t) * kTile;
          tma_load_2d(sm.q[t], &tm_q, 0, row, &sm.q_full);
          tma_load_2d(sm.q[t] + kHalfBytes, &tm_q, 64, row, &sm.q_full);
        }
      }
      __syncwarp();
      ++q_fills;
      for (int j = 0; ok && j + 1 < it.n_kv; ++j)
        ok = issue_stage(row_base + (it.kv0 + j) * kTile, row_base + (it.kv0 + j + 1) * kTile);
      pending_v = row_base + (it.kv0 + it.n_kv - 1) * kTile;
    }
    if (ok && pending_v >= 0) issue_stage(pending_v, -1);  // the last V, alone
    // Never leave with a copy in flight: wait (bounded) for the last fill of Q and of both stages.
    if (q_fills > 0) mbar_drain(&sm.q_full, (q_fills - 1) & 1, p.status);
    drain_kv_stages(sm, G, p.status);
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (whole warp, elect.sync issues)
    auto wait = [&](uint64_t* bar, uint32_t parity) { return mbar_wait_warp(bar, parity, abort, p.status); };
    const uint32_t q_lo = umma_desc_lo(smem_u32(sm.q[0]), 16);
    const uint32_t k_lo = umma_desc_lo(smem_u32(sm.kv[0]), 16);
    const uint32_t v_lo = umma_desc_lo(smem_u32(sm.kv[0]), kHalfBytes);
    constexpr uint32_t kTile16 = kTileBytes >> 4;
    auto qk = [&](int t, int slot) {
#pragma unroll
      for (int kc = 0; kc < 8; ++kc) {
        const uint32_t kcoff = (kc >> 2) * (kHalfBytes >> 4) + (kc & 3) * 2;
        umma_ss_warp_lo(tmem + t * 128, q_lo + t * kTile16 + kcoff, k_lo + slot * kTile16 + kcoff, kIdescQK,
                        kc > 0);
      }
    };
    uint32_t b0 = 0, items = 0;     // the item's first block (= its first K's stage), items done
    uint32_t blocks[2] = {0, 0};    // KV blocks done per tile: p_part phases consumed
    auto stage_ready = [&](uint32_t G) { return wait(&sm.kv_full[G % 2], (G / 2) & 1); };
    bool ok = true;
    for (int w = blockIdx.x; ok && w < p.n_units; w += gridDim.x) {
      const Item it = decode_item(p, w);
      // stage b0 (this item's first K) was waited for with the previous item's last V
      ok = wait(&sm.q_full, items & 1) && (b0 > 0 || stage_ready(0));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (t < it.nt) {
          qk(t, 2 * (b0 % 2) + 1);
          tc_commit_warp(&sm.s_full[t]);
        }
      }
      for (int j = 0; ok && j < it.n_kv; ++j) {
        const uint32_t st = b0 + j + 1;  // V_j and K_{j+1} (or the next item's first K)
        const bool last = (j == it.n_kv - 1);
        ok = stage_ready(st);
        if (!ok) break;
        const uint32_t vslot = v_lo + (2 * (st % 2)) * kTile16;
        const int kslot = 2 * (st % 2) + 1;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (t >= it.nt) break;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            ok = wait(&sm.p_part[t][c], (blocks[t] + j) & 1);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int kc = (i & 1) + 2 * c + 4 * (i >> 1);
              umma_ts_warp_lo(tmem + 256 + t * 128, tmem + t * 128 + p_col(kc), vslot + kc * (2048 >> 4), kIdescPV,
                              (j > 0 || c > 0 || i > 0) ? 1u : 0u);
            }
          }
          if (!ok) break;
          if (last) {
            tc_commit_warp(&sm.o_full[t]);
            continue;
          }
          qk(t, kslot);
          tc_commit_warp(&sm.s_full[t]);
        }
      }
      for (int t = 0; t < it.nt; ++t) blocks[t] += it.n_kv;
      b0 += it.n_kv;
      ++items;
    }
    tc_commit_warp(&sm.drain);
    mbar_drain(&sm.drain, 0, p.status);
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int sw = warp - 2;
    const int t = sw / kSoftmaxWarps;
    const int half = (sw % kSoftmaxWarps) / 4;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + t * 128 + half * 64;
    const uint32_t o_addr = tmem + lane_off + 256 + t * 128 + half * 64;
    uint32_t s_seen = 0, o_seen = 0, items = 0;  // s_full[t] / o_full[t] completions consumed, items of tile t
    uint32_t g0 = 0;                             // the item's first block (its first K's stage)
    // Once a wait has failed the warp does no more work, but it still meets its tile's named
    // barrier once per item, as its partner warps (which may not have seen the failure yet) do.
    bool ok = true;
    for (int w = blockIdx.x; w < p.n_units; w += gridDim.x) {
      const Item it = decode_item(p, w);
      const uint32_t item_g0 = g0;
      g0 += it.n_kv;
      if (t >= it.nt) continue;
      const bool releaser = t == it.nt - 1 && sw % kSoftmaxWarps == 0 && lane == 0;
      float2 l0 = make_float2(0.f, 0.f), l1 = make_float2(0.f, 0.f);
      for (int j = 0; ok && j < it.n_kv; ++j, ++s_seen) {
        ok = mbar_wait_warp(&sm.s_full[t], s_seen & 1, abort, p.status);
        if (!ok) break;
        tc_fence_after();
        uint32_t ra[32], rb[32], pk0[16], pk1[16];  // same order as attend_kernel (hand-over first)
        tmem_ld_32x32b_x32(s_addr, ra);
        tmem_wait_ld(ra);
        tmem_ld_32x32b_x32(s_addr + 32, rb);
        exp_chunk(ra, pk0);
        tmem_st_32x32b_x16(s_addr, pk0);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_part[t][0]);
        if (releaser) release_after_s(sm, item_g0 + j, j == it.n_kv - 1);
        tmem_wait_ld(rb);
        exp_chunk(rb, pk1);
        tmem_st_32x32b_x16(s_addr + 16, pk1);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.p_part[t][1]);
        row_sum_chunk(pk0, l0, l1);
        row_sum_chunk(pk1, l0, l1);
      }
      const int lb = items & 1;
      sm.l_part[lb][t][half][row] = (l0.x + l0.y) + (l1.x + l1.y);
      named_barrier_sync(1 + t, 32 * kSoftmaxWarps);
      const float l = sm.l_part[lb][t][0][row] + sm.l_part[lb][t][1][row];
      if (ok) ok = mbar_wait_warp(&sm.o_full[t], o_seen & 1, abort, p.status);
      ++o_seen;
      ++items;
      if (ok) {
        tc_fence_after();
        const size_t grow = static_cast<size_t>(it.bh) * p.S + (it.t0 + t) * kTile + row;
        store_rows(p, o_addr, grow, half, it.splits, it.pbase, l, nullptr);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// o = bf16(sum_i acc_i / sum_i l_i) over the pieces of the split items; one thread per 8 output
// columns of query rows [pa0, pb1) (rows [pa0, pa1) split s_a ways, [pa1, pb1) s_b ways), the
// pieces added in order.
struct CombineParams {
  long long pa0, pa1, pb1;
  int s_a, s_b, S;
};
__global__ void __launch_bounds__(256) combine_splits_kernel(const float* __restrict__ acc,
                                                             const float* __restrict__ lsum,
                                                             const __grid_constant__ CombineParams c,
                                                             const __grid_constant__ OutLayout L) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= (c.pb1 - c.pa0) * (kDim / 8)) return;
  const long long row = c.pa0 + idx / (kDim / 8);
  const int col = static_cast<int>(idx % (kDim / 8)) * 8;
  const bool tier_a = row < c.pa1;
  const int n = tier_a ? c.s_a : c.s_b;
  const long long first = tier_a ? row - c.pa0 : c.s_a * (c.pa1 - c.pa0) + (row - c.pa1);
  const long long stride = tier_a ? c.pa1 - c.pa0 : c.pb1 - c.pa1;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float l = 0.f;
  // Up to four pieces' loads in flight at once (written by the previous kernel, read-only here),
  // then added in piece order, as one piece at a time would.
  constexpr int kBatch = 4;
  for (int s0 = 0; s0 < n; s0 += kBatch) {
    float4 x[kBatch], y[kBatch];
    float ls[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (s0 + i < n) {
        const long long slot = first + (s0 + i) * stride;
        const float4* src = reinterpret_cast<const float4*>(acc + slot * kDim + col);
        x[i] = __ldg(src);
        y[i] = __ldg(src + 1);
        ls[i] = __ldg(lsum + slot);
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (s0 + i < n) {
        a[0] += x[i].x; a[1] += x[i].y; a[2] += x[i].z; a[3] += x[i].w;
        a[4] += y[i].x; a[5] += y[i].y; a[6] += y[i].z; a[7] += y[i].w;
        l += ls[i];
      }
    }
  }
  uint32_t pk[4];
  const float rl = __frcp_rn(l);
#pragma unroll
  for (int i = 0; i < 4; ++i) pk[i] = pack_bf16x2(quotient_rn(a[2 * i], l, rl), quotient_rn(a[2 * i + 1], l, rl));
  const size_t off = out_row(row, c.S, L) * kDim + col;
  if (L.multicast) {
    multimem_st16(L.o[0] + off, make_uint4(pk[0], pk[1], pk[2], pk[3]));
  } else {
#pragma unroll 1
    for (int d = 0; d < L.n_out; ++d) *reinterpret_cast<uint4*>(L.o[d] + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  if (L.n_out > 1 || L.multicast) __threadfence_system();
}

}  // namespace

// ---------------------------------------------------------------- host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
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

// [rows, 128] bf16 row-major viewed through 64-column x 128-row boxes with the 128-byte swizzle.
// Such a descriptor depends on nothing but (base, rows), so the last few are kept per host thread
// and a caller that reuses its buffers skips the driver's encoding on later calls.
struct TileMapEntry {
  const void* base;
  long long rows;
  CUtensorMap map;
};
static bool make_tile_map(CUtensorMap* map, const void* base, long long rows) {
  constexpr int kEntries = 8;
  thread_local TileMapEntry cache[kEntries] = {};
  thread_local int next = 0;
  for (const TileMapEntry& e : cache)
    if (e.base == base && e.rows == rows && base != nullptr) {
      *map = e.map;
      return true;
    }
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kDim) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kTile)};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  cache[next] = TileMapEntry{base, rows, *map};
  next = (next + 1) % kEntries;
  return true;
}

// Output map for the staged epilogue: [B*S rows, H_out*128 cols] bf16, 64 x 32 boxes, 128-byte swizzle.
static bool make_out_map(CUtensorMap* map, const void* base, long long rows, int cols) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {64, 32};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static size_t attend_smem_bytes() { return sizeof(Smem) + 1024; }
static_assert(sizeof(Smem) + 1024 <= 232448, "attend shared memory exceeds the 227 KB opt-in limit");

// First output row of item `item` (items are numbered (batch * H + head) * n_pairs + pair, each
// covering 256 consecutive query rows, or 128 for the odd last tile of a (batch, head)).
static long long item_row(int item, int n_pairs, int S) {
  return static_cast<long long>(item / n_pairs) * S + static_cast<long long>(item % n_pairs) * 2 * kTile;
}

AttendSchedule attend_unsplit(int B, int H, int S) {
  AttendSchedule sch;
  sch.n_items = static_cast<int>(std::min<long long>(INT32_MAX, static_cast<long long>(B) * H * ((S / kTile + 1) / 2)));
  sch.n_full = sch.n_items;
  return sch;
}

size_t attend_workspace_bytes(int B, int H, int S, const AttendSchedule& sch) {
  if (!sch.split()) return 0;
  const int n_pairs = (S / kTile + 1) / 2;
  const long long pa0 = item_row(sch.n_full, n_pairs, S), pa1 = item_row(sch.n_full + sch.n_a, n_pairs, S);
  const long long pb1 = static_cast<long long>(B) * H * S;
  const long long slots = sch.s_a * (pa1 - pa0) + sch.s_b * (pb1 - pa1);
  return static_cast<size_t>(slots) * (kDim + 1) * sizeof(float);
}

namespace {

// Estimated cost of a schedule, in units of one 128-row KV block of one work unit (~2700 SM
// cycles): the busiest CTA's blocks when unit u runs on CTA u % sms (the persistent kernel's
// order; the one-unit-per-CTA kernel is dispatched in the same order), plus a fixed cost per unit
// (its first S before any overlap, its epilogue; more for a piece, whose epilogue writes fp32
// partials) and per call (launch, ramp-up, drain), plus the combine pass: a launch and the
// partials' traffic (written and read back) at ~9.75 MB of HBM per block time. The constants are
// fitted to measured calls at S = 4608 and 16896 (11, 12, 13 and 3, 6, 12 heads on 148 SMs).
constexpr double kWholeBlocks = 0.5, kPieceBlocks = 2.0, kCallBlocks = 7.0, kCombineBlocks = 3.0,
                 kBytesPerBlock = 9.75e6;

double schedule_cost(const AttendSchedule& sch, int B, int H, int S, int sms) {
  const int n_tiles = S / kTile;
  const long long F = sch.n_full, A = static_cast<long long>(sch.n_a) * sch.s_a, U = sch.units();
  const double size_f = n_tiles + kWholeBlocks;
  const double size_a = (n_tiles + sch.s_a - 1) / sch.s_a + kPieceBlocks;
  const double size_b = (n_tiles + sch.s_b - 1) / sch.s_b + kPieceBlocks;
  // number of units u in [lo, hi) with u % sms == c
  auto count = [&](long long lo, long long hi, int c) -> long long {
    auto upto = [&](long long n) { return n <= c ? 0 : (n - 1 - c) / sms + 1; };  // u in [0, n)
    return hi > lo ? upto(hi) - upto(lo) : 0;
  };
  double worst = 0.0;
  for (int c = 0; c < sms && c < U; ++c)
    worst = std::max(worst, count(0, F, c) * size_f + count(F, F + A, c) * size_a + count(F + A, U, c) * size_b);
  double cost = worst + kCallBlocks;
  if (sch.split()) {
    const double slots = static_cast<double>(attend_workspace_bytes(B, H, S, sch)) / ((kDim + 1) * sizeof(float));
    const double rows = static_cast<double>(B) * H * S - item_row(sch.n_full, (n_tiles + 1) / 2, S);
    // partial rows written and read back, bf16 rows out
    cost += kCombineBlocks + (slots * (kDim + 1) * 4 * 2.0 + rows * kDim * 2) / kBytesPerBlock;
  }
  return cost;
}

}  // namespace

// The schedule for a shape on a device with `sms` SMs.
// Base rule: every item whole, unless (batch x heads x query-tile pairs) would fill at most half
// of the SMs; then every item is split evenly, into enough pieces to fill one wave.
// Tiered rule: the items that fill whole waves stay whole; of the rest, n_a are split s_a ways
// (at most one piece per SM) and the others s_b <= 16 ways (at most one more piece per SM), so the last
// wave is cut into pieces that end together instead of leaving SMs idle (216 items on 148 SMs:
// 36 + 18 blocks on the busiest SM instead of 2 x 36; measured 102 against 116 us). Taken when
// its estimated cost is at least 5 % below the base rule's.
static AttendSchedule compute_schedule(int B, int H, int S, int sms) {
  AttendSchedule base = attend_unsplit(B, H, S);
  const int n_tiles = S / kTile;
  const long long items = base.n_items;
  if (items <= 0 || sms <= 0 || n_tiles <= 0) return base;
  if (items * 2 <= sms) {
    const int s = static_cast<int>(std::min<long long>(n_tiles, std::max<long long>(1, sms / items)));
    if (s > 1) {
      base.n_full = 0;
      base.n_a = base.n_items;
      base.s_a = base.s_b = s;
    }
  }
  AttendSchedule best = base;
  const double base_cost = schedule_cost(base, B, H, S, sms);
  double best_cost = base_cost;
  const long long whole = (items / sms) * sms;  // items filling whole waves
  const long long rest = items - whole;
  for (int s_a = 2; rest > 0 && s_a <= std::min(n_tiles, 8); ++s_a) {
    AttendSchedule c;
    c.n_items = base.n_items;
    c.n_full = static_cast<int>(whole);
    c.n_a = static_cast<int>(std::min<long long>(rest, sms / s_a));
    c.s_a = s_a;
    const long long rb = rest - c.n_a;
    c.s_b = rb > 0 ? static_cast<int>(std::min<long long>({n_tiles, sms / rb, 16})) : s_a;
    if (c.n_a == 0 || c.s_b < 2 || c.units() > INT32_MAX) continue;
    const double cost = schedule_cost(c, B, H, S, sms);
    if (cost < best_cost) best = c, best_cost = cost;
  }
  return best_cost < 0.95 * base_cost ? best : base;
}

// The rule costs a few to ~20 us of host time (a scan of the CTAs per candidate); every call asks
// for it, so each host thread keeps its last few answers.
AttendSchedule attend_schedule(int B, int H, int S, int sms) {
  struct Entry {
    int B = 0, H = 0, S = -1, sms = 0;
    AttendSchedule sch;
  };
  constexpr int kEntries = 8;
  thread_local Entry cache[kEntries];
  thread_local unsigned next = 0;
  for (const Entry& e : cache)
    if (e.B == B && e.H == H && e.S == S && e.sms == sms) return e.sch;
  Entry& e = cache[next++ % kEntries];
  e.B = B, e.H = H, e.S = S, e.sms = sms;
  e.sch = compute_schedule(B, H, S, sms);
  return e.sch;
}

int launch_attend_out(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S,
                      const OutLayout& out, const AttendSchedule& sch, void* workspace, int* status,
                      cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FLK_ERR_CUDA;
  if (dev < 0 || dev >= 64) return FLK_ERR_UNSUPPORTED;
  // Per-device set-up on first use, under a lock: host threads making their first call on the
  // same device at the same time must not see the SM count before it is set.
  static std::mutex setup_mu;
  static bool configured[64] = {};
  static int sm_count[64] = {};
  int sms = 0;
  {
    std::lock_guard<std::mutex> lock(setup_mu);
    if (!configured[dev]) {
      int n = 0;
      if (cudaFuncSetAttribute(attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(attend_smem_bytes())) != cudaSuccess ||
          cudaFuncSetAttribute(attend_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(attend_smem_bytes())) != cudaSuccess ||
          cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return FLK_ERR_CUDA;
      sm_count[dev] = n;
      configured[dev] = true;
    }
    sms = sm_count[dev];
  }
  const long long rows = static_cast<long long>(B) * H * S;
  // Gathering calls in which CTAs write o themselves (some items whole) stage each warp's block
  // in shared memory (the Q buffers, free once the item's UMMAs are done) and store it as whole
  // rows: by TMA into every buffer, or by multimem stores through a multicast address. They run
  // one unit per CTA; the pieces of split items write partials there as in the persistent form.
  const bool staged = out.merged && (out.n_out > 1 || out.multicast) && sch.n_full > 0;
  const bool tma_out = staged && !out.multicast;
  const bool persistent = !staged;
  CUtensorMap mq, mk, mv;
  if (!make_tile_map(&mq, q, rows) || !make_tile_map(&mk, k, rows) || !make_tile_map(&mv, v, rows))
    return FLK_ERR_CUDA;
  Params p;
  p.S = S;
  p.n_tiles = S / kTile;
  p.BH = B * H;
  p.n_pairs = (p.n_tiles + 1) / 2;
  const long long units = sch.units();
  if (sch.n_items != static_cast<long long>(p.BH) * p.n_pairs || units > INT32_MAX) return FLK_ERR_UNSUPPORTED;
  p.n_full = sch.n_full;
  p.n_a = sch.n_a;
  p.s_a = sch.s_a;
  p.s_b = sch.s_b;
  p.n_units = static_cast<int>(units);
  p.pa0 = item_row(sch.n_full, p.n_pairs, S);
  p.pa1 = item_row(sch.n_full + sch.n_a, p.n_pairs, S);
  p.pb1 = rows;
  p.out = out;
  p.tma_out = tma_out ? 1 : 0;
  p.stage_mc = (staged && out.multicast) ? 1 : 0;
  if (p.tma_out)
    for (int d = 0; d < out.n_out; ++d)
      if (!make_out_map(&p.out_maps[d], out.o[d], static_cast<long long>(B) * S, out.H_out * kDim))
        return FLK_ERR_CUDA;
  const size_t slots = attend_workspace_bytes(B, H, S, sch) / ((kDim + 1) * sizeof(float));
  p.acc = sch.split() ? static_cast<float*>(workspace) : nullptr;
  p.lsum = sch.split() ? p.acc + slots * kDim : nullptr;
  p.status = status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(persistent ? std::min<long long>(units, sms) : units));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = attend_smem_bytes();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, persistent ? attend_persistent_kernel : attend_kernel, mq, mk, mv, p) !=
      cudaSuccess)
    return FLK_ERR_CUDA;
  if (cudaGetLastError() != cudaSuccess) return FLK_ERR_CUDA;
  if (sch.split()) {
    const CombineParams c{p.pa0, p.pa1, p.pb1, p.s_a, p.s_b, S};
    const long long threads = (p.pb1 - p.pa0) * (kDim / 8);
    combine_splits_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(p.acc, p.lsum, c, out);
    if (cudaGetLastError() != cudaSuccess) return FLK_ERR_CUDA;
  }
  return FLK_OK;
}

int launch_attend_layout(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, uint16_t* o,
                         int merged, const AttendSchedule& sch, void* workspace, int* status,
                         cudaStream_t stream) {
  OutLayout out{};
  out.merged = merged;
  out.H = H;
  out.H_out = H;
  out.h0 = 0;
  out.n_out = 1;
  out.o[0] = o;
  return launch_attend_out(q, k, v, B, H, S, out, sch, workspace, status, stream);
}

// Merged rows of H_out heads, this call's heads at [h0, h0 + H), written into each of the
// n_out buffers (this GPU's and peers' memory, all addressable from this device).
int launch_attend_gather(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S,
                         uint16_t* const* outs, int n_out, int H_out, int h0, const AttendSchedule& sch,
                         void* workspace, int* status, cudaStream_t stream) {
  if (n_out < 1 || n_out > kMaxOuts) return FLK_ERR_INVALID_ARGUMENT;
  OutLayout out{};
  out.merged = 1;
  out.H = H;
  out.H_out = H_out;
  out.h0 = h0;
  out.n_out = n_out;
  for (int d = 0; d < n_out; ++d) out.o[d] = outs[d];
  return launch_attend_out(q, k, v, B, H, S, out, sch, workspace, status, stream);
}

// Merged rows of H_out heads, this call's heads at [h0, h0 + H), stored once through the
// multicast address `out_mc`, which the NVSwitch replicates into every bound rank's buffer.
int launch_attend_gather_multicast(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S,
                                   uint16_t* out_mc, int H_out, int h0, const AttendSchedule& sch,
                                   void* workspace, int* status, cudaStream_t stream) {
  OutLayout out{};
  out.merged = 1;
  out.H = H;
  out.H_out = H_out;
  out.h0 = h0;
  out.n_out = 1;
  out.multicast = 1;
  out.o[0] = out_mc;
  return launch_attend_out(q, k, v, B, H, S, out, sch, workspace, status, stream);
}

int attend_binary_version(int* version) {
  cudaFuncAttributes a{};
  if (cudaFuncGetAttributes(&a, attend_persistent_kernel) != cudaSuccess) return FLK_ERR_CUDA;
  *version = a.binaryVersion;
  return FLK_OK;
}

// Head-major output ([B, H, S, 128]), the layout of kernels.attend.
int launch_attend(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, uint16_t* o,
                  const AttendSchedule& sch, void* workspace, int* status, cudaStream_t stream) {
  return launch_attend_layout(q, k, v, B, H, S, o, 0, sch, workspace, status, stream);
}

}  // namespace flk
