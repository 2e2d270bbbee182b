/*
 * flicker_b200 -- C ABI of the B200 (sm_100a) kernels for flicker's DiT attention hot path.
 *
 * Plain pointers and sizes only. Every tensor argument is a DEVICE pointer
 * into memory of the current CUDA device; bf16 tensors are passed as their
 * 16-bit patterns (uint16_t). `stream` is a cudaStream_t (NULL = legacy
 * default stream). Entry points enqueue work and return immediately; they
 * never synchronise, never allocate device memory, never abort or trap.
 *
 * Return codes: 0 on success, a negative FLK_ERR_* code otherwise
 * (flk_error_string() names it). A kernel that detects a problem while it
 * runs (a bounded wait that ran out) records it in a device-side status word
 * that flk_device_status() reads back.
 *
 * Layouts (row-major, contiguous):
 *   qkv      [B, L, 3*H*D]  columns ordered (3, H, D): q heads, then k heads, then v heads
 *   q, k, v  [B, H, L, D]   head-major
 *   o        [B, H, S, D]
 *   cos, sin [L, D] fp32    lane tables: cos[l, 2j] = cos[l, 2j+1] = cos(theta_lj),
 *                           sin[l, 2j] = -sin(theta_lj), sin[l, 2j+1] = +sin(theta_lj)
 * D must be 128.
 */
#ifndef FLICKER_B200_H
#define FLICKER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FLK_OK 0
#define FLK_ERR_INVALID_ARGUMENT (-1)  /* bad shape, null pointer or misaligned pointer */
#define FLK_ERR_UNSUPPORTED (-2)       /* shape this build does not support (e.g. D != 128) */
#define FLK_ERR_CUDA (-3)              /* a CUDA runtime/driver call failed (e.g. launch) */
#define FLK_ERR_WORKSPACE (-4)         /* workspace missing or smaller than required */
#define FLK_ERR_DEVICE_TIMEOUT (-5)    /* device status: a bounded in-kernel wait ran out */
#define FLK_ERR_NO_DEVICE (-6)         /* current device is not sm_100 */

/*
 * Fused head split + QK-RMSNorm + RoPE (+ q gain) for one attention call.
 * Replaces flicker kernels.qk_prep (src/flicker/kernels.py:57-91, body :35-53):
 *   q[b,h,l,:] = bf16(q_gain * rope(fp32(bf16(rmsnorm(x_q)) * q_scale)))
 *   k[b,h,l,:] = bf16(rope(fp32(bf16(rmsnorm(x_k)) * k_scale)))
 *   v[b,h,l,:] = x_v
 * rmsnorm(x) = x * rsqrt(mean(x^2) + 1e-6) in fp32; the bf16 multiply by the
 * scale rounds to bf16; rope(w)[i] = cos[l,i]*w[i] + sin[l,i]*w[i^1].
 * q_scale, k_scale: [D] bf16. Pointers 16-byte aligned.
 */
int flk_qk_prep(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale,
                const float* cos, const float* sin, float q_gain,
                int B, int L, int H, int D,
                uint16_t* q, uint16_t* k, uint16_t* v, void* stream);

/*
 * flk_qk_prep writing into a longer sequence: token l of this call goes to row row0 + l of
 * q, k, v viewed as [B, H, S_out, D] (0 <= row0, row0 + L <= S_out). Two calls (text stream at
 * row 0, image stream at row num_txt) build the joint q, k, v of a double block in place.
 * Replaces the kernel branch of modules.double_prepare_qkv (src/flicker/modules.py:127-138):
 * qkv_prep per stream, then jnp.concatenate([txt, img], axis=2), an extra HBM copy of q, k, v.
 */
int flk_qk_prep_into(const uint16_t* qkv, const uint16_t* q_scale, const uint16_t* k_scale,
                     const float* cos, const float* sin, float q_gain,
                     int B, int L, int H, int D,
                     uint16_t* q, uint16_t* k, uint16_t* v, int S_out, int row0, void* stream);

/*
 * Bounded (max-free) non-causal attention, q pre-scaled by 1/sqrt(D).
 * Replaces flicker kernels.attend (src/flicker/kernels.py:105-145):
 *   p = bf16(exp(q k^T)),  l = sum_j fp32(p_j),  o = bf16((sum_j p_j v_j) / l)
 * S must be a multiple of 128. `workspace`/`ws_bytes` is scratch the caller
 * owns; flk_attend_workspace_size() says how much a call needs (0 when the
 * call runs unsplit, in which case workspace may be NULL).
 */
int flk_attend(const uint16_t* q, const uint16_t* k, const uint16_t* v,
               int B, int H, int S, int D, uint16_t* o,
               void* workspace, size_t ws_bytes, void* stream);

/*
 * flk_attend with the heads merged on output: o is [B, S, H*D] (head h in columns
 * [h*D, (h+1)*D)), i.e. merge_heads(attend(q, k, v)) of modules.double_block / single_block
 * (src/flicker/modules.py:157,198 with merge_heads :63-65) without the transpose pass.
 * Same workspace rules as flk_attend.
 */
int flk_attend_merged(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      int B, int H, int S, int D, uint16_t* o,
                      void* workspace, size_t ws_bytes, void* stream);

/*
 * flk_attend_merged for one shard of heads, gathered by its own stores: this call's H heads
 * (q, k, v [B, H, S, D]) are heads [h0, h0 + H) of merged rows [B, S, H_total * D], and every
 * output row is written into each of the n_outs (1..8) buffers outs[] (a host array of device
 * pointers, all addressable from the current device: this GPU's output and peers' outputs
 * mapped into this process). When every rank of a head-sharded call does this, each rank's
 * buffer holds merge_heads of all H_total heads after the ranks synchronise, which replaces
 * the all-gather after attention (ncclAllGather over [H/n, S, D] slabs) and the merge_heads
 * transpose (src/flicker/modules.py:63-65,157). The kernel neither waits for peers nor signals
 * them: the caller orders the buffers' use across ranks (a barrier after the call). Same
 * workspace rules as flk_attend, for this call's B, H, S.
 */
int flk_attend_gather(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      int B, int H, int S, int D, uint16_t* const* outs, int n_outs,
                      int H_total, int h0, void* workspace, size_t ws_bytes, void* stream);

/*
 * flk_attend_gather with the rows stored once through an NVLink multicast address: out_mc is the
 * multicast mapping (NVSwitch, e.g. a symmetric-memory buffer's multicast pointer) bound to every
 * rank's merged output buffer [B, S, H_total * D]; each 16-byte store is a multimem.st, which the
 * switch writes into all bound buffers, so this rank's heads cross NVLink once instead of once per
 * peer (the egress of an all-gather drops from (n-1)/n of the output to 1/n of it). Replaces the
 * same ncclAllGather + merge_heads as flk_attend_gather (src/flicker/modules.py:63-65,157). As
 * there, the kernel neither waits for nor signals peers: the caller synchronises the ranks after
 * the call. Same workspace rules as flk_attend, for this call's B, H, S.
 */
int flk_attend_gather_multicast(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                int B, int H, int S, int D, uint16_t* out_mc,
                                int H_total, int h0, void* workspace, size_t ws_bytes, void* stream);

/* Bytes of workspace flk_attend needs for this shape on the current device. */
size_t flk_attend_workspace_size(int B, int H, int S, int D);

/*
 * How flk_attend (given its workspace) cuts the work of a B x H x S call over a device with `sms`
 * SMs. No counterpart in the reference (Pallas picks its grid itself); a host-only query for
 * tests and capacity planning, no GPU work. A work item is two 128-row query tiles of one
 * (batch, head); out[0..5] receive: items, items kept whole (the first ones), items split s_a
 * ways, s_a, s_b (the remaining items' split count) and work units. Returns FLK_OK or
 * FLK_ERR_INVALID_ARGUMENT / FLK_ERR_UNSUPPORTED for shapes flk_attend refuses.
 */
int flk_attend_schedule(int B, int H, int S, int D, int sms, long long* out);

/*
 * flk_attend for callers that cannot allocate device memory. No counterpart in the reference.
 * Same arguments as flk_attend minus the workspace, and the same result as flk_attend given the
 * workspace it asks for: when the shape runs (partly) split over KV, the partial results go to a
 * 32 MiB scratch array built into the library (held on every GPU that loads it) instead of caller
 * memory, so the call allocates nothing. Shapes whose schedule needs more than 32 MiB of scratch
 * (e.g. B=1, H=6, S=16896 on a 148-SM B200) return FLK_ERR_WORKSPACE, although flk_attend with
 * no workspace (NULL, 0) runs them unsplit: this entry point never silently changes the schedule.
 * The first call on a device sets up the scratch address (make it before any stream capture);
 * calls share the scratch, so calls whose kernels overlap on the GPU race and must be ordered
 * by the caller.
 */
int flk_attend_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                       int B, int H, int S, int D, uint16_t* o, void* stream);

/*
 * Load-time guard of the max-free softmax. Replaces kernels.logit_bound
 * (src/flicker/kernels.py:99-101) and the refusal in loader.check_logit_bound
 * (src/flicker/loader.py:115-128): returns sqrt(D) * max|q_scale| * max|k_scale|
 * for fp32 host arrays of length D in *bound, and FLK_OK when it is below
 * EXP_LIMIT = 80, FLK_ERR_INVALID_ARGUMENT otherwise. Host-only, no GPU work.
 */
int flk_logit_bound(const float* q_scale, const float* k_scale, int D, float* bound);

/*
 * linear: y[M, N] = bf16(x[M, K] @ w[K, N]) with fp32 accumulation on the bf16 tensor cores,
 * the weights given transposed (wt = w^T, [N, K], K contiguous; prepared once at load).
 * Replaces nn.linear (src/flicker/nn.py:13-14) on the QKV path. K % 8 == 0; pointers 16-byte
 * aligned.
 */
int flk_linear(const uint16_t* x, const uint16_t* wt, int M, int N, int K, uint16_t* y, void* stream);

/*
 * The QKV projection with qk_prep fused into its epilogue: equals flk_linear(x, wt) followed by
 * flk_qk_prep_into on its first 3*H*D columns, bit for bit, without writing the qkv block to
 * memory. x [B*L, K] (M = B*L tokens), wt [N, K] with N >= 3*H*D; q, k, v [B, H, S_out, D]
 * receive rows [row0, row0 + L); columns [3*H*D, N) (a single block's mlp part) go to rest
 * [M, N - 3*H*D] bf16 (NULL allowed when N == 3*H*D). cos, sin [L, D] fp32; scales [D] bf16.
 * Replaces linear + qkv_prep in modules.double_prepare_qkv / single_prepare_qkv
 * (src/flicker/modules.py:127-134,184-190).
 */
int flk_linear_qk_prep(const uint16_t* x, const uint16_t* wt, int M, int N, int K,
                       const uint16_t* q_scale, const uint16_t* k_scale, const float* cos, const float* sin,
                       float q_gain, int B, int L, int H, int D, uint16_t* q, uint16_t* k, uint16_t* v,
                       int S_out, int row0, uint16_t* rest, void* stream);

/*
 * W8A8 SmoothQuant linear, step 1 (per token). No counterpart in the reference (flicker's linear
 * is a bf16 x @ w, src/flicker/nn.py:13-14); arithmetic per SmoothQuant (Xiao et al., 2022):
 *   x'[i,k] = float(x[i,k]) * inv_smooth[k];  x_scale[i] = max_k |x'[i,k]| / 127 (1 if 0);
 *   xq[i,k] = clamp(rint(x'[i,k] / x_scale[i]), -127, 127)   (round half to even)
 * x [M, K] bf16, inv_smooth [K] fp32, xq [M, K] int8, x_scale [M] fp32. K % 8 == 0.
 */
int flk_w8a8_quantize_act(const uint16_t* x, const float* inv_smooth, int M, int K,
                          int8_t* xq, float* x_scale, void* stream);

/*
 * W8A8 SmoothQuant linear, step 2: y = bf16(float(xq @ wq^T) * (x_scale[i] * w_scale[n])) with
 * int32 accumulation on the int8 tensor cores. xq [M, K] int8, wq [N, K] int8 (per-output-channel
 * codes, K contiguous), x_scale [M], w_scale [N] fp32, y [M, N] bf16. K % 16 == 0.
 * No counterpart in the reference.
 */
int flk_w8a8_gemm(const int8_t* xq, const int8_t* wq, const float* x_scale, const float* w_scale,
                  int M, int N, int K, uint16_t* y, void* stream);

/* The raw int32 accumulators c [M, N] = a [M, K] @ b [N, K]^T of the same kernel (verification). */
int flk_i8_gemm_s32(const int8_t* a, const int8_t* b, int M, int N, int K, int32_t* c, void* stream);

/*
 * Self-test of the failure path (no counterpart in the reference): launches one warp that
 * waits on an mbarrier nothing arrives at. The bounded wait gives up after its ~2 s limit,
 * stores 0 in *result (a device int; 1 would mean the wait succeeded) and records
 * FLK_ERR_DEVICE_TIMEOUT, which the next flk_device_status() returns; the context stays usable.
 */
int flk_selftest_wait_timeout(int* result, void* stream);

/* Self-test of the attend epilogue's quotient (one correctly rounded reciprocal per row, then
 * Markstein's FMA correction per element): writes that quotient and __fdiv_rn's for n pairs of
 * device floats (a[i] / b[i]) into q_fast and q_ref. No reference counterpart (device check). */
int flk_selftest_quotient(const float* a, const float* b, long long n, float* q_fast, float* q_ref, void* stream);

/* Self-test of the attend kernel's exponentials (no reference counterpart; device check): for n
 * device floats x, poly[i] = 2^x[i] from the FMA-pipe polynomial that computes one exponential in
 * four of kernels.attend's p = exp(s) (src/flicker/kernels.py:124), mufu[i] = 2^x[i] from
 * ex2.approx (the other three). A test bounds both against float64 over the bounded-logit domain. */
int flk_selftest_exp2(const float* x, long long n, float* poly, float* mufu, void* stream);

/* binaryVersion (major * 10 + minor, 100 = sm_100) of the code the CUDA runtime loaded for this
 * library's kernels on the current device, or a negative FLK_ERR_* code. No reference counterpart. */
int flk_kernel_binary_version(void);

/* Reads (and clears) the device-side status word of the current device: 0 or FLK_ERR_DEVICE_TIMEOUT.
 * Synchronises the device. */
int flk_device_status(void);

/* Human-readable name of a FLK_* return code. */
const char* flk_error_string(int code);

/* ABI version of this library (major * 100 + minor). */
int flk_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FLICKER_B200_H */
