"""CPU oracle for the W8A8 SmoothQuant linear -- TEST INFRASTRUCTURE ONLY.

flicker has no int8 code (its `linear` is a plain bf16 `x @ w`, src/flicker/nn.py:13-14), so
this path has no reference implementation to pin against: parity for it is UNPINNED against
the reference. What this module pins is the arithmetic the CUDA path must reproduce, written
from the published method (SmoothQuant, Xiao et al., 2022):

* smoothing factors per input channel j:  s_j = max|X_:,j|^alpha / max|W_j,:|^(1 - alpha)
  (alpha = 0.5), so X' = X / s and W' = diag(s) W leave X W unchanged in exact arithmetic;
* activations: per-token symmetric int8, scale_x[i] = max_j |X'_ij| / 127,
  q = clamp(rint(X'_ij / scale_x[i]), -127, 127)   (round half to even);
* weights: per-output-channel symmetric int8, scale_w[n] = max_k |W'_kn| / 127,
  q = clamp(rint(W'_kn / scale_w[n]), -127, 127), stored N-major ([N, K], K contiguous);
* int32 accumulation acc[i, n] = sum_k Xq[i, k] * Wq[n, k]  (checked bit-exact against an
  int64 matmul);
* dequantisation y = bf16(float32(acc) * float32(scale_x[i] * scale_w[n])).

All float arithmetic is float32 with IEEE rounding (numpy float32 ops), matching the kernels'
__fdiv_rn / __fmul_rn and cvt.rn. A zero row/column gets scale 1 and all-zero codes.

Only tests/ and bench.py's CPU leg may import this module.
"""
from __future__ import annotations

import ml_dtypes
import numpy as np

F32 = np.float32
BF16 = ml_dtypes.bfloat16
ALPHA = 0.5


def make_inputs(m: int = 4608, k: int = 3072, n: int = 9216, outlier_frac: float = 0.01,
                outlier_scale: float = 20.0, seed: int = 0):
    """Config 4's synthetic operands: X ~ N(0,1) bf16 with 1 % of channels x20, W ~ N(0, 0.02) bf16 [K, N]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((m, k), dtype=F32)
    n_out = max(1, int(round(outlier_frac * k)))
    cols = rng.choice(k, n_out, replace=False)
    x[:, cols] *= F32(outlier_scale)
    w = (rng.standard_normal((k, n), dtype=F32) * F32(0.02))
    return x.astype(BF16), w.astype(BF16)


def smooth_factors(x_absmax: np.ndarray, w_absmax: np.ndarray, alpha: float = ALPHA) -> np.ndarray:
    """s_j = max|X_j|^alpha / max|W_j|^(1-alpha) in float32; channels with a zero max get s = 1."""
    xa = np.asarray(x_absmax, F32)
    wa = np.asarray(w_absmax, F32)
    s = np.power(xa, F32(alpha)) / np.power(wa, F32(1.0 - alpha))
    bad = ~np.isfinite(s) | (s <= 0)
    s = np.where(bad, F32(1.0), s).astype(F32)
    return s


def quantize_rows(v: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-row symmetric int8 of a float32 matrix: (codes int8, scale float32 per row)."""
    v = np.asarray(v, F32)
    amax = np.max(np.abs(v), axis=1)
    scale = (amax / F32(127.0)).astype(F32)
    safe = np.where(scale > 0, scale, F32(1.0)).astype(F32)
    q = np.rint(v / safe[:, None]).astype(F32)
    q = np.clip(q, -127, 127).astype(np.int8)
    return q, safe


def quantize_act(x: np.ndarray, inv_s: np.ndarray):
    """X bf16 [M, K] -> (Xq int8 [M, K], scale_x float32 [M]) with X' = float32(X) * inv_s."""
    xs = (np.asarray(x, F32) * np.asarray(inv_s, F32)[None, :]).astype(F32)
    return quantize_rows(xs)


def quantize_weight(w: np.ndarray, s: np.ndarray):
    """W bf16 [K, N] -> (Wq int8 [N, K] N-major, scale_w float32 [N]) with W' = float32(W) * s[:, None]."""
    ws = (np.asarray(w, F32) * np.asarray(s, F32)[:, None]).astype(F32)
    q, scale = quantize_rows(np.ascontiguousarray(ws.T))
    return q, scale


def prepare(x: np.ndarray, w: np.ndarray, alpha: float = ALPHA):
    """Smoothing factors from these operands, then both quantisations."""
    s = smooth_factors(np.max(np.abs(np.asarray(x, F32)), axis=0), np.max(np.abs(np.asarray(w, F32)), axis=1),
                       alpha)
    inv_s = (F32(1.0) / s).astype(F32)
    xq, sx = quantize_act(x, inv_s)
    wq, sw = quantize_weight(w, s)
    return s, inv_s, xq, sx, wq, sw


def int_gemm(xq: np.ndarray, wq_nk: np.ndarray, rows: np.ndarray | None = None) -> np.ndarray:
    """Exact integer product acc = Xq @ Wq^T as int64 (optionally only `rows` of Xq)."""
    a = np.asarray(xq if rows is None else xq[rows], np.int64)
    return a @ np.asarray(wq_nk, np.int64).T


def int_gemm_blas(xq: np.ndarray, wq_nk: np.ndarray) -> np.ndarray:
    """acc = Xq @ Wq^T through a float64 BLAS matmul, exact while |acc| < 2^53 (the CPU baseline's GEMM)."""
    return (np.asarray(xq, np.float64) @ np.asarray(wq_nk, np.float64).T).astype(np.int64)


def dequant(acc: np.ndarray, sx: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """y = bf16(float32(acc) * float32(sx[i] * sw[n]))."""
    scale = (np.asarray(sx, F32)[:, None] * np.asarray(sw, F32)[None, :]).astype(F32)
    return (np.asarray(acc, np.float64).astype(F32) * scale).astype(F32).astype(BF16)
