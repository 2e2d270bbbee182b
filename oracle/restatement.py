"""CPU restatement of flicker's DiT attention hot path -- TEST INFRASTRUCTURE ONLY.

This module is the parity oracle. It restates, in numpy (fp32 arithmetic with
``ml_dtypes.bfloat16`` rounding at exactly the points where the reference
rounds), the two paths the reference has for one attention call:

* the plain-XLA path the reference runs on every non-TPU backend
  (``src/flicker/modules.py:56-60,78-80``, ``src/flicker/nn.py:24-27,35-44``,
  ``src/flicker/rope.py:9-31``), and
* the Pallas kernel path (``src/flicker/kernels.py:28-53,105-145``): lane-pair
  RoPE, ``q_gain`` folded into q before the bf16 round, bf16 ``p = exp(s)``,
  fp32 ``l = sum(p)``, one division at the end.

Pinning: the reference is pure JAX and jax is not installable here, so its
own code is executed through a numpy stand-in for the few jax names it uses
(``tests/golden/make_golden.py``); the committed fixtures in ``tests/golden/``
come from that run and ``tests/test_oracle.py`` checks this restatement
against them. Those fixtures pin the algorithm, the order of operations and
the rounding points; they do not pin XLA's own ``exp``/``cos``/``rsqrt`` ulps.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU leg may
import this module. The ``flicker_b200`` package never does.
"""
from __future__ import annotations

import math
from typing import NamedTuple

import ml_dtypes
import numpy as np

BF16 = ml_dtypes.bfloat16
F32 = np.float32

# src/flicker/kernels.py:19-20,94-95
EPS = 1e-6
ROW_TILES = (2304, 1536, 1152, 512, 256, 128, 64)
SCORE_TILES = (2304, 1536, 1152, 512, 256, 128)
EXP_LIMIT = 80.0

# src/flicker/config.py:31,35-36 (Klein4B)
NUM_HEADS = 24
HEAD_DIM = 128
AXES_DIM = (32, 32, 32, 32)
THETA = 2000.0
NUM_TXT = 512


class Freqs(NamedTuple):
    """src/flicker/kernels.py:12-16 -- lane tables [L, 128] fp32 and the q gain."""

    cos: np.ndarray
    sin: np.ndarray
    q_gain: float = 1.0


def bf16(x: np.ndarray) -> np.ndarray:
    """Round to bfloat16 (round-to-nearest-even), like ``astype(jnp.bfloat16)``."""
    return np.asarray(x).astype(BF16)


def row_tile(length: int) -> int | None:
    """src/flicker/kernels.py:23-24."""
    return next((size for size in ROW_TILES if length % size == 0), None)


# ---------------------------------------------------------------------------
# RoPE tables: src/flicker/rope.py:9-50 and src/flicker/kernels.py:28-31
# ---------------------------------------------------------------------------

def rope_freqs(pos: np.ndarray, dim: int, theta: float = THETA) -> np.ndarray:
    """src/flicker/rope.py:9-14: per-pair 2x2 rotation [[cos,-sin],[sin,cos]] in fp32."""
    scale = np.arange(0, dim, 2, dtype=F32) / F32(dim)
    omega = F32(1.0) / (F32(theta) ** scale)
    angles = pos.astype(F32)[..., None] * omega
    stacked = np.stack([np.cos(angles), -np.sin(angles), np.sin(angles), np.cos(angles)], axis=-1)
    return stacked.reshape(*angles.shape, 2, 2).astype(F32)


def embed_nd(ids: np.ndarray, axes_dim=AXES_DIM, theta: float = THETA) -> np.ndarray:
    """src/flicker/rope.py:17-21: [B, L, 4] ids -> [B, 1, L, 64, 2, 2]."""
    if ids.ndim == 2:
        ids = ids[None]
    per_axis = [rope_freqs(ids[..., i], axes_dim[i], theta) for i in range(len(axes_dim))]
    return np.concatenate(per_axis, axis=-3)[:, None]


def img_ids(height: int, width: int, t: float = 0.0) -> np.ndarray:
    """src/flicker/rope.py:33-38: (t, row, col, 0) per image token."""
    flat = np.arange(height * width)
    ids = np.stack([np.full(height * width, t), flat // width, flat % width,
                    np.zeros(height * width)], axis=-1).astype(F32)
    return ids[None]


def txt_ids(length: int) -> np.ndarray:
    """src/flicker/rope.py:41-45: (0, 0, 0, i) per text token."""
    ids = np.stack([np.zeros(length), np.zeros(length), np.zeros(length),
                    np.arange(length)], axis=-1).astype(F32)
    return ids[None]


def joint_pe(grid_h: int, grid_w: int, num_txt: int = NUM_TXT) -> np.ndarray:
    """src/flicker/dit.py:44-46: text tables first, then image tables, along the sequence."""
    return np.concatenate([embed_nd(txt_ids(num_txt)), embed_nd(img_ids(grid_h, grid_w))], axis=2)


def lane_pair(pe: np.ndarray, q_gain: float = 1.0) -> Freqs:
    """src/flicker/kernels.py:28-31: cos lanes = repeat(cos, 2), sin lanes = (-sin, +sin) interleaved."""
    cos, sin = pe[..., 0, 0][0, 0], pe[..., 1, 0][0, 0]
    lanes = np.stack([-sin, sin], axis=-1).reshape(*sin.shape[:-1], 2 * sin.shape[-1])
    return Freqs(np.ascontiguousarray(np.repeat(cos, 2, axis=-1), F32),
                 np.ascontiguousarray(lanes, F32), q_gain)


# ---------------------------------------------------------------------------
# Plain-XLA path (the reference's non-TPU path)
# ---------------------------------------------------------------------------

def heads(qkv: np.ndarray, num_heads: int):
    """src/flicker/modules.py:56-60: [B, L, 3*H*D] -> three [B, H, L, D] (columns ordered (3, H, D))."""
    b, length, _ = qkv.shape
    head_dim = qkv.shape[-1] // (3 * num_heads)
    split = qkv.reshape(b, length, 3, num_heads, head_dim).transpose(2, 0, 3, 1, 4)
    return split[0], split[1], split[2]


def merge_heads(x: np.ndarray) -> np.ndarray:
    """src/flicker/modules.py:63-65: [B, H, L, D] -> [B, L, H*D]."""
    b, h, n, d = x.shape
    return x.transpose(0, 2, 1, 3).reshape(b, n, h * d)


def rms_norm(x: np.ndarray, scale: np.ndarray, eps: float = EPS) -> np.ndarray:
    """src/flicker/nn.py:24-27: fp32 norm, round to x.dtype, then multiply by scale in that dtype."""
    xf = x.astype(F32)
    normed = xf * (F32(1.0) / np.sqrt(np.mean(np.square(xf), axis=-1, keepdims=True) + F32(eps)))
    return normed.astype(x.dtype) * scale


def apply_rope(xq: np.ndarray, xk: np.ndarray, pe: np.ndarray):
    """src/flicker/rope.py:24-31: out = R @ (x[2j], x[2j+1]) in fp32, rounded to x.dtype."""

    def rotate(x: np.ndarray) -> np.ndarray:
        pairs = x.astype(F32).reshape(*x.shape[:-1], -1, 1, 2)
        out = pe[..., 0] * pairs[..., 0] + pe[..., 1] * pairs[..., 1]
        return out.reshape(*x.shape).astype(x.dtype)

    return rotate(xq), rotate(xk)


def qkv_prep_xla(qkv, q_scale, k_scale, pe, num_heads):
    """src/flicker/modules.py:78-80: heads -> qk_norm -> apply_rope (no q gain)."""
    q, k, v = heads(qkv, num_heads)
    q, k = rms_norm(q, q_scale), rms_norm(k, k_scale)
    q, k = apply_rope(q, k, pe)
    return q, k, v


def sdpa(q, k, v, rows: np.ndarray | None = None, q_block: int = 1024) -> np.ndarray:
    """src/flicker/nn.py:35-44: fp32 logits * 1/sqrt(D), max-subtracted softmax, fp32 PV, cast to v.dtype.

    Computed per (batch, head) and per block of query rows so the [S, S] logits
    never exist at once. ``rows`` (optional) restricts the output to those query
    rows: the result then has shape [B, H, len(rows), D].
    """
    b, h, length, d = q.shape
    scale = F32(1.0 / math.sqrt(d))
    sel = np.arange(length) if rows is None else np.asarray(rows)
    out = np.empty((b, h, len(sel), d), dtype=v.dtype)
    for bi in range(b):
        for hi in range(h):
            kf = k[bi, hi].astype(F32)
            vf = v[bi, hi].astype(F32)
            for r0 in range(0, len(sel), q_block):
                qf = q[bi, hi, sel[r0:r0 + q_block]].astype(F32)
                logits = (qf @ kf.T) * scale
                logits = logits - logits.max(axis=-1, keepdims=True)
                w = np.exp(logits)
                w = w / w.sum(axis=-1, keepdims=True)
                out[bi, hi, r0:r0 + q_block] = (w @ vf).astype(v.dtype)
    return out


# ---------------------------------------------------------------------------
# Kernel path (what kernels.qk_prep / kernels.attend compute)
# ---------------------------------------------------------------------------

def _prep_rows(value: np.ndarray, scale: np.ndarray, cos: np.ndarray, sin: np.ndarray,
               gain: float) -> np.ndarray:
    """src/flicker/kernels.py:42-49 on rows [..., L, D] with tables [L, D]."""
    wide = value.astype(F32)
    rms = np.mean(wide * wide, axis=-1, keepdims=True)
    normed = (wide * (F32(1.0) / np.sqrt(rms + F32(EPS)))).astype(value.dtype) * scale
    wide = normed.astype(F32)
    width = wide.shape[-1]
    even = (np.arange(width) % 2) == 0
    # pltpu.roll(x, width - 1) -> x[i + 1]; pltpu.roll(x, 1) -> x[i - 1]
    swap = np.where(even, np.roll(wide, width - 1, axis=-1), np.roll(wide, 1, axis=-1))
    rotated = cos * wide + sin * swap
    return (rotated if gain == 1.0 else F32(gain) * rotated).astype(value.dtype)


def qk_prep_kernel(qkv: np.ndarray, q_scale: np.ndarray, k_scale: np.ndarray, freqs: Freqs,
                   num_heads: int, rows: int | None = None):
    """src/flicker/kernels.py:57-91: fused head split + QK-RMSNorm + lane-pair RoPE (+ q gain); v copied.

    Raises ``ValueError`` when no row tile divides L, like the reference.
    """
    batch, length, width = qkv.shape
    head_dim = width // (3 * num_heads)
    tile_rows = rows or row_tile(length)
    if tile_rows is None or length % tile_rows:
        raise ValueError(f"qk_prep needs a row tile dividing L={length} (rows={tile_rows})")
    cos, sin, q_gain = freqs
    q, k, v = heads(qkv, num_heads)
    qs = np.asarray(q_scale).reshape(1, -1)
    ks = np.asarray(k_scale).reshape(1, -1)
    assert cos.shape == (length, head_dim)
    q = _prep_rows(q, qs, cos, sin, q_gain)
    k = _prep_rows(k, ks, cos, sin, 1.0)
    return np.ascontiguousarray(q), np.ascontiguousarray(k), np.ascontiguousarray(v)


def attend_kernel(q, k, v, block: int | None = None, rows: np.ndarray | None = None) -> np.ndarray:
    """src/flicker/kernels.py:105-145: no running max; p = bf16(exp(q k^T)); l += sum fp32(p); acc += p v.

    q already carries 1/sqrt(D). The KV loop runs in ``block``-sized steps like
    the reference grid's last axis; ``rows`` restricts the query rows computed.
    """
    b, h, length, d = q.shape
    block = block or next(size for size in SCORE_TILES if length % size == 0)
    sel = np.arange(length) if rows is None else np.asarray(rows)
    out = np.empty((b, h, len(sel), d), dtype=q.dtype)
    for bi in range(b):
        for hi in range(h):
            qf = q[bi, hi, sel].astype(F32)
            l_acc = np.zeros((len(sel), 1), F32)
            acc = np.zeros((len(sel), d), F32)
            for j in range(0, length, block):
                kf = k[bi, hi, j:j + block].astype(F32)
                vt = v[bi, hi, j:j + block]
                s = qf @ kf.T
                p = np.exp(s).astype(vt.dtype)
                l_acc += np.sum(p.astype(F32), axis=1)[:, None]
                acc += p.astype(F32) @ vt.astype(F32)
            out[bi, hi] = (acc / l_acc).astype(q.dtype)
    return out


def attention_fp32(q, k, v, rows: np.ndarray | None = None) -> np.ndarray:
    """softmax(q k^T) v entirely in fp32 (max-subtracted, no bf16 rounding) for pre-scaled q.

    The "reference computed in fp32" that bf16 attention outputs are held to
    (max-abs 2e-2, relative RMS 1e-2). Same ``rows`` convention as ``sdpa``.
    """
    b, h, length, d = q.shape
    sel = np.arange(length) if rows is None else np.asarray(rows)
    out = np.empty((b, h, len(sel), d), F32)
    for bi in range(b):
        for hi in range(h):
            kf = k[bi, hi].astype(F32)
            vf = v[bi, hi].astype(F32)
            for r0 in range(0, len(sel), 1024):
                s = q[bi, hi, sel[r0:r0 + 1024]].astype(F32) @ kf.T
                w = np.exp(s - s.max(axis=-1, keepdims=True))
                out[bi, hi, r0:r0 + 1024] = (w / w.sum(axis=-1, keepdims=True)) @ vf
    return out


# ---------------------------------------------------------------------------
# Load-time bound: src/flicker/kernels.py:99-101, src/flicker/loader.py:115-128
# ---------------------------------------------------------------------------

def logit_bound(q_scale, k_scale) -> np.ndarray:
    """src/flicker/kernels.py:99-101: sqrt(D) * max|q_scale| * max|k_scale| (per leading index)."""
    q_scale = np.asarray(q_scale, F32)
    k_scale = np.asarray(k_scale, F32)
    width = q_scale.shape[-1]
    return F32(math.sqrt(width)) * np.max(np.abs(q_scale), -1) * np.max(np.abs(k_scale), -1)


def check_logit_bound(blocks: dict) -> None:
    """src/flicker/loader.py:115-128: refuse bounded attention when stacked block scales allow exp overflow."""
    double, single = blocks["double_blocks"], blocks["single_blocks"]

    def joint(name: str) -> np.ndarray:
        return np.maximum(*(np.abs(np.asarray(double[f"{s}_attn.norm.{name}.scale"], F32))
                            for s in ("img", "txt")))

    bounds = (logit_bound(joint("query_norm"), joint("key_norm")),
              logit_bound(*(np.asarray(single[f"norm.{n}.scale"], F32)
                            for n in ("query_norm", "key_norm"))))
    worst = max(float(np.max(np.asarray(b))) for b in bounds)
    if worst >= EXP_LIMIT:
        raise ValueError(f"attention='bounded' needs logits under {EXP_LIMIT}; these weights allow "
                         f"{worst:.1f}. use attention='flash'")


# ---------------------------------------------------------------------------
# Seeded synthetic inputs with the shapes and distributions of the configs
# ---------------------------------------------------------------------------

# name -> (batch, image grid h, image grid w)
CONFIGS = {
    "512": (1, 32, 32),      # S = 512 + 1024 = 1536
    "1024": (1, 64, 64),     # S = 512 + 4096 = 4608
    "1024x8": (8, 64, 64),   # batch 8, one seed per batch element
    "2048": (1, 128, 128),   # S = 512 + 16384 = 16896
}


def make_qkv(batch: int, length: int, num_heads: int = NUM_HEADS, head_dim: int = HEAD_DIM,
             seed: int = 0) -> np.ndarray:
    """Fused QKV [B, L, 3*H*D] ~ N(0, 1) rounded to bf16; batch element b uses seed ``seed + b``."""
    out = np.empty((batch, length, 3 * num_heads * head_dim), BF16)
    for b in range(batch):
        rng = np.random.Generator(np.random.PCG64(seed + b))
        out[b] = bf16(rng.standard_normal((length, 3 * num_heads * head_dim), dtype=F32))
    return out


def make_scales(head_dim: int = HEAD_DIM, seed: int = 1):
    """QK-RMSNorm scales ~ U(0.5, 1.5) rounded to bf16 (q first, then k, one generator)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    q_scale = bf16(rng.uniform(0.5, 1.5, head_dim).astype(F32))
    k_scale = bf16(rng.uniform(0.5, 1.5, head_dim).astype(F32))
    return q_scale, k_scale


def make_config(name: str, num_heads: int = NUM_HEADS, seed: int = 0):
    """Inputs of one named config: (qkv, q_scale, k_scale, pe, freqs with q_gain = 1/sqrt(D))."""
    batch, gh, gw = CONFIGS[name]
    length = NUM_TXT + gh * gw
    qkv = make_qkv(batch, length, num_heads, HEAD_DIM, seed)
    q_scale, k_scale = make_scales(HEAD_DIM, seed + 1)
    pe = joint_pe(gh, gw)
    freqs = lane_pair(pe, 1.0 / math.sqrt(HEAD_DIM))
    return qkv, q_scale, k_scale, pe, freqs


# ---------------------------------------------------------------------------
# Tolerance used by every floating-point parity check
# ---------------------------------------------------------------------------

MAX_ABS_TOL = 2e-2
REL_RMS_TOL = 1e-2


def compare(got: np.ndarray, want: np.ndarray) -> tuple[float, float]:
    """(max-abs error, relative RMS error) of ``got`` against an fp32 ``want``."""
    g = np.asarray(got, F32)
    w = np.asarray(want, F32)
    err = g - w
    max_abs = float(np.max(np.abs(err))) if err.size else 0.0
    denom = float(np.sqrt(np.mean(w * w))) if w.size else 1.0
    rel_rms = float(np.sqrt(np.mean(err * err))) / max(denom, 1e-30) if err.size else 0.0
    return max_abs, rel_rms


def within_tolerance(got, want) -> bool:
    max_abs, rel_rms = compare(got, want)
    return max_abs <= MAX_ABS_TOL and rel_rms <= REL_RMS_TOL


def within_tolerance_scaled(got, want) -> bool:
    """Magnitude-aware form of the same bound for qk_prep outputs: |err| <= 2e-2 * max(1, |want|)
    element-wise and relative RMS <= 1e-2.

    q/k after QK-RMSNorm * scale reach |x| ~ 6, where one bf16 ulp is 0.031: a flat 2e-2 bound
    would reject a single last-bit rounding flip (fp32 sum-order differences inside the norm),
    which the reference's own bf16 output has as well.
    """
    g = np.asarray(got, F32)
    w = np.asarray(want, F32)
    ok = bool(np.all(np.abs(g - w) <= MAX_ABS_TOL * np.maximum(1.0, np.abs(w))))
    return ok and compare(g, w)[1] <= REL_RMS_TOL
