"""flicker's hot-path kernel API (``flicker.kernels``) on B200.

Same names, argument meanings and error behaviour as the reference module
``src/flicker/kernels.py``; arrays are CUDA ``torch.Tensor`` s instead of jax
arrays, and the work runs in the sm_100a kernels of ``libflicker_b200.so``
(through its C ABI) on the tensor's device and current torch stream.

* ``qk_prep`` -- kernels.py:57-91 (fused head split + QK-RMSNorm + RoPE + q gain)
* ``attend``  -- kernels.py:105-145 (bounded, max-free flash attention)
* ``Freqs``, ``EPS``, ``ROW_TILES``, ``row_tile``, ``lane_pair``, ``SCORE_TILES``,
  ``EXP_LIMIT``, ``logit_bound`` -- kernels.py:12-31,94-101

Two fused forms of the callers' glue around them (no counterpart in kernels.py):

* ``qk_prep_into`` / ``double_qk_prep`` -- the kernel branch of modules.double_prepare_qkv
  (src/flicker/modules.py:127-138) with each stream's qk_prep writing straight into the joint
  q, k, v instead of a jnp.concatenate copy afterwards;
* ``attend_merged`` -- merge_heads(attend(q, k, v)) (modules.py:63-65,157,198) with the heads
  merged by the attention epilogue's stores.

There is no CPU or eager fallback: if the library is missing the call raises.
"""
from __future__ import annotations

import math
from typing import NamedTuple

import numpy as np
import torch

from . import _lib

Array = torch.Tensor


class Freqs(NamedTuple):
    """kernels.py:12-16: RoPE lane tables ``cos``/``sin`` [L, 128] fp32 and the q gain."""

    cos: Array
    sin: Array
    q_gain: float = 1.0


EPS = 1e-6
ROW_TILES = (2304, 1536, 1152, 512, 256, 128, 64)
SCORE_TILES = (2304, 1536, 1152, 512, 256, 128)
EXP_LIMIT = 80.0
HEAD_DIM = 128


def row_tile(length: int) -> int | None:
    """kernels.py:23-24: first row tile that divides ``length``, or None."""
    tile = _ROW_TILE.get(length, 0)
    if tile == 0:
        tile = _ROW_TILE[length] = next((size for size in ROW_TILES if length % size == 0), None)
    return tile


_ROW_TILE: dict[int, int | None] = {}


def lane_pair(freqs: Array, q_gain: float = 1.0) -> Freqs:
    """kernels.py:28-31: RoPE table [1, 1, L, 64, 2, 2] -> lane tables [L, 128].

    cos lanes repeat cos(theta) twice; sin lanes interleave (-sin, +sin), so the
    rotation is ``cos * x + sin * pair_swap(x)``.
    """
    cos, sin = freqs[..., 0, 0][0, 0], freqs[..., 1, 0][0, 0]
    lanes = torch.stack([-sin, sin], dim=-1).reshape(*sin.shape[:-1], 2 * sin.shape[-1])
    return Freqs(torch.repeat_interleave(cos, 2, dim=-1).contiguous(), lanes.contiguous(), q_gain)


def logit_bound(q_scale, k_scale):
    """kernels.py:99-101: sqrt(D) * max|q_scale| * max|k_scale| along the last axis."""
    if isinstance(q_scale, torch.Tensor):
        width = q_scale.shape[-1]
        return math.sqrt(width) * q_scale.float().abs().amax(-1) * k_scale.float().abs().amax(-1)
    q_scale, k_scale = np.asarray(q_scale, np.float32), np.asarray(k_scale, np.float32)
    width = q_scale.shape[-1]
    return np.float32(math.sqrt(width)) * np.max(np.abs(q_scale), -1) * np.max(np.abs(k_scale), -1)


def _stream(t: Array) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _device_call(t: Array, call):
    """``call(stream)`` with ``t``'s device current and that device's current stream. The device
    context is entered only when another device is current: the API's host cost per call is what
    small shapes (and CUDA-graph-free serving loops) pay for every launch."""
    idx = t.get_device()
    if idx != torch.cuda.current_device():
        with torch.cuda.device(idx):
            return call(torch.cuda.current_stream().cuda_stream)
    return call(torch.cuda.current_stream().cuda_stream)


def _require_cuda_bf16(name: str, t: Array) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this package has no CPU path)")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16, got {t.dtype}")


def _qk_prep_args(qkv: Array, q_scale: Array, k_scale: Array, freqs: Freqs, num_heads: int, rows: int | None):
    """Validation shared by the qk_prep forms (kernels.py:66-73 error behaviour)."""
    _require_cuda_bf16("qkv", qkv)
    if qkv.dim() != 3:
        raise ValueError(f"qkv must be [B, L, 3*H*D], got shape {tuple(qkv.shape)}")
    batch, length, width = qkv.shape
    if num_heads <= 0 or width % (3 * num_heads):
        raise ValueError(f"width {width} is not 3 * num_heads * head_dim for num_heads={num_heads}")
    head_dim = width // (3 * num_heads)
    tile_rows = rows or row_tile(length)
    if tile_rows is None or length % tile_rows:
        raise ValueError(f"qk_prep needs a row tile dividing L={length} (rows={tile_rows})")
    if head_dim != HEAD_DIM:
        raise ValueError(f"head_dim must be {HEAD_DIM}, got {head_dim}")
    cos, sin, q_gain = freqs
    dev = qkv.get_device()
    for name, t in (("freqs.cos", cos), ("freqs.sin", sin)):
        if not isinstance(t, torch.Tensor) or t.get_device() != dev or t.dtype != torch.float32:
            raise ValueError(f"{name} must be a float32 tensor on {qkv.device}")
        if t.shape != (length, head_dim):
            raise ValueError(f"{name} must be [L, {head_dim}] = [{length}, {head_dim}], got {tuple(t.shape)}")
    scales = []
    for name, t in (("q_scale", q_scale), ("k_scale", k_scale)):
        _require_cuda_bf16(name, t)
        if t.numel() != head_dim or t.get_device() != dev:
            raise ValueError(f"{name} must hold {head_dim} values on {qkv.device}")
        scales.append(t if t.dim() == 1 and t.is_contiguous() else t.reshape(head_dim).contiguous())
    return qkv.contiguous(), scales, cos.contiguous(), sin.contiguous(), float(q_gain), batch, length, head_dim


def qk_prep(
    qkv: Array,
    q_scale: Array,
    k_scale: Array,
    freqs: Freqs,
    num_heads: int,
    *,
    rows: int | None = None,
    interpret: bool = False,
) -> tuple[Array, Array, Array]:
    """Fused head transpose + QK-RMSNorm + RoPE (+ q gain) in one HBM pass.

    ``qkv`` [B, L, 3*H*D] bf16 (columns ordered (3, H, D)) -> q, k, v [B, H, L, D] bf16.
    ``q = bf16(q_gain * rope(fp32(bf16(rmsnorm(x)) * q_scale)))``, k likewise without the
    gain, v copied (kernels.py:35-53). ``rows`` is the reference's row-tile hint: it is
    validated exactly as kernels.py:71-73 does (``ValueError`` when no tile divides L);
    the CUDA kernel does not need a row tile. ``interpret`` (Pallas interpret mode in the
    reference) is not available.
    """
    if interpret:
        raise NotImplementedError("interpret=True: this build runs only the sm_100a kernels")
    qkv, scales, cos, sin, q_gain, batch, length, head_dim = _qk_prep_args(qkv, q_scale, k_scale, freqs,
                                                                          num_heads, rows)
    # q, k, v as three views of one allocation (one call into the caching allocator)
    out = torch.empty((3, batch, num_heads, length, head_dim), dtype=qkv.dtype, device=qkv.device).unbind(0)
    lib = _lib.lib()
    code = _device_call(qkv, lambda stream: lib.flk_qk_prep(
        qkv.data_ptr(), scales[0].data_ptr(), scales[1].data_ptr(), cos.data_ptr(), sin.data_ptr(),
        q_gain, batch, length, num_heads, head_dim,
        out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(), stream))
    _lib.check("flk_qk_prep", code)
    return out[0], out[1], out[2]


def qk_prep_into(qkv: Array, q_scale: Array, k_scale: Array, freqs: Freqs, num_heads: int,
                 out: tuple[Array, Array, Array], row: int, *, rows: int | None = None) -> None:
    """qk_prep writing token l of ``qkv`` to row ``row + l`` of ``out`` = (q, k, v) [B, H, S, D].

    Same arithmetic, arguments and errors as ``qk_prep``; ``out`` must be contiguous bf16 of
    the same batch/heads/head_dim with ``row + L <= S``. Rows outside [row, row + L) are left
    untouched, so calls for the text and image streams fill one joint buffer.
    """
    qkv, scales, cos, sin, q_gain, batch, length, head_dim = _qk_prep_args(qkv, q_scale, k_scale, freqs,
                                                                          num_heads, rows)
    if len(out) != 3:
        raise ValueError("out must be the (q, k, v) buffers")
    seq = out[0].shape[2] if out[0].dim() == 4 else -1
    dev = qkv.get_device()
    for name, t in zip("qkv", out):
        _require_cuda_bf16(f"out.{name}", t)
        if (t.shape != (batch, num_heads, seq, head_dim) or not t.is_contiguous()
                or t.get_device() != dev):
            raise ValueError(f"out.{name} must be a contiguous [B, H, S, D] = [{batch}, {num_heads}, S, "
                             f"{head_dim}] tensor on {qkv.device}, got {tuple(t.shape)}")
    if row < 0 or row + length > seq:
        raise ValueError(f"rows [{row}, {row + length}) do not fit in S={seq}")
    lib = _lib.lib()
    code = _device_call(qkv, lambda stream: lib.flk_qk_prep_into(
        qkv.data_ptr(), scales[0].data_ptr(), scales[1].data_ptr(), cos.data_ptr(), sin.data_ptr(),
        q_gain, batch, length, num_heads, head_dim,
        out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(), seq, row, stream))
    _lib.check("flk_qk_prep_into", code)


def double_qk_prep(txt_qkv: Array, img_qkv: Array, txt_scales: tuple[Array, Array],
                   img_scales: tuple[Array, Array], freqs: Freqs, num_heads: int) -> tuple[Array, Array, Array]:
    """Joint q, k, v of a double block: text rows first, then image rows (modules.py:127-138).

    ``freqs`` holds the lane tables of the joint sequence ([num_txt + num_img, 128]); the text
    stream uses its first num_txt rows and the image stream the rest, as the reference slices
    them. Equal to concatenating the two streams' ``qk_prep`` outputs along the sequence axis,
    without that copy.
    """
    if txt_qkv.dim() != 3 or img_qkv.dim() != 3:
        raise ValueError("txt_qkv and img_qkv must be [B, L, 3*H*D]")
    num_txt, num_img = txt_qkv.shape[1], img_qkv.shape[1]
    cos, sin, q_gain = freqs
    if cos.shape[0] != num_txt + num_img or sin.shape[0] != num_txt + num_img:
        raise ValueError(f"freqs must cover {num_txt} + {num_img} rows, got {tuple(cos.shape)}")
    batch, width = txt_qkv.shape[0], txt_qkv.shape[2]
    if img_qkv.shape[0] != batch or img_qkv.shape[2] != width or num_heads <= 0 or width % (3 * num_heads):
        raise ValueError("txt_qkv and img_qkv must share batch and width 3 * num_heads * head_dim")
    head_dim = width // (3 * num_heads)
    out = torch.empty((3, batch, num_heads, num_txt + num_img, head_dim), dtype=txt_qkv.dtype,
                      device=txt_qkv.device).unbind(0)
    qk_prep_into(txt_qkv, *txt_scales, Freqs(cos[:num_txt], sin[:num_txt], q_gain), num_heads, out, 0)
    qk_prep_into(img_qkv, *img_scales, Freqs(cos[num_txt:], sin[num_txt:], q_gain), num_heads, out, num_txt)
    return out


def _attend_args(q: Array, k: Array, v: Array, block: int | None):
    dev = q.get_device() if isinstance(q, torch.Tensor) else None
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda_bf16(name, t)
        if t.dim() != 4 or t.shape != q.shape or t.get_device() != dev:
            raise ValueError(f"q, k, v must share one [B, H, S, D] shape and device; {name} is "
                             f"{tuple(t.shape)}")
    batch, heads, length, dim = q.shape
    if dim != HEAD_DIM:
        raise ValueError(f"head_dim must be {HEAD_DIM}, got {dim}")
    if length % 128:
        raise ValueError(f"attend needs S to be a multiple of 128, got {length}")
    if block is not None and (block <= 0 or block % 128 or length % block):
        raise ValueError(f"block={block} must be a multiple of 128 dividing S={length}")
    return q.contiguous(), k.contiguous(), v.contiguous(), batch, heads, length, dim


# Workspace bytes of a split-KV call, per (device, B, H, S): a function of the shape and the
# device's SM count only, so it is asked of the library once per shape.
_WS_BYTES: dict[tuple[int, int, int, int], int] = {}


def _run_attend(fn: str, q: Array, k: Array, v: Array, o: Array, batch: int, heads: int, length: int,
                dim: int) -> Array:
    lib = _lib.lib()
    entry = getattr(lib, fn)

    def call(stream: int) -> int:
        key = (q.get_device(), batch, heads, length)
        ws_bytes = _WS_BYTES.get(key)
        if ws_bytes is None:
            ws_bytes = _WS_BYTES[key] = lib.flk_attend_workspace_size(batch, heads, length, dim)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
        return entry(q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, heads, length, dim,
                     o.data_ptr(), ws.data_ptr() if ws is not None else None, ws_bytes, stream)

    _lib.check(fn, _device_call(q, call))
    return o


def attend(q: Array, k: Array, v: Array, *, block: int | None = None, interpret: bool = False) -> Array:
    """Bounded flash attention without a running max; q already carries 1/sqrt(D).

    q, k, v [B, H, S, D] bf16 -> o [B, H, S, D] bf16 with
    ``o = bf16((sum_j bf16(exp(q k_j^T)) v_j) / sum_j fp32(bf16(exp(q k_j^T))))``
    (kernels.py:113-130). ``block`` is the reference's score-tile hint; it must divide S
    and be a multiple of 128 (the kernel's own KV block). S must be a multiple of 128:
    the reference raises from ``next()`` there, this raises ``ValueError``.
    """
    if interpret:
        raise NotImplementedError("interpret=True: this build runs only the sm_100a kernels")
    q, k, v, batch, heads, length, dim = _attend_args(q, k, v, block)
    return _run_attend("flk_attend", q, k, v, torch.empty_like(q), batch, heads, length, dim)


def attend_merged(q: Array, k: Array, v: Array, *, block: int | None = None) -> Array:
    """``merge_heads(attend(q, k, v))`` in one kernel: o [B, S, H*D] bf16 (modules.py:63-65).

    Same arithmetic, arguments and errors as ``attend``; the epilogue stores each head's
    columns into the merged rows, so there is no separate transpose pass over o.
    """
    q, k, v, batch, heads, length, dim = _attend_args(q, k, v, block)
    o = torch.empty((batch, length, heads * dim), dtype=q.dtype, device=q.device)
    return _run_attend("flk_attend_merged", q, k, v, o, batch, heads, length, dim)


def device_status(device: torch.device | int | None = None) -> int:
    """Synchronise ``device`` and return (and clear) the kernels' device status word (0 = ok)."""
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        return _lib.lib().flk_device_status()
