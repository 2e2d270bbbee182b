"""The QKV projection of a DiT block with qk_prep fused into the GEMM's epilogue.

flicker computes ``qkv = linear(modulate(x, mod), w_qkv)`` (``nn.linear``, src/flicker/nn.py:13-14,
a bf16 ``x @ w``) and then ``qkv_prep`` (modules.py:68-80, 127-134, 184-190), which reads the
whole qkv block back from memory. Here one CTA-pair tcgen05 GEMM (bf16 in, fp32 accumulate)
applies qk_prep to each token's head rows while they are still in tensor memory and writes
q, k, v head-major, bit-identical to ``linear`` followed by ``qk_prep``.

* ``prepare_weight(w)`` -- [K, N] weight -> the [N, K] layout the GEMM reads (once, at load);
* ``linear(x, wt)`` -- ``x @ w`` (bf16 output, fp32 accumulation);
* ``qkv_projection(x, wt, q_scale, k_scale, freqs, num_heads, out=None, row=0)`` -- the fused
  projection: returns (q, k, v, rest), ``rest`` being the columns past the q, k, v block (a
  single block's mlp part) or None.
"""
from __future__ import annotations

import torch

from . import _lib
from .kernels import HEAD_DIM, Freqs, _device_call, _require_cuda_bf16

Array = torch.Tensor


def prepare_weight(w: Array) -> Array:
    """[K, N] bf16 weight (``x @ w``) -> [N, K] contiguous (K fastest), the GEMM's operand layout."""
    _require_cuda_bf16("w", w)
    if w.dim() != 2:
        raise ValueError(f"w must be [K, N], got {tuple(w.shape)}")
    return w.t().contiguous()


def _check_xw(x: Array, wt: Array) -> tuple[Array, int, int, int]:
    _require_cuda_bf16("x", x)
    _require_cuda_bf16("wt", wt)
    if wt.dim() != 2 or x.shape[-1] != wt.shape[1] or wt.device != x.device:
        raise ValueError(f"x [..., K] and wt [N, K] do not match: {tuple(x.shape)} vs {tuple(wt.shape)}")
    k = x.shape[-1]
    if k % 8:
        raise ValueError(f"K must be a multiple of 8, got {k}")
    x2 = x.reshape(-1, k).contiguous()
    return x2, x2.shape[0], wt.shape[0], k


def linear(x: Array, wt: Array) -> Array:
    """``x @ w`` for bf16 x [..., K] and wt = w^T [N, K]: bf16 [..., N], fp32 accumulation."""
    x2, m, n, k = _check_xw(x, wt)
    wt = wt.contiguous()
    y = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    lib = _lib.lib()
    code = _device_call(x2, lambda stream: lib.flk_linear(x2.data_ptr(), wt.data_ptr(), m, n, k, y.data_ptr(), stream))
    _lib.check("flk_linear", code)
    return y.reshape(*x.shape[:-1], n)


def qkv_projection(x: Array, wt: Array, q_scale: Array, k_scale: Array, freqs: Freqs, num_heads: int, *,
                   out: tuple[Array, Array, Array] | None = None, row: int = 0):
    """``qk_prep(linear(x, w)[..., :3HD])`` in one kernel, plus the remaining columns.

    x [B, L, K] bf16, wt [N, K] with N >= 3 * num_heads * 128. Returns (q, k, v, rest): q, k, v
    [B, H, L, 128] bf16 (or written into ``out`` = (q, k, v) [B, H, S, 128] at rows
    [row, row + L), as ``kernels.qk_prep_into``), and rest [B, L, N - 3HD] bf16 or None.
    Arithmetic and errors as ``linear`` and ``kernels.qk_prep``.
    """
    if x.dim() != 3:
        raise ValueError(f"x must be [B, L, K], got {tuple(x.shape)}")
    batch, length = x.shape[0], x.shape[1]
    x2, m, n, k = _check_xw(x, wt)
    n_qkv = 3 * num_heads * HEAD_DIM
    if num_heads <= 0 or n < n_qkv:
        raise ValueError(f"wt has {n} output columns; the q, k, v block needs {n_qkv}")
    cos, sin, q_gain = freqs
    for name, t in (("freqs.cos", cos), ("freqs.sin", sin)):
        if not isinstance(t, torch.Tensor) or t.dtype != torch.float32 or t.device != x.device:
            raise ValueError(f"{name} must be a float32 tensor on {x.device}")
        if tuple(t.shape) != (length, HEAD_DIM):
            raise ValueError(f"{name} must be [L, {HEAD_DIM}], got {tuple(t.shape)}")
    scales = []
    for name, t in (("q_scale", q_scale), ("k_scale", k_scale)):
        _require_cuda_bf16(name, t)
        if t.numel() != HEAD_DIM:
            raise ValueError(f"{name} must hold {HEAD_DIM} values")
        scales.append(t.reshape(HEAD_DIM).contiguous())
    if out is None:
        out = tuple(torch.empty((batch, num_heads, length, HEAD_DIM), dtype=torch.bfloat16, device=x.device)
                    for _ in range(3))
        row = 0
    seq = out[0].shape[2]
    for name, t in zip("qkv", out):
        _require_cuda_bf16(f"out.{name}", t)
        if tuple(t.shape) != (batch, num_heads, seq, HEAD_DIM) or not t.is_contiguous():
            raise ValueError(f"out.{name} must be a contiguous [B, H, S, 128] tensor, got {tuple(t.shape)}")
    if row < 0 or row + length > seq:
        raise ValueError(f"rows [{row}, {row + length}) do not fit in S={seq}")
    rest = torch.empty((m, n - n_qkv), dtype=torch.bfloat16, device=x.device) if n > n_qkv else None
    cos, sin, wt = cos.contiguous(), sin.contiguous(), wt.contiguous()
    lib = _lib.lib()
    code = _device_call(x2, lambda stream: lib.flk_linear_qk_prep(
        x2.data_ptr(), wt.data_ptr(), m, n, k, scales[0].data_ptr(), scales[1].data_ptr(), cos.data_ptr(),
        sin.data_ptr(), float(q_gain), batch, length, num_heads, HEAD_DIM, out[0].data_ptr(), out[1].data_ptr(),
        out[2].data_ptr(), seq, row, rest.data_ptr() if rest is not None else None, stream))
    _lib.check("flk_linear_qk_prep", code)
    return out[0], out[1], out[2], (rest.reshape(batch, length, n - n_qkv) if rest is not None else None)
