"""Timed CPU baseline: the reference's plain-XLA path restated with torch on all host cores.

TEST / BENCH INFRASTRUCTURE ONLY (used by ``bench.py``'s CPU leg and reference
arm). jax is not installable here, so the reference's own XLA-CPU path cannot be
jitted; this is the same computation -- ``modules.heads`` -> ``nn.rms_norm`` ->
``rope.apply_rope`` -> ``nn.sdpa`` (src/flicker/modules.py:56-60,78-80,
src/flicker/nn.py:24-27,35-44, src/flicker/rope.py:24-31) -- with the same bf16
rounding points, run as fp32 torch CPU kernels with every host thread. It is a
restatement ("port"), not the reference binary.
"""
from __future__ import annotations

import math
import os
import time

import torch


def _rms_norm(x: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    normed = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return normed.to(x.dtype) * scale


def _apply_rope(x: torch.Tensor, pe: torch.Tensor) -> torch.Tensor:
    pairs = x.float().reshape(*x.shape[:-1], -1, 1, 2)
    out = pe[..., 0] * pairs[..., 0] + pe[..., 1] * pairs[..., 1]
    return out.reshape(*x.shape).to(x.dtype)


def xla_path_heads(qkv: torch.Tensor, q_scale: torch.Tensor, k_scale: torch.Tensor, pe: torch.Tensor,
                   num_heads: int, heads: range) -> torch.Tensor:
    """Attention output [B, len(heads), L, D] bf16 of the plain-XLA path for the selected heads."""
    b, length, width = qkv.shape
    d = width // (3 * num_heads)
    split = qkv.reshape(b, length, 3, num_heads, d)
    sel = list(heads)
    q = split[:, :, 0, sel].permute(0, 2, 1, 3)
    k = split[:, :, 1, sel].permute(0, 2, 1, 3)
    v = split[:, :, 2, sel].permute(0, 2, 1, 3)
    q = _apply_rope(_rms_norm(q, q_scale), pe)
    k = _apply_rope(_rms_norm(k, k_scale), pe)
    qf, kf, vf = q.float(), k.float(), v.float()
    logits = torch.einsum("bhld,bhsd->bhls", qf, kf) * (1.0 / math.sqrt(d))
    weights = torch.softmax(logits, dim=-1)
    return torch.einsum("bhls,bhsd->bhld", weights, vf).to(v.dtype)


def time_heads(qkv, q_scale, k_scale, pe, num_heads: int, heads: range, threads: int | None = None):
    """Run the path once for ``heads`` and return (seconds, attend FLOPs covered, threads used)."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    b, length, _ = qkv.shape
    d = qkv.shape[-1] // (3 * num_heads)
    t0 = time.perf_counter()
    xla_path_heads(qkv, q_scale, k_scale, pe, num_heads, heads)
    dt = time.perf_counter() - t0
    flops = 4.0 * b * len(heads) * length * length * d
    return dt, flops, threads
