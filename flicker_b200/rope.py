"""RoPE position tables for the hot path, built with torch on the target device.

Restates ``src/flicker/rope.py:9-50`` (4-axis ids -> per-pair 2x2 rotations, fp32)
and the joint text-then-image ordering of ``src/flicker/dit.py:44-46``. These run
once per forward (not per block) and feed ``kernels.lane_pair``.
"""
from __future__ import annotations

import torch

AXES_DIM = (32, 32, 32, 32)  # src/flicker/config.py:35
THETA = 2000.0               # src/flicker/config.py:36


def rope_freqs(pos: torch.Tensor, dim: int, theta: float = THETA) -> torch.Tensor:
    """rope.py:9-14: [..., n] positions -> [..., n, dim/2, 2, 2] rotations [[cos, -sin], [sin, cos]]."""
    scale = torch.arange(0, dim, 2, dtype=torch.float32, device=pos.device) / dim
    omega = 1.0 / (theta ** scale)
    angles = pos.to(torch.float32)[..., None] * omega
    stacked = torch.stack([torch.cos(angles), -torch.sin(angles), torch.sin(angles), torch.cos(angles)], -1)
    return stacked.reshape(*angles.shape, 2, 2)


def embed_nd(ids: torch.Tensor, axes_dim=AXES_DIM, theta: float = THETA) -> torch.Tensor:
    """rope.py:17-21: [B, L, 4] ids -> [B, 1, L, sum(axes_dim)/2, 2, 2]."""
    if ids.dim() == 2:
        ids = ids[None]
    per_axis = [rope_freqs(ids[..., i], axes_dim[i], theta) for i in range(len(axes_dim))]
    return torch.cat(per_axis, dim=-3)[:, None]


def img_ids(height: int, width: int, t: float = 0.0, device=None) -> torch.Tensor:
    """rope.py:33-38: ids (t, row, col, 0) of an image grid, [1, h*w, 4] fp32."""
    flat = torch.arange(height * width, device=device)
    ids = torch.stack([torch.full_like(flat, 0) + t, flat // width, flat % width, torch.zeros_like(flat)], -1)
    return ids.to(torch.float32)[None]


def txt_ids(length: int, device=None) -> torch.Tensor:
    """rope.py:41-45: ids (0, 0, 0, i) of text tokens, [1, L, 4] fp32."""
    ar = torch.arange(length, device=device)
    z = torch.zeros_like(ar)
    return torch.stack([z, z, z, ar], -1).to(torch.float32)[None]


def joint_pe(num_txt: int, grid_h: int, grid_w: int, device=None) -> torch.Tensor:
    """dit.py:44-46: text tables first, then image tables, along the sequence axis."""
    return torch.cat([embed_nd(txt_ids(num_txt, device)), embed_nd(img_ids(grid_h, grid_w, device=device))], 2)
