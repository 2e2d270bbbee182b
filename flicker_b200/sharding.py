"""Splitting one attention call across the GPUs of a node (one process per GPU).

Heads are independent in both qk_prep and attend, and so are batch elements, so
the hot path shards without any exchange inside it:

* batch sharding (batch >= world): rank r owns whole batch elements; nothing is
  exchanged -- each rank's output feeds its own downstream layers;
* head sharding (batch 1): rank r owns heads [r*H/n, (r+1)*H/n). Its fused-QKV
  input holds only those heads' q, k and v columns (what a column-parallel QKV
  projection produces), it runs qk_prep + attend locally, and one all-gather
  assembles the [B, H, S, D] output that ``merge_heads`` needs.

The collective runs on whatever process group it is given: NCCL over NVLink on
the B200 box, gloo in the CPU tests of the layout logic.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def head_range(num_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Heads [h0, h1) owned by ``rank`` when ``num_heads`` are split evenly over ``world`` ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split evenly over {world} ranks")
    per = num_heads // world
    return rank * per, (rank + 1) * per


def batch_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Batch elements [b0, b1) owned by ``rank`` (contiguous, sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(batch, world)
    b0 = rank * base + min(rank, extra)
    return b0, b0 + base + (1 if rank < extra else 0)


def slice_qkv_heads(qkv: torch.Tensor, num_heads: int, h0: int, h1: int) -> torch.Tensor:
    """[B, L, 3*H*D] fused QKV -> [B, L, 3*(h1-h0)*D] holding only heads [h0, h1) of q, k and v."""
    b, length, width = qkv.shape
    d = width // (3 * num_heads)
    return qkv.reshape(b, length, 3, num_heads, d)[:, :, :, h0:h1].reshape(b, length, 3 * (h1 - h0) * d)


def gather_heads(o_local: torch.Tensor, out: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-rank head slabs [1, H/n, S, D] into ``out`` [n, 1, H/n, S, D].

    With batch 1 the rank-major result is exactly [1, H, S, D] in head order
    (``out.view(1, H, S, D)``). ``out`` is preallocated by the caller so the call
    allocates nothing and can be captured in a CUDA graph.
    """
    if o_local.shape[0] != 1:
        raise ValueError("head-sharded gather expects batch 1")
    o_local = o_local.contiguous()
    dist.all_gather_into_tensor(out.view(-1), o_local.view(-1), group=group)
    return out


def merge_heads(x: torch.Tensor) -> torch.Tensor:
    """src/flicker/modules.py:63-65: [B, H, N, D] -> [B, N, H*D]."""
    b, h, n, d = x.shape
    return x.transpose(1, 2).reshape(b, n, h * d)
