"""Splitting one attention call across the GPUs of a node (one process per GPU).

Heads are independent in both qk_prep and attend, and so are batch elements, so
the hot path shards without any exchange inside it:

* batch sharding (batch >= world): rank r owns whole batch elements; nothing is
  exchanged -- each rank's output feeds its own downstream layers;
* head sharding (batch 1): rank r owns heads [r*H/n, (r+1)*H/n). Its fused-QKV
  input holds only those heads' q, k and v columns (what a column-parallel QKV
  projection produces), it runs qk_prep + attend locally, and the ranks' heads
  are assembled either by one all-gather (``gather_heads``, then ``merge_heads``)
  or by the attention epilogue itself (``attend_gather_heads``): every rank stores
  its heads' merged rows into every rank's output buffer over NVLink
  (``PeerOutput``, torch symmetric memory), followed by one barrier -- once per
  peer through its pointer, or once through the buffers' NVLink multicast address
  (multimem stores, replicated by the NVSwitch).

The all-gather runs on whatever process group it is given: NCCL over NVLink on
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


class PeerOutput:
    """Merged-head output buffers [B, S, H_total * D] bf16 that every rank of ``group`` can store into.

    Allocated from torch symmetric memory and exchanged once (a collective), so each rank holds
    device pointers to all ranks' buffers (``ptrs``, in rank order). ``copies`` buffers are
    kept and used in turn: a rank storing into buffer i of step n + copies knows every peer has
    finished with that buffer's step-n contents, because it passed the barrier of step
    n + 1 ... after them (each rank consumes its output in stream order before its next call).
    """

    def __init__(self, shape, device, group, copies: int = 2):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.bufs, self.handles, self.ptrs, self.mc_ptrs = [], [], [], []
        for _ in range(copies):
            buf = symm_mem.empty(*shape, dtype=torch.bfloat16, device=device)
            handle = symm_mem.rendezvous(buf, group)
            self.bufs.append(buf)
            self.handles.append(handle)
            self.ptrs.append([int(p) for p in handle.buffer_ptrs])
            self.mc_ptrs.append(int(handle.multicast_ptr))  # 0 where the node has no NVLink multicast
        # multicast stores need every buffer bound to a multicast object on every rank
        flag = torch.tensor([1 if all(self.mc_ptrs) else 0], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        self.multicast = bool(flag.item())
        self.turn = 0
        self.last = 0  # buffer of the most recent call

    def barrier(self) -> None:
        """The barrier that ends a call made with ``sync=False``: after it, every rank's stores
        into the most recently used buffer are complete and visible."""
        self.handles[self.last].barrier()


def attend_gather_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, peer: PeerOutput, h0: int,
                        num_heads: int, sync: bool = True, multicast: bool | None = None) -> torch.Tensor:
    """Head-sharded attention whose epilogue stores this rank's heads [h0, h0 + H) of the merged
    rows into every rank's buffer; after the barrier, the returned local buffer holds
    merge_heads(attend(q, k, v)) over all ``num_heads`` heads on every rank. The stores go once
    per rank through the peers' pointers, or, with ``multicast``, once through the buffers'
    NVLink multicast address. The default (``None``) takes multicast from 4 ranks up where the
    buffers have it: on 2 GPUs the peer stores measured faster (188.5 vs 210.2 µs per step), on 8
    the multicast ones (115.5 vs 128.4 µs), since a rank's egress grows with the peer count only
    in the peer form. ``sync=False`` leaves
    the barrier to the caller (``peer.barrier()``), which must make it before using the buffer
    and before the next call."""
    import ctypes

    from . import _lib, kernels

    q, k, v, batch, heads, length, dim = kernels._attend_args(q, k, v, None)
    i = peer.turn
    peer.turn = (peer.turn + 1) % len(peer.bufs)
    peer.last = i
    buf, handle, ptrs = peer.bufs[i], peer.handles[i], peer.ptrs[i]
    if tuple(buf.shape) != (batch, length, num_heads * dim):
        raise ValueError(f"peer buffer {tuple(buf.shape)} is not [B, S, H*D] = {(batch, length, num_heads * dim)}")
    if multicast is None:
        multicast = peer.multicast and peer.world >= 4
    if multicast and not peer.multicast:
        raise ValueError("these buffers have no NVLink multicast address on every rank")
    lib = _lib.lib()
    with torch.cuda.device(q.device):
        ws_bytes = lib.flk_attend_workspace_size(batch, heads, length, dim)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
        ws_ptr = ws.data_ptr() if ws is not None else None
        if multicast:
            name = "flk_attend_gather_multicast"
            code = lib.flk_attend_gather_multicast(q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, heads, length,
                                                   dim, peer.mc_ptrs[i], num_heads, h0, ws_ptr, ws_bytes,
                                                   kernels._stream(q))
        else:
            name = "flk_attend_gather"
            outs = (ctypes.c_void_p * len(ptrs))(*ptrs)
            code = lib.flk_attend_gather(q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, heads, length, dim, outs,
                                         len(ptrs), num_heads, h0, ws_ptr, ws_bytes, kernels._stream(q))
    _lib.check(name, code)
    if sync:
        handle.barrier()
    return buf
