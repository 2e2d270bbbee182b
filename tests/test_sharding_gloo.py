"""Multi-GPU layout logic of flicker_b200.sharding, exercised on CPU with gloo ranks.

The per-rank compute here is the CPU oracle (the CUDA kernels need a B200); what is
under test is the sharding arithmetic, the head slicing of the fused QKV input and the
all-gather that reassembles the full-head output, plus host-side failure detection.
"""
from __future__ import annotations

import datetime
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flicker_b200 import sharding
from oracle import restatement as R


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_and_batch_ranges():
    assert [sharding.head_range(24, 8, r) for r in range(8)] == [(3 * r, 3 * r + 3) for r in range(8)]
    assert sharding.head_range(24, 1, 0) == (0, 24)
    with pytest.raises(ValueError):
        sharding.head_range(24, 5, 0)
    with pytest.raises(ValueError):
        sharding.head_range(24, 2, 2)
    spans = [sharding.batch_range(10, 4, r) for r in range(4)]
    assert spans == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert sharding.batch_range(8, 8, 7) == (7, 8)


def test_slice_qkv_heads_matches_full_oracle():
    h, length = 4, 256
    qkv = R.make_qkv(1, length, num_heads=h, seed=3)
    qs, ks = R.make_scales()
    f = R.lane_pair(R.joint_pe(8, 16, 128), 1 / math.sqrt(128))
    full = R.qk_prep_kernel(qkv, qs, ks, f, h)
    t = torch.from_numpy(qkv.view(np.int16)).view(torch.bfloat16)
    for h0, h1 in ((0, 2), (2, 4), (1, 3)):
        part = sharding.slice_qkv_heads(t, h, h0, h1).contiguous()
        part_np = part.view(torch.int16).numpy().view(R.BF16)
        got = R.qk_prep_kernel(part_np, qs, ks, f, h1 - h0)
        for g, w in zip(got, full):
            np.testing.assert_array_equal(g.view(np.uint16), w[:, h0:h1].view(np.uint16))


def _gather_worker(rank, world, port, heads, length, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    qkv = R.make_qkv(1, length, num_heads=heads, seed=5)
    qs, ks = R.make_scales()
    f = R.lane_pair(R.joint_pe(8, 16, 128), 1 / math.sqrt(128))
    h0, h1 = sharding.head_range(heads, world, rank)
    t = torch.from_numpy(qkv.view(np.int16)).view(torch.bfloat16)
    part = sharding.slice_qkv_heads(t, heads, h0, h1).contiguous().view(torch.int16).numpy().view(R.BF16)
    q, k, v = R.qk_prep_kernel(part, qs, ks, f, h1 - h0)
    o = R.attend_kernel(q, k, v)
    o_t = torch.from_numpy(np.ascontiguousarray(o).view(np.int16)).view(torch.bfloat16)
    gathered = torch.empty((world, 1, h1 - h0, length, 128), dtype=torch.bfloat16)
    sharding.gather_heads(o_t, gathered, None)
    full = gathered.view(1, heads, length, 128)
    merged = sharding.merge_heads(full)
    np.save(os.path.join(out_dir, f"o_{rank}.npy"), full.view(torch.int16).numpy())
    np.save(os.path.join(out_dir, f"m_{rank}.npy"), merged.view(torch.int16).numpy())
    dist.destroy_process_group()


def test_head_sharded_all_gather_reassembles_full_output(tmp_path):
    world, heads, length = 2, 4, 256
    mp.spawn(_gather_worker, args=(world, free_port(), heads, length, str(tmp_path)), nprocs=world, join=True)
    qkv = R.make_qkv(1, length, num_heads=heads, seed=5)
    qs, ks = R.make_scales()
    f = R.lane_pair(R.joint_pe(8, 16, 128), 1 / math.sqrt(128))
    want = R.attend_kernel(*R.qk_prep_kernel(qkv, qs, ks, f, heads))
    for rank in range(world):
        got = np.load(tmp_path / f"o_{rank}.npy").view(R.BF16)
        np.testing.assert_array_equal(got.view(np.uint16), want.view(np.uint16))
        merged = np.load(tmp_path / f"m_{rank}.npy").view(R.BF16)
        np.testing.assert_array_equal(merged.view(np.uint16), R.merge_heads(want).view(np.uint16))


def _leaver_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # This rank leaves between steps: it never joins the collective.
        open(os.path.join(out_dir, "left"), "w").close()
        os._exit(0)
    o = torch.zeros((1, 2, 128, 128), dtype=torch.bfloat16)
    out = torch.empty((world, 1, 2, 128, 128), dtype=torch.bfloat16)
    outcome = "completed"
    try:
        sharding.gather_heads(o, out, None)
    except Exception as exc:  # the collective must end with an error, not hang
        outcome = f"error: {type(exc).__name__}"
    with open(os.path.join(out_dir, "outcome"), "w") as fh:
        fh.write(outcome)
    os._exit(0)


def test_rank_that_leaves_makes_the_collective_fail_not_hang(tmp_path):
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_leaver_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    assert (tmp_path / "left").exists()
    outcome = (tmp_path / "outcome").read_text()
    assert outcome.startswith("error"), outcome
