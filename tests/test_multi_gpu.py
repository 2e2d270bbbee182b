"""Head-sharded attention across two GPUs, and across every GPU, of one node (skipped on a box with
fewer GPUs): the ranks' heads gathered by the attention epilogue's peer stores, and by its
multimem stores where the node has NVLink multicast, equal the NCCL all-gather of the same
per-rank results and match the single-GPU call. Runs tests/multi_gpu_worker.py under torchrun,
one process per GPU, inside a time limit so that a rank that stalls ends the run instead of
hanging it."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_worker(n: int) -> None:
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", f"--master-port={free_port()}",
           os.path.join(ROOT, "tests", "multi_gpu_worker.py")]
    res = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    print(res.stdout[-3000:], res.stderr[-3000:])
    assert res.returncode == 0
    assert res.stdout.count("fused == nccl True, fused ~ full True") == 4 * n  # 2 shapes x 2 steps per rank


def test_head_sharded_gather_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs on this node")
    run_worker(2)


def test_head_sharded_gather_on_every_gpu():
    """Every GPU of the node (4 or 8 on a B200 box): fewer heads per rank, split over KV, and the
    gather's default form from 4 ranks up (multimem stores through the multicast address)."""
    n = torch.cuda.device_count()
    if n < 4:
        pytest.skip("needs 4 or more GPUs on this node")
    run_worker(n)
