"""Failure detection on the B200 without a GPU fault: a kernel's bounded wait on a barrier that
nothing arrives at gives up, reports FLK_ERR_DEVICE_TIMEOUT through the device status word, and
the context keeps working (an attention call right after is correct and reports status 0)."""
from __future__ import annotations

import math
import time

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import flicker_b200 as fb  # noqa: E402
from flicker_b200 import _lib  # noqa: E402


def test_bounded_wait_times_out_and_context_survives():
    lib = _lib.lib()
    assert lib.flk_device_status() == 0
    result = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    assert lib.flk_selftest_wait_timeout(result.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    status = lib.flk_device_status()  # synchronises
    waited = time.perf_counter() - t0
    assert status == _lib.FLK_ERR_DEVICE_TIMEOUT
    assert int(result.item()) == 0
    assert 1.0 < waited < 30.0
    assert lib.flk_device_status() == 0  # read-and-clear
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    q = (torch.randn(1, 2, 256, 128, generator=g, device="cuda") / math.sqrt(128)).to(torch.bfloat16)
    k = torch.randn(1, 2, 256, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(1, 2, 256, 128, generator=g, device="cuda").to(torch.bfloat16)
    o = fb.attend(q, k, v).float()
    ref = torch.softmax(q.float() @ k.float().transpose(-1, -2), dim=-1) @ v.float()
    assert (o - ref).abs().max().item() < 2e-2
    assert lib.flk_device_status() == 0
