"""flk_attend_noalloc: attention for callers that cannot allocate device memory.

Some callers of this library are handed only their input and output buffers and a stream --
for example an XLA custom-call handler registered without a scratch buffer, where the runtime
owns all device memory and a cudaMalloc inside the handler would synchronise the device in the
middle of XLA's asynchronous work. flk_attend needs caller-provided workspace when a shape runs
(partly) split over KV; flk_attend_noalloc instead uses a 32 MiB scratch array built into the
library.

These tests call both entry points through the C ABI and check that the allocation-free one
gives the same result as flk_attend with a caller workspace, on two calls in a row (the scratch
is shared by every call and keeps the previous call's contents), and that it refuses shapes
whose schedule would need more than its 32 MiB.

This file is named so that pytest collects it last.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import bit_equal_fraction, to_device, to_host
from oracle import restatement as R

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from flicker_b200 import _lib  # noqa: E402


def qkv_inputs(b, h, s, seed):
    rng = np.random.default_rng(seed)
    q = R.bf16(rng.standard_normal((b, h, s, 128), dtype=np.float32) / np.float32(math.sqrt(128)))
    k = R.bf16(rng.standard_normal((b, h, s, 128), dtype=np.float32))
    v = R.bf16(rng.standard_normal((b, h, s, 128), dtype=np.float32))
    return to_device(q), to_device(k), to_device(v)


def with_workspace(lib, q, k, v):
    """The existing entry point, given the workspace it asks for (allocated by torch here)."""
    b, h, s, d = q.shape
    ws_bytes = lib.flk_attend_workspace_size(b, h, s, d)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
    o = torch.empty_like(q)
    code = lib.flk_attend(q.data_ptr(), k.data_ptr(), v.data_ptr(), b, h, s, d, o.data_ptr(),
                          ws.data_ptr() if ws_bytes else None, ws_bytes, None)
    assert code == 0, lib.flk_error_string(code)
    return o, ws_bytes


def no_alloc(lib, q, k, v):
    b, h, s, d = q.shape
    o = torch.empty_like(q)
    code = lib.flk_attend_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), b, h, s, d, o.data_ptr(), None)
    assert code == 0, lib.flk_error_string(code)
    return o


@pytest.mark.parametrize("b,h,s", [(1, 3, 4608), (1, 2, 512), (2, 1, 1152), (1, 24, 1024), (1, 12, 4608)])
def test_no_alloc_matches_workspace_entry_point_twice(b, h, s):
    lib = _lib.lib()
    first = qkv_inputs(b, h, s, seed=s + h)
    second = qkv_inputs(b, h, s, seed=s + h + 1)
    for inputs in (first, second):  # two calls in a row share (and overwrite) the scratch
        want, ws_bytes = with_workspace(lib, *inputs)
        got = no_alloc(lib, *inputs)
        torch.cuda.synchronize()
        g, w = to_host(got), to_host(want)
        assert R.within_tolerance(g, w.astype(np.float32)), R.compare(g, w)
        assert bit_equal_fraction(g, w) == 1.0  # same kernels, same split: identical results
    assert lib.flk_device_status() == 0


def test_no_alloc_refuses_shapes_beyond_its_scratch():
    lib = _lib.lib()
    # batch 1, 6 heads, S = 16896 (2048^2 on 4 GPUs) runs tiered on a 148-SM B200: two waves of
    # whole items, then 74 items in halves and 26 in fifths, whose partials need ~36.7 MB
    # (> 32 MiB) of scratch. On a device with another SM count the schedule may differ.
    if lib.flk_attend_workspace_size(1, 6, 16896, 128) <= 32 << 20:
        pytest.skip("this device's schedule for the shape fits the scratch")
    q, k, v = qkv_inputs(1, 6, 16896, seed=3)
    o = torch.empty_like(q)
    code = lib.flk_attend_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, 6, 16896, 128, o.data_ptr(), None)
    assert code == _lib.FLK_ERR_WORKSPACE
    assert lib.flk_device_status() == 0
