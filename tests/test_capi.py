"""The C-ABI library: it loads, exports every symbol include/*.h declares, and its host-side
checks answer without touching a GPU (no compute is launched in these tests)."""
from __future__ import annotations

import ctypes
import glob
import os
import re

import numpy as np
import pytest

from conftest import ROOT
from flicker_b200 import _lib


def declared_functions() -> set[str]:
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(flk_\w+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"flk_qk_prep", "flk_attend", "flk_attend_workspace_size", "flk_logit_bound",
            "flk_device_status", "flk_error_string", "flk_abi_version"} <= names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_lib.SIGNATURES) == declared_functions()


@pytest.mark.gpu
def test_library_runs_sm100_code():
    """The runtime loaded sm_100 code for the library's kernels (a kernel attribute, read through the C ABI)."""
    assert _lib.lib().flk_kernel_binary_version() == 100


def test_error_strings_and_version():
    lib = _lib.lib()
    assert lib.flk_abi_version() >= 100
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert lib.flk_error_string(code)
    assert b"unknown" in lib.flk_error_string(-99)


def test_logit_bound_host_entry_point():
    lib = _lib.lib()
    fp = ctypes.POINTER(ctypes.c_float)
    q = np.full(128, 1.5, np.float32)
    k = np.full(128, 1.5, np.float32)
    out = ctypes.c_float()
    code = lib.flk_logit_bound(q.ctypes.data_as(fp), k.ctypes.data_as(fp), 128, ctypes.byref(out))
    assert code == 0 and abs(out.value - np.sqrt(128) * 2.25) < 1e-4
    k[3] = -3.0  # |scale| counts
    code = lib.flk_logit_bound(q.ctypes.data_as(fp), k.ctypes.data_as(fp), 128, ctypes.byref(out))
    assert code == 0 and abs(out.value - np.sqrt(128) * 4.5) < 1e-4
    q[:] = 5.0
    code = lib.flk_logit_bound(q.ctypes.data_as(fp), k.ctypes.data_as(fp), 128, ctypes.byref(out))
    assert code == _lib.FLK_ERR_INVALID_ARGUMENT and out.value >= 80.0
    assert lib.flk_logit_bound(None, k.ctypes.data_as(fp), 128, ctypes.byref(out)) == _lib.FLK_ERR_INVALID_ARGUMENT


def test_shape_checks_run_before_any_device_work():
    """Invalid shapes are refused on the host with an error code (never a launch)."""
    lib = _lib.lib()
    fake = ctypes.c_void_p(0x10000)  # aligned, never dereferenced: the shape check fails first
    # head_dim != 128
    assert lib.flk_qk_prep(fake, fake, fake, fake, fake, 1.0, 1, 64, 2, 64, fake, fake, fake, None) \
        == _lib.FLK_ERR_UNSUPPORTED
    assert lib.flk_attend(fake, fake, fake, 1, 2, 128, 64, fake, None, 0, None) == _lib.FLK_ERR_UNSUPPORTED
    # S not a multiple of 128
    assert lib.flk_attend(fake, fake, fake, 1, 2, 100, 128, fake, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    # negative sizes / bad head count
    assert lib.flk_qk_prep(fake, fake, fake, fake, fake, 1.0, -1, 64, 2, 128, fake, fake, fake, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend(fake, fake, fake, 1, 0, 128, 128, fake, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    # empty problems are a no-op success
    assert lib.flk_qk_prep(fake, fake, fake, fake, fake, 1.0, 0, 64, 2, 128, fake, fake, fake, None) == 0
    assert lib.flk_attend(fake, fake, fake, 1, 2, 0, 128, fake, None, 0, None) == 0
    # misaligned pointer
    odd = ctypes.c_void_p(0x10002)
    assert lib.flk_attend(odd, fake, fake, 1, 2, 128, 128, fake, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    # non-finite gain
    assert lib.flk_qk_prep(fake, fake, fake, fake, fake, float("nan"), 1, 64, 2, 128, fake, fake, fake,
                           None) == _lib.FLK_ERR_INVALID_ARGUMENT
    # qk_prep into a longer sequence: the rows must fit, row0 >= 0
    assert lib.flk_qk_prep_into(fake, fake, fake, fake, fake, 1.0, 1, 64, 2, 128, fake, fake, fake, 100, 37,
                                None) == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_qk_prep_into(fake, fake, fake, fake, fake, 1.0, 1, 64, 2, 128, fake, fake, fake, 100, -1,
                                None) == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_qk_prep_into(fake, fake, fake, fake, fake, 1.0, 1, 64, 2, 64, fake, fake, fake, 100, 0,
                                None) == _lib.FLK_ERR_UNSUPPORTED
    assert lib.flk_qk_prep_into(fake, fake, fake, fake, fake, 1.0, 1, 0, 2, 128, fake, fake, fake, 100, 100,
                                None) == 0
    # gathering attend: 1..8 outputs, heads [h0, h0 + H) inside H_total
    outs = (ctypes.c_void_p * 9)(*([0x10000] * 9))
    assert lib.flk_attend_gather(fake, fake, fake, 1, 2, 128, 128, outs, 0, 4, 0, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_gather(fake, fake, fake, 1, 2, 128, 128, outs, 9, 4, 0, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_gather(fake, fake, fake, 1, 2, 128, 128, outs, 2, 4, 3, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_gather(fake, fake, fake, 1, 2, 128, 128, None, 2, 4, 0, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    odd_outs = (ctypes.c_void_p * 2)(0x10000, 0x10002)
    assert lib.flk_attend_gather(fake, fake, fake, 1, 2, 128, 128, odd_outs, 2, 4, 0, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_gather(fake, fake, fake, 1, 2, 0, 128, outs, 2, 4, 0, None, 0, None) == 0
    # gathering attend through a multicast address: one output pointer, heads inside H_total
    assert lib.flk_attend_gather_multicast(fake, fake, fake, 1, 2, 128, 64, fake, 4, 0, None, 0, None) \
        == _lib.FLK_ERR_UNSUPPORTED
    assert lib.flk_attend_gather_multicast(fake, fake, fake, 1, 2, 128, 128, fake, 4, 3, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_gather_multicast(fake, fake, fake, 1, 2, 128, 128, None, 4, 0, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_gather_multicast(fake, fake, fake, 1, 2, 128, 128, odd, 4, 0, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_gather_multicast(fake, fake, fake, 1, 2, 0, 128, fake, 4, 0, None, 0, None) == 0
    # merged-heads attend: the same shape rules as flk_attend
    assert lib.flk_attend_merged(fake, fake, fake, 1, 2, 128, 64, fake, None, 0, None) == _lib.FLK_ERR_UNSUPPORTED
    assert lib.flk_attend_merged(fake, fake, fake, 1, 2, 100, 128, fake, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_merged(odd, fake, fake, 1, 2, 128, 128, fake, None, 0, None) \
        == _lib.FLK_ERR_INVALID_ARGUMENT


def schedule(b, h, s, sms=148):
    out = (ctypes.c_longlong * 6)()
    assert _lib.lib().flk_attend_schedule(b, h, s, 128, sms, out) == 0
    return tuple(out)


def test_attend_schedule_host_query():
    """The work schedule flk_attend uses (host-only query, no GPU): on a 148-SM B200 the 1024^2
    call keeps its 432 items whole (three waves but for 12 idle SMs, too little to pay for a
    combine), 3 heads split every item in two (one wave), 12 heads keep the first wave whole and
    halve the last 68 items, 13 heads stay whole (the pieces would cost more than the idle SMs),
    7 heads at S=8192 add a second tier of smaller pieces."""
    assert schedule(1, 24, 4608) == (432, 432, 0, 1, 1, 432)
    assert schedule(1, 3, 4608) == (54, 0, 54, 2, 2, 108)
    assert schedule(1, 12, 4608) == (216, 148, 68, 2, 2, 284)
    assert schedule(1, 13, 4608) == (234, 234, 0, 1, 1, 234)
    assert schedule(1, 7, 8192) == (224, 148, 74, 2, 16, 328)
    assert schedule(1, 24, 1536) == (144, 144, 0, 1, 1, 144)
    lib = _lib.lib()
    out = (ctypes.c_longlong * 6)()
    assert lib.flk_attend_schedule(1, 2, 200, 128, 148, out) == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_attend_schedule(1, 2, 256, 64, 148, out) == _lib.FLK_ERR_UNSUPPORTED
    assert lib.flk_attend_schedule(1, 2, 256, 128, 0, out) == _lib.FLK_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("sms", [148, 132, 64])
def test_attend_schedule_invariants(sms):
    """For every shape: whole items fill whole waves (or all items), pieces are at least one KV
    block, and under the persistent kernel's order (unit u on CTA u % sms) no CTA gets more than
    one piece of each tier."""
    for s in (128, 256, 1152, 1536, 4608, 8192, 16896):
        n_tiles = s // 128
        for b, h in ((1, 1), (1, 2), (1, 3), (1, 6), (1, 11), (1, 12), (1, 13), (1, 24), (2, 24), (8, 24)):
            items, whole, n_a, s_a, s_b, units = schedule(b, h, s, sms)
            assert items == b * h * ((n_tiles + 1) // 2)
            rest = items - whole
            assert units == whole + n_a * s_a + (rest - n_a) * s_b
            assert 1 <= s_a <= n_tiles and 1 <= s_b <= n_tiles
            if whole in (0, items):
                continue
            assert whole % sms == 0 and s_a >= 2 and n_a * s_a <= sms
            if rest > n_a:
                assert s_b >= 2 and (rest - n_a) * s_b <= sms
