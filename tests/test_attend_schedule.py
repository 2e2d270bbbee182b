"""Index arithmetic of the KV-split schedule (CPU, no GPU): the partial rows that the pieces of
split items write (decode_item's pbase in flicker_b200/csrc/attend.cu) and the ones the combine
kernel reads back (combine_splits_kernel's first + s * stride) must be the same rows, each
written exactly once and read in piece order, all inside the s_a (pa1 - pa0) + s_b (pb1 - pa1)
partial rows that attend_workspace_bytes sizes. The schedules come from the library's own rule
(flk_attend_schedule); the formulas below restate attend.cu's."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from flicker_b200 import _lib


def schedule(b, h, s, sms):
    out = (ctypes.c_longlong * 6)()
    assert _lib.lib().flk_attend_schedule(b, h, s, 128, sms, out) == 0
    return tuple(int(x) for x in out)


def item_row(item, n_pairs, s):
    return (item // n_pairs) * s + (item % n_pairs) * 256


def units(b, h, s, sched):
    """decode_item for every unit: (item, split, splits, kv0, n_kv, pbase)."""
    items, n_full, n_a, s_a, s_b, n_units = sched
    n_tiles = s // 128
    n_pairs = (n_tiles + 1) // 2
    pa0, pa1, pb1 = item_row(n_full, n_pairs, s), item_row(n_full + n_a, n_pairs, s), b * h * s
    for w in range(n_units):
        if w < n_full:
            item, split, splits, pbase = w, 0, 1, 0
        elif w - n_full < n_a * s_a:
            u = w - n_full
            item, split, splits = n_full + u // s_a, u % s_a, s_a
            pbase = split * (pa1 - pa0) - pa0
        else:
            u = w - n_full - n_a * s_a
            item, split, splits = n_full + n_a + u // s_b, u % s_b, s_b
            pbase = s_a * (pa1 - pa0) + split * (pb1 - pa1) - pa1
        kv0 = n_tiles * split // splits
        yield item, split, splits, kv0, n_tiles * (split + 1) // splits - kv0, pbase


SHAPES = [(1, 12, 4608), (1, 9, 4608), (1, 7, 8192), (2, 6, 4608), (3, 4, 4480), (1, 3, 4608), (1, 2, 512),
          (2, 1, 1152), (1, 6, 16896), (1, 3, 16896), (1, 24, 4608), (1, 11, 4608), (1, 5, 1536), (2, 3, 384)]


@pytest.mark.parametrize("b,h,s", SHAPES)
@pytest.mark.parametrize("sms", [148, 132])
def test_partial_rows_written_once_and_read_in_piece_order(b, h, s, sms):
    sched = schedule(b, h, s, sms)
    items, n_full, n_a, s_a, s_b, n_units = sched
    n_tiles = s // 128
    n_pairs = (n_tiles + 1) // 2
    rows = b * h * s
    pa0, pa1 = item_row(n_full, n_pairs, s), item_row(n_full + n_a, n_pairs, s)
    slots = s_a * (pa1 - pa0) + s_b * (rows - pa1) if n_full < items else 0
    written = np.full(max(slots, 1), -1, np.int64)  # slot -> (row * 64 + piece)
    kv_seen = {}
    direct = np.zeros(rows, bool)
    for item, split, splits, kv0, n_kv, pbase in units(b, h, s, sched):
        assert 0 <= item < items and n_kv >= 1
        kv_seen.setdefault(item, []).append((kv0, n_kv))
        t0 = (item % n_pairs) * 2
        nt = min(2, n_tiles - t0)
        first_row = (item // n_pairs) * s + t0 * 128
        for grow in range(first_row, first_row + nt * 128):
            if splits == 1:
                assert not direct[grow]
                direct[grow] = True
            else:
                slot = pbase + grow
                assert 0 <= slot < slots
                assert written[slot] == -1, "two pieces write the same partial row"
                written[slot] = grow * 64 + split
    # every item's pieces cover its KV blocks exactly once, in order
    for item, parts in kv_seen.items():
        covered = sorted(parts)
        assert covered[0][0] == 0 and sum(n for _, n in covered) == n_tiles
        assert all(a[0] + a[1] == c[0] for a, c in zip(covered, covered[1:]))
    # rows of whole items are written directly, every other row goes through the combine
    assert direct[:pa0].all() and not direct[pa0:].any()
    if slots == 0:
        return
    assert (written >= 0).all(), "a partial row is never written"
    # combine_splits_kernel: rows [pa0, rows), pieces first + i * stride, i = 0 .. n - 1
    for row in range(pa0, rows, max(1, (rows - pa0) // 997)):
        tier_a = row < pa1
        n = s_a if tier_a else s_b
        first = row - pa0 if tier_a else s_a * (pa1 - pa0) + (row - pa1)
        stride = pa1 - pa0 if tier_a else rows - pa1
        assert [written[first + i * stride] for i in range(n)] == [row * 64 + i for i in range(n)]
