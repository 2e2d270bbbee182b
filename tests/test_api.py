"""Host-side behaviour of the flicker_b200.kernels API that needs no GPU: the reference's
error conventions and the absence of any CPU fallback."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import flicker_b200 as fb
from flicker_b200 import kernels, loader, rope
from oracle import restatement as R


def test_constants_match_reference():
    assert fb.EPS == 1e-6
    assert fb.ROW_TILES == (2304, 1536, 1152, 512, 256, 128, 64)
    assert fb.SCORE_TILES == (2304, 1536, 1152, 512, 256, 128)
    assert fb.EXP_LIMIT == 80.0
    for n in (64, 100, 128, 1536, 4608, 16896, 4096, 512):
        assert fb.row_tile(n) == R.row_tile(n)


def test_no_cpu_fallback():
    qkv = torch.zeros(1, 128, 3 * 128, dtype=torch.bfloat16)
    f = fb.Freqs(torch.zeros(128, 128), torch.zeros(128, 128))
    s = torch.ones(128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        fb.qk_prep(qkv, s, s, f, 1)
    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        fb.attend(q, q, q)
    with pytest.raises(NotImplementedError):
        fb.attend(q, q, q, interpret=True)
    with pytest.raises(NotImplementedError):
        fb.qk_prep(qkv, s, s, f, 1, interpret=True)


def test_lane_pair_matches_oracle():
    pe = R.joint_pe(4, 8, 32)
    want = R.lane_pair(pe, 0.5)
    got = fb.lane_pair(torch.from_numpy(pe), 0.5)
    np.testing.assert_array_equal(got.cos.numpy(), want.cos)
    np.testing.assert_array_equal(got.sin.numpy(), want.sin)
    assert got.q_gain == 0.5


def test_lane_pair_rotation_equals_apply_rope():
    """kernels.py:47-48 lane-pair rotation == rope.py:24-31 2x2 rotation (survey 4.2)."""
    rng = np.random.default_rng(3)
    pe = R.joint_pe(4, 4, 16)
    x = rng.standard_normal((1, 1, 32, 128)).astype(np.float32)
    f = R.lane_pair(pe)
    even = (np.arange(128) % 2) == 0
    swap = np.where(even, np.roll(x, 127, -1), np.roll(x, 1, -1))
    lane = f.cos * x + f.sin * swap
    pairs = x.reshape(1, 1, 32, 64, 1, 2)
    rot = (pe[..., 0] * pairs[..., 0] + pe[..., 1] * pairs[..., 1]).reshape(x.shape)
    np.testing.assert_allclose(lane, rot, rtol=0, atol=1e-6)


def test_torch_rope_tables_match_oracle():
    pe = rope.joint_pe(16, 4, 8)
    want = R.joint_pe(4, 8, 16)
    np.testing.assert_allclose(pe.numpy(), want, rtol=0, atol=2e-6)


def test_logit_bound_api_and_guard():
    qs = np.full(128, 1.5, np.float32)
    ks = np.full(128, 1.5, np.float32)
    assert math.isclose(float(fb.logit_bound(qs, ks)), math.sqrt(128) * 2.25, rel_tol=1e-6)
    t = fb.logit_bound(torch.from_numpy(qs), torch.from_numpy(ks))
    assert math.isclose(float(t), math.sqrt(128) * 2.25, rel_tol=1e-6)
    ok = {"double_blocks": {f"{s}_attn.norm.{n}.scale": np.ones((5, 128), np.float32)
                            for s in ("img", "txt") for n in ("query_norm", "key_norm")},
          "single_blocks": {f"norm.{n}.scale": np.ones((20, 128), np.float32)
                            for n in ("query_norm", "key_norm")}}
    loader.check_logit_bound(ok)
    bad = {**ok, "single_blocks": {**ok["single_blocks"],
                                   "norm.key_norm.scale": np.full((20, 128), 8.0, np.float32)}}
    with pytest.raises(ValueError, match="bounded"):
        loader.check_logit_bound(bad)
    bad2 = {**ok, "double_blocks": {**ok["double_blocks"],
                                    "txt_attn.norm.query_norm.scale": np.full((5, 128), -9.0, np.float32)}}
    with pytest.raises(ValueError, match="bounded"):
        loader.check_logit_bound(bad2)
