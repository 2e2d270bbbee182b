"""The CPU oracle against golden vectors produced by the reference's own code.

The fixtures in tests/golden/ were made by tests/golden/make_golden.py, which runs
the reference's kernels.qk_prep / kernels.attend / modules.qkv_prep / nn.sdpa /
rope.* / loader.check_logit_bound through a numpy stand-in for jax. These tests pin
oracle/restatement.py to them before any GPU result is compared with the oracle.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import GOLDEN_CASES, load_golden
from oracle import restatement as R


def bits(x):
    return np.asarray(x).astype(R.BF16).view(np.uint16)


def frac_equal(a, b) -> float:
    return float(np.mean(bits(a) == bits(b)))


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_rope_tables_match_reference(name):
    g = load_golden(name)
    gh, gw = (int(x) for x in g["grid"])
    pe = R.joint_pe(gh, gw, int(g["num_txt"]))
    np.testing.assert_array_equal(pe, g["pe"])
    freqs = R.lane_pair(pe, float(g["q_gain"]))
    np.testing.assert_array_equal(freqs.cos, g["cos"])
    np.testing.assert_array_equal(freqs.sin, g["sin"])


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_qk_prep_kernel_restatement_is_bit_exact(name):
    g = load_golden(name)
    freqs = R.Freqs(g["cos"], g["sin"], float(g["q_gain"]))
    q, k, v = R.qk_prep_kernel(g["qkv"], g["q_scale"], g["k_scale"], freqs, int(g["num_heads"]))
    assert frac_equal(q, g["q"]) == 1.0
    assert frac_equal(k, g["k"]) == 1.0
    assert frac_equal(v, g["v"]) == 1.0
    q1, _, _ = R.qk_prep_kernel(g["qkv"], g["q_scale"], g["k_scale"], freqs._replace(q_gain=1.0),
                                int(g["num_heads"]))
    assert frac_equal(q1, g["q_gain1"]) == 1.0


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_xla_path_restatement_is_bit_exact(name):
    g = load_golden(name)
    q, k, v = R.qkv_prep_xla(g["qkv"], g["q_scale"], g["k_scale"], g["pe"], int(g["num_heads"]))
    assert frac_equal(q, g["q_xla"]) == 1.0
    assert frac_equal(k, g["k_xla"]) == 1.0
    assert frac_equal(v, g["v"]) == 1.0


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_attend_restatement_matches_reference(name):
    g = load_golden(name)
    o = R.attend_kernel(g["q"], g["k"], g["v"])
    # fp32 GEMM summation order differs (BLAS blocking); bf16 outputs agree almost everywhere.
    assert frac_equal(o, g["o"]) > 0.99
    assert R.within_tolerance(o, g["o"].astype(np.float32))


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_sdpa_restatement_matches_reference(name):
    g = load_golden(name)
    o = R.sdpa(g["q_xla"], g["k_xla"], g["v"])
    assert frac_equal(o, g["o_xla"]) > 0.99
    assert R.within_tolerance(o, g["o_xla"].astype(np.float32))


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_kernel_path_agrees_with_xla_path(name):
    """The bounded path (gain folded into q, no max) and the plain-XLA path agree within tolerance."""
    g = load_golden(name)
    gain = float(g["q_gain"])
    assert R.within_tolerance(g["q"], g["q_xla"].astype(np.float32) * gain)
    assert R.within_tolerance(g["k"], g["k_xla"])
    assert R.within_tolerance(g["o"], g["o_xla"].astype(np.float32))


def test_logit_bound_matches_reference():
    with np.load(R.__file__.replace("oracle/restatement.py", "tests/golden/logit_bound.npz")) as z:
        cases = {}
        for key in z.files:
            idx, rest = key.split("|", 1)
            cases.setdefault(int(idx), {})[rest] = z[key]
    assert len(cases) == 5
    saw = set()
    for i in sorted(cases):
        c = cases[i]
        blocks = {"double_blocks": {}, "single_blocks": {}}
        for key, val in c.items():
            if "|" in key:
                grp, name = key.split("|", 1)
                blocks[grp][name] = val
        raised = 0
        try:
            R.check_logit_bound(blocks)
        except ValueError:
            raised = 1
        assert raised == int(c["raised"])
        saw.add(raised)
        single = R.logit_bound(blocks["single_blocks"]["norm.query_norm.scale"],
                               blocks["single_blocks"]["norm.key_norm.scale"])
        np.testing.assert_allclose(single, c["single_bound"], rtol=1e-6)
    assert saw == {0, 1}


def test_row_tile_and_errors():
    assert R.row_tile(4608) == 2304
    assert R.row_tile(1536) == 1536
    assert R.row_tile(16896) == 1536
    assert R.row_tile(512) == 512
    assert R.row_tile(100) is None
    qkv = np.zeros((1, 100, 3 * 128), R.BF16)
    f = R.Freqs(np.zeros((100, 128), np.float32), np.zeros((100, 128), np.float32))
    with pytest.raises(ValueError, match="row tile"):
        R.qk_prep_kernel(qkv, np.ones(128, R.BF16), np.ones(128, R.BF16), f, 1)


def test_config_generators_shapes():
    qkv, qs, ks, pe, freqs = R.make_config("512", num_heads=2)
    assert qkv.shape == (1, 1536, 3 * 2 * 128) and qkv.dtype == R.BF16
    assert qs.shape == (128,) and 0.5 <= float(qs.astype(np.float32).min())
    assert pe.shape == (1, 1, 1536, 64, 2, 2)
    assert freqs.cos.shape == (1536, 128) and math.isclose(freqs.q_gain, 1 / math.sqrt(128))
    assert float(R.logit_bound(qs, ks)) < R.EXP_LIMIT
