"""qk_prep on the B200 against the oracle and the reference-code golden vectors (through the C ABI)."""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

from conftest import GOLDEN_CASES, bit_equal_fraction, load_golden, to_device, to_host
from oracle import restatement as R

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import flicker_b200 as fb  # noqa: E402
from flicker_b200 import _lib  # noqa: E402


def run_qk_prep(qkv, q_scale, k_scale, cos, sin, gain, heads):
    f = fb.Freqs(to_device(cos), to_device(sin), gain)
    q, k, v = fb.qk_prep(to_device(qkv), to_device(q_scale), to_device(k_scale), f, heads)
    torch.cuda.synchronize()
    return to_host(q), to_host(k), to_host(v)


@pytest.mark.parametrize("name", GOLDEN_CASES)
@pytest.mark.parametrize("gain_key", ["q", "q_gain1"])
def test_golden(name, gain_key):
    g = load_golden(name)
    gain = float(g["q_gain"]) if gain_key == "q" else 1.0
    q, k, v = run_qk_prep(g["qkv"], g["q_scale"], g["k_scale"], g["cos"], g["sin"], gain,
                          int(g["num_heads"]))
    assert bit_equal_fraction(v, g["v"]) == 1.0
    # Only the fp32 sum-of-squares order differs from the reference body: near bit-exact.
    assert bit_equal_fraction(q, g[gain_key]) > 0.995
    assert bit_equal_fraction(k, g["k"]) > 0.995
    assert R.within_tolerance_scaled(q, g[gain_key].astype(np.float32))
    assert R.within_tolerance_scaled(k, g["k"].astype(np.float32))
    # ... and the plain-XLA path of the reference (gain folded into q).
    assert R.within_tolerance_scaled(q, g["q_xla"].astype(np.float32) * gain)
    assert R.within_tolerance_scaled(k, g["k_xla"].astype(np.float32))


@pytest.mark.parametrize("config", ["512", "1024"])
def test_config_full_size(config):
    qkv, qs, ks, pe, freqs = R.make_config(config)
    q, k, v = run_qk_prep(qkv, qs, ks, freqs.cos, freqs.sin, freqs.q_gain, R.NUM_HEADS)
    wq, wk, wv = R.qk_prep_kernel(qkv, qs, ks, freqs, R.NUM_HEADS)
    assert bit_equal_fraction(v, wv) == 1.0
    assert bit_equal_fraction(q, wq) > 0.995 and bit_equal_fraction(k, wk) > 0.995
    assert R.within_tolerance_scaled(q, wq.astype(np.float32))
    assert R.within_tolerance_scaled(k, wk.astype(np.float32))
    xq, xk, _ = R.qkv_prep_xla(qkv, qs, ks, pe, R.NUM_HEADS)
    assert R.within_tolerance_scaled(q, xq.astype(np.float32) * freqs.q_gain)
    assert R.within_tolerance_scaled(k, xk.astype(np.float32))


def test_batch8_seeds_independent():
    """Config 2's batch: element b is the single-batch result for seed b."""
    qkv = R.make_qkv(3, 512, num_heads=2, seed=0)
    qs, ks = R.make_scales()
    pe = R.joint_pe(16, 16, 256)
    f = R.lane_pair(pe, 1 / math.sqrt(128))
    q, k, v = run_qk_prep(qkv, qs, ks, f.cos, f.sin, f.q_gain, 2)
    for b in range(3):
        one = R.make_qkv(1, 512, num_heads=2, seed=b)
        q1, k1, v1 = run_qk_prep(one, qs, ks, f.cos, f.sin, f.q_gain, 2)
        assert bit_equal_fraction(q[b:b + 1], q1) == 1.0
        assert bit_equal_fraction(v[b:b + 1], v1) == 1.0


@pytest.mark.parametrize("B,L,H", [(2, 77, 3), (1, 1, 1), (3, 130, 5), (1, 64, 8)])
def test_ragged_shapes_through_c_abi(B, L, H):
    """Shapes the Python API's row-tile rule refuses still work through the C ABI."""
    rng = np.random.default_rng(B * 1000 + L * 10 + H)
    qkv = R.bf16(rng.standard_normal((B, L, 3 * H * 128), dtype=np.float32))
    qs = R.bf16(rng.uniform(0.5, 1.5, 128).astype(np.float32))
    ks = R.bf16(rng.uniform(0.5, 1.5, 128).astype(np.float32))
    ang = rng.uniform(-3, 3, (L, 64)).astype(np.float32)
    cos = np.repeat(np.cos(ang), 2, -1).astype(np.float32)
    sin = np.stack([-np.sin(ang), np.sin(ang)], -1).reshape(L, 128).astype(np.float32)
    d = [to_device(a) for a in (qkv, qs, ks, cos, sin)]
    outs = [torch.empty((B, H, L, 128), dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    code = _lib.lib().flk_qk_prep(*(t.data_ptr() for t in d), 0.25, B, L, H, 128,
                                  *(t.data_ptr() for t in outs), None)
    assert code == 0
    torch.cuda.synchronize()
    want = R.qk_prep_kernel(qkv, qs, ks, R.Freqs(cos, sin, 0.25), H, rows=L)
    for got, w in zip(outs, want):
        got = to_host(got)
        assert bit_equal_fraction(got, w) > 0.99
        assert R.within_tolerance_scaled(got, w.astype(np.float32))


def test_deterministic_and_stream_ordered():
    qkv, qs, ks, pe, freqs = R.make_config("512")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = run_qk_prep(qkv, qs, ks, freqs.cos, freqs.sin, freqs.q_gain, R.NUM_HEADS)
    b = run_qk_prep(qkv, qs, ks, freqs.cos, freqs.sin, freqs.q_gain, R.NUM_HEADS)
    for x, y in zip(a, b):
        assert bit_equal_fraction(x, y) == 1.0


def test_api_errors_on_device():
    qkv = torch.zeros(1, 100, 3 * 128, dtype=torch.bfloat16, device="cuda")
    f = fb.Freqs(torch.zeros(100, 128, device="cuda"), torch.zeros(100, 128, device="cuda"))
    s = torch.ones(128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="row tile"):
        fb.qk_prep(qkv, s, s, f, 1)
    qkv = torch.zeros(1, 128, 3 * 2 * 64, dtype=torch.bfloat16, device="cuda")
    f = fb.Freqs(torch.zeros(128, 64, device="cuda"), torch.zeros(128, 64, device="cuda"))
    with pytest.raises(ValueError, match="head_dim"):
        fb.qk_prep(qkv, s[:64], s[:64], f, 2)
    with pytest.raises(ValueError, match="width"):
        fb.qk_prep(torch.zeros(1, 128, 1000, dtype=torch.bfloat16, device="cuda"), s, s, f, 2)
    assert fb.device_status() == 0
