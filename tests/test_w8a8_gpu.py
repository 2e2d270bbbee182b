"""W8A8 SmoothQuant linear on the B200 against the oracle (oracle/smoothquant.py), through the C ABI.

Bars: int8 codes and fp32 scales bit-exact; int32 accumulators bit-exact (checked against a
float64 matmul, which is exact here: |acc| <= K * 127^2 < 2^53); bf16 outputs bit-exact to the
oracle's dequantisation of those accumulators. Parity against flicker itself is unpinned (it has
no int8 path); the error against the bf16 x @ w is reported as information.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import to_device, to_host
from oracle import smoothquant as SQ

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from flicker_b200 import w8a8  # noqa: E402


def exact_acc(xq, wq, rows=None):
    a = xq.astype(np.float64) if rows is None else xq[rows].astype(np.float64)
    return (a @ wq.astype(np.float64).T).astype(np.int64)


def dev_i8(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("m,k,n", [(256, 384, 512), (200, 208, 300), (128, 128, 256), (1, 16, 1),
                                   (4608, 3072, 9216)])
def test_pipeline_bit_exact(m, k, n):
    x, w = SQ.make_inputs(m, k, n, seed=m + k + n)
    s, inv_s, xq, sx, wq, sw = SQ.prepare(x, w)
    if k % 8 == 0:
        gq, gsx = w8a8.quantize_act(to_device(x), to_device(inv_s))
        np.testing.assert_array_equal(gq.cpu().numpy(), xq)
        np.testing.assert_array_equal(gsx.cpu().numpy().view(np.uint32), sx.view(np.uint32))
    gwq, gsw = w8a8.quantize_weight(to_device(w), to_device(s))
    np.testing.assert_array_equal(gwq.cpu().numpy(), wq)
    np.testing.assert_array_equal(gsw.cpu().numpy().view(np.uint32), sw.view(np.uint32))
    a, b = dev_i8(xq), dev_i8(wq)
    acc = w8a8.gemm_s32(a, b)
    y = w8a8.gemm(a, b, to_device(sx), to_device(sw))
    torch.cuda.synchronize()
    rows = np.arange(m) if m * n * k <= 2 ** 28 else np.sort(np.random.default_rng(0).choice(m, 96, replace=False))
    want = exact_acc(xq, wq, rows)
    got = acc.cpu().numpy()[rows]
    np.testing.assert_array_equal(got, want)
    yw = SQ.dequant(want, sx[rows], sw)
    np.testing.assert_array_equal(to_host(y)[rows].view(np.uint16), yw.view(np.uint16))


@pytest.mark.parametrize("m,k,n", [(300, 400, 600), (520, 272, 1300), (256, 128, 700)])
def test_full_accumulator_tile_columns_and_tail(m, k, n):
    """Every output element of multi-tile ragged shapes checked (tails in M, N and K; several
    256 x 256 pair tiles per row and column, the last ones mostly past M or N)."""
    rng = np.random.default_rng(1)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    b = rng.integers(-127, 128, (n, k), dtype=np.int8)
    got = w8a8.gemm_s32(dev_i8(a), dev_i8(b)).cpu().numpy()
    np.testing.assert_array_equal(got, exact_acc(a, b))


def test_extreme_codes_do_not_overflow():
    """All codes at +-127 with K = 3072: |acc| = 49.5e6, far inside int32."""
    m, k, n = 128, 3072, 256
    a = np.full((m, k), 127, np.int8)
    b = np.full((n, k), -127, np.int8)
    got = w8a8.gemm_s32(dev_i8(a), dev_i8(b)).cpu().numpy()
    assert (got == -127 * 127 * k).all()


def test_layer_against_bf16_linear_is_close():
    """Information: the quantised layer against the bf16 x @ w of the same operands (config 4)."""
    x, w = SQ.make_inputs(seed=4)
    xd, wd = to_device(x), to_device(w)
    layer = w8a8.SmoothQuantLinear.from_float(wd, xd.float().abs().amax(dim=0))
    y = layer(xd).float()
    ref = xd.float() @ wd.float()
    rel = ((y - ref).norm() / ref.norm()).item()
    print(f"W8A8 vs bf16 linear: relative Frobenius error {rel:.4f}")
    assert rel < 0.05
    from flicker_b200 import _lib
    assert _lib.lib().flk_device_status() == 0


def test_errors():
    a = torch.zeros(16, 24, dtype=torch.int8, device="cuda")
    with pytest.raises(ValueError, match="multiple of 16"):
        w8a8.gemm(a, a, torch.ones(16, device="cuda"), torch.ones(16, device="cuda"))
    with pytest.raises(ValueError, match="CUDA"):
        w8a8.quantize_act(torch.zeros(4, 8, dtype=torch.bfloat16), torch.ones(8))


@pytest.mark.parametrize("m,k", [(64, 8), (33, 1000), (11, 1536), (17, 2056), (7, 3072), (9, 4096), (5, 4104)])
def test_quantize_act_widths(m, k):
    """Every row-width branch of the activation quantiser (register-held rows and the two-pass kernel)."""
    rng = np.random.default_rng(k)
    x = SQ.BF16 and rng.standard_normal((m, k)).astype(np.float32).astype(SQ.BF16)
    inv_s = rng.uniform(0.2, 3.0, k).astype(np.float32)
    want_q, want_s = SQ.quantize_act(x, inv_s)
    gq, gs = w8a8.quantize_act(to_device(x), to_device(inv_s))
    np.testing.assert_array_equal(gq.cpu().numpy(), want_q)
    np.testing.assert_array_equal(gs.cpu().numpy().view(np.uint32), want_s.view(np.uint32))


def test_quantize_ties_and_near_ties():
    """Quotients x'/scale exactly on, and a few ulps either side of, every half-integer k + 0.5:
    the codes must still round half to even exactly as numpy's float32 division does."""
    m, k = 6, 1024
    rng = np.random.default_rng(5)
    x = np.ones((m, k), dtype=np.float32).astype(SQ.BF16)
    inv_s = np.empty((m, k), dtype=np.float32)
    for r in range(m):
        amax = np.float32(rng.uniform(0.01, 50.0))
        scale = np.float32(amax / np.float32(127.0))
        inv_s[r, 0] = amax  # x'[r, 0] = 1 * amax sets the row's absmax
        for j in range(1, k):
            target = np.float32((j % 127 + 0.5) * np.float64(scale))
            step = (j // 127) % 7 - 3  # -3 .. 3 ulps around the tie
            for _ in range(abs(step)):
                target = np.nextafter(target, np.float32(np.inf if step > 0 else -np.inf), dtype=np.float32)
            inv_s[r, j] = -target if j % 2 else target
    # one inv_smooth vector per row: quantise each row on its own
    for r in range(m):
        want_q, want_s = SQ.quantize_act(x[r:r + 1], inv_s[r])
        gq, gs = w8a8.quantize_act(to_device(x[r:r + 1]), to_device(inv_s[r]))
        np.testing.assert_array_equal(gs.cpu().numpy().view(np.uint32), want_s.view(np.uint32))
        np.testing.assert_array_equal(gq.cpu().numpy(), want_q)
