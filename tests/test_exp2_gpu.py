"""The attend kernel's two exponentials against float64, on the B200.

kernels.attend computes p = exp(s) (src/flicker/kernels.py:124) as 2^(s * log2(e)); three of
every four values come from ex2.approx on the SFU and one from a degree-4 minimax polynomial on
the FMA pipe (derived by flicker_b200/csrc/exp2_poly.py: relative error 3.6e-6 in fp32 Horner).
The bounded-logit check keeps |s| < 80, i.e. |x| < 80 * log2(e) < 116, so the sweep covers
[-116, 116] densely plus the integers and half-integers, where the polynomial's range reduction
switches.
"""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from flicker_b200 import _lib  # noqa: E402

POLY_REL_BOUND = 4e-6       # the polynomial's stated 3.6e-6 plus the final scaling's rounding
MUFU_REL_BOUND = 2.0 ** -21  # ex2.approx


def exps(x):
    poly, mufu = torch.empty_like(x), torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.lib().flk_selftest_exp2(x.data_ptr(), x.numel(), poly.data_ptr(), mufu.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    return poly, mufu


def rel_err(got, x):
    want = torch.exp2(x.double())
    return ((got.double() - want).abs() / want).max().item()


def test_exp2_dense_sweep_within_bounds():
    n = (1 << 24) + 1
    x = torch.linspace(-116.0, 116.0, n, device="cuda", dtype=torch.float64).float()
    poly, mufu = exps(x)
    assert rel_err(poly, x) <= POLY_REL_BOUND
    assert rel_err(mufu, x) <= MUFU_REL_BOUND


def test_exp2_range_reduction_edges():
    """Integers, half-integers and their float neighbours: where rint() and the exponent add switch."""
    base = torch.arange(-232, 233, device="cuda", dtype=torch.float32) * 0.5
    up = torch.nextafter(base, torch.full_like(base, 1e9))
    down = torch.nextafter(base, torch.full_like(base, -1e9))
    x = torch.cat([base, up, down])
    poly, mufu = exps(x)
    assert rel_err(poly, x) <= POLY_REL_BOUND
    assert rel_err(mufu, x) <= MUFU_REL_BOUND
    ints = base[base == base.round()]
    p_int, _ = exps(ints)
    assert torch.equal(p_int.double(), torch.exp2(ints.double()))  # p(0) = 1 exactly: 2^n is exact


def test_exp2_random_logits():
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    s = (torch.rand(1 << 22, generator=g, device="cuda") * 2 - 1) * 80.0  # logits within the bound
    x = s * 1.4426950408889634
    poly, mufu = exps(x)
    assert rel_err(poly, x) <= POLY_REL_BOUND
    assert rel_err(mufu, x) <= MUFU_REL_BOUND
