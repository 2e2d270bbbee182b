"""The attend epilogue's quotient o = acc / l (one correctly rounded reciprocal per row, then
Markstein's FMA correction per element) against __fdiv_rn, bit for bit, on the B200."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from flicker_b200 import _lib  # noqa: E402


def quotients(a, b):
    q_fast, q_ref = torch.empty_like(a), torch.empty_like(a)
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.lib().flk_selftest_quotient(a.data_ptr(), b.data_ptr(), a.numel(), q_fast.data_ptr(),
                                            q_ref.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    return q_fast, q_ref


def log_uniform(n, lo, hi, gen):
    e = torch.rand(n, generator=gen, device="cuda", dtype=torch.float64) * (hi - lo) + lo
    return torch.pow(10.0, e).float()


def special_divisors(gen, n):
    """Divisors whose significand is all ones, 1.0 or 1 + 1 ulp, at random exponents."""
    exps = torch.randint(100, 160, (n,), generator=gen, device="cuda", dtype=torch.int32)
    mant = torch.tensor([0x7FFFFF, 0, 1, 0x7FFFFE, 0x400000], device="cuda", dtype=torch.int32)
    m = mant[torch.randint(0, mant.numel(), (n,), generator=gen, device="cuda")]
    return ((exps << 23) | m).view(torch.float32)


def test_quotient_matches_fdiv_rn():
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    n = 1 << 23
    # accumulators of either sign over a wide range; row sums from tiny to huge, and divisors
    # with extreme significands
    a = log_uniform(n, -25.0, 30.0, g) * torch.where(torch.rand(n, generator=g, device="cuda") < 0.5, -1.0, 1.0)
    b = torch.cat([log_uniform(n - n // 4, -4.0, 8.0, g), special_divisors(g, n // 4)])
    a[:1024] = 0.0
    q_fast, q_ref = quotients(a, b)
    assert torch.equal(q_fast.view(torch.int32), q_ref.view(torch.int32)), int((q_fast != q_ref).sum())


def test_quotient_exact_cases():
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    n = 1 << 20
    # quotients that are exact (a = k * b for small integers k) must come out exact
    b = log_uniform(n, -3.0, 6.0, g)
    k = torch.randint(-4096, 4097, (n,), generator=g, device="cuda").float()
    a = k * b
    exact = (a / b == k) & torch.isfinite(a)
    q_fast, q_ref = quotients(a, b)
    assert torch.equal(q_fast[exact], k[exact])
    assert torch.equal(q_fast.view(torch.int32), q_ref.view(torch.int32))
