"""The QKV projection GEMM on the B200: ``linear`` (x @ w, bf16 tensor cores, fp32 accumulation)
against an fp32 reference, and the projection with qk_prep fused into the GEMM's epilogue
against ``linear`` followed by ``qk_prep`` -- bit for bit, since the fused epilogue rounds and
reduces exactly as the two separate kernels do."""
from __future__ import annotations

import math

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import flicker_b200 as fb  # noqa: E402
from flicker_b200 import _lib, projection  # noqa: E402


def rand_bf16(shape, gen, scale=1.0):
    return (torch.randn(*shape, generator=gen, device="cuda") * scale).to(torch.bfloat16)


def tables(length, gen, gain=1.0 / math.sqrt(128)):
    ang = torch.rand(length, 64, generator=gen, device="cuda") * 6.0 - 3.0
    cos = torch.repeat_interleave(torch.cos(ang), 2, dim=-1).contiguous()
    sin = torch.stack([-torch.sin(ang), torch.sin(ang)], -1).reshape(length, 128).contiguous()
    return fb.Freqs(cos, sin, gain)


# (M, N, K): config-1 single block rows x (qkv + mlp) columns, ragged edges, tiny, odd M
@pytest.mark.parametrize("m,n,k", [(4608, 9216, 3072), (300, 520, 136), (1, 16, 8), (257, 1024, 64), (640, 2048, 1024)])
def test_linear_against_fp32(m, n, k):
    g = torch.Generator(device="cuda")
    g.manual_seed(m + n + k)
    x = rand_bf16((m, k), g)
    w = rand_bf16((k, n), g, 0.02)
    y = projection.linear(x, projection.prepare_weight(w))
    ref = x.float() @ w.float()
    err = (y.float() - ref).abs()
    tol = 2e-2 * ref.abs().clamp(min=1.0)
    assert bool((err <= tol).all()), float(err.max())
    # fp32 accumulation then one bf16 rounding: within half a bf16 ulp of the fp32 product plus
    # accumulation-order noise
    rel = (err / ref.abs().clamp(min=1e-3)).median().item()
    assert rel < 4e-3


@pytest.mark.parametrize("b,length,h,extra,row0,s_out", [(1, 512, 4, 0, 0, 512), (2, 384, 3, 640, 0, 384),
                                                           (1, 300, 2, 128, 77, 500), (1, 4096, 24, 0, 512, 4608)])
def test_fused_projection_equals_linear_then_qk_prep(b, length, h, extra, row0, s_out):
    g = torch.Generator(device="cuda")
    g.manual_seed(b * 1000 + length + h)
    k_dim = 256 if h < 24 else 3072
    n = 3 * h * 128 + extra
    x = rand_bf16((b, length, k_dim), g)
    w = rand_bf16((k_dim, n), g, 1.0 / math.sqrt(k_dim))
    wt = projection.prepare_weight(w)
    qs = (torch.rand(128, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
    ks = (torch.rand(128, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
    freqs = tables(length, g)
    outs = tuple(torch.full((b, h, s_out, 128), 3.0, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    q, k, v, rest = projection.qkv_projection(x, wt, qs, ks, freqs, h, out=outs, row=row0)
    qkv = projection.linear(x, wt)
    want = [torch.full_like(o, 3.0) for o in outs]
    fb.qk_prep_into(qkv[..., :3 * h * 128].contiguous(), qs, ks, freqs, h, tuple(want), row0,
                    rows=length if length % 64 else None)
    for got, exp in zip((q, k, v), want):
        assert torch.equal(got, exp)
    if extra:
        assert torch.equal(rest, qkv[..., 3 * h * 128:])
    else:
        assert rest is None
    assert _lib.lib().flk_device_status() == 0


def test_fused_projection_errors():
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    x = rand_bf16((1, 128, 64), g)
    wt = rand_bf16((3 * 2 * 128, 64), g)
    qs = torch.ones(128, dtype=torch.bfloat16, device="cuda")
    freqs = tables(128, g)
    with pytest.raises(ValueError):
        projection.qkv_projection(x, wt, qs, qs, freqs, 3)  # 3 heads need 1152 columns
    with pytest.raises(ValueError):
        projection.qkv_projection(x[..., :60], wt[:, :60], qs, qs, freqs, 2)  # K % 8
    with pytest.raises(ValueError):
        projection.qkv_projection(x, wt, qs, qs, tables(64, g), 2)
    fake = x.data_ptr()
    lib = _lib.lib()
    # M != B * L, rows past S_out, head_dim != 128
    assert lib.flk_linear_qk_prep(fake, fake, 100, 768, 64, fake, fake, fake, fake, 1.0, 1, 128, 2, 128, fake,
                                  fake, fake, 128, 0, None, None) == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_linear_qk_prep(fake, fake, 128, 768, 64, fake, fake, fake, fake, 1.0, 1, 128, 2, 128, fake,
                                  fake, fake, 128, 5, None, None) == _lib.FLK_ERR_INVALID_ARGUMENT
    assert lib.flk_linear_qk_prep(fake, fake, 128, 768, 64, fake, fake, fake, fake, 1.0, 1, 128, 2, 64, fake,
                                  fake, fake, 128, 0, None, None) == _lib.FLK_ERR_UNSUPPORTED
