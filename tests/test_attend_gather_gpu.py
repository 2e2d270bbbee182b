"""The gathering attend epilogue on one B200: shards of heads, each call storing its heads'
merged rows into several output buffers (on one GPU here; on a node, this GPU's and its peers'
buffers). After all shards have run, every buffer must equal merge_heads(attend) over all
heads bit for bit (the stores only change where rows go)."""
from __future__ import annotations

import ctypes
import math

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import flicker_b200 as fb  # noqa: E402
from flicker_b200 import _lib  # noqa: E402


def random_qkv(b, h, s, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = (torch.randn(b, h, s, 128, generator=g, device="cuda") / math.sqrt(128)).to(torch.bfloat16)
    k = torch.randn(b, h, s, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(b, h, s, 128, generator=g, device="cuda").to(torch.bfloat16)
    return q, k, v


def gather_call(q, k, v, outs, h_total, h0):
    b, h, s, d = q.shape
    lib = _lib.lib()
    ws_bytes = lib.flk_attend_workspace_size(b, h, s, d)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda") if ws_bytes else None
    ptrs = (ctypes.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
    code = lib.flk_attend_gather(q.data_ptr(), k.data_ptr(), v.data_ptr(), b, h, s, d, ptrs, len(outs), h_total,
                                 h0, ws.data_ptr() if ws is not None else None, ws_bytes,
                                 torch.cuda.current_stream().cuda_stream)
    assert code == 0, code


# On 148 SMs: (24 heads in 2 shards of 12) and (14 at S=8192 in 2 of 7) run tiered (the first wave
# of items whole, stored by the attention epilogue; the rest split over KV, stored by the combine
# kernel);
# (8 heads in 4 shards of 2) and (6 in 3 of 2, B=2) run split over KV, so the combine kernel does
# all the gathering stores; (32 heads in 2 shards of 16) runs unsplit.
@pytest.mark.parametrize("b,h,s,shards", [(1, 24, 4608, 2), (1, 14, 8192, 2), (1, 8, 1024, 4), (2, 6, 512, 3),
                                          (1, 32, 2048, 2)])
def test_shards_gathered_into_every_buffer(b, h, s, shards):
    """Each shard's heads land at their columns of every buffer, exactly as the shard's own
    merged attention (a shard may run with a different KV split count than the full call, so the
    comparison with the all-heads call is within the attention tolerance, not bit for bit)."""
    q, k, v = random_qkv(b, h, s, h * 7 + shards)
    outs = [torch.full((b, s, h * 128), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(shards)]
    per = h // shards
    want = torch.empty((b, s, h, 128), dtype=torch.bfloat16, device="cuda")
    for r in range(shards):
        sl = slice(r * per, (r + 1) * per)
        qs, ks, vs = q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous()
        gather_call(qs, ks, vs, outs, h, r * per)
        want[:, :, sl] = fb.attend_merged(qs, ks, vs).view(b, s, per, 128)
    torch.cuda.synchronize()
    want = want.view(b, s, h * 128)
    for o in outs:
        assert torch.equal(o, want)
    full = fb.attend_merged(q, k, v).float()
    err = (outs[0].float() - full).abs().max().item()
    assert err <= 2e-2


# attend_merged runs the persistent kernel, while a gathering call into two local buffers runs
# the one-item-per-CTA kernel with its TMA-staged epilogue whenever some items are whole:
# (1, 24, 4608) is 432 items on 148 CTAs, (2, 24, 1536) 288 items, (3, 2, 128) single-tile items,
# (2, 24, 1152) nine tiles per head (items of two and of one query tile mixed); (1, 12, 4608) and
# (1, 7, 8192) run tiered on 148 SMs (whole items, then pieces whose partials the combine adds).
@pytest.mark.parametrize("b,h,s", [(1, 24, 4608), (2, 24, 1536), (3, 2, 128), (1, 16, 2048), (2, 24, 1152),
                                   (1, 12, 4608), (1, 7, 8192)])
def test_attend_persistent_matches(b, h, s):
    """The persistent kernel (units walked by one CTA per SM, barriers counting across units)
    computes exactly what one CTA per unit computes: bit-identical outputs."""
    q, k, v = random_qkv(b, h, s, b * 100 + h + s)
    lib = _lib.lib()
    persistent = fb.attend_merged(q, k, v)
    outs = [torch.full((b, s, h * 128), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    gather_call(q, k, v, outs, h, 0)
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, persistent)
    assert lib.flk_device_status() == 0
