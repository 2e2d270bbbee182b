"""The fused caller glue on the B200: qk_prep writing into the joint buffers (the double block's
concatenation, src/flicker/modules.py:127-138) and attend storing merged heads (merge_heads,
modules.py:63-65). Both must equal the unfused composition bit for bit, since they only move
where each output row is stored."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import bit_equal_fraction, to_device, to_host
from oracle import restatement as R

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import flicker_b200 as fb  # noqa: E402
from flicker_b200 import _lib  # noqa: E402


def stream_inputs(b, length, h, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    qkv = torch.randn(b, length, 3 * h * 128, generator=g, device="cuda").to(torch.bfloat16)
    qs = torch.empty(128, device="cuda").uniform_(0.5, 1.5, generator=g).to(torch.bfloat16)
    ks = torch.empty(128, device="cuda").uniform_(0.5, 1.5, generator=g).to(torch.bfloat16)
    return qkv, qs, ks


def joint_freqs(num_txt, num_img, gain=1.0 / math.sqrt(128)):
    pe = R.joint_pe(int(math.isqrt(num_img)), int(math.isqrt(num_img)), num_txt)
    f = R.lane_pair(pe, gain)
    return fb.Freqs(to_device(f.cos), to_device(f.sin), f.q_gain)


@pytest.mark.parametrize("num_txt,num_img,h,b", [(512, 4096, 24, 1), (512, 1024, 4, 2), (128, 256, 3, 1)])
def test_double_qk_prep_equals_concatenated_streams(num_txt, num_img, h, b):
    txt, img = stream_inputs(b, num_txt, h, 1), stream_inputs(b, num_img, h, 2)
    freqs = joint_freqs(num_txt, num_img)
    q, k, v = fb.double_qk_prep(txt[0], img[0], txt[1:], img[1:], freqs, h)
    ft = fb.Freqs(freqs.cos[:num_txt], freqs.sin[:num_txt], freqs.q_gain)
    fi = fb.Freqs(freqs.cos[num_txt:], freqs.sin[num_txt:], freqs.q_gain)
    a = fb.qk_prep(txt[0], txt[1], txt[2], ft, h)
    c = fb.qk_prep(img[0], img[1], img[2], fi, h)
    for got, x, y in zip((q, k, v), a, c):
        assert torch.equal(got, torch.cat([x, y], dim=2))


def test_qk_prep_into_ragged_rows_through_c_abi():
    """Odd row offsets and lengths (refused by the row-tile rule of the Python API) through the
    C ABI, against the oracle, with the rows outside the written range left untouched."""
    B, H, S_out = 2, 3, 333
    rng = np.random.default_rng(7)
    outs = [torch.full((B, H, S_out, 128), 7.0, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    pieces = [(0, 77), (77, 129), (206, 101)]  # [row0, row0 + L) tile rows [0, 307)
    for row0, L in pieces:
        qkv = R.bf16(rng.standard_normal((B, L, 3 * H * 128), dtype=np.float32))
        qs = R.bf16(rng.uniform(0.5, 1.5, 128).astype(np.float32))
        ks = R.bf16(rng.uniform(0.5, 1.5, 128).astype(np.float32))
        ang = rng.uniform(-3, 3, (L, 64)).astype(np.float32)
        cos = np.repeat(np.cos(ang), 2, -1).astype(np.float32)
        sin = np.stack([-np.sin(ang), np.sin(ang)], -1).reshape(L, 128).astype(np.float32)
        d = [to_device(x) for x in (qkv, qs, ks, cos, sin)]
        code = _lib.lib().flk_qk_prep_into(*(t.data_ptr() for t in d), 0.5, B, L, H, 128,
                                           *(t.data_ptr() for t in outs), S_out, row0, None)
        assert code == 0
        torch.cuda.synchronize()
        want = R.qk_prep_kernel(qkv, qs, ks, R.Freqs(cos, sin, 0.5), H, rows=L)
        for got, w in zip(outs, want):
            got = to_host(got[:, :, row0:row0 + L])
            assert bit_equal_fraction(got, w) > 0.99
            assert R.within_tolerance_scaled(got, w.astype(np.float32))
    for t in outs:
        assert torch.all(t[:, :, 307:] == 7.0)


def test_qk_prep_into_errors():
    qkv, qs, ks = stream_inputs(1, 128, 2, 3)
    f = joint_freqs(128, 256)
    f = fb.Freqs(f.cos[:128], f.sin[:128], 1.0)
    out = tuple(torch.empty(1, 2, 200, 128, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    with pytest.raises(ValueError):
        fb.qk_prep_into(qkv, qs, ks, f, 2, out, 100)  # rows [100, 228) do not fit in 200
    with pytest.raises(ValueError):
        fb.qk_prep_into(qkv, qs, ks, f, 2, out[:2], 0)
    bad = (out[0], out[1], torch.empty(1, 3, 200, 128, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(ValueError):
        fb.qk_prep_into(qkv, qs, ks, f, 2, bad, 0)
    fake = out[0].data_ptr()
    assert _lib.lib().flk_qk_prep_into(fake, fake, fake, fake, fake, 1.0, 1, 128, 2, 128, fake, fake, fake,
                                       200, 73, None) == _lib.FLK_ERR_INVALID_ARGUMENT


def random_qkv(b, h, s, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = (torch.randn(b, h, s, 128, generator=g, device="cuda") / math.sqrt(128)).to(torch.bfloat16)
    k = torch.randn(b, h, s, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(b, h, s, 128, generator=g, device="cuda").to(torch.bfloat16)
    return q, k, v


# (1, 24, 4608) runs unsplit; (1, 2, 1024) and (2, 3, 512) run split over KV with the combine
# kernel storing the merged rows.
@pytest.mark.parametrize("b,h,s", [(1, 24, 4608), (1, 2, 1024), (2, 3, 512), (2, 5, 384)])
def test_attend_merged_equals_merge_heads(b, h, s):
    q, k, v = random_qkv(b, h, s, b * 100 + h)
    o = fb.attend_merged(q, k, v)
    ref = fb.attend(q, k, v)
    assert o.shape == (b, s, h * 128)
    assert torch.equal(o, ref.transpose(1, 2).reshape(b, s, h * 128))


def test_double_block_attention_against_oracle():
    """Joint q, k, v of a small double block (text + image streams) -> merged attention output,
    against the oracle's plain-XLA path (per-stream norm + RoPE on the concatenation, sdpa,
    merge_heads) on sampled rows."""
    num_txt, num_img, h = 128, 256, 2
    txt, img = stream_inputs(1, num_txt, h, 11), stream_inputs(1, num_img, h, 12)
    freqs = joint_freqs(num_txt, num_img)
    q, k, v = fb.double_qk_prep(txt[0], img[0], txt[1:], img[1:], freqs, h)
    o = to_host(fb.attend_merged(q, k, v))
    pe = R.joint_pe(16, 16, num_txt)
    parts = []
    for (qkv, qs, ks), pe_s in ((txt, pe[:, :, :num_txt]), (img, pe[:, :, num_txt:])):
        parts.append(R.qkv_prep_xla(to_host(qkv), to_host(qs), to_host(ks), pe_s, h))
    # the XLA path scales q by 1/sqrt(D) inside sdpa; the kernel path folds it in as q_gain
    qx = np.concatenate([parts[0][0], parts[1][0]], axis=2)
    kx = np.concatenate([parts[0][1], parts[1][1]], axis=2)
    vx = np.concatenate([parts[0][2], parts[1][2]], axis=2)
    want = R.merge_heads(R.sdpa(qx, kx, vx))
    assert R.within_tolerance(o, want.astype(np.float32))
