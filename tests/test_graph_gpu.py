"""The API inside a CUDA graph: qk_prep + attend (and the fused double-block section) captured
once and replayed with new inputs give exactly the eager calls' results.

A serving loop replays a captured forward instead of re-entering Python for every launch (the
API's host cost is ~15-20 us per call, more than the GPU time of a 512^2 attention call). The
calls capture cleanly: no allocation outside torch's caching allocator, no synchronisation, the
attention kernel's programmatic (PDL) launch becomes a programmatic edge of the graph. The one
requirement is a first, eager call per device and shape family before capturing (it queries
the device and sets kernel attributes).
"""
from __future__ import annotations

import math

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import flicker_b200 as fb  # noqa: E402


def tables(length, gen):
    ang = torch.rand(length, 64, generator=gen, device="cuda") * 6.0 - 3.0
    cos = torch.repeat_interleave(torch.cos(ang), 2, dim=-1).contiguous()
    sin = torch.stack([-torch.sin(ang), torch.sin(ang)], -1).reshape(length, 128).contiguous()
    return fb.Freqs(cos, sin, 1.0 / math.sqrt(128))


def inputs(b, length, h, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    qkv = torch.randn(b, length, 3 * h * 128, generator=g, device="cuda").to(torch.bfloat16)
    qs = (torch.rand(128, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
    ks = (torch.rand(128, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
    return qkv, qs, ks, tables(length, g)


def capture(fn, *static_args):
    """Warm up on a side stream (torch's recipe), then capture fn(*static_args) in a graph."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn(*static_args)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fn(*static_args)
    return graph, out


# the 1024^2 call (432 persistent work items), and 3 heads at S=4608 (split over KV: the combine
# kernel and a workspace from the graph's memory pool)
@pytest.mark.parametrize("b,length,h", [(1, 4608, 24), (1, 4608, 3)])
def test_qk_prep_attend_graph_replays_match_eager(b, length, h):
    qkv, qs, ks, freqs = inputs(b, length, h, 1)

    def step(x):
        q, k, v = fb.qk_prep(x, qs, ks, freqs, h)
        return fb.attend(q, k, v)

    static_qkv = qkv.clone()
    graph, out = capture(step, static_qkv)
    for seed in (2, 3):
        fresh = inputs(b, length, h, seed)[0]
        static_qkv.copy_(fresh)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, step(fresh))
    for _ in range(50):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, step(static_qkv))
    assert fb.device_status() == 0


def test_double_block_section_graph():
    """Both streams' qk_prep written into the joint buffers, then attention with merged heads."""
    h, num_txt, num_img = 24, 512, 1024
    txt, qs_t, ks_t, _ = inputs(1, num_txt, h, 4)
    img, qs_i, ks_i, _ = inputs(1, num_img, h, 5)
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    freqs = tables(num_txt + num_img, g)

    def section(t, i):
        q, k, v = fb.double_qk_prep(t, i, (qs_t, ks_t), (qs_i, ks_i), freqs, h)
        return fb.attend_merged(q, k, v)

    st, si = txt.clone(), img.clone()
    graph, out = capture(section, st, si)
    st.copy_(inputs(1, num_txt, h, 7)[0])
    si.copy_(inputs(1, num_img, h, 8)[0])
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, section(st, si))
    assert fb.device_status() == 0
