"""Generate the golden vectors in this folder by running the REFERENCE's own code.

Run (in a container that has the reference source; the GPU box does not need it):

    python tests/golden/make_golden.py [--reference-src <path to flicker's src/>]

jax is not installable here, so ``jax_stand_in.install()`` first registers a
numpy stand-in for the jax names the reference uses (see that module for what
it maps and what it cannot pin). The script then imports the reference's
``flicker.kernels``, ``flicker.modules``, ``flicker.nn``, ``flicker.rope`` and
``flicker.loader`` unmodified and records, for small seeded inputs:

* the RoPE tables: ``rope.embed_nd`` of text + image ids, ``kernels.lane_pair``;
* ``kernels.qk_prep`` (the Pallas body executed by the stand-in grid walker),
  with q_gain = 1/sqrt(D) and with q_gain = 1;
* ``kernels.attend`` on those q, k, v;
* the plain-XLA path ``modules.qkv_prep(..., freqs=None)`` + ``nn.sdpa``;
* ``kernels.logit_bound`` / ``loader.check_logit_bound`` outcomes.

bf16 arrays are stored as their uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import ml_dtypes
import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BF16 = ml_dtypes.bfloat16


def bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x).astype(BF16)).view(np.uint16)


def case(ref, name: str, num_heads: int, num_txt: int, grid_h: int, grid_w: int, seed: int):
    kernels, modules, nn, rope = ref["kernels"], ref["modules"], ref["nn"], ref["rope"]
    head_dim = 128
    length = num_txt + grid_h * grid_w
    rng = np.random.Generator(np.random.PCG64(seed))
    qkv = rng.standard_normal((1, length, 3 * num_heads * head_dim), dtype=np.float32).astype(BF16)
    srng = np.random.Generator(np.random.PCG64(seed + 1))
    q_scale = srng.uniform(0.5, 1.5, head_dim).astype(np.float32).astype(BF16)
    k_scale = srng.uniform(0.5, 1.5, head_dim).astype(np.float32).astype(BF16)

    # src/flicker/dit.py:44-47
    pe = np.concatenate([rope.embed_nd(rope.txt_ids(num_txt)),
                         rope.embed_nd(rope.img_ids(grid_h, grid_w))], axis=2)
    q_gain = 1.0 / math.sqrt(head_dim)
    freqs = kernels.lane_pair(pe, q_gain)
    freqs1 = kernels.lane_pair(pe, 1.0)

    q, k, v = kernels.qk_prep(qkv, q_scale, k_scale, freqs, num_heads)
    q1, _, _ = kernels.qk_prep(qkv, q_scale, k_scale, freqs1, num_heads)
    o = kernels.attend(q, k, v)
    qx, kx, vx = modules.qkv_prep(qkv, q_scale, k_scale, pe, None, num_heads)
    ox = nn.sdpa(qx, kx, vx)
    assert np.array_equal(bits(v), bits(vx))
    out = dict(
        qkv=bits(qkv), q_scale=bits(q_scale), k_scale=bits(k_scale),
        pe=np.asarray(pe, np.float32), cos=np.asarray(freqs.cos, np.float32),
        sin=np.asarray(freqs.sin, np.float32), q_gain=np.float32(q_gain),
        num_heads=np.int32(num_heads), num_txt=np.int32(num_txt),
        grid=np.array([grid_h, grid_w], np.int32),
        q=bits(q), k=bits(k), v=bits(v), o=bits(o), q_gain1=bits(q1),
        q_xla=bits(qx), k_xla=bits(kx), o_xla=bits(ox),
    )
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: S={length} H={num_heads}")


def bound_cases(ref):
    kernels, loader = ref["kernels"], ref["loader"]
    rng = np.random.Generator(np.random.PCG64(7))
    rows = []
    for i, hi in enumerate((1.5, 2.0, 2.5, 2.6, 3.0)):
        blocks = {"double_blocks": {}, "single_blocks": {}}
        for s in ("img", "txt"):
            for n in ("query_norm", "key_norm"):
                blocks["double_blocks"][f"{s}_attn.norm.{n}.scale"] = rng.uniform(
                    0.5, hi, (5, 128)).astype(np.float32)
        for n in ("query_norm", "key_norm"):
            blocks["single_blocks"][f"norm.{n}.scale"] = rng.uniform(0.5, hi, (20, 128)).astype(
                np.float32)
        try:
            loader.check_logit_bound(blocks)
            raised = 0
        except ValueError:
            raised = 1
        single = np.asarray(kernels.logit_bound(blocks["single_blocks"]["norm.query_norm.scale"],
                                                blocks["single_blocks"]["norm.key_norm.scale"]))
        rows.append((blocks, raised, single))
    out = {}
    for i, (blocks, raised, single) in enumerate(rows):
        for grp, d in blocks.items():
            for key, val in d.items():
                out[f"{i}|{grp}|{key}"] = val
        out[f"{i}|raised"] = np.int32(raised)
        out[f"{i}|single_bound"] = single.astype(np.float32)
    path = os.path.join(HERE, "logit_bound.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: raised={[r[1] for r in rows]}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("FLICKER_REFERENCE_SRC"),
                    help="the reference checkout's src/ directory (or set FLICKER_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("pass --reference-src or set FLICKER_REFERENCE_SRC to the reference's src/ directory")
    sys.path.insert(0, HERE)
    import jax_stand_in

    jax_stand_in.install()
    sys.path.insert(0, args.reference_src)
    import flicker.kernels as kernels  # noqa: E402
    import flicker.loader as loader  # noqa: E402
    import flicker.modules as modules  # noqa: E402
    import flicker.nn as nn  # noqa: E402
    import flicker.rope as rope  # noqa: E402

    ref = dict(kernels=kernels, modules=modules, nn=nn, rope=rope, loader=loader)
    case(ref, "joint_s256_h2", num_heads=2, num_txt=128, grid_h=8, grid_w=16, seed=0)
    case(ref, "joint_s384_h1", num_heads=1, num_txt=128, grid_h=16, grid_w=16, seed=10)
    bound_cases(ref)


if __name__ == "__main__":
    main()
