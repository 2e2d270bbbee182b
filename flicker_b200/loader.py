"""Load-time guard for the max-free softmax (``src/flicker/loader.py:115-128``).

``attend`` never subtracts a running max, so it is only exact while every logit
stays below ``EXP_LIMIT`` (exp overflows fp32 near 88.7). With QK-RMSNorm the
logits are bounded by sqrt(D) * max|q_scale| * max|k_scale| (q carries 1/sqrt(D)).
"""
from __future__ import annotations

import numpy as np

from .kernels import EXP_LIMIT, logit_bound


def check_logit_bound(blocks: dict) -> None:
    """Raise ``ValueError`` when the stacked block scales allow a logit >= EXP_LIMIT.

    ``blocks`` has the reference's stacked layout: ``blocks["double_blocks"]`` with
    ``{img,txt}_attn.norm.{query,key}_norm.scale`` [depth, D] and ``blocks["single_blocks"]``
    with ``norm.{query,key}_norm.scale`` [depth, D]. The two streams of a double block
    share one attention, so their scales are combined by per-lane max of |scale|.
    """
    double, single = blocks["double_blocks"], blocks["single_blocks"]

    def host(x) -> np.ndarray:
        return np.asarray(x.float().cpu() if hasattr(x, "cpu") else x, np.float32)

    def joint(name: str) -> np.ndarray:
        return np.maximum(*(np.abs(host(double[f"{s}_attn.norm.{name}.scale"])) for s in ("img", "txt")))

    bounds = (logit_bound(joint("query_norm"), joint("key_norm")),
              logit_bound(*(host(single[f"norm.{n}.scale"]) for n in ("query_norm", "key_norm"))))
    worst = max(float(np.max(np.asarray(b))) for b in bounds)
    if worst >= EXP_LIMIT:
        raise ValueError(f"attention='bounded' needs logits under {EXP_LIMIT}; these weights allow "
                         f"{worst:.1f}. use attention='flash'")
