"""flicker_b200: flicker's DiT attention hot path (qk_prep -> attend) as sm_100a CUDA kernels.

``flicker_b200.kernels`` mirrors the reference module ``flicker.kernels``;
``flicker_b200.loader.check_logit_bound`` mirrors the reference's load-time guard;
``flicker_b200.rope`` builds the RoPE tables on device; ``flicker_b200.sharding``
splits one call across GPUs. The kernels live in ``libflicker_b200.so`` (C ABI in
``include/flicker_b200.h``), built by ``python -m flicker_b200.build``.
"""
from .kernels import (EPS, EXP_LIMIT, ROW_TILES, SCORE_TILES, Freqs, attend, attend_merged, device_status,
                      double_qk_prep, lane_pair, logit_bound, qk_prep, qk_prep_into, row_tile)

__all__ = ["EPS", "EXP_LIMIT", "ROW_TILES", "SCORE_TILES", "Freqs", "attend", "attend_merged", "device_status",
           "double_qk_prep", "lane_pair", "logit_bound", "qk_prep", "qk_prep_into", "row_tile"]
