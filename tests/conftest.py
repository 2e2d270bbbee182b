"""Shared pytest set-up: the `gpu` marker, repo-root imports and golden-vector loading."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def has_b200() -> bool:
    try:
        import torch
    except ImportError:
        return False
    if not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(0) == (10, 0)


def pytest_collection_modifyitems(config, items):
    if has_b200():
        return
    skip = pytest.mark.skip(reason="needs a B200 GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> dict:
    """Golden case from tests/golden/<name>.npz; uint16 arrays are bf16 bit patterns."""
    import ml_dtypes

    bf16_keys = {"qkv", "q_scale", "k_scale", "q", "k", "v", "o", "q_gain1", "q_xla", "k_xla", "o_xla"}
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        out = {}
        for key in z.files:
            arr = z[key]
            out[key] = arr.view(ml_dtypes.bfloat16) if key in bf16_keys else arr
    return out


GOLDEN_CASES = ("joint_s256_h2", "joint_s384_h1")


def to_device(arr: np.ndarray, device="cuda"):
    """numpy (ml_dtypes.bfloat16 or float32) -> torch tensor on `device`, same bits."""
    import ml_dtypes
    import torch

    arr = np.ascontiguousarray(arr)
    if arr.dtype == ml_dtypes.bfloat16:
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(arr.copy()).to(device)


def to_host(t) -> np.ndarray:
    """torch tensor -> numpy with the same bits (bf16 -> ml_dtypes.bfloat16)."""
    import ml_dtypes
    import torch

    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(ml_dtypes.bfloat16)
    return t.numpy()


def bit_equal_fraction(a, b) -> float:
    import ml_dtypes

    a = np.asarray(a).astype(ml_dtypes.bfloat16).view(np.uint16)
    b = np.asarray(b).astype(ml_dtypes.bfloat16).view(np.uint16)
    return float(np.mean(a == b))
