"""W8A8 SmoothQuant linear on B200 int8 tensor cores (tcgen05.mma kind::i8).

flicker itself has no int8 path (its `linear` is a plain bf16 `x @ w`, src/flicker/nn.py:13-14);
this module implements the SmoothQuant method (Xiao et al., 2022) for the DiT's fused-QKV
projection shape:

* ``smooth_factors``: s_j = max|X_j|^alpha / max|W_j|^(1-alpha) per input channel (alpha = 0.5);
* ``quantize_weight`` (load time, torch): W' = W * s[:, None], per-output-channel symmetric int8,
  stored N-major [N, K] (K contiguous) for the tensor-core B operand;
* ``quantize_act`` (CUDA): X' = X / s, per-token symmetric int8 (round half to even);
* ``gemm`` (CUDA): y = bf16(float(int32 acc) * x_scale[i] * w_scale[n]);
* ``SmoothQuantLinear``: the three steps as one layer.
"""
from __future__ import annotations

import torch

from . import _lib
from .kernels import _device_call

ALPHA = 0.5


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check(name: str, t: torch.Tensor, dtype: torch.dtype, dim: int) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this package has no CPU path)")
    if t.dtype != dtype or t.dim() != dim:
        raise ValueError(f"{name} must be a {dim}-D {dtype} tensor, got {t.dtype} {tuple(t.shape)}")


def smooth_factors(x_absmax: torch.Tensor, w_absmax: torch.Tensor, alpha: float = ALPHA) -> torch.Tensor:
    """Per-input-channel smoothing factors (fp32); channels with a zero max get 1."""
    s = x_absmax.float().pow(alpha) / w_absmax.float().pow(1.0 - alpha)
    return torch.where(torch.isfinite(s) & (s > 0), s, torch.ones_like(s))


def quantize_weight(w: torch.Tensor, s: torch.Tensor):
    """W [K, N] (bf16) -> (Wq [N, K] int8, w_scale [N] fp32) of W' = float(W) * s[:, None].

    Runs the per-row quantisation kernel on W^T with `s` as its per-column multiplier, which is
    exactly per-output-channel quantisation of W' (same IEEE division as the activations).
    """
    return quantize_act(w.t().contiguous(), s.float().contiguous())


def quantize_act(x: torch.Tensor, inv_s: torch.Tensor):
    """X [M, K] bf16 -> (Xq [M, K] int8, x_scale [M] fp32) with X' = float(X) * inv_s (CUDA kernel)."""
    _check("x", x, torch.bfloat16, 2)
    _check("inv_s", inv_s, torch.float32, 1)
    m, k = x.shape
    if inv_s.numel() != k or k % 8:
        raise ValueError(f"inv_s must hold K={k} values and K must be a multiple of 8")
    x, inv_s = x.contiguous(), inv_s.contiguous()
    xq = torch.empty((m, k), dtype=torch.int8, device=x.device)
    sx = torch.empty((m,), dtype=torch.float32, device=x.device)
    lib = _lib.lib()
    code = _device_call(x, lambda stream: lib.flk_w8a8_quantize_act(x.data_ptr(), inv_s.data_ptr(), m, k,
                                                                    xq.data_ptr(), sx.data_ptr(), stream))
    _lib.check("flk_w8a8_quantize_act", code)
    return xq, sx


def gemm(xq: torch.Tensor, wq: torch.Tensor, x_scale: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    """y [M, N] bf16 = bf16(float(xq @ wq^T) * x_scale[:, None] * w_scale[None, :]) (CUDA kernel)."""
    _check("xq", xq, torch.int8, 2)
    _check("wq", wq, torch.int8, 2)
    m, k = xq.shape
    n = wq.shape[0]
    if wq.shape[1] != k or k % 16:
        raise ValueError(f"wq must be [N, K={k}] and K must be a multiple of 16")
    y = torch.empty((m, n), dtype=torch.bfloat16, device=xq.device)
    xq, wq, x_scale, w_scale = xq.contiguous(), wq.contiguous(), x_scale.contiguous(), w_scale.contiguous()
    lib = _lib.lib()
    code = _device_call(xq, lambda stream: lib.flk_w8a8_gemm(xq.data_ptr(), wq.data_ptr(), x_scale.data_ptr(),
                                                             w_scale.data_ptr(), m, n, k, y.data_ptr(), stream))
    _lib.check("flk_w8a8_gemm", code)
    return y


def gemm_s32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Raw int32 accumulators a [M, K] @ b [N, K]^T of the same kernel (for verification)."""
    _check("a", a, torch.int8, 2)
    _check("b", b, torch.int8, 2)
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty((m, n), dtype=torch.int32, device=a.device)
    with torch.cuda.device(a.device):
        code = _lib.lib().flk_i8_gemm_s32(a.contiguous().data_ptr(), b.contiguous().data_ptr(), m, n, k,
                                          c.data_ptr(), _stream(a))
    _lib.check("flk_i8_gemm_s32", code)
    return c


class SmoothQuantLinear:
    """y = x @ w through SmoothQuant W8A8: weights prepared once, activations quantised per call."""

    def __init__(self, wq: torch.Tensor, w_scale: torch.Tensor, inv_s: torch.Tensor):
        self.wq, self.w_scale, self.inv_s = wq, w_scale, inv_s

    @classmethod
    def from_float(cls, w: torch.Tensor, x_absmax: torch.Tensor, alpha: float = ALPHA) -> "SmoothQuantLinear":
        """w [K, N]; x_absmax [K] = per-channel max |activation| from calibration data."""
        s = smooth_factors(x_absmax, w.float().abs().amax(dim=1), alpha)
        wq, w_scale = quantize_weight(w, s)
        return cls(wq, w_scale, (1.0 / s).float())

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        xq, x_scale = quantize_act(x, self.inv_s)
        return gemm(xq, self.wq, x_scale, self.w_scale)
