"""RMSNorm prologue, linear and epilogues restated on the CPU (test oracle).

  * ``rmsnorm_breeze``: BreezeRMSNorm.forward, models/breeze.py:115-120
    (fp32 variance, x_hat rounded to the input dtype, then weight * x_hat in
    the weight's dtype).
  * ``rmsnorm_fp32``: the fused Triton prologue, models/fused/kernels.py:65-81
    (x * inv * gamma kept in fp32, inv = 1/sqrt(mean(x^2) + eps)).
  * ``linear_epilogue``: F.linear in fp32 followed by the epilogues of
    gemv_epilogue_kernel, models/fused/kernels.py:116-137 (0: none,
    1: silu(gate) * up over [gate | up], 2: + residual) and the bench's
    reference, bench_gemv.py:30-35.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

EPI_NONE, EPI_SILU_MUL, EPI_ADD_RESIDUAL = 0, 1, 2


def rmsnorm_breeze(x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    input_dtype = x.dtype
    h = x.to(torch.float32)
    variance = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(variance + eps)
    return gamma * h.to(input_dtype)


def rmsnorm_fp32(x: torch.Tensor, gamma: torch.Tensor | None, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    inv = 1.0 / torch.sqrt((xf * xf).sum(-1, keepdim=True) / x.shape[-1] + eps)
    y = xf * inv
    if gamma is not None:
        y = y * gamma.float()
    return y


def linear_epilogue(xhat: torch.Tensor, w: torch.Tensor, epilogue: int = EPI_NONE,
                    residual: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 out = epilogue(xhat @ w.T (+ bias))."""
    y = F.linear(xhat.float(), w.float(), None if bias is None else bias.float())
    if epilogue == EPI_SILU_MUL:
        n = y.shape[-1] // 2
        g, u = y[..., :n], y[..., n:]
        return F.silu(g) * u
    if epilogue == EPI_ADD_RESIDUAL:
        return y + residual.float()
    return y


def fused_reference(x: torch.Tensor, w: torch.Tensor, gamma: torch.Tensor | None, eps: float,
                    epilogue: int, residual: torch.Tensor | None = None,
                    bias: torch.Tensor | None = None, norm: str = "fp32") -> torch.Tensor:
    """Whole rms_gemv in fp32: optional RMSNorm, linear with the dequantized
    weight ``w``, epilogue. ``norm`` picks the Triton ("fp32") or the
    BreezeRMSNorm ("breeze") prologue."""
    if gamma is None:
        xhat = x.float()
    elif norm == "breeze":
        xhat = rmsnorm_breeze(x, gamma, eps).float()
    else:
        xhat = rmsnorm_fp32(x, gamma, eps)
    return linear_epilogue(xhat, w, epilogue, residual, bias)


def max_rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max |got - ref| / max |ref|, the reference's own metric
    (bench_gemv.py:53, models/fused/test_layer.py:86-88)."""
    got, ref = got.double(), ref.double()
    return ((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()
