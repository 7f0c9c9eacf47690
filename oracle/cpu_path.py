"""The reference's CPU path for the decode GEMV, for timing (test oracle).

This is the path the reference itself runs on host cores: dequantize with
torch ops and call F.linear (bench_gemv.py:29-52 -- RMSNorm, then
``q * scale + min`` repeated over each 128-group, then ``xn @ w_eff.T`` in
fp32; models/int8_linear.py:50-53 for int8). It uses every thread torch has.
bench.py's cpu_baseline leg and ``--impl reference`` time it; nothing in the
product calls it.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_gemv_int4_plain(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, mn: torch.Tensor,
                        gamma: torch.Tensor | None, eps: float = 1e-6, group: int = 128) -> torch.Tensor:
    """x (M, K) bf16, packed (N, K/2) uint8 even-k low, scale/min (N, K/g) bf16."""
    n = packed.shape[0]
    q = torch.stack([packed & 15, packed >> 4], -1).reshape(n, -1).float()
    w = q * scale.float().repeat_interleave(group, 1) + mn.float().repeat_interleave(group, 1)
    xf = x.float()
    if gamma is not None:
        xf = F.rms_norm(xf, (xf.shape[-1],), gamma.float(), eps)
    return F.linear(xf, w).to(torch.bfloat16)


def gemv_fp8(x: torch.Tensor, wq: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    w = wq.float() * scale.reshape(-1, 1).float()
    return F.linear(x.float(), w).to(torch.bfloat16)
