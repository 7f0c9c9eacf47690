"""FP8 (e4m3) Linear, drop-in for models/fp8_linear.py.

Buffers are the reference's (models/fp8_linear.py:56-66): ``weight_fp8``
e4m3fn [N, K] and ``weight_scale`` fp32 [1, N] = amax / 448 per output
channel, so existing modules and state dicts load unchanged.

Difference, on purpose: the reference forward also quantizes activations
per row and runs ``torch._scaled_mm`` (W8A8, ~3 % output error on the
recorded fixtures). Here the forward is weight-only -- one bq_gemv launch
that dequantizes e4m3 in registers and keeps bf16-class activations -- the
semantics of the reference's fused fp8 path (models/fused/kernels.py:124-134).
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib

FP8_MAX = 448.0
FP8_DTYPE = torch.float8_e4m3fn
MIN_QUANT_BYTES = 8 * 1024 * 1024
DEFAULT_TARGET_NAMES = ("gate_proj", "up_proj", "down_proj")


class Fp8Linear(nn.Module):
    """Drop-in replacement for a bias-free nn.Linear using FP8 weights."""

    def __init__(self, linear: nn.Linear) -> None:
        super().__init__()
        if linear.bias is not None:
            raise ValueError("Fp8Linear expects a bias-free Linear")
        weight = linear.weight.data
        self.in_features = int(weight.shape[1])
        self.out_features = int(weight.shape[0])
        amax = weight.abs().amax(dim=1, keepdim=True).float().clamp(min=1e-12)
        weight_scale = amax / FP8_MAX
        q = (weight.float() / weight_scale).clamp(-FP8_MAX, FP8_MAX)
        self.register_buffer("weight_fp8", q.to(FP8_DTYPE).contiguous())
        self.register_buffer("weight_scale", weight_scale.reshape(1, -1).contiguous())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        if flat.stride(-1) != 1:
            flat = flat.contiguous()
        out = _lib.gemv(flat, self.weight_fp8, _lib.W_FP8_E4M3, self.out_features,
                        scale=self.weight_scale.reshape(-1), out_dtype=x.dtype, flags=_lib.default_flags())
        return out.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, fp8=True"


def quantize_module_fp8(root: nn.Module, *, target_names: tuple[str, ...] = DEFAULT_TARGET_NAMES,
                        min_bytes: int = MIN_QUANT_BYTES) -> dict[str, int]:
    """Swap qualifying Linear layers for Fp8Linear (models/fp8_linear.py:89-122)."""
    stats = {"converted": 0, "skipped_below_threshold": 0, "weight_bytes_saved": 0}
    for module in root.modules():
        for name, child in list(module.named_children()):
            if not isinstance(child, nn.Linear) or child.bias is not None:
                continue
            if target_names and name not in target_names:
                continue
            nbytes = child.weight.numel() * child.weight.element_size()
            if nbytes < min_bytes:
                stats["skipped_below_threshold"] += 1
                continue
            setattr(module, name, Fp8Linear(child))
            stats["converted"] += 1
            stats["weight_bytes_saved"] += nbytes // 2
    return stats
