"""int8 Linear, drop-in for models/int8_linear.py.

Buffers as in the reference (models/int8_linear.py:35-47): ``weight_int8``
[N, K] int8 (codes clamped to +-127), ``weight_scale`` fp32 [N, 1] = amax /
127, optional ``bias``. The reference dequantizes a full bf16 copy of W and
calls F.linear (moving more bytes than bf16, :3-6); here the forward reads
the int8 codes once in bq_gemv and applies the per-row scale -- rounded to
the activation dtype first when that is bf16, as the reference's
``weight_scale.to(x.dtype)`` does -- to the fp32 accumulator.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib

MIN_QUANT_BYTES = 1024 * 1024


class Int8Linear(nn.Module):
    """nn.Linear with int8-stored weights."""

    def __init__(self, linear: nn.Linear) -> None:
        super().__init__()
        weight = linear.weight.data
        self.out_features, self.in_features = weight.shape
        amax = weight.abs().amax(dim=1, keepdim=True).float().clamp(min=1e-12)
        scale = amax / 127.0
        q = (weight.float() / scale).round().clamp(-127, 127).to(torch.int8)
        self.register_buffer("weight_int8", q.contiguous())
        self.register_buffer("weight_scale", scale.to(torch.float32).contiguous())
        self.register_buffer("bias", linear.bias.data.clone() if linear.bias is not None else None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        if flat.stride(-1) != 1:
            flat = flat.contiguous()
        flags = _lib.default_flags()
        if x.dtype == torch.bfloat16:
            flags |= _lib.FLAG_SCALE_ROUND_BF16
        out = _lib.gemv(flat, self.weight_int8, _lib.W_INT8, self.out_features,
                        scale=self.weight_scale.reshape(-1), bias=self.bias, out_dtype=x.dtype, flags=flags)
        return out.reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, int8=True"

    # manifest record of a quantized checkpoint (quantized_checkpoint.py:50-59 of the reference)
    MANIFEST_KIND = "int8"
    MANIFEST_BUFFERS = (("weight_int8", torch.int8), ("weight_scale", torch.float32))

    def manifest_entry(self) -> dict:
        return {"kind": self.MANIFEST_KIND, "in_features": self.in_features, "out_features": self.out_features,
                "has_bias": self.bias is not None,
                "shapes": {name: list(getattr(self, name).shape) for name, _ in self.MANIFEST_BUFFERS}}

    @classmethod
    def from_manifest(cls, entry: dict, device) -> "Int8Linear":
        """An uninitialised module with the recorded geometry (and a bias slot
        when the entry has one), for a checkpoint's tensors to be assigned into."""
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.in_features, m.out_features = entry["in_features"], entry["out_features"]
        for name, dtype in cls.MANIFEST_BUFFERS:
            m.register_buffer(name, torch.empty(entry["shapes"][name], dtype=dtype, device=device))
        m.register_buffer("bias", torch.empty(m.out_features, dtype=torch.bfloat16, device=device)
                          if entry.get("has_bias") else None)
        return m


def quantize_module_int8(root: nn.Module, *, target_names: tuple[str, ...] | None = None,
                         min_bytes: int = MIN_QUANT_BYTES) -> dict[str, int]:
    """Store qualifying Linear weights as int8 (models/int8_linear.py:62-91).
    ``None`` targets every Linear."""
    stats = {"converted": 0, "skipped_below_threshold": 0, "weight_bytes_saved": 0}
    for module in root.modules():
        for name, child in list(module.named_children()):
            if not isinstance(child, nn.Linear):
                continue
            if target_names is not None and name not in target_names:
                continue
            nbytes = child.weight.numel() * child.weight.element_size()
            if nbytes < min_bytes:
                stats["skipped_below_threshold"] += 1
                continue
            setattr(module, name, Int8Linear(child))
            stats["converted"] += 1
            stats["weight_bytes_saved"] += nbytes // 2
    return stats
