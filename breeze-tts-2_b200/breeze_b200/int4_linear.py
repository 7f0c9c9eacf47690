"""Weight-only int4 Linear, drop-in for models/int4_linear.py.

Same class name, constructor, buffers and checkpoint layout as the
reference (models/int4_linear.py:47-163):

  * ``weight_int4``: int32 [N/8, K/128, 32, 4] -- PyTorch's tinygemm tiles
    (innerKTiles = 8), produced on the GPU by bq_int4_tinygemm_pack, which
    re-tiles bit-for-bit like ``torch._convert_weight_to_int4pack``;
  * ``scales_zeros``: bf16 [K/g, N, 2] holding (scale, lo + 8 * scale);
  * ``w = (q - 8) * scale + zero``, codes in 0..15, odd k in the low nibble
    of the packed bytes.

Quantized checkpoints written by the reference load unchanged. The forward
pass is one bq_gemv launch (sm_100a, tensor-core dot products on
in-register dequantized weights) instead of ``torch._weight_int4pack_mm``.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib

GROUP_SIZE = 128
INNER_K_TILES = 8
# Layers below this size are L2-resident and launch-bound (reference
# models/int4_linear.py:39-42); kept for the same selection behaviour.
MIN_QUANT_BYTES = 8 * 1024 * 1024
DEFAULT_TARGET_NAMES = ("gate_proj", "up_proj", "down_proj")


def quantize_int4(weight: torch.Tensor, group_size: int = GROUP_SIZE):
    """Group-wise asymmetric int4 in the tinygemm layout (CUDA tensors).

    The code/scale arithmetic is the reference's (models/int4_linear.py:49-63)
    so packed checkpoints are bit-identical; the re-tiling runs in
    bq_int4_tinygemm_pack.
    """
    n, k = weight.shape
    g = weight.float().reshape(n, k // group_size, group_size)
    lo = g.amin(dim=-1, keepdim=True)
    scale = ((g.amax(dim=-1, keepdim=True) - lo) / 15).clamp(min=1e-8)
    codes = ((g - lo) / scale).round().clamp(0, 15).to(torch.uint8).reshape(n, k)
    packed = (codes[:, 1::2] | (codes[:, 0::2] << 4)).contiguous()
    inner = _lib.tinygemm_pack(packed, INNER_K_TILES)
    s = scale.squeeze(-1)
    sz = torch.stack([s.t().contiguous(), (lo.squeeze(-1) + 8 * s).t().contiguous()], dim=-1)
    return inner, sz.to(torch.bfloat16).contiguous()


class Int4Linear(nn.Module):
    """Drop-in replacement for a bias-free nn.Linear using int4 weights."""

    def __init__(self, linear: nn.Linear, group_size: int = GROUP_SIZE,
                 device: torch.device | str | None = None) -> None:
        super().__init__()
        if linear.bias is not None:
            raise ValueError("Int4Linear expects a bias-free Linear")
        weight = linear.weight.data
        if device is not None:
            weight = weight.to(device)
        self.out_features = int(weight.shape[0])
        self.in_features = int(weight.shape[1])
        self.group_size = group_size
        if self.in_features % group_size:
            raise ValueError(f"in_features {self.in_features} not divisible by group {group_size}")
        inner, scales_zeros = quantize_int4(weight, group_size)
        self.register_buffer("weight_int4", inner)
        self.register_buffer("scales_zeros", scales_zeros)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        if flat.stride(-1) != 1:
            flat = flat.contiguous()
        if flat.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            flat = flat.to(torch.bfloat16)
        out = _lib.gemv(flat, self.weight_int4, _lib.W_INT4_TINYGEMM, self.out_features,
                        scale=self.scales_zeros, group=self.group_size, out_dtype=x.dtype
                        if x.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.bfloat16,
                        flags=_lib.default_flags())
        return out.to(x.dtype).reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"int4=True, group={self.group_size}")

    # manifest record of a quantized checkpoint (quantized_checkpoint.py:39-48 of the reference)
    MANIFEST_KIND = "int4"
    MANIFEST_BUFFERS = (("weight_int4", torch.int32), ("scales_zeros", torch.bfloat16))

    def manifest_entry(self) -> dict:
        return {"kind": self.MANIFEST_KIND, "in_features": self.in_features, "out_features": self.out_features,
                "group_size": self.group_size,
                "shapes": {name: list(getattr(self, name).shape) for name, _ in self.MANIFEST_BUFFERS}}

    @classmethod
    def from_manifest(cls, entry: dict, device) -> "Int4Linear":
        """An uninitialised module with the recorded geometry, for a checkpoint's
        tensors to be assigned into; the packed shapes come from the manifest."""
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.in_features, m.out_features, m.group_size = entry["in_features"], entry["out_features"], entry["group_size"]
        for name, dtype in cls.MANIFEST_BUFFERS:
            m.register_buffer(name, torch.empty(entry["shapes"][name], dtype=dtype, device=device))
        return m


def quantize_module_int4(root: nn.Module, *, target_names: tuple[str, ...] = DEFAULT_TARGET_NAMES,
                         min_bytes: int = MIN_QUANT_BYTES, device: torch.device | str | None = None,
                         group_size: int = GROUP_SIZE) -> dict[str, int]:
    """Swap qualifying Linear layers under ``root`` for Int4Linear.

    Selection and the returned stats follow models/int4_linear.py:118-163:
    bias-free Linears named in ``target_names`` with at least ``min_bytes``
    of weights; a layer that cannot be packed is counted as
    ``skipped_unsupported`` and left untouched.
    """
    stats = {"converted": 0, "skipped_below_threshold": 0, "skipped_unsupported": 0, "weight_bytes_saved": 0}
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
            try:
                replacement = Int4Linear(child, group_size=group_size, device=device)
            except Exception:  # noqa: BLE001 - shape/geometry rejections, as the reference
                stats["skipped_unsupported"] += 1
                continue
            setattr(module, name, replacement)
            child.weight = None
            stats["converted"] += 1
            stats["weight_bytes_saved"] += nbytes - nbytes // 4
    return stats
