"""Seeded weight/activation builders shared by the GPU tests and smoke().

Each builder returns CPU tensors in the packed layout the kernel reads plus
the oracle's fp32 dequantized weight, so a test can run the CUDA path on
copies and check it against the oracle.
"""

from __future__ import annotations

import torch

from oracle import quant

FORMATS = ("bf16", "int4_tinygemm", "int4_plain", "fp8", "int8")


def make_weight(fmt: str, n: int, k: int, seed: int = 0, group: int = 128):
    """-> dict(w, scale, group, wfmt_name, deq) with CPU tensors."""
    g = torch.Generator().manual_seed(seed)
    if fmt == "bf16":
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        return {"w": w, "scale": None, "group": 128, "deq": w.float()}
    if fmt in ("int4_tinygemm", "int4_plain"):
        codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32).to(torch.uint8)
        gs = group if fmt == "int4_tinygemm" else 128
        s = ((torch.randn(k // gs, n, generator=g) * 0.02).abs() / 7 + 1e-4).to(torch.bfloat16)
        z = (torch.randn(k // gs, n, generator=g) * 0.01).to(torch.bfloat16)
        sz = torch.stack([s, z], -1).contiguous()
        if fmt == "int4_tinygemm":
            w = quant.tinygemm_pack(quant.pack_odd_low(codes))
            deq = quant.dequant_int4_tinygemm(w, sz, gs)
        else:
            w = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
            deq = quant.dequant_int4_plain(w, s.t().contiguous(), z.t().contiguous())
        return {"w": w, "scale": sz, "group": gs, "deq": deq}
    if fmt == "fp8":
        b = torch.randint(0, 256, (n, k), generator=g, dtype=torch.int32).to(torch.uint8)
        b[(b & 0x7F) == 0x7F] = 0x3C  # no NaN codes (the quantizers never emit them)
        w = b.view(torch.float8_e4m3fn)
        s = (torch.rand(n, generator=g) * 1e-3 + 1e-5).float()
        return {"w": w, "scale": s, "group": 128, "deq": quant.dequant_fp8(w, s)}
    if fmt == "int8":
        q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int32).to(torch.int8)
        s = (torch.rand(n, generator=g) * 1e-3 + 1e-5).float()
        # the GEMV applies the fp32 scale to the fp32 accumulator
        return {"w": q, "scale": s, "group": 128, "deq": q.float() * s[:, None]}
    raise ValueError(fmt)


def wfmt_code(fmt: str) -> int:
    from breeze_b200 import _lib

    return {"bf16": _lib.W_BF16, "int4_tinygemm": _lib.W_INT4_TINYGEMM, "int4_plain": _lib.W_INT4_PLAIN,
            "fp8": _lib.W_FP8_E4M3, "int8": _lib.W_INT8}[fmt]


def dequant_qweight(qw) -> torch.Tensor:
    """The oracle's fp32 (N, K) weight for a breeze_b200 QWeight, whatever its format."""
    from breeze_b200 import _lib

    w, s = qw.w.cpu(), None if qw.scale is None else qw.scale.cpu()
    if qw.wfmt == _lib.W_INT4_TINYGEMM:
        return quant.dequant_int4_tinygemm(w, s, qw.group)
    if qw.wfmt == _lib.W_INT4_PLAIN:
        return quant.dequant_int4_plain(w, s[..., 0].t().contiguous(), s[..., 1].t().contiguous(), qw.group)
    if qw.wfmt == _lib.W_FP8_E4M3:
        return quant.dequant_fp8(w, s)
    if qw.wfmt == _lib.W_INT8:
        return quant.dequant_int8(w, s, dtype=torch.float32)
    return w.float()
