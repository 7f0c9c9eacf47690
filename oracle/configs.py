"""Seeded synthetic inputs for the BASELINE configurations (test oracle).

Every tensor is drawn from one ``torch.Generator().manual_seed(seed)`` on
the CPU, in the order the fields are listed in each docstring, so a test, a
fixture script and bench.py's CPU leg all regenerate identical inputs.
There is no public dataset behind these shapes; the distributions are the
ones BASELINE.json states for each config.
"""

from __future__ import annotations

import torch

from . import quant


def int4_codes_scales(n: int, k: int, g: torch.Generator, group: int = 128):
    """Config-0 weights: codes uniform 0..15 (N, K) uint8, then
    scale = |N(0, 0.02)| / 7 as bf16 (N, K/group). Zero-point 8."""
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32).to(torch.uint8)
    scale = ((torch.randn(n, k // group, generator=g) * 0.02).abs() / 7).to(torch.bfloat16)
    return codes, scale


def int4_tinygemm_from_codes(codes: torch.Tensor, scale: torch.Tensor):
    """Zero-point 8 in the tinygemm convention: zero = 0, so w = (q-8)*s.
    Returns (weight_int4, scales_zeros [K/g, N, 2] bf16)."""
    w = quant.tinygemm_pack(quant.pack_odd_low(codes))
    sz = torch.stack([scale.t().float(), torch.zeros(scale.shape[1], scale.shape[0])], -1)
    return w, sz.to(torch.bfloat16).contiguous()


def int4_plain_from_codes(codes: torch.Tensor, scale: torch.Tensor):
    """Zero-point 8 in the plain convention: min = -8*scale (exact in bf16).
    Returns (packed even-low (N, K/2) uint8, scale, min)."""
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    mn = (-8.0 * scale.float()).to(torch.bfloat16)
    return packed, scale.contiguous(), mn.contiguous()


def config0(seed: int = 0, n: int = 2048, k: int = 2048, m: int = 1):
    """Config 0: codes, scale, x ~ bf16 N(0,1) (M, K)."""
    g = torch.Generator().manual_seed(seed)
    codes, scale = int4_codes_scales(n, k, g)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    return {"codes": codes, "scale": scale, "x": x}


def config1(seed: int = 0, n: int = 6144, k: int = 2048, m: int = 1):
    """Config 1: codes, scale, residual x ~ bf16 N(0,1) (M, K),
    gamma = bf16(1 + N(0, 0.1)) (K,), eps 1e-6."""
    g = torch.Generator().manual_seed(seed)
    codes, scale = int4_codes_scales(n, k, g)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    return {"codes": codes, "scale": scale, "x": x, "gamma": gamma, "eps": 1e-6}


def fp8_weight(n: int, k: int, g: torch.Generator):
    """Config-2 weight: N(0, 0.02) quantized as Fp8Linear does
    (models/fp8_linear.py:58-66)."""
    w = torch.randn(n, k, generator=g) * 0.02
    return quant.quantize_fp8_linear(w)


def config2(seed: int = 0, shape: str = "gate_up", m: int = 1):
    """Config 2: fp8 weight (N(0,0.02) -> e4m3, scale absmax/448), x ~ bf16
    N(0,1) (M, K), residual ~ bf16 N(0,1) for the down projection.
    gate_up: K=2048, N=16384, SiLU epilogue; down: K=8192, N=2048, +residual."""
    g = torch.Generator().manual_seed(seed)
    n, k = (16384, 2048) if shape == "gate_up" else (2048, 8192)
    wq, ws = fp8_weight(n, k, g)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16) if shape == "down" else None
    return {"w": wq, "scale": ws, "x": x, "residual": res, "n": n, "k": k}


def int8_weight(n: int, k: int, g: torch.Generator):
    """Config-3 int8 weight: codes uniform in -127..127, per-row fp32 scale
    absmax/127 with absmax = 0.06 * (1 + 0.1 |N(0,1)|)."""
    q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int32).to(torch.int8)
    amax = 0.06 * (1 + 0.1 * torch.randn(n, 1, generator=g).abs())
    return q, (amax * quant._recip(127.0)).float()


# The decode-step stack of config 3 / 4: per layer (name, K, N, epilogue, norm).
LAYER_SHAPES = (
    ("qkv", 2048, 6144, 0, True),
    ("o", 2048, 2048, 2, False),
    ("gate_up", 2048, 16384, 1, True),
    ("down", 8192, 2048, 2, False),
)
HEAD_SHAPE = ("head", 2048, 8192, 0, True)
N_LAYERS = 28
