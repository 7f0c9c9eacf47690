"""Quantization, packing and dequantization restated on the CPU (test oracle).

Formats (reference project paths):
  * int4 tinygemm -- models/int4_linear.py:47-64. Codes q in 0..15 per group
    of ``group`` along K, ``scale = (hi-lo)/15`` (clamped at 1e-8), packed two
    per byte with the ODD k in the low nibble (:58), then re-tiled by
    ``torch._convert_weight_to_int4pack(packed, 8)`` (third-party ATen op,
    torch==2.9.1 per requirements.txt:1; restated here as ``tinygemm_pack``).
    ``scales_zeros[K/g, N, 2]`` bf16 holds (scale, lo + 8*scale) and the
    weight is ``w = (q - 8) * scale + zero`` (docstring :25-28).
  * int4 plain (fused Triton path) -- models/fused/kernels.py:141-150. (N, K/2)
    uint8 with the EVEN k in the low nibble, scale/min (N, K/128) bf16,
    ``w = q * scale + min``.
  * fp8 e4m3 -- models/fp8_linear.py:56-66 (Fp8Linear, amax clamp 1e-12) and
    models/fused/kernels.py:153-158 (pack_fp8, clamp 1e-8); per-row fp32 scale
    ``amax/448``; weight-only use is ``w = float(q) * scale_n``
    (bench_gemv.py:49, kernels.py:124-134).
  * int8 -- models/int8_linear.py:40-53. ``scale = amax/127``, codes rounded
    and clamped to +-127; forward dequantizes IN THE ACTIVATION DTYPE:
    ``w = dtype(q) * dtype(scale)`` (:52).
"""

from __future__ import annotations

import numpy as np
import torch

GROUP_SIZE = 128  # models/int4_linear.py:36
INNER_K_TILES = 8  # models/int4_linear.py:37
FP8_MAX = 448.0  # models/fp8_linear.py:33


def _recip(v: float) -> torch.Tensor:
    """fp32 reciprocal of a Python scalar.

    The reference quantizes on CUDA tensors (Int4Linear's pack has no CPU
    kernel), and PyTorch's CUDA true-divide by a Python scalar is computed as
    ``a * (1.0f / b)``. Restating ``x / 15`` as ``x * _recip(15)`` reproduces
    the reference's codes and scales bit-for-bit (checked against the
    recorded buffers in tests/golden/*.npz); a true division differs by an
    ulp on some groups and flips codes.
    """
    return torch.tensor(1.0 / v, dtype=torch.float32)


# --------------------------------------------------------------------------
# int4, tinygemm layout
# --------------------------------------------------------------------------

def quantize_int4_codes(weight: torch.Tensor, group_size: int = GROUP_SIZE):
    """Codes and fp32 (scale, lo) per models/int4_linear.py:49-56.

    Returns q (N, K) uint8 in 0..15, scale (N, K/g) fp32, lo (N, K/g) fp32.
    """
    n, k = weight.shape
    grouped = weight.float().reshape(n, k // group_size, group_size)
    lo = grouped.amin(dim=-1, keepdim=True)
    hi = grouped.amax(dim=-1, keepdim=True)
    scale = ((hi - lo) * _recip(15)).clamp(min=1e-8)
    q = ((grouped - lo) / scale).round().clamp(0, 15).to(torch.uint8)
    return q.reshape(n, k), scale.squeeze(-1), lo.squeeze(-1)


def pack_odd_low(q: torch.Tensor) -> torch.Tensor:
    """(N, K) codes -> (N, K/2) uint8, odd k low nibble (int4_linear.py:58)."""
    return (q[:, 1::2] | (q[:, 0::2] << 4)).contiguous()


def _tinygemm_byte_index(n: int, k: int, inner_k_tiles: int):
    """For every int32 of the tinygemm tensor, its 4 source (row, byte) pairs.

    Restates the re-tiling done by torch._convert_weight_to_int4pack for a
    uint8 (N, K/2) input (pinned bit-for-bit against the op's output on a
    B200, tests/golden/tinygemm_pack.npz). Output shape is
    (N/8, K/(ik*16), 32, ik/2). The word at [nt, ko, lane, j] serves row
    n = 8*nt + lane//4 and the k-tile pair (ko*ik + 2j, ko*ik + 2j + 1); its
    source bytes are B_i = 8*(ko*ik + 2j) + lane%4 + 4*i for i = 0..3.
    """
    assert n % 8 == 0 and k % (inner_k_tiles * 16) == 0
    nt = np.arange(n // 8)[:, None, None, None, None]
    ko = np.arange(k // (inner_k_tiles * 16))[None, :, None, None, None]
    lane = np.arange(32)[None, None, :, None, None]
    j = np.arange(inner_k_tiles // 2)[None, None, None, :, None]
    i = np.arange(4)[None, None, None, None, :]
    row = nt * 8 + lane // 4
    byte = (ko * inner_k_tiles + 2 * j) * 8 + lane % 4 + 4 * i
    shape = (n // 8, k // (inner_k_tiles * 16), 32, inner_k_tiles // 2, 4)
    return np.broadcast_to(row, shape), np.broadcast_to(byte, shape)


def tinygemm_pack(packed_u8: torch.Tensor, inner_k_tiles: int = INNER_K_TILES) -> torch.Tensor:
    """(N, K/2) uint8 -> tinygemm int32 tiles (restates the ATen op).

    Nibble p of the word (bits 4p..4p+3) is the HIGH nibble of byte B_p for
    p < 4 and the LOW nibble of byte B_{p-4} for p >= 4. With the reference's
    odd-k-low byte convention that puts k = K0 + 2*(lane%4) + 8*(p%4) + p//4
    (K0 = 16*(ko*ik + 2j)) in nibble p, so the 16-bit halves selected by the
    masks 0x000F000F / 0x00F000F0 (and the same after >> 8) hold the k pairs
    {2t, 2t+1}, {2t+8, 2t+9}, {2t+16, 2t+17}, {2t+24, 2t+25}: the operand
    fragments of m16n8k16 for k-tiles 2j and 2j+1.
    """
    src = packed_u8.numpy()
    n, kh = src.shape
    row, byte = _tinygemm_byte_index(n, kh * 2, inner_k_tiles)
    v = src[row, byte].astype(np.uint32)
    hi, lo = v >> 4, v & 15
    word = np.zeros(v.shape[:-1], dtype=np.uint32)
    for i in range(4):
        word |= hi[..., i] << (4 * i)
        word |= lo[..., i] << (16 + 4 * i)
    return torch.from_numpy(word.view(np.int32).copy())


def tinygemm_unpack_indexed(weight_int4: torch.Tensor) -> torch.Tensor:
    """Inverse of tinygemm_pack through the explicit index map (slow; the
    check for ``tinygemm_unpack``)."""
    w = weight_int4.numpy().view(np.uint32)
    nt, kt, _, half = w.shape
    n, k, ik = nt * 8, kt * half * 2 * 16, half * 2
    row, byte = _tinygemm_byte_index(n, k, ik)
    out = np.zeros((n, k // 2), dtype=np.uint8)
    for i in range(4):
        hi = (w >> (4 * i)) & 15
        lo = (w >> (16 + 4 * i)) & 15
        out[row[..., i], byte[..., i]] = ((hi << 4) | lo).astype(np.uint8)
    return torch.from_numpy(out)


def tinygemm_unpack(weight_int4: torch.Tensor) -> torch.Tensor:
    """Inverse of tinygemm_pack: int32 tiles -> (N, K/2) uint8 (odd k low).

    The index map of ``_tinygemm_byte_index`` is a permutation of axes: with
    lane = 4r + c, word [nt, ko, lane, j] byte i lands in row 8nt + r at byte
    ko*ik*8 + 16j + 4i + c, i.e. a row's bytes run in (ko, j, i, c) order. So
    the unpack is one transpose of [nt, ko, r, c, j, i] to [nt, r, ko, j, i, c]
    (identical to the indexed form, which the oracle tests compare)."""
    w = weight_int4.numpy().view(np.uint32)
    nt, kt, _, half = w.shape
    by = np.stack([(((w >> (4 * i)) & 15) << 4) | ((w >> (16 + 4 * i)) & 15) for i in range(4)], -1)
    by = by.astype(np.uint8).reshape(nt, kt, 8, 4, half, 4)  # [nt, ko, r, c, j, i]
    return torch.from_numpy(np.ascontiguousarray(by.transpose(0, 2, 1, 4, 5, 3)).reshape(nt * 8, kt * half * 16))


def codes_from_odd_low(packed_u8: torch.Tensor) -> torch.Tensor:
    """(N, K/2) odd-low bytes -> (N, K) codes."""
    p = packed_u8.to(torch.int32)
    n, kh = p.shape
    q = torch.empty(n, kh * 2, dtype=torch.int32)
    q[:, 0::2] = p >> 4
    q[:, 1::2] = p & 15
    return q


def scales_zeros(scale: torch.Tensor, lo: torch.Tensor) -> torch.Tensor:
    """(N, K/g) fp32 scale and lo -> [K/g, N, 2] bf16 (int4_linear.py:61-63)."""
    s = scale.t().contiguous()
    z = (lo + 8 * scale).t().contiguous()
    return torch.stack([s, z], dim=-1).to(torch.bfloat16).contiguous()


def quantize_int4(weight: torch.Tensor, group_size: int = GROUP_SIZE):
    """Whole Int4Linear construction: (weight_int4, scales_zeros)."""
    q, scale, lo = quantize_int4_codes(weight, group_size)
    return tinygemm_pack(pack_odd_low(q)), scales_zeros(scale, lo)


def _grouped_fma(q: np.ndarray, s: np.ndarray, z: np.ndarray, group: int) -> np.ndarray:
    """fp32 W[N, K] = q * s + z per group of ``group`` along K, with q (N, K)
    small integers and s, z (N, K/group) bf16-valued. q * s is exact in fp32
    (a 4-bit integer times an 8-bit significand), so the single rounding of
    the add equals fmaf(q, s, z), the reference's dequant rounding."""
    n, k = q.shape
    w = q.astype(np.float32).reshape(n, k // group, group) * s[..., None] + z[..., None]
    return w.reshape(n, k)


def dequant_int4_tinygemm(weight_int4: torch.Tensor, sz: torch.Tensor, group_size: int) -> torch.Tensor:
    """fp32 W[N, K] = (q - 8) * scale + zero, one rounding (fmaf)."""
    q = codes_from_odd_low(tinygemm_unpack(weight_int4)).numpy()
    szf = sz.float().numpy()  # [K/g, N, 2]
    return torch.from_numpy(_grouped_fma(q - 8, np.ascontiguousarray(szf[..., 0].T),
                                         np.ascontiguousarray(szf[..., 1].T), group_size))


# --------------------------------------------------------------------------
# int4, plain layout (fused Triton path)
# --------------------------------------------------------------------------

def pack_int4_plain(weight: torch.Tensor, group: int = 128):
    """models/fused/kernels.py:141-150: packed even-low, scale, min (bf16)."""
    n, k = weight.shape
    g = weight.float().reshape(n, k // group, group)
    lo, hi = g.amin(-1, keepdim=True), g.amax(-1, keepdim=True)
    scale = ((hi - lo) * _recip(15)).clamp_min(1e-8)
    q = ((g - lo) / scale).round().clamp(0, 15).to(torch.uint8).reshape(n, k)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()
    return packed, scale.squeeze(-1).to(torch.bfloat16).contiguous(), lo.squeeze(-1).to(torch.bfloat16).contiguous()


def codes_from_even_low(packed_u8: torch.Tensor) -> torch.Tensor:
    p = packed_u8.to(torch.int32)
    n, kh = p.shape
    q = torch.empty(n, kh * 2, dtype=torch.int32)
    q[:, 0::2] = p & 15
    q[:, 1::2] = p >> 4
    return q


def dequant_int4_plain(packed: torch.Tensor, scale: torch.Tensor, mn: torch.Tensor, group: int = 128) -> torch.Tensor:
    """fp32 W = q * scale + min (bench_gemv.py:51-52; q*s is exact, one rounding)."""
    q = codes_from_even_low(packed).numpy()
    return torch.from_numpy(_grouped_fma(q, scale.float().numpy(), mn.float().numpy(), group))


# --------------------------------------------------------------------------
# fp8 e4m3
# --------------------------------------------------------------------------

def quantize_fp8_linear(weight: torch.Tensor):
    """Fp8Linear.__init__ (fp8_linear.py:58-66): (weight_fp8 [N,K], weight_scale [1,N])."""
    amax = weight.abs().amax(dim=1, keepdim=True).float().clamp(min=1e-12)
    weight_scale = amax * _recip(FP8_MAX)
    quantized = (weight.float() / weight_scale).clamp(-FP8_MAX, FP8_MAX)
    return quantized.to(torch.float8_e4m3fn).contiguous(), weight_scale.reshape(1, -1).contiguous()


def pack_fp8(weight: torch.Tensor):
    """models/fused/kernels.py:153-158: (q [N,K] e4m3, scale [N] fp32)."""
    amax = weight.float().abs().amax(-1, keepdim=True).clamp_min(1e-8)
    scale = amax * _recip(448.0)
    q = (weight.float() / scale).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.contiguous(), scale.squeeze(-1).float().contiguous()


def dequant_fp8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp32 W = float(q) * scale_n (bench_gemv.py:49), one rounding."""
    return q.float() * scale.reshape(-1, 1).float()


# --------------------------------------------------------------------------
# int8
# --------------------------------------------------------------------------

def quantize_int8(weight: torch.Tensor):
    """Int8Linear.__init__ (int8_linear.py:40-47): (weight_int8 [N,K], weight_scale [N,1] fp32)."""
    amax = weight.abs().amax(dim=1, keepdim=True).float().clamp(min=1e-12)
    scale = amax * _recip(127.0)
    q = (weight.float() / scale).round().clamp(-127, 127).to(torch.int8)
    return q.contiguous(), scale.to(torch.float32).contiguous()


def dequant_int8(q: torch.Tensor, scale: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """Int8Linear.forward's weight (int8_linear.py:52): dtype(q) * dtype(scale)."""
    return q.to(dtype) * scale.reshape(-1, 1).to(dtype)


# --------------------------------------------------------------------------
# bit helpers shared by tests
# --------------------------------------------------------------------------

def from_bits(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """Inverse of tests/golden/make_golden.py:bits()."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype == torch.bfloat16:
        return t.view(torch.int16).view(torch.bfloat16)
    if dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).view(torch.float8_e4m3fn)
    return t.to(dtype)
