"""Decode attention step restated on the CPU (test oracle only).

Follows models/fused/kernels.py:355-536 (``attention_step``):
  * per-head RMSNorm of q and k when norm weights are given (``_rms_head``,
    kernels.py:357-359): v * (1 / sqrt(mean(v^2) + eps)) * w, in fp32;
  * RoPE with rotate_half (``_rope``, kernels.py:363-373): v * cos +
    cat(-v[D/2:], v[:D/2]) * sin, in fp32;
  * the new k (normed, roped) and v written into the static cache at
    ``cache_position`` (kernels.py:397-401), cast to the cache dtype;
  * softmax((q * D^-0.5) k^T + mask) v over cache positions [0, pos]
    (kernels.py:409-455), fp32, output cast to bf16; the additive mask is
    (B, S) (kernels.py:492-502: bool masks become 0 / -1e30).
Grouped-query attention: q head h reads kv head h // (HQ / HKV).
"""

from __future__ import annotations

import torch


def rms_head(v: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    var = (v * v).sum(-1, keepdim=True) / v.shape[-1]
    return v * (1.0 / torch.sqrt(var + eps)) * w.float()


def rope(v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = v.shape[-1] // 2
    rot = torch.cat([-v[..., half:], v[..., :half]], -1)
    return v * cos + rot * sin


def additive_mask(mask: torch.Tensor, b: int, s: int) -> torch.Tensor:
    if mask.dtype == torch.bool:
        return torch.where(mask.reshape(b, -1)[:, :s], 0.0, -1e30).float()
    return mask.reshape(b, -1)[:, :s].float()


def attention_step(qkv, cos, sin, pos: int, keys, values, mask, q_norm_w=None, k_norm_w=None, eps=1e-6):
    """Returns (out (B, HQ*D) bf16, keys, values) with the caches updated in
    place (CPU tensors)."""
    b = qkv.shape[0]
    _, hkv, s, d = keys.shape
    hq = (qkv.shape[1] - 2 * hkv * d) // d
    x = qkv.float().reshape(b, hq + 2 * hkv, d)
    c = cos.reshape(cos.shape[0], -1).float()
    sn = sin.reshape(sin.shape[0], -1).float()
    if c.shape[0] != b:
        c, sn = c.expand(b, d), sn.expand(b, d)
    q = x[:, :hq]
    k = x[:, hq:hq + hkv]
    v = qkv.reshape(b, hq + 2 * hkv, d)[:, hq + hkv:]
    if q_norm_w is not None:
        q = rms_head(q, q_norm_w, eps)
        k = rms_head(k, k_norm_w, eps)
    q = rope(q, c[:, None], sn[:, None])
    k = rope(k, c[:, None], sn[:, None])
    keys[:, :, pos] = k.to(keys.dtype)
    values[:, :, pos] = v.to(values.dtype)
    m = additive_mask(mask, b, s)[:, : pos + 1]
    g = hq // hkv
    kk = keys[:, :, : pos + 1].float().repeat_interleave(g, dim=1)  # (B, HQ, L, D)
    vv = values[:, :, : pos + 1].float().repeat_interleave(g, dim=1)
    scores = torch.einsum("bhd,bhld->bhl", q * d ** -0.5, kk) + m[:, None, :]
    p = torch.softmax(scores, -1)
    out = torch.einsum("bhl,bhld->bhd", p, vv)
    return out.reshape(b, hq * d).to(torch.bfloat16), keys, values
