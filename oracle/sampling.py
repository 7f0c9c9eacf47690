"""CFG mix, token sampling and the fp32 output heads restated on the CPU (test
oracle only: imported by tests/, never by the library).

Sampling follows DepthDecoderGraph._cfg_sample
(models/cudagraph/depth_decoder_graph.py:487-558) and sample_logits
(models/cudagraph/sampling.py:36-87):
  * cfg = uncond + g * (cond - uncond) for paired rows (:498-501), else cond;
  * mask_invalid_codec_token_logits (models/logits_process.py:7-25): logits in
    [codebook_size, token_vocab_size) become -inf;
  * the HF repetition penalty over the unique history tokens
    (sampling.py:14-33) and the suppress mask (sampling.py:58-61);
  * greedy = argmax of those logits (depth_decoder_graph.py:550);
  * temperature (:511), top-k (:514-523: the first k ranks of torch.topk; or,
    as sample_logits does at :65-69, every logit >= the k-th value), top-p
    (:525-540: sort, softmax, cumsum, drop where the mass before a token
    exceeds top_p, the first always kept), softmax (:543).
The draw itself is the library's: the first token, in descending-probability
order (a stable sort, ties by ascending index), whose cumulative probability
exceeds u. torch.multinomial's own draw depends on its generator's stream and
is not restated; tests give u explicitly, and the Philox4x32-10 generator the
library uses is restated below (philox4x32_10) so its u can be checked too.

The heads follow BreezeCodebooksHead.forward (models/breeze.py:598-613:
F.linear(h, W[codebook].T) in fp32) after the depth model's final norm
(BreezeRMSNorm, breeze.py:115-120: xh = bf16(x * rsqrt(mean(x^2) + eps)),
y = bf16(gamma * xh)), and the backbone lm_head.float()
(models/cudagraph/backbone_graph.py:70, 272-273).
"""

from __future__ import annotations

import numpy as np
import torch

_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK32 = 0xFFFFFFFF


def philox4x32_10(counter: tuple[int, int, int, int], key: tuple[int, int]) -> tuple[int, int, int, int]:
    """Philox4x32 with 10 rounds (Salmon, Moraes, Dror and Shaw, SC 2011)."""
    c0, c1, c2, c3 = counter
    k0, k1 = key
    for _ in range(10):
        p0, p1 = _M0 * c0, _M1 * c2
        hi0, lo0 = p0 >> 32, p0 & _MASK32
        hi1, lo1 = p1 >> 32, p1 & _MASK32
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & _MASK32, lo1, (hi0 ^ c3 ^ k1) & _MASK32, lo0
        k0, k1 = (k0 + _W0) & _MASK32, (k1 + _W1) & _MASK32
    return c0, c1, c2, c3


def philox_uniform(seed: int, call: int, row: int) -> float:
    """The library's u for (seed, call counter, row): first Philox word >> 8, times 2^-24."""
    w = philox4x32_10((call & _MASK32, (call >> 32) & _MASK32, row, 0), (seed & _MASK32, (seed >> 32) & _MASK32))
    return float(np.float32(w[0] >> 8) * np.float32(1.0 / 16777216.0))


def mixed_logits(logits: torch.Tensor, rows: int, guidance=None, mask=(0, 0), rep_penalty: float = 1.0,
                 history=None, history_len=None, suppress=None) -> torch.Tensor:
    """(rows, V) fp32: CFG mix, codec mask, repetition penalty, suppress mask."""
    lg = logits.float()
    if guidance is not None:
        cond, unc = lg[:rows], lg[rows:2 * rows]
        g = guidance.float().reshape(rows, 1)
        cfg = unc + g * (cond - unc)
    else:
        cfg = lg[:rows].clone()
    lo, hi = mask
    if hi > lo:
        cfg[:, lo:hi] = float("-inf")
    if history is not None and rep_penalty != 1.0:
        for r in range(rows):
            toks = history[r, : int(history_len[r])].long()
            toks = toks[(toks >= 0) & (toks < cfg.shape[1])].unique()
            v = cfg[r, toks]
            cfg[r, toks] = torch.where(v > 0, v / rep_penalty, v * rep_penalty)
    if suppress is not None:
        cfg[:, suppress.bool()] = float("-inf")
    return cfg


def sample_probs(cfg_row: torch.Tensor, temperature: float, top_k: int, top_p: float, max_k: int,
                 topk_by_value: bool = False) -> torch.Tensor:
    """(V,) fp32 probabilities in vocabulary order after temperature, top-k,
    top-p and the softmax: what the reference hands to torch.multinomial."""
    v = cfg_row.shape[0]
    scaled = cfg_row.float() / temperature
    k = max_k if top_k <= 0 else top_k
    k = max(1, min(k, max_k, v))
    vals, idx = torch.sort(scaled, descending=True, stable=True)
    kept = (vals >= vals[k - 1]) if topk_by_value else (torch.arange(v) < k)
    kept &= vals > float("-inf")
    e = torch.where(kept, torch.exp(vals - vals[0]), torch.zeros_like(vals))
    z = e.sum()
    excl = torch.cumsum(e, 0) - e
    remove = (excl / z > top_p) & (torch.arange(v) >= 1)
    e = torch.where(remove, torch.zeros_like(e), e)
    probs = torch.zeros(v, dtype=torch.float32)
    probs[idx] = e / e.sum()
    return probs


def sample_row(cfg_row: torch.Tensor, temperature: float, top_k: int, top_p: float, do_sample: bool, u: float,
               max_k: int, topk_by_value: bool = False, clamp_hi: int | None = None) -> int:
    """One token from one row of mixed logits (see the module docstring)."""
    v = cfg_row.shape[0]
    greedy = int(torch.argmax(cfg_row).item())
    scaled = cfg_row / temperature
    k = max_k if top_k <= 0 else top_k
    k = max(1, min(k, max_k, v))
    vals, idx = torch.sort(scaled, descending=True, stable=True)
    if topk_by_value:
        kept = vals >= vals[k - 1]
    else:
        kept = torch.arange(v) < k
    kept &= vals > float("-inf")
    tok = greedy
    if do_sample and bool(kept.any()):
        e = torch.where(kept, torch.exp(vals - vals[0]), torch.zeros_like(vals))
        z = e.sum()
        excl = torch.cumsum(e, 0) - e
        remove = (excl / z > top_p) & (torch.arange(v) >= 1)
        e = torch.where(remove, torch.zeros_like(e), e)
        cum = torch.cumsum(e, 0)
        target = u * cum[-1]
        hit = ((cum > target) & (e > 0)).nonzero()
        sel = int(hit[0]) if len(hit) else int((e > 0).nonzero()[-1])
        tok = int(idx[sel])
    hi = v - 1 if clamp_hi is None else clamp_hi
    return min(max(tok, 0), hi)


def draw_margin(cfg_row: torch.Tensor, temperature: float, top_k: int, top_p: float, u: float, max_k: int,
                topk_by_value: bool = False) -> float:
    """Distance of u * mass from the nearest cumulative boundary and of the
    top-p test from its threshold (relative); a draw with a tiny margin can
    legitimately differ between fp32 summation orders."""
    v = cfg_row.shape[0]
    scaled = cfg_row / temperature
    k = max_k if top_k <= 0 else top_k
    k = max(1, min(k, max_k, v))
    vals, _ = torch.sort(scaled.double(), descending=True, stable=True)
    kept = (vals >= vals[k - 1]) if topk_by_value else (torch.arange(v) < k)
    kept &= vals > float("-inf")
    e = torch.where(kept, torch.exp(vals - vals[0]), torch.zeros_like(vals))
    z = e.sum()
    excl = torch.cumsum(e, 0) - e
    m1 = float((excl[kept] / z - top_p).abs().min()) if bool(kept.any()) else 1.0
    remove = (excl / z > top_p) & (torch.arange(v) >= 1)
    e = torch.where(remove, torch.zeros_like(e), e)
    cum = torch.cumsum(e, 0) / e.sum()
    m2 = float((cum[e > 0] - u).abs().min())
    return min(m1, m2)


def rmsnorm_bf16(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    """BreezeRMSNorm (breeze.py:115-120), returned as fp32 values of the bf16 result."""
    x32 = x.float()
    var = x32.pow(2).mean(-1, keepdim=True)
    xh = (x32 * torch.rsqrt(var + eps)).to(torch.bfloat16)
    return (gamma.to(torch.bfloat16) * xh).float()


def head(x: torch.Tensor, w: torch.Tensor, layout_kn: bool, gamma=None, eps: float = 1e-6) -> torch.Tensor:
    """fp32 head in float64: (M, N) = y @ W (layout_kn: W is (K, N), else (N, K))."""
    y = rmsnorm_bf16(x, gamma, eps) if gamma is not None else x.float()
    wt = w.double() if layout_kn else w.double().t()
    return (y.double() @ wt).float()
