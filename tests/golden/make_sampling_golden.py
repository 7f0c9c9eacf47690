"""Golden fixtures for the sampling oracle, from the reference itself (CPU).

Calls the reference's own ``DepthDecoderGraph._cfg_sample``
(models/cudagraph/depth_decoder_graph.py:487-558) and ``sample_logits``
(models/cudagraph/sampling.py:36-87) on seeded CPU logits. Both end in
``torch.multinomial``; it is replaced for the duration of a call by a
recorder that stores the probability vector it is handed (and returns its
argmax), so the fixture holds exactly the distribution the reference samples
from. Greedy cases (do_sample off) store the reference's token.

    python tests/golden/make_sampling_golden.py --ref <reference tree> --out tests/golden
"""

from __future__ import annotations

import argparse
import sys
import types
from pathlib import Path

import numpy as np
import torch

# (rows, cfg, V, codebook_size, max_k, temperature, top_k, top_p, do_sample, guidance, seed)
DEPTH_CASES = [
    (1, False, 2051, 2048, 1024, 0.9, 50, 0.95, 1, 1.0, 1),
    (2, True, 2051, 2048, 1024, 0.7, 0, 0.9, 1, 3.0, 2),
    (2, True, 2051, 2048, 1024, 1.0, 8, 1.0, 1, 1.5, 3),
    (1, True, 2051, 2048, 1024, 1.3, 300, 0.5, 1, 2.0, 4),
    (1, False, 2051, 2048, 1024, 0.8, 50, 0.9, 0, 1.0, 5),
    (2, True, 2051, 2048, 1024, 0.8, 50, 0.9, 0, 2.5, 7),
    (1, False, 4099, 4096, 1024, 1.1, 1024, 0.99, 1, 1.0, 6),
]
# (V, temperature, top_k, top_p, do_sample, rep_penalty, hist_len, n_suppress, seed)
BACKBONE_CASES = [
    (2049, 0.9, 50, 0.95, True, 1.1, 40, 1, 11),
    (2049, 1.0, 0, 0.8, True, 1.3, 200, 2, 12),
    (2049, 0.7, 20, 1.0, True, 1.0, 0, 0, 13),
    (2049, 0.9, 50, 0.95, False, 1.2, 64, 1, 14),
]


class _Recorder:
    def __init__(self):
        self.probs = []

    def __call__(self, probs, num_samples, *a, **k):
        self.probs.append(probs.detach().clone())
        return torch.argmax(probs, dim=-1, keepdim=True)


def depth_case(dd, rows, cfg, v, cb, max_k, temp, top_k, top_p, do_sample, g, seed):
    gen = torch.Generator().manual_seed(seed)
    batch = 2 * rows if cfg else rows
    logits = torch.randn(batch, 1, v, generator=gen) * 3.0
    ns = types.SimpleNamespace(
        batch_size=batch, half=rows, codec_codebook_size=cb, vocab_size=v, _max_k=max_k,
        _topk_ranks=torch.arange(max_k), guidance_scale=torch.full((rows, 1), g),
        temperature_buf=torch.full((rows, 1), temp), top_k_buf=torch.full((rows, 1), top_k, dtype=torch.long),
        top_p_buf=torch.full((rows, 1), top_p), do_sample_buf=torch.full((rows,), do_sample, dtype=torch.long),
        _debug_probs_slot=None, _tok_buf=torch.zeros(batch, dtype=torch.long))
    rec = _Recorder()
    orig = torch.multinomial
    torch.multinomial = rec
    try:
        dd.DepthDecoderGraph._cfg_sample(ns, logits)
    finally:
        torch.multinomial = orig
    return logits[:, 0, :].numpy(), rec.probs[0].numpy(), ns._tok_buf.numpy()


def backbone_case(sm, v, temp, top_k, top_p, do_sample, pen, hist_len, n_sup, seed):
    gen = torch.Generator().manual_seed(seed)
    logits = torch.randn(1, v, generator=gen) * 3.0
    hist = torch.randint(0, v, (max(hist_len, 1),), generator=gen)[:hist_len]
    sup = torch.zeros(v, dtype=torch.bool)
    if n_sup:
        sup[torch.randint(0, v, (n_sup,), generator=gen)] = True
    rec = _Recorder()
    orig = torch.multinomial
    torch.multinomial = rec
    try:
        tok = sm.sample_logits(logits, temperature=temp, top_k=top_k, top_p=top_p, do_sample=do_sample,
                               token_history=hist, repetition_penalty=pen, suppress_mask=sup if n_sup else None)
    finally:
        torch.multinomial = orig
    probs = rec.probs[0].numpy() if rec.probs else np.zeros((1, v), np.float32)
    return logits.numpy(), hist.numpy(), sup.numpy(), probs, np.asarray(tok).reshape(-1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    from models.cudagraph import depth_decoder_graph as dd
    from models.cudagraph import sampling as sm

    out = {}
    for i, c in enumerate(DEPTH_CASES):
        logits, probs, toks = depth_case(dd, *c)
        out[f"depth{i}_case"] = np.asarray(c, dtype=np.float64)
        out[f"depth{i}_logits"] = logits
        out[f"depth{i}_probs"] = probs
        out[f"depth{i}_tokens"] = toks
    for i, c in enumerate(BACKBONE_CASES):
        logits, hist, sup, probs, tok = backbone_case(sm, *c)
        out[f"bb{i}_case"] = np.asarray(c, dtype=np.float64)
        out[f"bb{i}_logits"] = logits
        out[f"bb{i}_history"] = hist
        out[f"bb{i}_suppress"] = sup
        out[f"bb{i}_probs"] = probs
        out[f"bb{i}_token"] = tok
    np.savez_compressed(Path(a.out) / "sampling.npz", **out)
    print("wrote", Path(a.out) / "sampling.npz", len(out), "arrays")


if __name__ == "__main__":
    main()
