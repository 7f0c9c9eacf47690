"""Depth-decoder frame (breeze_b200.fused.depth.DepthDecoderLoop).

CPU: construction, buffer shapes, launch counts, and no CPU path. GPU: a
small seeded depth decoder run as one frame (prefill at positions 0-1, then
single steps) is compared step by step with the teacher-forced CPU oracle
(oracle/depth.py): every step's fp32 logits within max rel err 1e-2; greedy
tokens equal the argmax of the oracle's CFG-mixed, masked logits (where the
top two differ by more than 1e-3 of the logit scale); sampled tokens equal the
sampler oracle's draw from the GPU's own logits with the Philox u of that
launch; graph replay of a greedy frame equals the eager run.
"""

import pytest
import torch

from oracle import depth as od
from oracle import gemv as og
from oracle import quant
from oracle import sampling as osm

TOL = 1e-2
CFG = dict(hidden=256, inter=256, q_heads=2, kv_heads=1, head_dim=128, emb_width=384, vocab=300, num_codebooks=5)
CODEBOOK = 296


def _build(fmt, dev, batch, attn_fmt=None, **kw):
    from breeze_b200.fused import depth

    layers, norm_w, head, embed, in_proj = depth.synthetic_depth(fmt, 2, dev, seed=5, attn_fmt=attn_fmt, **CFG)
    loop = depth.DepthDecoderLoop(layers, norm_w, head, embed, in_proj, batch, codebook_size=CODEBOOK,
                                  kv_heads=CFG["kv_heads"], **kw)
    return loop


def test_depth_loop_shapes_cpu():
    loop = _build("int8", "cpu", 2)
    assert loop.half == 1 and loop.cfg and loop.n_dec == 4 and loop.kv_len == 6
    assert loop.output_tokens.shape == (2, 4) and loop.step_logits.shape == (4, 2, 300)
    assert loop.launches == (1 + 1 + 6 * 2 + 2) + 3 * (2 + 5 * 2 + 2)
    assert loop.backbone_hidden_buf.shape == (2, 384)
    with pytest.raises(Exception):
        loop.run()
    with pytest.raises(ValueError):
        loop.set_top_k(5000)
    # bf16 O: the single steps fuse attention, O projection and residual (one launch fewer per layer)
    fused = _build("int8", "cpu", 2, attn_fmt="bf16")
    assert fused.launches == (1 + 1 + 6 * 2 + 2) + 3 * (2 + 4 * 2 + 2)
    assert _build("int8", "cpu", 2, attn_fmt="bf16", fuse_attention_o=False).launches == loop.launches


def _deq(qw):
    from breeze_b200 import _lib as L

    w, s = qw.w.cpu(), None if qw.scale is None else qw.scale.cpu()
    if qw.wfmt == L.W_INT4_TINYGEMM:
        return quant.dequant_int4_tinygemm(w, s, qw.group)
    if qw.wfmt == L.W_FP8_E4M3:
        return quant.dequant_fp8(w, s)
    if qw.wfmt == L.W_INT8:
        return quant.dequant_int8(w, s, dtype=torch.float32)
    return w.float()


def _oracle_logits(loop, bb, first):
    layers = [dict(wqkv=_deq(l.wqkv), wo=_deq(l.wo), wgu=_deq(l.wgu), wd=_deq(l.wd), ln1=l.ln1.cpu(), ln2=l.ln2.cpu(),
                   qn=l.q_norm.cpu(), kn=l.k_norm.cpu()) for l in loop.layers]
    return od.frame_logits(bb, first, loop.output_tokens.cpu(), layers, loop.norm_w.cpu(), loop.head_w.cpu(),
                           loop.embed.cpu(), _deq(loop.in_proj), loop.cos.cpu(), loop.sin.cpu(), loop.n_dec, loop.hkv,
                           loop.head_dim)


def _inputs(loop, seed):
    g = torch.Generator().manual_seed(seed)
    bb = torch.randn(loop.B, loop.backbone_hidden_buf.shape[1], generator=g).to(torch.bfloat16)
    first = torch.randint(0, CODEBOOK, (loop.half,), generator=g)
    first = torch.cat([first, first]) if loop.cfg else first
    loop.backbone_hidden_buf.copy_(bb)
    loop.first_cb_token_buf.copy_(first)
    return bb, first


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,attn_fmt", [("int4", None), ("fp8", None), ("int4", "bf16")])
@pytest.mark.parametrize("batch", [1, 2, 4])
def test_depth_greedy_frame_matches_oracle(fmt, attn_fmt, batch):
    """attn_fmt bf16 runs the single steps through the fused attention + O launch."""
    dev = torch.device("cuda", 0)
    loop = _build(fmt, dev, batch, attn_fmt=attn_fmt, do_sample=False, guidance_scale=2.0)
    bb, first = _inputs(loop, 11 + batch)
    loop.run()
    torch.cuda.synchronize()
    ref = _oracle_logits(loop, bb, first)
    got = loop.step_logits.cpu()
    toks = loop.output_tokens.cpu()
    for j in range(loop.n_dec):
        assert og.max_rel_err(got[j], ref[j]) < TOL, f"step {j}"
        mixed = osm.mixed_logits(ref[j], loop.half, torch.full((loop.half,), 2.0) if loop.cfg else None,
                                 mask=(CODEBOOK, loop.vocab))
        for r in range(loop.half):
            top2 = torch.topk(mixed[r], 2).values
            if float(top2[0] - top2[1]) > 1e-3 * float(mixed[r][mixed[r] > -1e30].abs().max()):
                assert int(toks[r, j]) == int(torch.argmax(mixed[r])), f"step {j} row {r}"
            if loop.cfg:
                assert int(toks[r + loop.half, j]) == int(toks[r, j])


@pytest.mark.gpu
def test_depth_sampled_frame_uses_philox_draws():
    dev = torch.device("cuda", 0)
    loop = _build("int4", dev, 2, do_sample=True, temperature=0.9, top_k=20, top_p=0.9, guidance_scale=3.0,
                  seed=1234)
    bb, first = _inputs(loop, 5)
    loop.run()
    torch.cuda.synchronize()
    assert int(loop.rng[1]) == loop.n_dec
    got = loop.step_logits.cpu()
    ref = _oracle_logits(loop, bb, first)
    toks = loop.output_tokens.cpu()
    checked = 0
    for j in range(loop.n_dec):
        assert og.max_rel_err(got[j], ref[j]) < TOL
        mixed = osm.mixed_logits(got[j], 1, torch.full((1,), 3.0), mask=(CODEBOOK, loop.vocab))
        u = osm.philox_uniform(1234, j, 0)
        if osm.draw_margin(mixed[0], 0.9, 20, 0.9, u, loop.max_k) < 1e-5:
            continue
        assert int(toks[0, j]) == osm.sample_row(mixed[0], 0.9, 20, 0.9, True, u, loop.max_k)
        checked += 1
    assert checked >= loop.n_dec - 1


@pytest.mark.gpu
@pytest.mark.parametrize("attn_fmt", [None, "bf16"])
def test_depth_graph_replay_matches_eager(attn_fmt):
    dev = torch.device("cuda", 0)
    loop = _build("int4", dev, 2, attn_fmt=attn_fmt, do_sample=False)
    _inputs(loop, 21)
    loop.run()
    torch.cuda.synchronize()
    eager_tok = loop.output_tokens.clone()
    eager_logits = loop.step_logits.clone()
    loop.capture()
    loop.output_tokens.zero_()
    loop.step_logits.zero_()
    loop.replay()
    torch.cuda.synchronize()
    assert torch.equal(loop.output_tokens, eager_tok)
    assert torch.equal(loop.step_logits, eager_logits)
    # sampling switched on without a recapture: draws advance with every replay
    loop.set_do_sample(True)
    c0 = int(loop.rng[1])
    loop.replay()
    loop.replay()
    torch.cuda.synchronize()
    assert int(loop.rng[1]) == c0 + 2 * loop.n_dec
    from breeze_b200 import _lib

    assert _lib.device_status(0) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 2])
def test_depth_fused_attention_o_matches_separate_launches(batch):
    """The fused attention + O step against attention_step + O GEMV on the same
    weights and inputs: caches within bf16 rounding of each other, per-step
    logits within 1e-2, greedy tokens equal where the margin allows."""
    dev = torch.device("cuda", 0)
    runs = []
    for fuse in (False, True):
        loop = _build("int4", dev, batch, attn_fmt="bf16", do_sample=False, guidance_scale=2.0, fuse_attention_o=fuse)
        _inputs(loop, 31 + batch)
        loop.run()
        torch.cuda.synchronize()
        runs.append(loop)
    a, b = runs
    assert b.launches == a.launches - (a.n_dec - 1) * len(a.layers)
    # compare until the first token that may differ (a near-tie); later steps depend on it
    same = True
    for j in range(a.n_dec):
        assert og.max_rel_err(b.step_logits[j].cpu(), a.step_logits[j].cpu()) < TOL, f"step {j}"
        mixed = osm.mixed_logits(a.step_logits[j].cpu(), a.half, torch.full((a.half,), 2.0) if a.cfg else None,
                                 mask=(CODEBOOK, a.vocab))
        for r in range(a.half):
            top2 = torch.topk(mixed[r], 2).values
            if float(top2[0] - top2[1]) > 1e-2 * float(mixed[r][mixed[r] > -1e30].abs().max()):
                assert int(b.output_tokens[r, j]) == int(a.output_tokens[r, j]), f"step {j} row {r}"
        if not torch.equal(b.output_tokens[:, j], a.output_tokens[:, j]):
            same = False
            break
    if same:
        for i in range(len(a.layers)):
            for ca, cb in ((a.k_cache[i], b.k_cache[i]), (a.v_cache[i], b.v_cache[i])):
                assert og.max_rel_err(cb.float().cpu(), ca.float().cpu()) < TOL
