"""Decode-step projection chain (breeze_b200.fused.stack).

CPU: construction, shape validation, launch and byte counts, and that the
chain refuses to run without the CUDA library path. GPU: every launch of a
two-layer chain checked against the oracle on the inputs it actually read
(max |err| / max |ref| <= TOL), eager and graph replay bit-identical.
"""

import pytest
import torch

from oracle import gemv as og
from oracle import quant

TOL = 1e-2


def _stack():
    from breeze_b200.fused import stack

    return stack


def _small(fmt, device, n_layers=2, seed=0):
    S = _stack()
    return S.synthetic_stack(fmt, n_layers, device, seed=seed, hidden=256, qkv=768, inter=512, head=384)


def test_stack_shapes_and_counts_cpu():
    S = _stack()
    layers, head, ln_f = _small("int8", "cpu")
    st = S.DecodeStack(layers, head, ln_f, rows=3)
    assert st.launches == 4 * 2 + 1
    per_layer = 768 * 256 + 256 * 256 + 1024 * 256 + 256 * 512
    scales = 4 * (768 + 256 + 1024 + 256)
    assert st.weight_bytes == 2 * (per_layer + scales + 2 * 256 * 2) + 384 * 256 + 4 * 384 + 256 * 2
    assert st.logits.shape == (3, 384) and st.logits.dtype == torch.float32


def test_stack_int4_bytes_cpu():
    layers, head, ln_f = _small("int4", "cpu", n_layers=1)
    l = layers[0]
    assert l.wqkv.w.shape == (768 // 8, 256 // 128, 32, 4) and l.wqkv.w.dtype == torch.int32
    assert l.wqkv.scale.shape == (2, 768, 2) and l.wqkv.scale.dtype == torch.bfloat16
    assert l.wqkv.nbytes == 768 * 256 // 2 + 2 * 768 * 2 * 2


def test_stack_rejects_mismatched_layers_cpu():
    S = _stack()
    layers, head, ln_f = _small("fp8", "cpu")
    bad = S.DecodeLayer(layers[1].wqkv, layers[1].wo, layers[1].wgu, layers[0].wqkv, layers[1].ln1, layers[1].ln2)
    with pytest.raises(ValueError):
        S.DecodeStack([layers[0], bad], head, ln_f, rows=1)
    with pytest.raises(ValueError):
        S.DecodeStack([], head, ln_f, rows=1)
    with pytest.raises(ValueError):
        S.DecodeStack(layers, layers[0].wo, ln_f, rows=1, attn_cols=128)


def test_stack_has_no_cpu_path():
    S = _stack()
    layers, head, ln_f = _small("int8", "cpu", n_layers=1)
    st = S.DecodeStack(layers, head, ln_f, rows=1)
    with pytest.raises(Exception):
        st.run()


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


def _check(name, got, x, qw, gamma=None, epilogue=0, residual=None):
    ref = og.fused_reference(x.cpu(), _deq(qw), None if gamma is None else gamma.cpu(), 1e-6, epilogue,
                             None if residual is None else residual.cpu())
    err = og.max_rel_err(got.cpu().float(), ref)
    assert err <= TOL, f"{name}: max rel err {err:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("chain", [False, True])
@pytest.mark.parametrize("fmt", ["int4", "fp8", "int8", "bf16"])
@pytest.mark.parametrize("rows", [1, 2, 5])
def test_stack_stages_match_oracle(fmt, rows, chain):
    S = _stack()
    dev = torch.device("cuda", 0)
    layers, head, ln_f = _small(fmt, dev)
    st = S.DecodeStack(layers, head, ln_f, rows=rows, chain=chain)
    g = torch.Generator().manual_seed(1)
    st.x.copy_(torch.randn(rows, 256, generator=g).to(torch.bfloat16))
    st.run()
    torch.cuda.synchronize()
    # buffers now hold the last layer's intermediates; res[0] is its input
    l = layers[1]
    xin = st.res[0]
    _check("qkv", st.qkv, xin, l.wqkv, gamma=l.ln1)
    _check("o", st.h, st.qkv[:, :256], l.wo, epilogue=2, residual=xin)
    _check("gate_up", st.act, st.h, l.wgu, gamma=l.ln2, epilogue=1)
    _check("down", st.res[1], st.act, l.wd, epilogue=2, residual=st.h)
    _check("head", st.logits, st.res[1], head, gamma=ln_f)
    # first layer, through a one-layer chain on the same input
    st1 = S.DecodeStack(layers[:1], head, ln_f, rows=rows, chain=chain)
    st1.x.copy_(st.x)
    st1.run()
    torch.cuda.synchronize()
    assert torch.equal(st1.res[0], st.res[0])
    _check("qkv0", st1.qkv, st1.x, layers[0].wqkv, gamma=layers[0].ln1)
    _check("down0", st1.res[0], st1.act, layers[0].wd, epilogue=2, residual=st1.h)


@pytest.mark.gpu
@pytest.mark.parametrize("chain", [False, True])
def test_stack_graph_replay_matches_eager(chain):
    S = _stack()
    dev = torch.device("cuda", 0)
    layers, head, ln_f = _small("int4", dev, n_layers=3)
    st = S.DecodeStack(layers, head, ln_f, rows=2, chain=chain)
    st.x.copy_(torch.randn(2, 256, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16))
    st.run()
    torch.cuda.synchronize()
    eager = st.logits.clone()
    st.logits.zero_()
    st.capture()
    st.logits.zero_()
    st.replay()
    torch.cuda.synchronize()
    assert torch.equal(st.logits, eager)
    from breeze_b200 import _lib

    assert _lib.device_status(0) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["int4", "fp8"])
def test_chain_full_size_layer_matches_per_op(fmt):
    """Two full-size decode layers plus the head (the benchmark shapes): the
    chain launch and the per-projection launches agree within tolerance."""
    S = _stack()
    dev = torch.device("cuda", 0)
    layers, head, ln_f = S.synthetic_stack(fmt, 2, dev, seed=3)
    a = S.DecodeStack(layers, head, ln_f, rows=2)
    b = S.DecodeStack(layers, head, ln_f, rows=2, chain=True)
    x = torch.randn(2, 2048, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    a.x.copy_(x)
    b.x.copy_(x)
    a.run()
    b.run()
    torch.cuda.synchronize()
    assert og.max_rel_err(b.logits.cpu(), a.logits.cpu().float()) < TOL


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [1, 2])
def test_stack_with_attention_matches_oracle(rows):
    """attention=True: the attention step sits between QKV and O; its output
    matches the oracle on the QKV output and the caches it read, and O, gate+up,
    down and the head still match stage by stage."""
    from oracle import attention as oa

    S = _stack()
    dev = torch.device("cuda", 0)
    layers, head, ln_f = _small("int4", dev)
    st = S.DecodeStack(layers, head, ln_f, rows=rows, attention=True, kv_len=64)
    assert (st.hq, st.hkv) == (2, 2) and st.launches == 11
    g = torch.Generator().manual_seed(9)
    st.x.copy_(torch.randn(rows, 256, generator=g).to(torch.bfloat16))
    for c in st.k_cache + st.v_cache:
        c.copy_((torch.randn(c.shape, generator=g) * 0.5).to(torch.bfloat16))
    k_before = [c.cpu() for c in st.k_cache]
    v_before = [c.cpu() for c in st.v_cache]
    st.pos.fill_(40)
    st.run()
    torch.cuda.synchronize()
    l = layers[1]
    ref, _, _ = oa.attention_step(st.qkv.cpu(), st.cos.cpu(), st.sin.cpu(), 40, k_before[1].clone(),
                                  v_before[1].clone(), torch.zeros(rows, 64), l.q_norm.cpu(), l.k_norm.cpu(), 1e-6)
    assert og.max_rel_err(st.attn_out.cpu().float(), ref.float()) < TOL
    _check("o", st.h, st.attn_out, l.wo, epilogue=2, residual=st.res[0])
    _check("gate_up", st.act, st.h, l.wgu, gamma=l.ln2, epilogue=1)
    _check("head", st.logits, st.res[1], head, gamma=ln_f)


@pytest.mark.gpu
def test_stack_fp32_lm_head_and_in_graph_sampling():
    """lm_head (fp32, norm fused) replaces the quantized head; the token is
    drawn in the graph with CFG, repetition penalty over the appended history,
    the suppressed range, and the EOS flag."""
    from oracle import sampling as osm

    S = _stack()
    dev = torch.device("cuda", 0)
    layers, _, ln_f = _small("int4", dev)
    g = torch.Generator().manual_seed(21)
    lm = torch.randn(300, 256, generator=g) * 0.05
    st = S.DecodeStack(layers, None, ln_f, rows=2, lm_head=lm.to(dev),
                       sampling=dict(do_sample=False, repetition_penalty=1.3, suppress=(296, 299), guidance_scale=2.0,
                                     history_cap=8))
    assert st.launches == 4 * 2 + 2
    st.x.copy_(torch.randn(2, 256, generator=g).to(torch.bfloat16))
    st.token.fill_(7)
    st.capture()  # one eager warm-up step, then the graph
    torch.cuda.synchronize()
    assert int(st.history_len[0]) == 1 and int(st.history[0, 0]) == 7
    ref = osm.head(st.res[1].cpu(), lm, False, ln_f.cpu(), 1e-6)
    assert og.max_rel_err(st.logits.cpu(), ref) < 2e-3
    mixed = osm.mixed_logits(st.logits.cpu(), 1, torch.tensor([2.0]), mask=(296, 299), rep_penalty=1.3,
                             history=st.history.cpu(), history_len=st.history_len.cpu())
    tok = int(torch.argmax(mixed[0]))
    assert int(st.token[0]) == tok and int(st.token[1]) == tok
    assert int(st.eos_flag[0]) == 0
    prev = tok
    st.replay()
    torch.cuda.synchronize()
    assert int(st.history_len[0]) == 2 and int(st.history[0, 1]) == prev
    # EOS: a stack whose eos_id is the token it will draw raises the flag
    st2 = S.DecodeStack(layers, None, ln_f, rows=2, lm_head=lm.to(dev),
                        sampling=dict(do_sample=False, repetition_penalty=1.3, suppress=(296, 299),
                                      guidance_scale=2.0, history_cap=8, eos_id=tok))
    st2.x.copy_(st.x)
    st2.token.fill_(7)
    st2.run()
    torch.cuda.synchronize()
    assert int(st2.token[0]) == tok and int(st2.eos_flag[0]) == 1
