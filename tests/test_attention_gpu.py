"""Decode attention step (bq_attention_step) against the reference's Triton
attention_step recorded on a B200 (tests/golden/attention_step.npz) and the
CPU oracle (oracle/attention.py) on seeded cases: output within max rel err
1e-2, the new v written bit-exactly, the new k within one bf16 ulp, every
other cache position untouched."""

import pytest
import torch

from oracle import attention as oa
from oracle import gemv as og
from oracle.quant import from_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-2


def _attn():
    from breeze_b200.fused.kernels import attention_step

    return attention_step


def _check(out, keys, values, ref_out, ref_k, ref_v, k0, pos):
    assert og.max_rel_err(out.cpu().float(), ref_out.float()) < TOL
    assert torch.equal(values.cpu()[:, :, pos], ref_v)
    kd = (keys.cpu()[:, :, pos].float() - ref_k.float()).abs()
    assert (kd <= ref_k.float().abs() * 2 ** -7 + 1e-6).all()
    other = torch.ones(keys.shape[2], dtype=torch.bool)
    other[pos] = False
    assert torch.equal(keys.cpu()[:, :, other], k0[:, :, other])


@pytest.mark.parametrize("tag", ["c0", "c1"])
def test_attention_matches_reference_golden(golden, tag):
    d = golden("attention_step.npz")
    bf = torch.bfloat16
    g = {k: from_bits(d[f"{k}_{tag}"], bf) for k in ("qkv", "k", "v", "qn", "kn", "cos", "sin", "mask", "out",
                                                     "k_after", "v_after")}
    pos = int(d[f"pos_{tag}"][0])
    keys, values = g["k"].to(DEV), g["v"].to(DEV)
    out = _attn()(g["qkv"].to(DEV), g["cos"].to(DEV), g["sin"].to(DEV), torch.tensor([pos], device=DEV), keys, values,
                  g["mask"].to(DEV), g["qn"].to(DEV), g["kn"].to(DEV), 1e-6)
    torch.cuda.synchronize()
    _check(out, keys, values, g["out"], g["k_after"], g["v_after"], g["k"], pos)


CASES = [
    # B, HQ, HKV, D, S, pos, norm, mask, bcast_rope
    (1, 16, 16, 128, 256, 255, True, "float", False),
    (2, 16, 16, 128, 256, 100, True, "bool", True),
    (5, 8, 1, 128, 1024, 777, False, None, False),
    (2, 4, 2, 64, 48, 0, True, "float", False),
    (3, 6, 3, 64, 600, 599, False, "bool", False),
    (2, 32, 8, 128, 4096, 3000, True, "float", True),
    # 256 (row, kv head) pairs after the smaller cases: the workspace's counter
    # region must not overlap what earlier calls wrote as partials
    (16, 16, 16, 128, 512, 300, False, None, True),
]


@pytest.mark.parametrize("case", CASES)
def test_attention_matches_oracle(case):
    B, HQ, HKV, D, S, pos, norm, mk, bcast = case
    g = torch.Generator().manual_seed(B * 1000 + HQ * 10 + D + S)
    qkv = torch.randn(B, (HQ + 2 * HKV) * D, generator=g).to(torch.bfloat16)
    k0 = (torch.randn(B, HKV, S, D, generator=g) * 0.5).to(torch.bfloat16)
    v0 = torch.randn(B, HKV, S, D, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16) if norm else None
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16) if norm else None
    rb = 1 if bcast else B
    ang = torch.rand(rb, 1, D // 2, generator=g) * 6.0
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    if mk == "bool":
        mask = torch.zeros(B, 1, 1, S, dtype=torch.bool)
        mask[:, :, :, : pos + 1] = True
        if B > 1:
            mask[1, :, :, : min(3, pos)] = False
    elif mk == "float":
        mask = torch.full((B, 1, 1, S), torch.finfo(torch.bfloat16).min)
        mask[:, :, :, : pos + 1] = 0.0
        mask = mask.to(torch.bfloat16)
    else:
        mask = None
    ref_out, ref_k, ref_v = oa.attention_step(qkv, cos, sin, pos, k0.clone(), v0.clone(),
                                             mask if mask is not None else torch.zeros(B, S), qn, kn, 1e-6)
    keys, values = k0.to(DEV), v0.to(DEV)
    out = _attn()(qkv.to(DEV), cos.to(DEV), sin.to(DEV), torch.tensor([pos], device=DEV), keys, values,
                  None if mask is None else mask.to(DEV), None if qn is None else qn.to(DEV),
                  None if kn is None else kn.to(DEV), 1e-6)
    torch.cuda.synchronize()
    _check(out, keys, values, ref_out, ref_k[:, :, pos], ref_v[:, :, pos], k0, pos)


def test_attention_graph_replay_follows_cache_position():
    """Captured once, replayed with the device-side position advanced: each
    replay writes its own cache slot and attends over [0, pos]."""
    B, HQ, HKV, D, S = 2, 16, 16, 128, 256
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn(B, (HQ + 2 * HKV) * D, generator=g).to(torch.bfloat16).to(DEV)
    keys = (torch.randn(B, HKV, S, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    values = torch.randn(B, HKV, S, D, generator=g).to(torch.bfloat16).to(DEV)
    cos = torch.ones(B, 1, D, dtype=torch.bfloat16, device=DEV)
    sin = torch.zeros(B, 1, D, dtype=torch.bfloat16, device=DEV)
    pos = torch.tensor([10], device=DEV)
    out = torch.empty(B, HQ * D, dtype=torch.bfloat16, device=DEV)
    attn = _attn()
    attn(qkv, cos, sin, pos, keys, values, None, out=out)
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            attn(qkv, cos, sin, pos, keys, values, None, out=out)
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    for p_ in (11, 200):
        pos.fill_(p_)
        k_before = keys.cpu()
        graph.replay()
        torch.cuda.synchronize()
        ref_out, ref_k, ref_v = oa.attention_step(qkv.cpu(), cos.cpu(), sin.cpu(), p_, k_before.clone(),
                                                 values.cpu().clone(), torch.zeros(B, S))
        _check(out, keys, values, ref_out, ref_k[:, :, p_], ref_v[:, :, p_], k_before, p_)
    from breeze_b200 import _lib

    assert _lib.device_status(0) == 0


FUSED_O_CASES = [
    # B, HQ, HKV, D, S, pos, norm, N, bcast_rope, mask
    (1, 8, 8, 128, 17, 16, True, 1024, True, None),    # depth decoder step
    (2, 8, 8, 128, 17, 0, True, 1024, True, None),
    (3, 4, 2, 64, 48, 30, False, 256, False, "bool"),
    (4, 16, 8, 128, 256, 255, True, 2048, False, "float"),
    (1, 8, 8, 128, 64, 40, True, 48, True, None),      # 16-row chunks
    (2, 8, 8, 128, 17, 9, True, 1024, True, "float"),  # the HF causal mask of a decoder layer
    (2, 16, 16, 128, 64, 30, True, 512, True, None),   # HKV > 8: global partials, no cluster
]


@pytest.mark.parametrize("case", FUSED_O_CASES)
def test_attention_o_step_matches_oracle(case):
    """bq_attention_o_step: residual + attention @ Wo^T in one launch, against
    the attention oracle (output rounded to bf16, as the unfused step stores
    it) followed by an fp32 projection: within 1e-2; caches written as by
    attention_step; a rerun is bit-identical."""
    from breeze_b200 import _lib as L

    B, HQ, HKV, D, S, pos, norm, N, bcast, mk = case
    g = torch.Generator().manual_seed(B * 7 + HQ + D + S + N)
    qkv = torch.randn(B, (HQ + 2 * HKV) * D, generator=g).to(torch.bfloat16)
    k0 = (torch.randn(B, HKV, S, D, generator=g) * 0.5).to(torch.bfloat16)
    v0 = torch.randn(B, HKV, S, D, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16) if norm else None
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16) if norm else None
    ang = torch.rand(1 if bcast else B, 1, D // 2, generator=g) * 6.0
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    wo = (torch.randn(N, HQ * D, generator=g) * 0.02).to(torch.bfloat16)
    res = torch.randn(B, N, generator=g).to(torch.bfloat16)
    mask = None
    if mk == "bool":
        mask = torch.zeros(B, 1, 1, S, dtype=torch.bool)
        mask[:, :, :, : pos + 1] = True
        mask[1, :, :, : min(3, pos)] = False
    elif mk == "float":
        mask = torch.full((B, 1, 1, S), torch.finfo(torch.bfloat16).min)
        mask[:, :, :, : pos + 1] = 0.0
        mask = mask.to(torch.bfloat16)
    ref_attn, ref_k, ref_v = oa.attention_step(qkv, cos, sin, pos, k0.clone(), v0.clone(),
                                               mask if mask is not None else torch.zeros(B, S), qn, kn, 1e-6)
    ref = res.float() + ref_attn.float() @ wo.float().T
    keys, values = k0.to(DEV), v0.to(DEV)
    args = (qkv.to(DEV), cos.to(DEV), sin.to(DEV), torch.tensor([pos], device=DEV), keys, values,
            None if qn is None else qn.to(DEV), None if kn is None else kn.to(DEV), 1e-6, wo.to(DEV), res.to(DEV))
    m = None if mask is None else mask.to(DEV)
    out = L.attention_o_step(*args, flags=L.default_flags(), mask=m)
    again = L.attention_o_step(*args, flags=L.default_flags(), mask=m)
    torch.cuda.synchronize()
    assert out.shape == (B, N)
    assert og.max_rel_err(out.cpu().float(), ref) < TOL
    assert torch.equal(out, again)
    assert torch.equal(values.cpu()[:, :, pos], ref_v[:, :, pos])
    kd = (keys.cpu()[:, :, pos].float() - ref_k[:, :, pos].float()).abs()
    assert (kd <= ref_k[:, :, pos].float().abs() * 2 ** -7 + 1e-6).all()
    other = torch.ones(S, dtype=torch.bool)
    other[pos] = False
    assert torch.equal(keys.cpu()[:, :, other], k0[:, :, other])
    assert L.device_status() == 0
