"""FusedDecoderLayer and install_fused_* (breeze_b200.fused.layer / install).

Built around a small transformers Qwen3 decoder layer (the backbone's layer
type, q/k norms included) with bf16, fp8 (Fp8Linear) and int4 (Int4Linear)
MLPs.

CPU: construction, the weight set it builds, and which calls it takes.

GPU: one call over T new positions (T = 1, and T = 2 for the depth decoder's
two-position prefill) with every library launch the layer makes recorded as
it happens. Each stage is checked against the oracle on the inputs it
actually read, at max rel err 1e-2: the QKV GEMV (RMSNorm fused), each
position's attention step (output, and the new k / v written into the cache:
v bit-exact, k within one bf16 ulp), the O GEMV (+ residual) or the fused
attention + O launch, gate+up (RMSNorm, SiLU*up) and down (+ residual). The
whole call is also checked against the oracle run end to end in fp32 from
the layer's input (1e-2), and, as a cross-check with a different rounding
scheme, against the wrapped layer's own eager forward on a copy of the same
cache (2e-2: the wrapped layer rounds every intermediate to bf16 -- norm
output, q / k / v, attention output, MLP activations -- which the oracle
does not).
"""

import copy
import types

import pytest
import torch

from gpu_cases import dequant_qweight
from oracle import attention as oa
from oracle import gemv as og

H, HEADS, KVH, HD, INTER = 256, 2, 1, 128, 256
TOL = 1e-2
EPS = 1e-6


def _config():
    from transformers import Qwen3Config

    cfg = Qwen3Config(hidden_size=H, num_attention_heads=HEADS, num_key_value_heads=KVH, head_dim=HD,
                      intermediate_size=INTER, num_hidden_layers=2, rms_norm_eps=EPS, vocab_size=64,
                      max_position_embeddings=64)
    cfg._attn_implementation = "eager"
    return cfg


def _layer(device, dtype=torch.bfloat16, seed=0):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3DecoderLayer

    torch.manual_seed(seed)
    layer = Qwen3DecoderLayer(_config(), 0).to(device=device, dtype=dtype).eval()
    with torch.no_grad():
        for p in layer.parameters():
            if p.dim() == 1:
                p.copy_(1 + 0.1 * torch.randn_like(p))
    return layer


def test_fused_layer_construction_cpu():
    from breeze_b200 import _lib
    from breeze_b200.fused.layer import FusedDecoderLayer

    fl = FusedDecoderLayer(_layer("cpu"), 0)
    w = fl.weights
    assert fl.kv_heads == KVH and fl.head_dim == HD and fl.layer_idx == 0
    assert (w.wqkv.N, w.wqkv.K) == ((HEADS + 2 * KVH) * HD, H) and (w.wo.N, w.wo.K) == (H, HEADS * HD)
    assert (w.wgu.N, w.wgu.K) == (2 * INTER, H) and (w.wd.N, w.wd.K) == (H, INTER)
    assert w.wqkv.wfmt == _lib.W_BF16 and w.wgu.wfmt == _lib.W_BF16
    assert w.q_norm is not None and w.k_norm is not None
    fl8 = FusedDecoderLayer(_layer("cpu"), 1, mlp_bits=8, attn_bits=8)
    assert fl8.weights.wqkv.wfmt == _lib.W_FP8_E4M3 and fl8.weights.wd.wfmt == _lib.W_FP8_E4M3


def test_fused_layer_dispatch_cpu():
    """Long prefills, calls without a static cache or without rotary
    embeddings / mask go to the wrapped layer."""
    from breeze_b200.fused.layer import MAX_NEW_POSITIONS, FusedDecoderLayer

    fl = FusedDecoderLayer(_layer("cpu"), 0)
    cache = types.SimpleNamespace(layers=[None])
    pe = (torch.ones(1), torch.zeros(1))
    mask, pos = torch.zeros(1), torch.zeros(1)

    def x(t):
        return torch.zeros(2, t, H)

    assert fl.handles(x(1), mask, cache, pos, pe) and fl.handles(x(MAX_NEW_POSITIONS), mask, cache, pos, pe)
    assert not fl.handles(x(MAX_NEW_POSITIONS + 1), mask, cache, pos, pe)
    assert not fl.handles(x(1), mask, None, pos, pe)
    assert not fl.handles(x(1), None, cache, pos, pe)
    assert not fl.handles(x(1), mask, cache, pos, None)
    assert not fl.handles(x(1), mask, cache, None, pe)


def _mask(b, s, first, t, dtype, device):
    """(b, 1, t, s) additive causal mask for positions first .. first + t - 1."""
    m = torch.full((b, 1, t, s), torch.finfo(dtype).min, dtype=dtype, device=device)
    for i in range(t):
        m[:, :, i, : first + i + 1] = 0
    return m


class _Recorder:
    """Wraps the library calls the layer makes and keeps CPU copies of what
    each one read and wrote."""

    def __init__(self, monkeypatch):
        from breeze_b200 import _lib

        self.calls = []
        real_gemv, real_attn, real_attn_o = _lib.gemv, _lib.attention_step, _lib.attention_o_step

        def gemv(x, w, wfmt, n, **kw):
            out = real_gemv(x, w, wfmt, n, **kw)
            self.calls.append(("gemv", dict(x=x.cpu(), w=w, wfmt=wfmt, n=n, scale=kw.get("scale"),
                                            group=kw.get("group", 128), gamma=_cpu(kw.get("gamma")),
                                            epilogue=kw.get("epilogue", 0), residual=_cpu(kw.get("residual")),
                                            out=out.cpu())))
            return out

        def attention_step(qkv, cos, sin, pos, keys, values, mask, qn, kn, eps, out=None, flags=0):
            before = (keys.cpu(), values.cpu())
            res = real_attn(qkv, cos, sin, pos, keys, values, mask, qn, kn, eps, out=out, flags=flags)
            self.calls.append(("attn", dict(qkv=qkv.cpu(), cos=cos.cpu(), sin=sin.cpu(), pos=int(pos[0]),
                                            before=before, after=(keys.cpu(), values.cpu()), mask=mask.cpu(),
                                            qn=_cpu(qn), kn=_cpu(kn), out=res.cpu())))
            return res

        def attention_o_step(qkv, cos, sin, pos, keys, values, qn, kn, eps, wo, residual, out=None, flags=0,
                             mask=None):
            before = (keys.cpu(), values.cpu())
            res = real_attn_o(qkv, cos, sin, pos, keys, values, qn, kn, eps, wo, residual, out=out, flags=flags,
                              mask=mask)
            self.calls.append(("attn_o", dict(qkv=qkv.cpu(), cos=cos.cpu(), sin=sin.cpu(), pos=int(pos[0]),
                                              before=before, after=(keys.cpu(), values.cpu()), mask=mask.cpu(),
                                              qn=_cpu(qn), kn=_cpu(kn), wo=wo.cpu(), residual=residual.cpu(),
                                              out=res.cpu())))
            return res

        monkeypatch.setattr(_lib, "gemv", gemv)
        monkeypatch.setattr(_lib, "attention_step", attention_step)
        monkeypatch.setattr(_lib, "attention_o_step", attention_o_step)


def _cpu(t):
    return None if t is None else t.cpu()


def _check_attention(c, name):
    """Output and cache writes of one attention launch against the oracle."""
    k0, v0 = c["before"]
    ref, rk, rv = oa.attention_step(c["qkv"], c["cos"], c["sin"], c["pos"], k0.clone(), v0.clone(), c["mask"],
                                    c["qn"], c["kn"], EPS)
    p = c["pos"]
    k1, v1 = c["after"]
    assert torch.equal(v1[:, :, p], rv[:, :, p]), f"{name}: v written at {p}"
    kd = (k1[:, :, p].float() - rk[:, :, p].float()).abs()
    assert (kd <= rk[:, :, p].float().abs() * 2 ** -7 + 1e-6).all(), f"{name}: k written at {p}"
    return ref


def _check_call(rec, fl, t, b):
    """Every recorded launch of one layer call, in the order the layer makes them."""
    from breeze_b200 import _lib

    w = fl.weights
    kinds = [k for k, _ in rec.calls]
    fused_o = "attn_o" in kinds
    assert kinds == ["gemv"] + ["attn_o" if fused_o else "attn"] * t + ([] if fused_o else ["gemv"]) + ["gemv"] * 2
    calls = [c for _, c in rec.calls]
    qkv = calls[0]
    assert qkv["x"].shape[0] == t * b
    ref = og.fused_reference(qkv["x"], dequant_qweight(w.wqkv), qkv["gamma"], EPS, 0)
    assert og.max_rel_err(qkv["out"].float(), ref) <= TOL, "qkv"
    for i in range(t):
        c = calls[1 + i]
        attn = _check_attention(c, f"attention {i}")
        if fused_o:
            ref = og.linear_epilogue(attn.float(), c["wo"].float(), _lib.EPI_ADD_RESIDUAL, c["residual"])
            assert og.max_rel_err(c["out"].float(), ref) <= TOL, f"attention+O {i}"
        else:
            assert og.max_rel_err(c["out"].float(), attn.float()) <= TOL, f"attention {i}"
    rest = calls[1 + t:]
    if not fused_o:
        o = rest.pop(0)
        ref = og.fused_reference(o["x"], dequant_qweight(w.wo), None, EPS, _lib.EPI_ADD_RESIDUAL, o["residual"])
        assert og.max_rel_err(o["out"].float(), ref) <= TOL, "o"
    gu, dn = rest
    ref = og.fused_reference(gu["x"], dequant_qweight(w.wgu), gu["gamma"], EPS, _lib.EPI_SILU_MUL)
    assert og.max_rel_err(gu["out"].float(), ref) <= TOL, "gate_up"
    ref = og.fused_reference(dn["x"], dequant_qweight(w.wd), None, EPS, _lib.EPI_ADD_RESIDUAL, dn["residual"])
    assert og.max_rel_err(dn["out"].float(), ref) <= TOL, "down"


def _oracle_layer(fl, x, cos, sin, first, keys, values, mask):
    """The whole call in fp32 on the CPU from the layer's input (B, T, H)."""
    from breeze_b200 import _lib

    w = fl.weights
    b, t, _ = x.shape
    xr = x.transpose(0, 1).reshape(t * b, -1)
    qkv = og.fused_reference(xr, dequant_qweight(w.wqkv), w.ln1.cpu(), EPS, 0).to(torch.bfloat16)
    attn = []
    for p in range(t):
        a, keys, values = oa.attention_step(qkv[p * b:(p + 1) * b], cos[:, p:p + 1], sin[:, p:p + 1], first + p,
                                            keys, values, mask[:, :, p:p + 1], w.q_norm.cpu(), w.k_norm.cpu(), EPS)
        attn.append(a)
    h = og.linear_epilogue(torch.cat(attn).float(), dequant_qweight(w.wo), _lib.EPI_ADD_RESIDUAL, xr)
    act = og.fused_reference(h, dequant_qweight(w.wgu), w.ln2.cpu(), EPS, _lib.EPI_SILU_MUL)
    out = og.linear_epilogue(act, dequant_qweight(w.wd), _lib.EPI_ADD_RESIDUAL, h)
    return out.reshape(t, b, -1).transpose(0, 1)


@pytest.mark.gpu
@pytest.mark.parametrize("t", [1, 2])
@pytest.mark.parametrize("mlp", ["bf16", "fp8", "int4"])
@pytest.mark.parametrize("cache_len", [16, 300])
def test_fused_layer_stages_match_oracle(mlp, t, cache_len, monkeypatch):
    """cache_len 16 takes the fused attention + O launch (bf16 O, short
    cache), 300 the separate attention step and O GEMV."""
    from transformers import StaticCache
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    from breeze_b200.fused.layer import FusedDecoderLayer

    dev = torch.device("cuda", 0)
    layer = _layer(dev)
    if mlp == "int4":
        from breeze_b200.int4_linear import quantize_module_int4

        quantize_module_int4(layer, min_bytes=0)
    elif mlp == "fp8":
        from breeze_b200.fp8_linear import quantize_module_fp8

        quantize_module_fp8(layer, min_bytes=0)
    cfg = _config()
    cfg.max_position_embeddings = 512
    rope = Qwen3RotaryEmbedding(cfg).to(dev)
    b, t0 = 2, 5
    g = torch.Generator(device=dev).manual_seed(1)
    xs = torch.randn(b, t0 + t, H, device=dev, generator=g).to(torch.bfloat16)
    cache = StaticCache(config=cfg, max_cache_len=cache_len)
    pos_ids = torch.arange(t0 + t, device=dev)[None].expand(b, -1)
    cos, sin = rope(xs, pos_ids)
    with torch.no_grad():
        layer(xs[:, :t0], attention_mask=_mask(b, cache_len, 0, t0, torch.bfloat16, dev),
              position_ids=pos_ids[:, :t0], past_key_values=cache, use_cache=True,
              cache_position=torch.arange(t0, device=dev), position_embeddings=(cos[:, :t0], sin[:, :t0]))
        ref_cache = copy.deepcopy(cache)
        mask = _mask(b, cache_len, t0, t, torch.bfloat16, dev)
        step = dict(attention_mask=mask, position_ids=pos_ids[:, t0:], use_cache=True,
                    cache_position=torch.arange(t0, t0 + t, device=dev),
                    position_embeddings=(cos[:, t0:], sin[:, t0:]))
        wrapped = layer(xs[:, t0:], past_key_values=ref_cache, **step)
        wrapped = wrapped[0] if isinstance(wrapped, tuple) else wrapped
        fl = FusedDecoderLayer(layer, 0)
        if mlp == "int4":
            gw, uw = layer.mlp.gate_proj.weight_int4, layer.mlp.up_proj.weight_int4
            assert gw.data_ptr() == fl.weights.wgu.w.data_ptr()
            assert uw.data_ptr() == fl.weights.wgu.w.data_ptr() + gw.numel() * gw.element_size()
        n0 = int(cache.layers[0].cumulative_length) if hasattr(cache.layers[0], "cumulative_length") else None
        k_in, v_in = cache.layers[0].keys.cpu(), cache.layers[0].values.cpu()
        rec = _Recorder(monkeypatch)
        got = fl(xs[:, t0:], past_key_values=cache, **step)
    torch.cuda.synchronize()
    monkeypatch.undo()
    assert got.shape == (b, t, H) and got.is_contiguous()
    _check_call(rec, fl, t, b)
    ref = _oracle_layer(fl, xs[:, t0:].cpu(), cos[:, t0:].cpu(), sin[:, t0:].cpu(), t0, k_in.clone(), v_in.clone(),
                        mask.cpu())
    assert og.max_rel_err(got.float().cpu(), ref) <= TOL
    assert og.max_rel_err(got.float().cpu(), wrapped.float().cpu()) < 2e-2
    if n0 is not None:
        assert int(cache.layers[0].cumulative_length) == n0 + t


@pytest.mark.gpu
def test_install_fused_depth_wraps_and_warms():
    from transformers.models.qwen3.modeling_qwen3 import Qwen3Model

    from breeze_b200.fused.install import install_fused_depth
    from breeze_b200.fused.layer import FusedDecoderLayer

    cfg = _config()
    cfg.num_codebooks = 4
    torch.manual_seed(0)
    dm = Qwen3Model(cfg).to(device="cuda", dtype=torch.bfloat16).eval()
    model = types.SimpleNamespace(depth_decoder=types.SimpleNamespace(model=dm))
    assert install_fused_depth(model, batch_size=2) == 2
    assert all(isinstance(l, FusedDecoderLayer) for l in dm.layers)
    assert install_fused_depth(model, batch_size=2) == 0  # already installed
    from breeze_b200 import _lib

    assert _lib.device_status(0) == 0
