"""FusedDecoderLayer and install_fused_* (breeze_b200.fused.layer / install).

Built around a small transformers Qwen3 decoder layer (the backbone's layer
type; q/k norms included). CPU: construction keeps the reference's attributes
and refuses nothing it accepts. GPU: after a 5-token prefill through the
wrapped layer, one decode step through FusedDecoderLayer (bf16, fp8 and int4
MLPs) matches the wrapped layer's own eager forward on a copy of the same
static cache within max rel err 2e-2 (bf16 end to end), writes k / v at the
cache position within 2 % (the projections round differently: fused RMSNorm in
fp32 here, bf16 norm then matmul in the wrapped layer), and keeps the cache's own length counter; the int4
gate and up modules end up as views of one tensor (no duplicate weight
memory); install_fused_depth wraps every layer and runs its warm-up step.
"""

import copy
import types

import pytest
import torch

from oracle import gemv as og

H, HEADS, KVH, HD, INTER = 256, 2, 1, 128, 256


def _config():
    from transformers import Qwen3Config

    cfg = Qwen3Config(hidden_size=H, num_attention_heads=HEADS, num_key_value_heads=KVH, head_dim=HD,
                      intermediate_size=INTER, num_hidden_layers=2, rms_norm_eps=1e-6, vocab_size=64,
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
    from breeze_b200.fused.layer import FusedDecoderLayer

    fl = FusedDecoderLayer(_layer("cpu"), 0)
    assert fl.hkv == KVH and fl.hd == HD and fl.layer_idx == 0
    assert fl.wqkv.N == (HEADS + 2 * KVH) * HD and fl.wqkv.K == H and fl.wo.N == H
    assert fl.wgu.N == 2 * INTER and fl.wd.K == INTER
    assert fl.qn is not None and fl.kn is not None


def _mask(b, s, upto, dtype, device):
    m = torch.full((b, 1, 1, s), torch.finfo(dtype).min, dtype=dtype, device=device)
    m[..., : upto + 1] = 0
    return m


@pytest.mark.gpu
@pytest.mark.parametrize("mlp", ["bf16", "fp8", "int4"])
def test_fused_layer_decode_step_matches_wrapped_layer(mlp):
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
    rope = Qwen3RotaryEmbedding(cfg).to(dev)
    b, s, t0 = 2, 16, 5
    g = torch.Generator(device=dev).manual_seed(1)
    xs = torch.randn(b, t0 + 1, H, device=dev, generator=g).to(torch.bfloat16)
    cache = StaticCache(config=cfg, max_cache_len=s)
    pos_ids = torch.arange(t0 + 1, device=dev)[None].expand(b, -1)
    cos, sin = rope(xs, pos_ids)
    with torch.no_grad():
        causal = torch.full((b, 1, t0, s), torch.finfo(torch.bfloat16).min, dtype=torch.bfloat16, device=dev)
        for i in range(t0):
            causal[:, :, i, : i + 1] = 0
        layer(xs[:, :t0], attention_mask=causal, position_ids=pos_ids[:, :t0], past_key_values=cache, use_cache=True,
              cache_position=torch.arange(t0, device=dev), position_embeddings=(cos[:, :t0], sin[:, :t0]))
        ref_cache = copy.deepcopy(cache)
        mask = _mask(b, s, t0, torch.bfloat16, dev)
        step = dict(attention_mask=mask, position_ids=pos_ids[:, t0:], use_cache=True,
                    cache_position=torch.tensor([t0], device=dev), position_embeddings=(cos[:, t0:], sin[:, t0:]))
        ref = layer(xs[:, t0:], past_key_values=ref_cache, **step)
        ref = ref[0] if isinstance(ref, tuple) else ref
        fl = FusedDecoderLayer(layer, 0)
        if mlp == "int4":
            assert fl.qgu is not None
            gw, uw = layer.mlp.gate_proj.weight_int4, layer.mlp.up_proj.weight_int4
            assert gw.data_ptr() == fl.qgu.w.data_ptr()
            assert uw.data_ptr() == fl.qgu.w.data_ptr() + gw.numel() * gw.element_size()
        n0 = int(cache.layers[0].cumulative_length) if hasattr(cache.layers[0], "cumulative_length") else None
        got = fl(xs[:, t0:], past_key_values=cache, **step)
    torch.cuda.synchronize()
    assert got.shape == ref.shape
    assert og.max_rel_err(got.float().cpu(), ref.float().cpu()) < 2e-2
    kd = (cache.layers[0].keys[:, :, t0].float() - ref_cache.layers[0].keys[:, :, t0].float()).abs()
    assert float(kd.max()) <= 0.02 * float(ref_cache.layers[0].keys[:, :, t0].float().abs().max())
    vd = (cache.layers[0].values[:, :, t0].float() - ref_cache.layers[0].values[:, :, t0].float()).abs()
    assert float(vd.max()) <= 0.02 * float(ref_cache.layers[0].values[:, :, t0].float().abs().max())
    if n0 is not None:
        assert int(cache.layers[0].cumulative_length) == n0 + 1


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
