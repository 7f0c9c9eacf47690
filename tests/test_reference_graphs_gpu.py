"""This package's FusedDecoderLayer inside the reference's OWN CUDA-graph classes.

The reference captures its decode steps with two classes -- DepthDecoderGraph
(the 15-step depth loop: 2-position prefill, then single steps, fp32
per-codebook head, CFG sampling; models/cudagraph/depth_decoder_graph.py:
560-660, 775-812) and BackboneGraph (one backbone step, fp32 lm_head, CFG;
models/cudagraph/backbone_graph.py:254-320). Their premise is that a fused
layer is a drop-in: the graph code calls every decoder layer with its static
cache, masks and rotary embeddings and records the result.

Here the unmodified classes, imported from the reference installed in
baseline/_ref, capture and replay two copies of one small random model: one
with the stock decoder layers, one after this package's install_fused_depth /
install_fused_backbone (the reference-side re-export INTEGRATION.md shows).
The replayed logits of every step agree within max rel err 2e-2 (the stock
layers round every intermediate to bf16 -- norm output, q / k / v, attention
output, MLP activations -- where the fused kernels keep fp32; the kernels
themselves are held to 1e-2 against the oracle elsewhere) and the greedy
tokens agree wherever the reference's top two logits are further apart than
that error.

The reference pins transformers 4.57.3; this image has 5.5, and three API
changes between them are bridged for the duration of each test (nothing of
the reference is edited): the "default" RoPE initialiser (inverse
frequencies 1 / theta^(2i/d), scaling 1), the rotary module's
compute_default_rope_parameters that 5.5's weight initialisation asks for,
and StaticLayer.lazy_initialization with the keys only, as the reference's
graph classes call it.
"""

import copy
import types
from pathlib import Path

import pytest
import torch

from oracle import gemv as og

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
TOL = 2e-2
DEV = "cuda:0"


def _default_rope(config=None, device=None, seq_len=None, *args, **kwargs):  # noqa: ARG001
    dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
    inv = 1.0 / (config.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float().to(device) / dim))
    return inv, 1.0


@pytest.fixture()
def ref(monkeypatch):
    """The reference package from baseline/_ref, with the transformers bridges."""
    if not (REF / "models" / "cudagraph" / "depth_decoder_graph.py").exists():
        pytest.skip("the reference is not installed in baseline/_ref")
    monkeypatch.syspath_prepend(str(REF))
    from transformers import cache_utils
    from transformers import modeling_rope_utils as rope

    monkeypatch.setitem(rope.ROPE_INIT_FUNCTIONS, "default", _default_rope)
    orig = cache_utils.StaticLayer.lazy_initialization

    def lazy_initialization(self, key_states, value_states=None):
        return orig(self, key_states, key_states if value_states is None else value_states)

    monkeypatch.setattr(cache_utils.StaticLayer, "lazy_initialization", lazy_initialization)
    import models.breeze as breeze

    monkeypatch.setattr(breeze.BreezeRotaryEmbedding, "compute_default_rope_parameters", staticmethod(_default_rope),
                        raising=False)
    return types.SimpleNamespace(breeze=breeze)


def _randomize(model, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 1:  # norm weights
                p.copy_((1 + 0.1 * torch.randn(p.shape, generator=g)).to(p.dtype))
            else:
                p.copy_((torch.randn(p.shape, generator=g) * 0.05).to(p.dtype))


def _compare(name, got, want):
    err = og.max_rel_err(got.float().cpu(), want.float().cpu())
    assert err < TOL, f"{name}: logits max rel err {err:.3e}"


def test_depth_decoder_graph_with_fused_layers(ref):
    from breeze_b200.fused.install import install_fused_depth
    from breeze_b200.fused.layer import FusedDecoderLayer
    from models.breeze_base_config import BreezeDepthDecoderConfig
    from models.cudagraph.depth_decoder_graph import DepthDecoderGraph

    cfg = BreezeDepthDecoderConfig(num_codebooks=6, backbone_hidden_size=256, vocab_size=96, hidden_size=256,
                                   intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
                                   num_key_value_heads=2, head_dim=128, max_position_embeddings=33, rope_theta=10000,
                                   rms_norm_eps=1e-6)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    stock = ref.breeze.BreezeDepthDecoderForCausalLM(cfg)
    _randomize(stock, 1)
    stock = stock.to(device=DEV, dtype=torch.bfloat16).eval()
    fused = copy.deepcopy(stock)
    assert install_fused_depth(types.SimpleNamespace(depth_decoder=fused), batch_size=2) == 2
    assert all(isinstance(l, FusedDecoderLayer) for l in fused.model.layers)

    g = torch.Generator(device=DEV).manual_seed(2)
    backbone_h = torch.randn(2, 256, device=DEV, generator=g).to(torch.bfloat16)
    first_tok = torch.tensor([5, 5], device=DEV)
    results = []
    for model in (stock, fused):
        graph = DepthDecoderGraph(model, cfg, device=DEV, do_sample=False, guidance_scale=1.5, debug=True,
                                  batch_size=2)
        graph.capture(num_warmup=1)
        # what run() does for a full bucket, minus its debug-mode multinomial hook
        # (a keyword only the reference's own debugging patch accepts)
        with torch.inference_mode():  # the graph's buffers were made in inference mode, as run() writes them
            graph.backbone_hidden_buf.copy_(backbone_h)
            graph.first_cb_token_buf.copy_(first_tok)
            graph.static_cache.reset()
            graph.graph.replay()
        torch.cuda.synchronize()
        results.append((graph.output_tokens[: graph.half].clone(), graph.debug_logits.clone()))
        del graph
    (t_stock, l_stock), (t_fused, l_fused) = results
    assert l_stock.shape == l_fused.shape and torch.isfinite(l_fused).all()
    # step by step: every step's raw fp32 logits (cond and uncond rows) agree; the
    # greedy token, drawn from the CFG mix uncond + g (cond - uncond), agrees
    # whenever the stock mix separates its top two by more than the error can
    # move them; after a near-tie that the two runs broke differently the
    # inputs differ, so the comparison stops there
    g_cfg = 1.5
    compared = 0
    for step in range(l_stock.shape[0]):
        err = og.max_rel_err(l_fused[step].float().cpu(), l_stock[step].float().cpu())
        assert err < TOL, f"depth graph step {step}: logits max rel err {err:.3e}"
        compared += 1
        raw = l_stock[step].float().cpu()
        mixed = raw[1] + g_cfg * (raw[0] - raw[1])
        top2 = mixed.topk(2).values
        decisive = float(top2[0] - top2[1]) > 4 * TOL * float(raw.abs().max())
        same = int(t_fused[0, step]) == int(t_stock[0, step])
        assert same or not decisive, f"depth graph step {step}: greedy tokens differ"
        if not same:
            break
    assert compared >= l_stock.shape[0] // 2
    from breeze_b200 import _lib

    assert _lib.device_status(0) == 0


def test_backbone_graph_with_fused_layers(ref):
    from transformers import DynamicCache, Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3Model

    from breeze_b200.fused.install import install_fused_backbone
    from breeze_b200.fused.layer import FusedDecoderLayer
    from models.cudagraph.backbone_graph import BackboneGraph

    cfg = Qwen3Config(hidden_size=256, num_attention_heads=2, num_key_value_heads=2, head_dim=128,
                      intermediate_size=512, num_hidden_layers=2, rms_norm_eps=1e-6, vocab_size=64,
                      max_position_embeddings=512)
    cfg._attn_implementation = "eager"
    cfg.num_codebooks = 4
    torch.manual_seed(0)
    stock = Qwen3Model(cfg)
    _randomize(stock, 3)
    stock = stock.to(device=DEV, dtype=torch.bfloat16).eval()
    embed = ref.breeze.BreezeBackboneModelEmbeddings(cfg)
    _randomize(embed, 4)
    embed = embed.to(device=DEV, dtype=torch.bfloat16)
    head = torch.nn.Linear(256, 64, bias=False)
    _randomize(head, 5)
    head = head.to(device=DEV, dtype=torch.bfloat16)
    fused = copy.deepcopy(stock)
    assert install_fused_backbone(types.SimpleNamespace(backbone_model=fused), batch_size=2, max_seq_len=128) == 2
    assert all(isinstance(l, FusedDecoderLayer) for l in fused.layers)

    g = torch.Generator(device=DEV).manual_seed(6)
    prompt = torch.randint(0, 64, (2, 12, 4), device=DEV, generator=g)
    steps = torch.randint(0, 64, (3, 2, 1, 4), device=DEV, generator=g)
    results = []
    for model in (stock, fused):
        graph = BackboneGraph(model, copy.deepcopy(head), embed, cfg, device=DEV, max_seq_len=128, guidance_scale=2.0,
                              batch_size=2)
        with torch.no_grad():  # the prompt goes through the stock model eagerly, as the reference's prefill graph does
            kv = DynamicCache(config=cfg)
            stock(inputs_embeds=embed(prompt), past_key_values=kv, use_cache=True)
        graph.capture(prefill_len=12, num_warmup=1)
        graph.prefill_kv([(layer.keys, layer.values) for layer in kv.layers])  # 5.5 caches are not subscriptable
        outs = []
        for i in range(steps.shape[0]):
            _, cfg_logits = graph.run(steps[i], i)
            outs.append(graph.logits_buf.clone())
        torch.cuda.synchronize()
        results.append(torch.stack(outs))
        del graph
    _compare("backbone graph", results[1], results[0])
    from breeze_b200 import _lib

    assert _lib.device_status(0) == 0
