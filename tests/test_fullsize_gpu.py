"""Decode-step parity at the benchmark's real shapes (BASELINE configs 3 and 4).

One decoder layer plus the output head at full size -- QKV 2048->6144, O
2048->2048, gate+up 2048->16384, down 8192->2048, head 2048->8192 -- in int4
g128 (tinygemm tiles), fp8 per-channel and int8 per-channel, for M = 1, 2, 4,
8, 16 (config 3's MTP-verify rows) and 32, 64 (config 4's concurrent
streams), with and without the attention step (16 q / 16 kv heads of 128
over a 256-position cache). Every stage is checked against the CPU oracle on
the inputs it actually read, at max rel err 1e-2: QKV (RMSNorm fused), the
attention output and the k / v it wrote, O (+ residual), gate+up (RMSNorm,
SiLU*up), down (+ residual) and the fp32 head (RMSNorm fused).

The same checks run through the one-launch decode chain (DecodeStack
chain=True, the persistent kernel) at M = 1, 2, 4 and 8, the rows whose
staged activations fit beside its weight ring at K = 8192.

The whole 28-layer step the benchmark times is also run per format (M = 1
and 16 launch by launch, M = 1 and 4 as one chain launch), and its last
layer and head are checked the same way.
"""

import pytest
import torch

from gpu_cases import dequant_qweight
from oracle import attention as oa
from oracle import gemv as og

pytestmark = pytest.mark.gpu
TOL = 1e-2
EPS = 1e-6
ROWS = (1, 2, 4, 8, 16, 32, 64)
_CACHE: dict = {}


def _stack_weights(fmt: str, n_layers: int):
    """Full-size synthetic layers + head on the GPU, and the oracle's fp32
    weights of the last layer and the head (built once per format)."""
    from breeze_b200.fused.stack import synthetic_stack

    key = (fmt, n_layers)
    if key not in _CACHE:
        _CACHE.clear()
        torch.cuda.empty_cache()
        layers, head, ln_f = synthetic_stack(fmt, n_layers, torch.device("cuda", 0), seed=11)
        last = layers[-1]
        deq = {name: dequant_qweight(getattr(last, name)) for name in ("wqkv", "wo", "wgu", "wd")}
        deq["head"] = dequant_qweight(head)
        _CACHE[key] = (layers, head, ln_f, deq)
    return _CACHE[key]


def _check(name, got, x, w, gamma=None, epilogue=0, residual=None):
    ref = og.fused_reference(x.cpu(), w, None if gamma is None else gamma.cpu(), EPS, epilogue,
                             None if residual is None else residual.cpu())
    err = og.max_rel_err(got.cpu().float(), ref)
    assert err <= TOL, f"{name}: max rel err {err:.3e}"


def _run_and_check(fmt, rows, n_layers, attention, chain=False):
    from breeze_b200 import _lib
    from breeze_b200.fused.stack import DecodeStack

    layers, head, ln_f, deq = _stack_weights(fmt, n_layers)
    st = DecodeStack(layers, head, ln_f, rows=rows, attention=attention, chain=chain)
    g = torch.Generator().manual_seed(100 + rows)
    st.x.copy_(torch.randn(rows, st.hidden, generator=g).to(torch.bfloat16))
    li = n_layers - 1
    if attention:
        for c in st.k_cache + st.v_cache:
            c.copy_((torch.randn(c.shape, generator=g) * 0.5).to(torch.bfloat16))
        k_before, v_before = st.k_cache[li].cpu(), st.v_cache[li].cpu()
    st.run()
    torch.cuda.synchronize()
    assert _lib.device_status(0) == 0
    last = layers[li]
    xin = st.x if n_layers == 1 else st.res[(li - 1) % 2]
    y = st.res[li % 2]
    tag = f"{fmt} M={rows} layers={n_layers} attention={attention} chain={chain}"
    _check(f"qkv [{tag}]", st.qkv, xin, deq["wqkv"], gamma=last.ln1)
    if attention:
        pos = int(st.pos.item())
        ref, rk, rv = oa.attention_step(st.qkv.cpu(), st.cos.cpu(), st.sin.cpu(), pos, k_before.clone(),
                                        v_before.clone(), torch.zeros(rows, st.kv_len), last.q_norm.cpu(),
                                        last.k_norm.cpu(), EPS)
        err = og.max_rel_err(st.attn_out.cpu().float(), ref.float())
        assert err <= TOL, f"attention [{tag}]: {err:.3e}"
        assert torch.equal(st.v_cache[li].cpu()[:, :, pos], rv[:, :, pos]), f"v written [{tag}]"
        kd = (st.k_cache[li].cpu()[:, :, pos].float() - rk[:, :, pos].float()).abs()
        assert (kd <= rk[:, :, pos].float().abs() * 2 ** -7 + 1e-6).all(), f"k written [{tag}]"
        attn_in = st.attn_out
    else:
        attn_in = st.qkv[:, : st.attn_cols]
    _check(f"o [{tag}]", st.h, attn_in, deq["wo"], epilogue=_lib.EPI_ADD_RESIDUAL, residual=xin)
    _check(f"gate_up [{tag}]", st.act, st.h, deq["wgu"], gamma=last.ln2, epilogue=_lib.EPI_SILU_MUL)
    _check(f"down [{tag}]", y, st.act, deq["wd"], epilogue=_lib.EPI_ADD_RESIDUAL, residual=st.h)
    _check(f"head [{tag}]", st.logits, y, deq["head"], gamma=ln_f)


@pytest.mark.parametrize("attention", [False, True], ids=["projections", "attention"])
@pytest.mark.parametrize("rows", ROWS)
@pytest.mark.parametrize("fmt", ["int4", "fp8", "int8"])
def test_full_size_layer_stages_match_oracle(fmt, rows, attention):
    _run_and_check(fmt, rows, 1, attention)


@pytest.mark.parametrize("rows", [1, 2, 4, 8])
@pytest.mark.parametrize("fmt", ["int4", "fp8", "int8"])
def test_full_size_layer_stages_match_oracle_one_launch(fmt, rows):
    _run_and_check(fmt, rows, 1, False, chain=True)


@pytest.mark.parametrize("rows,chain", [(1, False), (16, False), (1, True), (4, True)])
@pytest.mark.parametrize("fmt", ["int4", "fp8", "int8"])
def test_full_28_layer_step_last_layer_matches_oracle(fmt, rows, chain):
    _run_and_check(fmt, rows, 28, False, chain=chain)
