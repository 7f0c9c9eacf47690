"""Quantized-checkpoint load path (breeze_b200.quantized_checkpoint).

tests/golden/ckpt_ref/ was written by the reference's own save_quantized
(tests/golden/make_ckpt_golden.py). CPU: it loads into this package's
Int4Linear / Int8Linear shells with nothing missing or unexpected, every
tensor bit-identical to the file, describe() reproduces the reference's
manifest, a save/load round trip is lossless, and a wrong format version is
refused. GPU: the loaded modules' forward passes match the oracle's
dequantize + linear within 1e-2, and the decode-graph views share storage
with the loaded buffers (no repack, no copy).
"""

import json
import shutil
import sys
from pathlib import Path

import pytest
import torch
from safetensors.torch import load_file

from oracle import gemv as og
from oracle import quant

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from make_ckpt_golden import toy_model  # noqa: E402

GOLD = Path(__file__).resolve().parent / "golden" / "ckpt_ref"


def _qc():
    from breeze_b200 import quantized_checkpoint as qc

    return qc


def _load(device="cpu", src=GOLD, **kw):
    qc = _qc()
    man = qc.read_manifest(src)
    model = toy_model()
    n = qc.install_shells(model, man, device)
    stats = qc.load_quantized_state(model, src, device, **kw)
    return model, man, n, stats


def test_reference_checkpoint_loads_into_our_modules():
    from breeze_b200.int4_linear import Int4Linear
    from breeze_b200.int8_linear import Int8Linear

    model, man, n, stats = _load()
    assert n == 6 and stats["missing"] == 0 and stats["unexpected"] == 0
    assert isinstance(model.layers[0].mlp.gate_proj, Int4Linear)
    assert isinstance(model.layers[1].o_proj, Int8Linear)
    state = load_file(str(GOLD / "quantized.safetensors"))
    sd = model.state_dict()
    assert set(sd) == set(state)
    for k, v in sd.items():
        assert v.dtype == state[k].dtype and torch.equal(v, state[k]), k
    assert _qc().describe(model) == man["modules"]


def test_save_load_round_trip(tmp_path):
    qc = _qc()
    model, man, _, _ = _load()
    out = tmp_path / "ckpt"
    m2 = qc.save_quantized(model, out, man["quant_config"], "round trip")
    assert m2["modules"] == man["modules"] and m2["tensor_count"] == man["tensor_count"]
    again, _, _, stats = _load(src=out)
    assert stats["missing"] == 0 and stats["unexpected"] == 0
    for (k, a), (_, b) in zip(sorted(model.state_dict().items()), sorted(again.state_dict().items())):
        assert torch.equal(a, b), k


def test_host_prefixes_and_version_check(tmp_path):
    model, _, _, stats = _load(host_prefixes=("embed_tokens.",))
    assert stats["loaded"] > 0 and model.embed_tokens.weight.device.type == "cpu"
    bad = tmp_path / "bad"
    shutil.copytree(GOLD, bad)
    man = json.loads((bad / "quant_manifest.json").read_text())
    man["version"] = 2
    (bad / "quant_manifest.json").write_text(json.dumps(man))
    with pytest.raises(ValueError):
        _qc().read_manifest(bad)


@pytest.mark.gpu
def test_loaded_modules_forward_match_oracle():
    qc = _qc()
    dev = torch.device("cuda", 0)
    model, _, _, _ = _load(device=dev)
    x = torch.randn(3, 128, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    g = model.layers[0].mlp.gate_proj
    y = g(x.to(dev))
    w = quant.dequant_int4_tinygemm(g.weight_int4.cpu(), g.scales_zeros.cpu(), 128)
    assert og.max_rel_err(y.cpu().float(), x.float() @ w.t()) < 1e-2
    o = model.layers[1].o_proj
    y8 = o(x.to(dev))
    w8 = quant.dequant_int8(o.weight_int8.cpu(), o.weight_scale.cpu(), dtype=torch.float32)
    assert og.max_rel_err(y8.cpu().float(), x.float() @ w8.t()) < 1e-2
    views = qc.attach_decode_weights(model)
    assert len(views) == 6
    assert views["layers.0.mlp.gate_proj"].w.data_ptr() == g.weight_int4.data_ptr()
    assert views["layers.1.o_proj"].w.data_ptr() == o.weight_int8.data_ptr()
