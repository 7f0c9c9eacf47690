"""A small quantized checkpoint written by the reference's own saver.

Builds ``toy_model()`` (the module tree tests/test_checkpoint.py rebuilds),
swaps in the reference's Int4Linear / Int8Linear shells
(models/quantized_checkpoint.py:91-124), fills their buffers from
``torch.Generator().manual_seed(0)`` in module order, and writes the
checkpoint with the reference's ``save_quantized`` (:64-88) into
tests/golden/ckpt_ref/ (quantized.safetensors + quant_manifest.json).

    python tests/golden/make_ckpt_golden.py --ref <reference tree>
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch
from torch import nn

HERE = Path(__file__).resolve().parent


def toy_model() -> nn.Module:
    torch.manual_seed(0)
    root = nn.Module()
    root.layers = nn.ModuleList()
    for _ in range(2):
        layer = nn.Module()
        layer.mlp = nn.Module()
        layer.mlp.gate_proj = nn.Linear(128, 256, bias=False)
        layer.mlp.down_proj = nn.Linear(256, 128, bias=False)
        layer.o_proj = nn.Linear(128, 128, bias=False)
        root.layers.append(layer)
    root.norm = nn.LayerNorm(128)
    root.embed_tokens = nn.Embedding(32, 128)
    return root


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    from models import quantized_checkpoint as qc

    model = toy_model()
    g = torch.Generator().manual_seed(0)
    for i, layer in enumerate(model.layers):
        for name, (n, k) in (("gate_proj", (256, 128)), ("down_proj", (128, 256))):
            spec = {"in_features": k, "out_features": n, "group_size": 128,
                    "shapes": {"weight_int4": [n // 8, k // 128, 32, 4], "scales_zeros": [k // 128, n, 2]}}
            m = qc._empty_int4(spec, "cpu")
            m.weight_int4.copy_(torch.randint(-(2 ** 31), 2 ** 31 - 1, m.weight_int4.shape, generator=g,
                                              dtype=torch.int64).to(torch.int32))
            s = (torch.rand(k // 128, n, generator=g) * 0.004 + 1e-4)
            z = torch.randn(k // 128, n, generator=g) * 0.01
            m.scales_zeros.copy_(torch.stack([s, z], -1).to(torch.bfloat16))
            setattr(layer.mlp, name, m)
        spec8 = {"in_features": 128, "out_features": 128, "shapes": {"weight_int8": [128, 128], "weight_scale": [128, 1]}}
        m8 = qc._empty_int8(spec8, "cpu")
        m8.weight_int8.copy_(torch.randint(-127, 128, (128, 128), generator=g, dtype=torch.int8))
        m8.weight_scale.copy_(torch.rand(128, 1, generator=g) * 0.001 + 1e-5)
        layer.o_proj = m8
    out = HERE / "ckpt_ref"
    qc.save_quantized(model, out, {"policy": "synthetic test: int4 gate/down, int8 o_proj"}, "toy_model")
    print("wrote", out)


if __name__ == "__main__":
    main()
