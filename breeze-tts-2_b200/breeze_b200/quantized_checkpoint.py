"""Save and load an already-quantized checkpoint, into this package's modules.

Same on-disk format and functions as the reference's
models/quantized_checkpoint.py (FORMAT_VERSION 1: ``quantized.safetensors``
plus ``quant_manifest.json`` recording every quantized module's kind,
features, group size and buffer shapes, :35-88), so a checkpoint written by
either side loads into the other:

  * describe(model)            -> manifest "modules" (reference :35-61)
  * save_quantized(...)        -> writes both files (:64-88)
  * install_shells(...)        -> swaps in empty Int4Linear / Int8Linear
                                  shells of THIS package (:91-135)
  * load_quantized_state(...)  -> assigns the tensors, optionally keeping
                                  some prefixes in host memory (:138-166)
  * read_manifest(dir)         -> version-checked manifest (:169-173)

No repack is needed at load time: the GEMV consumes Int4Linear's tinygemm
tiles exactly as stored (each 16-bit half of a packed word is one
m16n8k16 operand pair {k, k+1}), and the fp8 / int8 buffers are row-major
as saved. ``attach_decode_weights`` is the load-time step that does exist:
it builds the QWeight views the decode graphs launch on, sharing storage
with the loaded buffers (no copy, nothing rewritten).
"""

from __future__ import annotations

import json
from pathlib import Path

import torch
from safetensors.torch import load_file, save_file
from torch import nn

from .int4_linear import Int4Linear
from .int8_linear import Int8Linear

FORMAT_VERSION = 1
WEIGHTS_NAME = "quantized.safetensors"
TEXT_EMBEDDING_PREFIXES = ("embed_text_tokens.", "text_encoder.embed_tokens.")
MANIFEST_NAME = "quant_manifest.json"


def _kind(module: nn.Module) -> str | None:
    """Quantized kind by class name, so the reference's own modules describe
    the same way as this package's (the reference dispatches on names too,
    models/fused/layer.py:52-61)."""
    name = type(module).__name__
    return {"Int4Linear": "int4", "Int8Linear": "int8"}.get(name)


def describe(model: nn.Module) -> dict[str, dict]:
    """Every quantized module, so the loader can recreate its shell."""
    described: dict[str, dict] = {}
    for path, module in model.named_modules():
        kind = _kind(module)
        if kind == "int4":
            described[path] = {
                "kind": "int4",
                "in_features": module.in_features,
                "out_features": module.out_features,
                "group_size": module.group_size,
                "shapes": {"weight_int4": list(module.weight_int4.shape),
                           "scales_zeros": list(module.scales_zeros.shape)},
            }
        elif kind == "int8":
            described[path] = {
                "kind": "int8",
                "in_features": module.in_features,
                "out_features": module.out_features,
                "has_bias": module.bias is not None,
                "shapes": {"weight_int8": list(module.weight_int8.shape),
                           "weight_scale": list(module.weight_scale.shape)},
            }
    return described


def save_quantized(model: nn.Module, out_dir: Path, quant_config: dict, source: str) -> dict:
    """Write the weights (contiguous host copies) and the manifest."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    modules = describe(model)
    state = {k: v.detach().cpu().contiguous().clone() for k, v in model.state_dict().items()}
    save_file(state, str(out_dir / WEIGHTS_NAME))
    manifest = {
        "version": FORMAT_VERSION,
        "source": source,
        "quant_config": quant_config,
        "modules": modules,
        "tensor_count": len(state),
        "bytes": sum(v.numel() * v.element_size() for v in state.values()),
    }
    (out_dir / MANIFEST_NAME).write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def _empty_int4(spec: dict, device) -> Int4Linear:
    module = Int4Linear.__new__(Int4Linear)
    nn.Module.__init__(module)
    module.in_features = spec["in_features"]
    module.out_features = spec["out_features"]
    module.group_size = spec["group_size"]
    module.register_buffer("weight_int4", torch.empty(spec["shapes"]["weight_int4"], dtype=torch.int32,
                                                      device=device))
    module.register_buffer("scales_zeros", torch.empty(spec["shapes"]["scales_zeros"], dtype=torch.bfloat16,
                                                       device=device))
    return module


def _empty_int8(spec: dict, device) -> Int8Linear:
    module = Int8Linear.__new__(Int8Linear)
    nn.Module.__init__(module)
    module.in_features = spec["in_features"]
    module.out_features = spec["out_features"]
    module.register_buffer("weight_int8", torch.empty(spec["shapes"]["weight_int8"], dtype=torch.int8, device=device))
    module.register_buffer("weight_scale", torch.empty(spec["shapes"]["weight_scale"], dtype=torch.float32,
                                                       device=device))
    if spec.get("has_bias"):
        module.register_buffer("bias", torch.empty(spec["out_features"], dtype=torch.bfloat16, device=device))
    else:
        module.register_buffer("bias", None)
    return module


def _set_submodule(root: nn.Module, path: str, replacement: nn.Module) -> None:
    parts = path.split(".")
    parent = root
    for part in parts[:-1]:
        parent = getattr(parent, part)
    setattr(parent, parts[-1], replacement)


def install_shells(model: nn.Module, manifest: dict, device) -> int:
    """Swap in empty quantized modules so the state dict has somewhere to land."""
    for path, spec in manifest["modules"].items():
        builder = _empty_int4 if spec["kind"] == "int4" else _empty_int8
        _set_submodule(model, path, builder(spec, device))
    return len(manifest["modules"])


def load_quantized_state(model: nn.Module, out_dir: Path, device, host_prefixes: tuple[str, ...] = ()) -> dict:
    """Load the weights into a model whose shells are installed; tensors whose
    names start with ``host_prefixes`` stay in host memory."""
    out_dir = Path(out_dir)
    if host_prefixes:
        from safetensors import safe_open

        state = {}
        with safe_open(str(out_dir / WEIGHTS_NAME), framework="pt") as handle:
            for key in handle.keys():  # noqa: SIM118 - safetensors API
                target = "cpu" if key.startswith(host_prefixes) else str(device)
                state[key] = handle.get_tensor(key).to(target)
    else:
        state = load_file(str(out_dir / WEIGHTS_NAME), device=str(device))
    missing, unexpected = model.load_state_dict(state, strict=False, assign=True)
    return {
        "loaded": len(state),
        "missing": len(missing),
        "unexpected": len(unexpected),
        "missing_sample": list(missing)[:5],
        "unexpected_sample": list(unexpected)[:5],
    }


def read_manifest(out_dir: Path) -> dict:
    manifest = json.loads((Path(out_dir) / MANIFEST_NAME).read_text())
    if manifest.get("version") != FORMAT_VERSION:
        raise ValueError(f"unsupported checkpoint version {manifest.get('version')!r}")
    return manifest


def attach_decode_weights(model: nn.Module) -> dict[str, "object"]:
    """QWeight views (breeze_b200.fused.stack.QWeight) of every loaded
    Int4Linear / Fp8Linear / Int8Linear, keyed by module path. The views share
    storage with the module buffers; nothing is copied or repacked."""
    from .fused.stack import QWeight

    out = {}
    for path, module in model.named_modules():
        if type(module).__name__ in ("Int4Linear", "Fp8Linear") or (
                type(module).__name__ == "Int8Linear" and module.bias is None):
            out[path] = QWeight.from_module(module)
    return out
