"""Pre-quantized checkpoints: write one, and load one into this package's modules.

The files are the reference's format (models/quantized_checkpoint.py,
FORMAT_VERSION 1), so a checkpoint moves either way between the two:

  quantized.safetensors  every tensor of the model's state dict (host copies)
  quant_manifest.json    {"version", "source", "quant_config", "modules",
                          "tensor_count", "bytes"}; "modules" maps the path of
                          each quantized module to its kind, feature sizes and
                          buffer shapes (reference :35-61, :64-88)

Loading never builds a bf16 weight: each recorded path gets an empty module
of the recorded kind, sized from the manifest (the tinygemm tile shape is
recorded, not derived), and the file's tensors are then assigned into the
model in place. The modules themselves know their manifest record
(``Int4Linear.manifest_entry`` / ``from_manifest``, the same for
``Int8Linear``); this file only walks the model and the files.

No repack happens at load time: the GEMV reads Int4Linear's tinygemm tiles as
stored, and fp8 / int8 buffers are row-major as saved. ``attach_decode_weights``
gives the decode graphs QWeight views that share the loaded storage.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch
from safetensors import safe_open
from safetensors.torch import save_file
from torch import nn

from .int4_linear import Int4Linear
from .int8_linear import Int8Linear

FORMAT_VERSION = 1
WEIGHTS_NAME = "quantized.safetensors"
MANIFEST_NAME = "quant_manifest.json"
# tensors an offloading runtime keeps in host memory (reference :29-31)
TEXT_EMBEDDING_PREFIXES = ("embed_text_tokens.", "text_encoder.embed_tokens.")

# Manifest kinds, by class NAME: a model holding the reference's own
# Int4Linear / Int8Linear describes the same as one holding this package's
# (the reference dispatches on class names too, models/fused/layer.py:52-61).
_CLASS_OF_KIND = {Int4Linear.MANIFEST_KIND: Int4Linear, Int8Linear.MANIFEST_KIND: Int8Linear}
_KIND_OF_NAME = {cls.__name__: kind for kind, cls in _CLASS_OF_KIND.items()}


def describe(model: nn.Module) -> dict[str, dict]:
    """The manifest's "modules" table: path -> record of every quantized module."""
    table = {}
    for path, module in model.named_modules():
        kind = _KIND_OF_NAME.get(type(module).__name__)
        if kind is not None:
            table[path] = _CLASS_OF_KIND[kind].manifest_entry(module)
    return table


def save_quantized(model: nn.Module, out_dir: Path, quant_config: dict, source: str) -> dict:
    """Write ``model``'s state and its manifest to ``out_dir``; returns the manifest.

    Every tensor is written from a private contiguous host copy, so views,
    tied weights and device tensors all serialise."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    tensors = {name: t.detach().to("cpu", copy=True).contiguous() for name, t in model.state_dict().items()}
    save_file(tensors, str(out / WEIGHTS_NAME))
    manifest = {"version": FORMAT_VERSION, "source": source, "quant_config": quant_config,
                "modules": describe(model), "tensor_count": len(tensors),
                "bytes": sum(t.numel() * t.element_size() for t in tensors.values())}
    (out / MANIFEST_NAME).write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def read_manifest(out_dir: Path) -> dict:
    """The checkpoint's manifest; ValueError unless it is format version 1."""
    manifest = json.loads((Path(out_dir) / MANIFEST_NAME).read_text())
    found = manifest.get("version")
    if found != FORMAT_VERSION:
        raise ValueError(f"unsupported checkpoint version {found!r} (this loader reads {FORMAT_VERSION})")
    return manifest


def install_shells(model: nn.Module, manifest: dict, device) -> int:
    """Put an empty quantized module of the recorded kind at every path the
    manifest lists; returns how many were placed."""
    table = manifest["modules"]
    for path, entry in table.items():
        parent, _, leaf = path.rpartition(".")
        setattr(model.get_submodule(parent), leaf, _CLASS_OF_KIND[entry["kind"]].from_manifest(entry, device))
    return len(table)


def load_quantized_state(model: nn.Module, out_dir: Path, device, host_prefixes: tuple[str, ...] = ()) -> dict:
    """Assign the checkpoint's tensors into ``model`` (shells installed first).

    Tensors are read one at a time and placed directly: names starting with
    one of ``host_prefixes`` stay in host memory, the rest go to ``device``,
    so host-resident tables never pass through device memory. Returns the
    reference's counts: loaded, missing, unexpected (+ five-name samples)."""
    prefixes = tuple(host_prefixes)
    placed = {}
    with safe_open(str(Path(out_dir) / WEIGHTS_NAME), framework="pt", device="cpu") as f:
        for name in f.keys():  # noqa: SIM118 - safetensors handle, not a dict
            target = "cpu" if prefixes and name.startswith(prefixes) else device
            placed[name] = f.get_tensor(name).to(target)
    missing, unexpected = model.load_state_dict(placed, strict=False, assign=True)
    return {"loaded": len(placed), "missing": len(missing), "unexpected": len(unexpected),
            "missing_sample": list(missing)[:5], "unexpected_sample": list(unexpected)[:5]}


def attach_decode_weights(model: nn.Module) -> dict[str, "object"]:
    """QWeight views (breeze_b200.fused.stack.QWeight) of every loaded
    Int4Linear / Fp8Linear / bias-free Int8Linear, keyed by module path. The
    views share storage with the module buffers; nothing is copied or repacked."""
    from .fused.stack import QWeight

    views = {}
    for path, module in model.named_modules():
        name = type(module).__name__
        if name in ("Int4Linear", "Fp8Linear") or (name == "Int8Linear" and module.bias is None):
            views[path] = QWeight.from_module(module)
    return views
