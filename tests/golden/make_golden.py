"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs on a CUDA machine (the reference's int4 pack and fp8 rowwise matmul have
no CPU kernels). It imports the reference's own modules from ``--ref`` (an
unmodified copy of the reference tree; nothing here restates them) and calls:

  * ``torch._convert_weight_to_int4pack`` on seeded uint8 inputs at several
    (N, K, inner_k_tiles): the tinygemm packed layout, as a black box
    (models/int4_linear.py:59 is the reference call site);
  * ``models.int4_linear.Int4Linear`` (quantize_int4 + tinygemm forward,
    models/int4_linear.py:47-109), also on hand-built config-0 codes;
  * ``models.fp8_linear.Fp8Linear`` (models/fp8_linear.py:44-83);
  * ``models.int8_linear.Int8Linear`` (models/int8_linear.py:32-53);
  * ``models.fused.kernels.rms_gemv`` / ``FusedWeight`` / ``rmsnorm`` /
    ``silu_mul`` / ``attention_step`` (models/fused/kernels.py), the Triton
    fused decode path, with a fixed launch config so no autotuning runs.

Every input is drawn from ``torch.Generator().manual_seed(seed)`` on the CPU
in the order written below, then moved to the device, so the CPU tests can
regenerate the same inputs. Outputs land in ``--out`` as .npz files (bf16 is
stored as its uint16 bit pattern, fp8 as uint8) plus meta.json.

    python tests/golden/make_golden.py --ref baseline/_ref --out <dir>
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch


def bits(t: torch.Tensor) -> np.ndarray:
    """Tensor -> numpy, keeping exact bit patterns for bf16 / fp8."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="baseline/_ref")
    ap.add_argument("--out", default="tests/golden/regen")
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("BREEZE_FUSED_TUNE", str(out / "fused_tune.json"))
    sys.path.insert(0, str(Path(args.ref).resolve()))
    dev = "cuda"

    meta = {
        "torch": torch.__version__,
        "device": torch.cuda.get_device_name(0),
        "capability": list(torch.cuda.get_device_capability(0)),
        "files": {},
    }

    # ---- 1. tinygemm pack layout, black box -------------------------------
    pack_cases = [(16, 256, 8), (24, 512, 8), (32, 128, 2), (32, 128, 4), (40, 384, 8)]
    arrays = {}
    for i, (n, k, ik) in enumerate(pack_cases):
        g = gen(100 + i)
        src = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int32).to(torch.uint8)
        packed = torch._convert_weight_to_int4pack(src.to(dev), ik)
        arrays[f"in_{n}_{k}_{ik}"] = bits(src)
        arrays[f"out_{n}_{k}_{ik}"] = bits(packed)
    np.savez_compressed(out / "tinygemm_pack.npz", **arrays)
    meta["files"]["tinygemm_pack.npz"] = {"cases": pack_cases}

    # ---- 2. Int4Linear (reference module) ---------------------------------
    from models.int4_linear import Int4Linear

    int4_cases = [(256, 512, 128), (128, 1024, 64), (64, 256, 32), (256, 512, 256)]
    arrays = {}
    for i, (n, k, gs) in enumerate(int4_cases):
        g = gen(200 + i)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        lin = torch.nn.Linear(k, n, bias=False, dtype=torch.bfloat16)
        lin.weight.data = w.to(dev)
        mod = Int4Linear(lin, group_size=gs)
        tag = f"{n}_{k}_{gs}"
        arrays[f"w_{tag}"] = bits(w)
        arrays[f"weight_int4_{tag}"] = bits(mod.weight_int4)
        arrays[f"scales_zeros_{tag}"] = bits(mod.scales_zeros)
        for m in (1, 2, 3, 16):
            x = torch.randn(m, k, generator=g).to(torch.bfloat16)
            y = mod(x.to(dev))
            arrays[f"x_{tag}_m{m}"] = bits(x)
            arrays[f"y_{tag}_m{m}"] = bits(y)
    np.savez_compressed(out / "int4_linear.npz", **arrays)
    meta["files"]["int4_linear.npz"] = {"cases": int4_cases, "m": [1, 2, 3, 16]}

    # ---- 2b. config-0 style codes straight into the tinygemm op -----------
    # codes uniform 0..15, scale |N(0,0.02)|/7 bf16, zero-point 8 (zero = 0).
    arrays = {}
    n = k = 256
    g = gen(0)
    codes = torch.randint(0, 16, (n, k), generator=g, dtype=torch.int32).to(torch.uint8)
    scale = (torch.randn(n, k // 128, generator=g) * 0.02).abs() / 7
    scale = scale.to(torch.bfloat16)
    x = torch.randn(1, k, generator=g).to(torch.bfloat16)
    # the reference's nibble convention: odd k low, even k high (int4_linear.py:58)
    packed_u8 = (codes[:, 1::2] | (codes[:, 0::2] << 4)).contiguous()
    inner = torch._convert_weight_to_int4pack(packed_u8.to(dev), 8)
    sz = torch.stack([scale.t().float(), torch.zeros(k // 128, n)], -1).to(torch.bfloat16).contiguous()
    y = torch._weight_int4pack_mm(x.to(dev), inner, 128, sz.to(dev))
    arrays.update(codes=bits(codes), scale=bits(scale), x=bits(x), weight_int4=bits(inner),
                  scales_zeros=bits(sz), y=bits(y))
    np.savez_compressed(out / "config0_small.npz", **arrays)
    meta["files"]["config0_small.npz"] = {"n": n, "k": k, "seed": 0}

    # ---- 3. Fp8Linear (reference module, W8A8 via _scaled_mm) -------------
    from models.fp8_linear import Fp8Linear

    arrays = {}
    for i, (n, k) in enumerate([(256, 512), (128, 1024)]):
        g = gen(300 + i)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        lin = torch.nn.Linear(k, n, bias=False, dtype=torch.bfloat16)
        lin.weight.data = w.to(dev)
        mod = Fp8Linear(lin)
        tag = f"{n}_{k}"
        arrays[f"w_{tag}"] = bits(w)
        arrays[f"weight_fp8_{tag}"] = bits(mod.weight_fp8)
        arrays[f"weight_scale_{tag}"] = bits(mod.weight_scale)
        for m in (1, 2):
            x = torch.randn(m, k, generator=g).to(torch.bfloat16)
            arrays[f"x_{tag}_m{m}"] = bits(x)
            arrays[f"y_{tag}_m{m}"] = bits(mod(x.to(dev)))
    np.savez_compressed(out / "fp8_linear.npz", **arrays)

    # ---- 4. Int8Linear (reference module) ---------------------------------
    from models.int8_linear import Int8Linear

    arrays = {}
    for i, (n, k, has_bias) in enumerate([(256, 512, False), (96, 384, True)]):
        g = gen(400 + i)
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
        lin = torch.nn.Linear(k, n, bias=has_bias, dtype=torch.bfloat16)
        lin.weight.data = w.to(dev)
        if has_bias:
            lin.bias.data = b.to(dev)
        mod = Int8Linear(lin)
        tag = f"{n}_{k}_{int(has_bias)}"
        arrays[f"w_{tag}"] = bits(w)
        arrays[f"b_{tag}"] = bits(b)
        arrays[f"weight_int8_{tag}"] = bits(mod.weight_int8)
        arrays[f"weight_scale_{tag}"] = bits(mod.weight_scale)
        for m in (1, 2):
            x = torch.randn(m, k, generator=g).to(torch.bfloat16)
            arrays[f"x_{tag}_m{m}"] = bits(x)
            arrays[f"y_{tag}_m{m}"] = bits(mod(x.to(dev)))
    np.savez_compressed(out / "int8_linear.npz", **arrays)

    # ---- 5. Triton fused path (rms_gemv, glue kernels) --------------------
    from models.fused import kernels as fk

    arrays = {}
    n, k = 512, 1024
    cfg = (16, 2, 512, 4, 2)  # BLOCK_N, SPLIT_K, BLOCK_K, warps, stages: fixed, no tuning
    g = gen(500)
    w = torch.randn(n, k, generator=g) * 0.02
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    arrays.update(w=bits(w), gamma=bits(gamma))
    for bits_ in (4, 8, 16):
        fw = fk.FusedWeight(w.to(dev), bits_)
        arrays[f"fw{bits_}_w"] = bits(fw.w)
        if fw.s is not None:
            arrays[f"fw{bits_}_s"] = bits(fw.s)
        if fw.z is not None:
            arrays[f"fw{bits_}_z"] = bits(fw.z)
        for epi in (0, 1, 2):
            key = (n, k, bits_, epi, epi != 2, str(torch.device(dev)))
            fk._BEST[key] = cfg
            fk._BEST[(n, k, bits_, epi, epi != 2, "cuda:0")] = cfg
            for m in (1, 2):
                x = torch.randn(m, k, generator=g).to(torch.bfloat16)
                n_out = n // 2 if epi == 1 else n
                res = torch.randn(m, n_out, generator=g).to(torch.bfloat16)
                xd = x.to(dev)
                y = fk.rms_gemv(
                    xd, fw, gamma.to(dev) if epi != 2 else None, 1e-6, epilogue=epi,
                    residual=res.to(dev) if epi == 2 else None,
                )
                tag = f"b{bits_}_e{epi}_m{m}"
                arrays[f"x_{tag}"] = bits(x)
                arrays[f"res_{tag}"] = bits(res)
                arrays[f"y_{tag}"] = bits(y)
    xg = torch.randn(2, k, generator=g).to(torch.bfloat16)
    arrays["rmsnorm_x"] = bits(xg)
    arrays["rmsnorm_y"] = bits(fk.rmsnorm(xg.to(dev), gamma.to(dev), 1e-6))
    gg = torch.randn(2, 384, generator=g).to(torch.bfloat16)
    uu = torch.randn(2, 384, generator=g).to(torch.bfloat16)
    arrays.update(silu_g=bits(gg), silu_u=bits(uu), silu_y=bits(fk.silu_mul(gg.to(dev), uu.to(dev))))
    np.savez_compressed(out / "fused_triton.npz", **arrays)
    meta["files"]["fused_triton.npz"] = {"n": n, "k": k, "cfg": list(cfg), "eps": 1e-6}

    # ---- 6. attention_step (Triton decode attention) -----------------------
    arrays = {}
    for ci, (B, HQ, HKV, D, S, pos) in enumerate([(2, 4, 2, 128, 64, 37), (2, 4, 2, 128, 320, 300)]):
        g = gen(600 + ci)
        qkv = torch.randn(B, (HQ + 2 * HKV) * D, generator=g).to(torch.bfloat16)
        kc = (torch.randn(B, HKV, S, D, generator=g) * 0.5).to(torch.bfloat16)
        vc = torch.randn(B, HKV, S, D, generator=g).to(torch.bfloat16)
        qn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
        kn = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
        inv_freq = 1.0 / (1e6 ** (torch.arange(0, D, 2).float() / D))
        ang = torch.tensor([float(pos), float(pos - 3)])[:, None] * inv_freq[None, :]
        emb = torch.cat([ang, ang], -1)
        cos = emb.cos().to(torch.bfloat16).reshape(B, 1, D)
        sin = emb.sin().to(torch.bfloat16).reshape(B, 1, D)
        mask = torch.full((B, 1, 1, S), torch.finfo(torch.bfloat16).min)
        mask[:, :, :, : pos + 1] = 0.0
        mask[1, :, :, :5] = torch.finfo(torch.bfloat16).min  # a padded row
        mask = mask.to(torch.bfloat16)
        cp = torch.tensor([pos], dtype=torch.long)
        kd, vd = kc.to(dev).clone(), vc.to(dev).clone()
        o = fk.attention_step(qkv.to(dev), cos.to(dev), sin.to(dev), cp.to(dev), kd, vd,
                              mask.to(dev), qn.to(dev), kn.to(dev), 1e-6)
        tag = f"c{ci}"
        arrays.update({
            f"qkv_{tag}": bits(qkv), f"k_{tag}": bits(kc), f"v_{tag}": bits(vc),
            f"qn_{tag}": bits(qn), f"kn_{tag}": bits(kn), f"cos_{tag}": bits(cos),
            f"sin_{tag}": bits(sin), f"mask_{tag}": bits(mask), f"pos_{tag}": np.array([pos]),
            f"out_{tag}": bits(o), f"k_after_{tag}": bits(kd[:, :, pos]),
            f"v_after_{tag}": bits(vd[:, :, pos]),
            f"shape_{tag}": np.array([B, HQ, HKV, D, S]),
        })
    np.savez_compressed(out / "attention_step.npz", **arrays)

    (out / "meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("golden fixtures written to", out)
    for f in sorted(out.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
