"""The CPU oracle against the reference's own outputs recorded on a B200.

These pin the oracle before it is trusted as the checker for the CUDA path:
layouts and quantizers must reproduce the reference's buffers bit-for-bit,
and the restated dequant-then-linear must match the reference modules'
outputs within the tolerance the reference's own checks use.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import configs, gemv, quant
from oracle.quant import from_bits

TOL = 1e-2  # max |err| / max |ref|, the north-star bound for bf16 outputs


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("n,k,ik", [(16, 256, 8), (24, 512, 8), (32, 128, 2), (32, 128, 4), (40, 384, 8)])
def test_tinygemm_pack_matches_aten(golden, n, k, ik):
    d = golden("tinygemm_pack.npz")
    src = torch.from_numpy(d[f"in_{n}_{k}_{ik}"])
    ref = d[f"out_{n}_{k}_{ik}"]
    mine = quant.tinygemm_pack(src, ik).numpy()
    assert mine.shape == ref.shape
    assert (mine == ref).all()
    assert torch.equal(quant.tinygemm_unpack(torch.from_numpy(ref)), src)


def test_tinygemm_unpack_transpose_equals_index_map():
    """The fast unpack (an axis permutation) against the explicit index map."""
    g = torch.Generator().manual_seed(3)
    for n, k, ik in ((8, 128, 8), (64, 512, 8), (16, 512, 2), (24, 1024, 4)):
        packed = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int32).to(torch.uint8)
        w = quant.tinygemm_pack(packed, ik)
        assert torch.equal(quant.tinygemm_unpack(w), quant.tinygemm_unpack_indexed(w))
        assert torch.equal(quant.tinygemm_unpack(w), packed)


def test_grouped_dequant_is_one_rounding():
    """fp32 (q - 8) * s + z equals the fma formed in float64 and rounded once."""
    g = torch.Generator().manual_seed(4)
    q = torch.randint(0, 16, (64, 512), generator=g, dtype=torch.int32).numpy()
    s = ((torch.randn(64, 4, generator=g) * 0.02).abs() / 7).to(torch.bfloat16).float().numpy()
    z = (torch.randn(64, 4, generator=g) * 0.01).to(torch.bfloat16).float().numpy()
    got = quant._grouped_fma(q - 8, s, z, 128)
    want = ((q - 8).astype(np.float64) * np.repeat(s, 128, 1).astype(np.float64)
            + np.repeat(z, 128, 1).astype(np.float64)).astype(np.float32)
    assert (got.view(np.uint32) == want.view(np.uint32)).all()


@pytest.mark.parametrize("n,k,gs", [(256, 512, 128), (128, 1024, 64), (64, 256, 32), (256, 512, 256)])
def test_int4_linear_quantize_and_forward(golden, n, k, gs):
    d = golden("int4_linear.npz")
    tag = f"{n}_{k}_{gs}"
    w = from_bits(d[f"w_{tag}"], torch.bfloat16)
    wi, sz = quant.quantize_int4(w, gs)
    assert (wi.numpy() == d[f"weight_int4_{tag}"]).all()
    assert (u16(sz) == d[f"scales_zeros_{tag}"]).all()
    W = quant.dequant_int4_tinygemm(wi, sz, gs)
    for m in (1, 2, 3, 16):
        x = from_bits(d[f"x_{tag}_m{m}"], torch.bfloat16)
        y = from_bits(d[f"y_{tag}_m{m}"], torch.bfloat16)
        assert gemv.max_rel_err(y.float(), x.float() @ W.T) < TOL


def test_config0_small_codes(golden):
    d = golden("config0_small.npz")
    cfg = configs.config0(seed=0, n=256, k=256)
    assert (cfg["codes"].numpy() == d["codes"]).all()
    assert (u16(cfg["scale"]) == d["scale"]).all()
    assert (u16(cfg["x"]) == d["x"]).all()
    wi, sz = configs.int4_tinygemm_from_codes(cfg["codes"], cfg["scale"])
    assert (wi.numpy() == d["weight_int4"]).all()
    assert (u16(sz) == d["scales_zeros"]).all()
    W = quant.dequant_int4_tinygemm(wi, sz, 128)
    # zero-point 8 with zero = 0 is w = (q - 8) * s exactly
    exact = (cfg["codes"].float() - 8) * cfg["scale"].float().repeat_interleave(128, 1)
    assert torch.equal(W, exact)
    # the plain layout with min = -8 s dequantizes to the same weights
    pk, s, mn = configs.int4_plain_from_codes(cfg["codes"], cfg["scale"])
    assert torch.equal(quant.dequant_int4_plain(pk, s, mn), exact)
    y = from_bits(d["y"], torch.bfloat16)
    assert gemv.max_rel_err(y.float(), cfg["x"].float() @ W.T) < TOL


@pytest.mark.parametrize("n,k", [(256, 512), (128, 1024)])
def test_fp8_linear_quantize(golden, n, k):
    d = golden("fp8_linear.npz")
    tag = f"{n}_{k}"
    w = from_bits(d[f"w_{tag}"], torch.bfloat16)
    wq, ws = quant.quantize_fp8_linear(w)
    assert (wq.view(torch.uint8).numpy() == d[f"weight_fp8_{tag}"]).all()
    assert (ws.numpy() == d[f"weight_scale_{tag}"]).all()
    W = quant.dequant_fp8(wq, ws)
    for m in (1, 2):
        x = from_bits(d[f"x_{tag}_m{m}"], torch.bfloat16)
        y = from_bits(d[f"y_{tag}_m{m}"], torch.bfloat16)
        # Fp8Linear.forward also quantizes activations (W8A8); the weight-only
        # path differs from it by the activation quantization error only.
        assert gemv.max_rel_err(y.float(), x.float() @ W.T) < 6e-2


@pytest.mark.parametrize("n,k,hb", [(256, 512, 0), (96, 384, 1)])
def test_int8_linear(golden, n, k, hb):
    d = golden("int8_linear.npz")
    tag = f"{n}_{k}_{hb}"
    w = from_bits(d[f"w_{tag}"], torch.bfloat16)
    q, s = quant.quantize_int8(w)
    assert (q.numpy() == d[f"weight_int8_{tag}"]).all()
    assert (s.numpy() == d[f"weight_scale_{tag}"]).all()
    W = quant.dequant_int8(q, s)
    b = from_bits(d[f"b_{tag}"], torch.bfloat16) if hb else None
    for m in (1, 2):
        x = from_bits(d[f"x_{tag}_m{m}"], torch.bfloat16)
        y = from_bits(d[f"y_{tag}_m{m}"], torch.bfloat16)
        assert gemv.max_rel_err(y.float(), gemv.linear_epilogue(x, W, bias=b)) < TOL


def _fused_weights(d):
    w = torch.from_numpy(d["w"])
    pk, s, mn = quant.pack_int4_plain(w)
    q8, s8 = quant.pack_fp8(w)
    return w, {
        4: (pk, s, mn, quant.dequant_int4_plain(pk, s, mn)),
        8: (q8, s8, None, quant.dequant_fp8(q8, s8)),
        16: (w.to(torch.bfloat16), None, None, w.to(torch.bfloat16).float()),
    }


def test_fused_pack_bit_exact(golden):
    d = golden("fused_triton.npz")
    _, fw = _fused_weights(d)
    pk, s, mn, _ = fw[4]
    assert (pk.numpy() == d["fw4_w"]).all()
    assert (u16(s) == d["fw4_s"]).all() and (u16(mn) == d["fw4_z"]).all()
    q8, s8, _, _ = fw[8]
    assert (q8.view(torch.uint8).numpy() == d["fw8_w"]).all()
    assert (s8.numpy() == d["fw8_s"]).all()


@pytest.mark.parametrize("bits", [4, 8, 16])
@pytest.mark.parametrize("epi", [0, 1, 2])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("norm", ["fp32", "breeze"])
def test_fused_rms_gemv_outputs(golden, bits, epi, m, norm):
    d = golden("fused_triton.npz")
    _, fw = _fused_weights(d)
    gamma = from_bits(d["gamma"], torch.bfloat16)
    t = f"b{bits}_e{epi}_m{m}"
    x = from_bits(d[f"x_{t}"], torch.bfloat16)
    res = from_bits(d[f"res_{t}"], torch.bfloat16)
    y = from_bits(d[f"y_{t}"], torch.bfloat16)
    ref = gemv.fused_reference(x, fw[bits][3], gamma if epi != 2 else None, 1e-6, epi,
                               res if epi == 2 else None, norm=norm)
    assert gemv.max_rel_err(y.float(), ref) < TOL


def test_glue_kernels(golden):
    d = golden("fused_triton.npz")
    gamma = from_bits(d["gamma"], torch.bfloat16)
    x = from_bits(d["rmsnorm_x"], torch.bfloat16)
    assert gemv.max_rel_err(from_bits(d["rmsnorm_y"], torch.bfloat16).float(), gemv.rmsnorm_fp32(x, gamma)) < TOL
    g = from_bits(d["silu_g"], torch.bfloat16)
    u = from_bits(d["silu_u"], torch.bfloat16)
    ref = F.silu(g.float()) * u.float()
    assert gemv.max_rel_err(from_bits(d["silu_y"], torch.bfloat16).float(), ref) < TOL


def test_oracle_detects_a_planted_layout_bug(golden):
    """A mistake planted in the oracle (the natural even-low nibble order the
    reference warns about, models/int4_linear.py:25-28) must be caught."""
    d = golden("tinygemm_pack.npz")
    src = torch.from_numpy(d["in_16_256_8"])
    swapped = ((src & 15) << 4) | (src >> 4)
    assert not (quant.tinygemm_pack(swapped, 8).numpy() == d["out_16_256_8"]).all()


# ---------------------------------------------------------------- attention
def _attn_case(golden, tag):
    d = golden("attention_step.npz")
    bf = torch.bfloat16
    B, HQ, HKV, D, S = (int(v) for v in d[f"shape_{tag}"])
    return dict(
        qkv=from_bits(d[f"qkv_{tag}"], bf), k=from_bits(d[f"k_{tag}"], bf), v=from_bits(d[f"v_{tag}"], bf),
        qn=from_bits(d[f"qn_{tag}"], bf), kn=from_bits(d[f"kn_{tag}"], bf), cos=from_bits(d[f"cos_{tag}"], bf),
        sin=from_bits(d[f"sin_{tag}"], bf), mask=from_bits(d[f"mask_{tag}"], bf), pos=int(d[f"pos_{tag}"][0]),
        out=from_bits(d[f"out_{tag}"], bf), k_after=from_bits(d[f"k_after_{tag}"], bf),
        v_after=from_bits(d[f"v_after_{tag}"], bf), shape=(B, HQ, HKV, D, S))


@pytest.mark.parametrize("tag", ["c0", "c1"])
def test_attention_step_matches_reference(golden, tag):
    """The oracle against the reference's Triton attention_step recorded on a
    B200 (one split at S=64, eight splits at S=320, a padded row)."""
    from oracle import attention

    c = _attn_case(golden, tag)
    keys, values = c["k"].clone(), c["v"].clone()
    out, keys, values = attention.attention_step(c["qkv"], c["cos"], c["sin"], c["pos"], keys, values, c["mask"],
                                                 c["qn"], c["kn"], 1e-6)
    # cache writes: v copied exactly, k within one bf16 ulp (fp32 sum order)
    assert torch.equal(values[:, :, c["pos"]], c["v_after"])
    kd = (keys[:, :, c["pos"]].float() - c["k_after"].float()).abs()
    assert (kd <= c["k_after"].float().abs() * 2 ** -7 + 1e-6).all()
    assert gemv.max_rel_err(out.float(), c["out"].float()) < 1e-2
    # every other cache position is untouched
    other = torch.ones(keys.shape[2], dtype=torch.bool)
    other[c["pos"]] = False
    assert torch.equal(keys[:, :, other], c["k"][:, :, other])
