"""Parity of the CUDA path (through the C ABI) against the CPU oracle.

Bars: dequantized weights and int4 re-tiling bit-exact; GEMV outputs within
max |err| / max |ref| <= 1e-2 of the oracle's fp32 dequant-then-linear
(TOL below), for every weight format, epilogue and M = 1..20.
"""

import numpy as np
import pytest
import torch

from gpu_cases import FORMATS, make_weight, wfmt_code
from oracle import configs, gemv, quant
from oracle.quant import from_bits

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda"


def _lib():
    from breeze_b200 import _lib as L

    return L


def run_gemv(case, x, n, *, gamma=None, eps=1e-6, epilogue=0, residual=None, out_dtype=torch.bfloat16, fmt="bf16"):
    L = _lib()
    w = case["w"].to(DEV)
    scale = None if case["scale"] is None else case["scale"].to(DEV)
    return L.gemv(x.to(DEV), w, wfmt_code(fmt), n, scale=scale, group=case["group"],
                  gamma=None if gamma is None else gamma.to(DEV), eps=eps, epilogue=epilogue,
                  residual=None if residual is None else residual.to(DEV), out_dtype=out_dtype,
                  flags=L.default_flags()).cpu()


# ---------------------------------------------------------------- layouts
@pytest.mark.parametrize("n,k,ik", [(16, 256, 8), (24, 512, 8), (32, 128, 2), (32, 128, 4), (40, 384, 8)])
def test_tinygemm_pack_bit_exact(golden, n, k, ik):
    L = _lib()
    d = golden("tinygemm_pack.npz")
    src = torch.from_numpy(d[f"in_{n}_{k}_{ik}"]).to(DEV)
    out = L.tinygemm_pack(src, ik).cpu().numpy()
    assert (out == d[f"out_{n}_{k}_{ik}"]).all()
    back = L.tinygemm_unpack(torch.from_numpy(d[f"out_{n}_{k}_{ik}"]).to(DEV))
    assert torch.equal(back.cpu(), src.cpu())


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("group", [32, 64, 128, 256])
def test_dequant_bit_exact(fmt, group):
    if fmt != "int4_tinygemm" and group != 128:
        pytest.skip("group size applies to tinygemm int4 only")
    n, k = 72, 512
    case = make_weight(fmt, n, k, seed=group, group=group)
    L = _lib()
    got = L.dequant(case["w"].to(DEV), wfmt_code(fmt), n, k,
                    scale=None if case["scale"] is None else case["scale"].to(DEV), group=case["group"]).cpu()
    if fmt == "int8":
        ref = quant.dequant_int8(case["w"], case["scale"]).float()  # bf16 weights, as Int8Linear.forward
    else:
        ref = case["deq"]
    assert torch.equal(got, ref)


def test_fp8_all_codes_exact():
    """Every e4m3 byte (except the two NaNs) dequantizes exactly."""
    L = _lib()
    b = torch.arange(256, dtype=torch.int32).to(torch.uint8).repeat(8, 2)  # (8, 512)
    b[(b & 0x7F) == 0x7F] = 0
    w = b.view(torch.float8_e4m3fn)
    s = torch.ones(8)
    got = L.dequant(w.to(DEV), L.W_FP8_E4M3, 8, 512, scale=s.to(DEV)).cpu()
    assert torch.equal(got, w.float())


# ---------------------------------------------------------------- GEMV sweep
SHAPES = [(256, 512), (200, 384), (96, 1024)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 16, 20])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemv_parity(fmt, m, epi):
    for n, k in SHAPES:
        if fmt.startswith("int4") and (n % 8 or (epi == 1 and (n // 2) % 8)):
            continue
        case = make_weight(fmt, n, k, seed=n + k + m + epi)
        g = torch.Generator().manual_seed(7 * m + epi)
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16) if epi != 2 else None
        n_out = n // 2 if epi == 1 else n
        res = torch.randn(m, n_out, generator=g).to(torch.bfloat16) if epi == 2 else None
        got = run_gemv(case, x, n, gamma=gamma, epilogue=epi, residual=res, fmt=fmt)
        ref = gemv.fused_reference(x, case["deq"], gamma, 1e-6, epi, res)
        assert got.shape == ref.shape
        err = gemv.max_rel_err(got.float(), ref)
        assert err < TOL, (fmt, m, epi, n, k, err)


@pytest.mark.parametrize("fmt", ["int4_tinygemm"])
@pytest.mark.parametrize("group", [32, 64, 256])
@pytest.mark.parametrize("m", [1, 9])
def test_gemv_group_sizes(fmt, group, m):
    n, k = 128, 1024
    case = make_weight(fmt, n, k, seed=group + m, group=group)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(group)).to(torch.bfloat16)
    got = run_gemv(case, x, n, fmt=fmt)
    assert gemv.max_rel_err(got.float(), x.float() @ case["deq"].T) < TOL


@pytest.mark.parametrize("xdt", [torch.float16, torch.float32])
@pytest.mark.parametrize("fmt", ["int4_tinygemm", "fp8", "bf16"])
def test_gemv_activation_dtypes(xdt, fmt):
    n, k, m = 128, 512, 2
    case = make_weight(fmt, n, k, seed=3)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(4)).to(xdt)
    got = run_gemv(case, x, n, fmt=fmt, out_dtype=xdt)
    assert got.dtype == xdt
    assert gemv.max_rel_err(got.float(), x.float() @ case["deq"].T) < TOL


def test_gemv_extreme_activation_scale():
    """Rows of very different magnitude (1e-30 .. 1e30) keep full relative
    accuracy: each row is rescaled by a power of two before the f16 MMA."""
    n, k = 64, 256
    case = make_weight("fp8", n, k, seed=5)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4, k, generator=g)
    x = x * torch.tensor([1e-30, 1e-3, 1e4, 1e30])[:, None]
    x = x.to(torch.float32)
    got = run_gemv(case, x, n, fmt="fp8", out_dtype=torch.float32)
    ref = x.double() @ case["deq"].double().T
    for r in range(4):
        assert gemv.max_rel_err(got[r], ref[r]) < TOL


# ---------------------------------------------------------------- drop-in modules vs golden
@pytest.mark.parametrize("n,k,gs", [(256, 512, 128), (128, 1024, 64), (64, 256, 32), (256, 512, 256)])
def test_int4_linear_module_golden(golden, n, k, gs):
    from breeze_b200.int4_linear import Int4Linear

    d = golden("int4_linear.npz")
    tag = f"{n}_{k}_{gs}"
    w = from_bits(d[f"w_{tag}"], torch.bfloat16)
    lin = torch.nn.Linear(k, n, bias=False, dtype=torch.bfloat16)
    lin.weight.data = w.to(DEV)
    mod = Int4Linear(lin, group_size=gs)
    assert (mod.weight_int4.cpu().numpy() == d[f"weight_int4_{tag}"]).all()
    assert (mod.scales_zeros.cpu().view(torch.int16).numpy().view(np.uint16) == d[f"scales_zeros_{tag}"]).all()
    W = quant.dequant_int4_tinygemm(mod.weight_int4.cpu(), mod.scales_zeros.cpu(), gs)
    for m in (1, 2, 3, 16):
        x = from_bits(d[f"x_{tag}_m{m}"], torch.bfloat16)
        y_ref_module = from_bits(d[f"y_{tag}_m{m}"], torch.bfloat16)
        y = mod(x.to(DEV)).cpu()
        assert y.dtype == torch.bfloat16 and y.shape == (m, n)
        assert gemv.max_rel_err(y.float(), x.float() @ W.T) < TOL
        assert gemv.max_rel_err(y.float(), y_ref_module.float()) < TOL


def test_int4_linear_3d_input():
    from breeze_b200.int4_linear import Int4Linear

    lin = torch.nn.Linear(512, 256, bias=False, dtype=torch.bfloat16, device=DEV)
    mod = Int4Linear(lin)
    x = torch.randn(2, 3, 512, device=DEV, dtype=torch.bfloat16)
    y = mod(x)
    assert y.shape == (2, 3, 256)
    W = quant.dequant_int4_tinygemm(mod.weight_int4.cpu(), mod.scales_zeros.cpu(), 128)
    assert gemv.max_rel_err(y.cpu().float().reshape(6, 256), x.cpu().float().reshape(6, 512) @ W.T) < TOL


@pytest.mark.parametrize("n,k", [(256, 512), (128, 1024)])
def test_fp8_linear_module_golden(golden, n, k):
    from breeze_b200.fp8_linear import Fp8Linear

    d = golden("fp8_linear.npz")
    tag = f"{n}_{k}"
    w = from_bits(d[f"w_{tag}"], torch.bfloat16)
    lin = torch.nn.Linear(k, n, bias=False, dtype=torch.bfloat16)
    lin.weight.data = w.to(DEV)
    mod = Fp8Linear(lin)
    assert (mod.weight_fp8.cpu().view(torch.uint8).numpy() == d[f"weight_fp8_{tag}"]).all()
    assert (mod.weight_scale.cpu().numpy() == d[f"weight_scale_{tag}"]).all()
    W = quant.dequant_fp8(mod.weight_fp8.cpu(), mod.weight_scale.cpu())
    for m in (1, 2):
        x = from_bits(d[f"x_{tag}_m{m}"], torch.bfloat16)
        y = mod(x.to(DEV)).cpu()
        assert gemv.max_rel_err(y.float(), x.float() @ W.T) < TOL
        # the reference module is W8A8; weight-only stays within its error
        assert gemv.max_rel_err(y.float(), from_bits(d[f"y_{tag}_m{m}"], torch.bfloat16).float()) < 6e-2


@pytest.mark.parametrize("n,k,hb", [(256, 512, 0), (96, 384, 1)])
def test_int8_linear_module_golden(golden, n, k, hb):
    from breeze_b200.int8_linear import Int8Linear

    d = golden("int8_linear.npz")
    tag = f"{n}_{k}_{hb}"
    w = from_bits(d[f"w_{tag}"], torch.bfloat16)
    lin = torch.nn.Linear(k, n, bias=bool(hb), dtype=torch.bfloat16)
    lin.weight.data = w.to(DEV)
    if hb:
        lin.bias.data = from_bits(d[f"b_{tag}"], torch.bfloat16).to(DEV)
    mod = Int8Linear(lin)
    assert (mod.weight_int8.cpu().numpy() == d[f"weight_int8_{tag}"]).all()
    assert (mod.weight_scale.cpu().numpy() == d[f"weight_scale_{tag}"]).all()
    W = quant.dequant_int8(mod.weight_int8.cpu(), mod.weight_scale.cpu())
    b = mod.bias.cpu() if hb else None
    for m in (1, 2):
        x = from_bits(d[f"x_{tag}_m{m}"], torch.bfloat16)
        y = mod(x.to(DEV)).cpu()
        assert gemv.max_rel_err(y.float(), gemv.linear_epilogue(x, W, bias=b)) < TOL
        assert gemv.max_rel_err(y.float(), from_bits(d[f"y_{tag}_m{m}"], torch.bfloat16).float()) < TOL


@pytest.mark.parametrize("bits", [4, 8, 16])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_rms_gemv_golden(golden, bits, epi):
    from breeze_b200.fused.kernels import FusedWeight, rms_gemv

    d = golden("fused_triton.npz")
    w = torch.from_numpy(d["w"])
    gamma = from_bits(d["gamma"], torch.bfloat16)
    fw = FusedWeight(w.to(DEV), bits)
    if bits == 4:
        assert (fw.w.cpu().numpy() == d["fw4_w"]).all()
        assert (fw.s.cpu().contiguous().view(torch.int16).numpy().view(np.uint16) == d["fw4_s"]).all()
        assert (fw.z.cpu().contiguous().view(torch.int16).numpy().view(np.uint16) == d["fw4_z"]).all()
        W = quant.dequant_int4_plain(fw.w.cpu(), fw.s.cpu().contiguous(), fw.z.cpu().contiguous())
    elif bits == 8:
        assert (fw.w.cpu().view(torch.uint8).numpy() == d["fw8_w"]).all()
        assert (fw.s.cpu().numpy() == d["fw8_s"]).all()
        W = quant.dequant_fp8(fw.w.cpu(), fw.s.cpu())
    else:
        W = fw.w.cpu().float()
    for m in (1, 2):
        t = f"b{bits}_e{epi}_m{m}"
        x = from_bits(d[f"x_{t}"], torch.bfloat16)
        res = from_bits(d[f"res_{t}"], torch.bfloat16)
        y = rms_gemv(x.to(DEV), fw, gamma.to(DEV) if epi != 2 else None, 1e-6, epilogue=epi,
                     residual=res.to(DEV) if epi == 2 else None).cpu()
        ref = gemv.fused_reference(x, W, gamma if epi != 2 else None, 1e-6, epi, res if epi == 2 else None)
        assert gemv.max_rel_err(y.float(), ref) < TOL
        assert gemv.max_rel_err(y.float(), from_bits(d[f"y_{t}"], torch.bfloat16).float()) < TOL


def test_glue_kernels_golden(golden):
    from breeze_b200.fused.kernels import rmsnorm, silu_mul

    d = golden("fused_triton.npz")
    gamma = from_bits(d["gamma"], torch.bfloat16)
    x = from_bits(d["rmsnorm_x"], torch.bfloat16)
    y = rmsnorm(x.to(DEV), gamma.to(DEV)).cpu()
    assert gemv.max_rel_err(y.float(), from_bits(d["rmsnorm_y"], torch.bfloat16).float()) < TOL
    g = from_bits(d["silu_g"], torch.bfloat16)
    u = from_bits(d["silu_u"], torch.bfloat16)
    y = silu_mul(g.to(DEV), u.to(DEV)).cpu()
    assert gemv.max_rel_err(y.float(), from_bits(d["silu_y"], torch.bfloat16).float()) < TOL


# ---------------------------------------------------------------- BASELINE configs at full size
def test_config0_full():
    L = _lib()
    cfg = configs.config0(seed=0)
    w, sz = configs.int4_tinygemm_from_codes(cfg["codes"], cfg["scale"])
    case = {"w": w, "scale": sz, "group": 128}
    got = run_gemv(case, cfg["x"], 2048, fmt="int4_tinygemm")
    W = quant.dequant_int4_tinygemm(w, sz, 128)
    assert gemv.max_rel_err(got.float(), cfg["x"].float() @ W.T) < TOL
    # dequant bit-exact at full size
    deq = L.dequant(w.to(DEV), L.W_INT4_TINYGEMM, 2048, 2048, scale=sz.to(DEV)).cpu()
    assert torch.equal(deq, W)


@pytest.mark.parametrize("layout", ["int4_tinygemm", "int4_plain"])
def test_config1_full(layout):
    cfg = configs.config1(seed=0)
    if layout == "int4_tinygemm":
        w, sz = configs.int4_tinygemm_from_codes(cfg["codes"], cfg["scale"])
        W = quant.dequant_int4_tinygemm(w, sz, 128)
    else:
        w, s, mn = configs.int4_plain_from_codes(cfg["codes"], cfg["scale"])
        sz = torch.stack([s.t(), mn.t()], -1).contiguous()
        W = quant.dequant_int4_plain(w, s, mn)
    case = {"w": w, "scale": sz, "group": 128}
    got = run_gemv(case, cfg["x"], 6144, gamma=cfg["gamma"], eps=cfg["eps"], fmt=layout)
    for norm in ("fp32", "breeze"):
        ref = gemv.fused_reference(cfg["x"], W, cfg["gamma"], cfg["eps"], 0, norm=norm)
        assert gemv.max_rel_err(got.float(), ref) < TOL


@pytest.mark.parametrize("shape", ["gate_up", "down"])
@pytest.mark.parametrize("m", [1, 2])
def test_config2_full(shape, m):
    cfg = configs.config2(seed=0, shape=shape, m=m)
    case = {"w": cfg["w"], "scale": cfg["scale"].reshape(-1), "group": 128}
    epi = 1 if shape == "gate_up" else 2
    got = run_gemv(case, cfg["x"], cfg["n"], epilogue=epi, residual=cfg["residual"], fmt="fp8")
    W = quant.dequant_fp8(cfg["w"], cfg["scale"])
    ref = gemv.fused_reference(cfg["x"], W, None, 1e-6, epi, cfg["residual"])
    assert gemv.max_rel_err(got.float(), ref) < TOL


# ---------------------------------------------------------------- graphs, determinism, errors
def test_cuda_graph_capture_and_determinism():
    from breeze_b200.fused.kernels import FusedWeight, rms_gemv

    g = torch.Generator().manual_seed(11)
    w = torch.randn(1024, 2048, generator=g) * 0.02
    fw = FusedWeight(w.to(DEV), 4)
    x = torch.randn(2, 2048, generator=g).to(torch.bfloat16).to(DEV)
    gamma = torch.ones(2048, dtype=torch.bfloat16, device=DEV)
    eager = rms_gemv(x, fw, gamma)
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        rms_gemv(x, fw, gamma, out=out)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            rms_gemv(x, fw, gamma, out=out)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)  # bit-identical: fixed summation order


def test_invalid_arguments_raise():
    L = _lib()
    x = torch.randn(1, 200, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(64, 200, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="multiple of 128"):
        L.gemv(x, w, L.W_BF16, 64)
    x = torch.randn(1, 256, device=DEV, dtype=torch.bfloat16)
    w4 = torch.zeros(60 // 8, 2, 32, 4, device=DEV, dtype=torch.int32)
    with pytest.raises(ValueError, match="N % 8"):
        L.gemv(x, w4, L.W_INT4_TINYGEMM, 60, scale=torch.zeros(2, 60, 2, device=DEV, dtype=torch.bfloat16))


def test_device_status_clean():
    assert _lib().device_status() == 0


def test_workspace_shared_across_shapes():
    """Calls of very different shapes share one workspace: a small-N call's
    partial sums must never land on the arrival counters a large-N call
    reads (multi-chunk workers, many units)."""
    for (n, k) in [(64, 256), (6144, 2048), (32, 128), (6144, 2048), (4096, 1024)]:
        case = make_weight("int4_tinygemm", n, k, seed=n)
        x = torch.randn(1, k, generator=torch.Generator().manual_seed(n)).to(torch.bfloat16)
        got = run_gemv(case, x, n, fmt="int4_tinygemm")
        assert gemv.max_rel_err(got.float(), x.float() @ case["deq"].T) < TOL, (n, k)


# ---------------------------------------------------------------- one-row kernels, k-blocks per warp
@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 5])
@pytest.mark.parametrize("k", [1024, 1280, 2048, 3072, 4096])
@pytest.mark.parametrize("epi", [0, 2])
def test_gemv_one_row_kernel_k_blocks_per_warp(fmt, m, k, epi):
    """One-row kernels (M <= 8) carry two k-blocks per ring slot. Each warp
    owns an eighth of K (of a K slice when K is split): K = 2048 and 4096 give
    every warp an even count (the variant without the half-slot path), 1024
    and 3072 an odd one (last slot half full), 1280 a mix. With a norm
    (epi 0) K is never split; without one (epi 2) it may be. Parity with the
    oracle and bit-identical reruns either way."""
    n = 256
    case = make_weight(fmt, n, k, seed=k + m + epi)
    g = torch.Generator().manual_seed(k * 5 + m)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16) if epi == 0 else None
    res = torch.randn(m, n, generator=g).to(torch.bfloat16) if epi == 2 else None
    got = run_gemv(case, x, n, gamma=gamma, epilogue=epi, residual=res, fmt=fmt)
    again = run_gemv(case, x, n, gamma=gamma, epilogue=epi, residual=res, fmt=fmt)
    ref = gemv.fused_reference(x, case["deq"], gamma, 1e-6, epi, res)
    assert gemv.max_rel_err(got.float(), ref) < TOL, (fmt, m, k, epi)
    assert torch.equal(got, again)


# ---------------------------------------------------------------- K split across CTAs
@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m,n,k,epi", [(16, 2048, 8192, 2), (32, 1024, 8192, 0), (8, 512, 16384, 2),
                                       (12, 2048, 4096, 2), (16, 6144, 2048, 0)])
def test_gemv_k_split_large_m(fmt, m, n, k, epi):
    """Without a norm, activations that do not fit one CTA beside a dependent
    CTA split K across CTAs (rectangles of units x K slices, summed by the last
    arriver in slice order): parity with the oracle and bit-identical reruns."""
    case = make_weight(fmt, n, k, seed=m + n + k)
    g = torch.Generator().manual_seed(m * 3 + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16) if epi == 2 else None
    got = run_gemv(case, x, n, epilogue=epi, residual=res, fmt=fmt)
    again = run_gemv(case, x, n, epilogue=epi, residual=res, fmt=fmt)
    ref = gemv.fused_reference(x, case["deq"], None, 1e-6, epi, res)
    assert gemv.max_rel_err(got.float(), ref) < TOL
    assert torch.equal(got, again)


@pytest.mark.parametrize("fmt", ["int4_plain", "int4_tinygemm", "fp8"])
@pytest.mark.parametrize("m,epi", [(1, 0), (2, 1), (3, 2)])
def test_gemv_host_io_matches_device_call(fmt, m, epi):
    """bq_gemv_host_io (host input and output, copies enqueued with the GEMV)
    gives bit-for-bit the output of bq_gemv on the same data."""
    L = _lib()
    n, k = 256, 512
    case = make_weight(fmt, n, k, seed=m + epi)
    g = torch.Generator().manual_seed(17 * m + epi)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16) if epi != 2 else None
    n_out = n // 2 if epi == 1 else n
    res = torch.randn(m, n_out, generator=g).to(torch.bfloat16) if epi == 2 else None
    ref = run_gemv(case, x, n, gamma=gamma, epilogue=epi, residual=res, fmt=fmt)
    w = case["w"].to(DEV)
    scale = None if case["scale"] is None else case["scale"].to(DEV)
    xd = torch.zeros(m, k, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(m, n_out, device=DEV, dtype=torch.bfloat16)
    x_host, out_host = x.pin_memory(), torch.zeros(m, n_out, dtype=torch.bfloat16).pin_memory()
    got = L.gemv_host_io(x_host, xd, w, wfmt_code(fmt), n, out=out, out_host=out_host, scale=scale,
                         group=case["group"], gamma=None if gamma is None else gamma.to(DEV), eps=1e-6, epilogue=epi,
                         residual=None if res is None else res.to(DEV), flags=L.default_flags())
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    assert torch.equal(xd.cpu(), x)


@pytest.mark.parametrize("fmt", ["int8", "bf16", "int4_plain"])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_bias_in_output_dtype_through_raw_abi(fmt, out_dtype):
    """The descriptor's bias holds [N] values of the output's dtype (the
    header's contract). Called through ctypes with a descriptor built by hand
    from the tensors, no Python-side conversion."""
    import ctypes

    L = _lib()
    n, k, m = 384, 512, 3
    case = make_weight(fmt, n, k, seed=31)
    g = torch.Generator().manual_seed(32)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(n, generator=g) * 0.5).to(out_dtype).to(DEV)
    out = torch.full((m, n), float("nan"), dtype=out_dtype, device=DEV)
    w = case["w"].to(DEV)
    scale = None if case["scale"] is None else case["scale"].to(DEV)
    d = L.make_desc(x, w, wfmt_code(fmt), n, scale=scale, group=case["group"], bias=bias, out=out,
                    flags=L.default_flags())
    need = ctypes.c_size_t(0)
    L.check(L.load().bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(need)), "bq_gemv_workspace_bytes")
    ws = torch.zeros(max(need.value, 256), dtype=torch.uint8, device=DEV)
    L.check(L.load().bq_gemv(ctypes.byref(d), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream),
            "bq_gemv")
    torch.cuda.synchronize()
    ref = gemv.linear_epilogue(x.cpu().float(), case["deq"], bias=bias.cpu().float())
    assert gemv.max_rel_err(out.cpu().float(), ref) < TOL
