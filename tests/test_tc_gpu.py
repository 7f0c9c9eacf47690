"""Parity of the tensor-core GEMV (tcgen05, 17..128 activation rows, weights
read once) against the CPU oracle, through the C ABI.

bq_gemv takes this path by itself for 17..128 bf16 rows when N is a multiple
of 128; BQ_FLAG_NO_TC keeps a call on the mma.sync kernel, which re-streams
the weights per 16 rows. Bar: max |err| / max |ref| <= 1e-2 against the
oracle's fp32 dequant-then-linear (TOL), every weight format and epilogue, with
and without the RMSNorm; bit-identical reruns (the K slices of a unit are
summed in cluster-rank order).
"""

import functools

import pytest
import torch

from gpu_cases import FORMATS, make_weight, wfmt_code
from oracle import gemv

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda"


def _run(case, fmt, x, n, *, gamma=None, epilogue=0, residual=None, bias=None, out_dtype=torch.bfloat16, flags=None):
    from breeze_b200 import _lib as L

    scale = None if case["scale"] is None else case["scale"].to(DEV)
    fl = L.default_flags() if flags is None else flags
    return L.gemv(x.to(DEV), case["w"].to(DEV), wfmt_code(fmt), n, scale=scale, group=case["group"],
                  gamma=None if gamma is None else gamma.to(DEV), eps=1e-6, epilogue=epilogue,
                  residual=None if residual is None else residual.to(DEV),
                  bias=None if bias is None else bias.to(DEV), out_dtype=out_dtype, flags=fl).cpu()


def _inputs(m, n, k, epi, norm, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16) if norm else None
    n_out = n // 2 if epi == 1 else n
    res = torch.randn(m, n_out, generator=g).to(torch.bfloat16) if epi == 2 else None
    return x, gamma, res


@functools.lru_cache(maxsize=64)
def _case(fmt, n, k):
    return make_weight(fmt, n, k, seed=n + 3 * k)


# (N, K): two units of 128 rows, each split into up to 8 K slices (256x1024), eight
# units (1024x2048), 48 units in uneven K slices (6144x2048: 3 slices of 16 k-blocks)
SHAPES = [(256, 1024), (1024, 2048), (6144, 2048)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [17, 32, 64, 128])
@pytest.mark.parametrize("epi,norm", [(0, False), (0, True), (1, True), (2, False)])
def test_tc_parity(fmt, m, epi, norm):
    for n, k in SHAPES:
        if fmt == "bf16" and m > 64 and n == 6144:
            continue  # bf16 weights above 64 rows keep the mma.sync kernel (shared memory)
        case = _case(fmt, n, k)
        x, gamma, res = _inputs(m, n, k, epi, norm, 7 * m + epi + int(norm))
        got = _run(case, fmt, x, n, gamma=gamma, epilogue=epi, residual=res)
        ref = gemv.fused_reference(x, case["deq"], gamma, 1e-6, epi, res)
        assert got.shape == ref.shape
        err = gemv.max_rel_err(got.float(), ref)
        assert err < TOL, (fmt, m, epi, norm, n, k, err)


@pytest.mark.parametrize("group", [32, 64, 256])
def test_tc_tinygemm_groups(group):
    n, k, m = 512, 2048, 40
    case = make_weight("int4_tinygemm", n, k, seed=group, group=group)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(group)).to(torch.bfloat16)
    got = _run(case, "int4_tinygemm", x, n)
    assert gemv.max_rel_err(got.float(), x.float() @ case["deq"].T) < TOL


@pytest.mark.parametrize("fmt", ["int4_tinygemm", "fp8"])
def test_tc_bias_f32_out_and_rows_not_multiple_of_16(fmt):
    n, k, m = 384, 1024, 45
    case = make_weight(fmt, n, k, seed=3)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    bias = torch.randn(n, generator=g)
    got = _run(case, fmt, x, n, bias=bias, out_dtype=torch.float32)
    ref = x.float() @ case["deq"].T + bias
    assert got.dtype == torch.float32
    assert gemv.max_rel_err(got, ref) < TOL


def test_tc_int8_scale_rounding():
    from breeze_b200 import _lib as L

    n, k, m = 256, 1024, 33
    case = make_weight("int8", n, k, seed=5)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
    got = _run(case, "int8", x, n, flags=L.default_flags() | L.FLAG_SCALE_ROUND_BF16)
    s = case["scale"].to(torch.bfloat16).float()
    ref = x.float() @ (case["w"].float() * s[:, None]).T
    assert gemv.max_rel_err(got.float(), ref) < TOL


@pytest.mark.parametrize("fmt", ["int4_tinygemm", "int4_plain", "fp8", "int8", "bf16"])
def test_tc_matches_row_block_kernel_and_is_deterministic(fmt):
    """The same call on both kernels (BQ_FLAG_NO_TC forces the mma.sync row
    blocks) agrees within the tolerance; reruns of the tensor-core kernel are
    bit-identical."""
    from breeze_b200 import _lib as L

    n, k, m = 2048, 2048, 48
    case = make_weight(fmt, n, k, seed=11)
    x, gamma, res = _inputs(m, n, k, 2, False, 12)
    a = _run(case, fmt, x, n, epilogue=2, residual=res)
    b = _run(case, fmt, x, n, epilogue=2, residual=res)
    c = _run(case, fmt, x, n, epilogue=2, residual=res, flags=L.default_flags() | L.FLAG_NO_TC)
    assert torch.equal(a, b)
    assert gemv.max_rel_err(a.float(), c.float()) < TOL


def test_tc_graph_chain_with_norms():
    """Three dependent GEMVs (norm -> gate+up SiLU, down + residual, norm -> QKV)
    captured in one CUDA graph with programmatic dependent launch: replays give
    the eager result bit for bit and match the oracle."""
    from breeze_b200 import _lib as L

    m, h, inter = 64, 1024, 4096
    gu = make_weight("int4_tinygemm", 2 * inter, h, seed=21)
    dn = make_weight("int4_tinygemm", h, inter, seed=22)
    qk = make_weight("int4_tinygemm", 3 * h, h, seed=23)
    g = torch.Generator().manual_seed(24)
    x = torch.randn(m, h, generator=g).to(torch.bfloat16).to(DEV)
    g1 = (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16).to(DEV)
    g2 = (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16).to(DEV)
    act = torch.empty(m, inter, dtype=torch.bfloat16, device=DEV)
    h2 = torch.empty(m, h, dtype=torch.bfloat16, device=DEV)
    qkv = torch.empty(m, 3 * h, dtype=torch.bfloat16, device=DEV)
    fl = L.default_flags()
    dev = {name: (c["w"].to(DEV), c["scale"].to(DEV)) for name, c in (("gu", gu), ("dn", dn), ("qk", qk))}

    def step():
        L.gemv(x, dev["gu"][0], L.W_INT4_TINYGEMM, 2 * inter, scale=dev["gu"][1], group=128, gamma=g1,
               epilogue=L.EPI_SILU_MUL, out=act, flags=fl)
        L.gemv(act, dev["dn"][0], L.W_INT4_TINYGEMM, h, scale=dev["dn"][1], group=128,
               epilogue=L.EPI_ADD_RESIDUAL, residual=x, out=h2, flags=fl)
        L.gemv(h2, dev["qk"][0], L.W_INT4_TINYGEMM, 3 * h, scale=dev["qk"][1], group=128, gamma=g2, out=qkv, flags=fl)

    step()
    torch.cuda.synchronize()
    eager = (act.clone(), h2.clone(), qkv.clone())
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        act.zero_()
        qkv.zero_()
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(act, eager[0]) and torch.equal(h2, eager[1]) and torch.equal(qkv, eager[2])
    xc = x.cpu()
    a_ref = gemv.fused_reference(xc, gu["deq"], g1.cpu(), 1e-6, 1, None)
    assert gemv.max_rel_err(act.cpu().float(), a_ref) < TOL
    h_ref = gemv.fused_reference(act.cpu(), dn["deq"], None, 1e-6, 2, xc)
    assert gemv.max_rel_err(h2.cpu().float(), h_ref) < TOL
    q_ref = gemv.fused_reference(h2.cpu(), qk["deq"], g2.cpu(), 1e-6, 0, None)
    assert gemv.max_rel_err(qkv.cpu().float(), q_ref) < TOL
    assert L.device_status(0) == 0
