"""The two kernels behind one- and two-row GEMVs, each against the CPU oracle.

bq_gemv runs one or two activation rows on the resident-slice kernel (the
CTA's whole weight slice copied to shared memory before the dependent-launch
wait); BQ_FLAG_RING_KERNEL keeps such a call on the ring-streaming kernel,
which also serves three to sixteen rows and the shapes the former declines.
Shapes with fewer 16-row units than half the SMs run the resident-slice kernel
with K split across a cluster of two CTAs per unit (partial sums added in
distributed shared memory). All must meet the suite's bar --
max |err| / max |ref| <= 1e-2 against the oracle's fp32 dequant-then-linear --
for every weight format, epilogue and the RMSNorm prologue, on shapes that
give CTAs one to four units (ragged last unit included), and the
resident-slice kernel must give bit-identical results on a rerun.
"""

import pytest
import torch

from gpu_cases import FORMATS, make_weight, wfmt_code
from oracle import gemv

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda"

# (N, K): 128 units of 16 rows (one per CTA), 384 units (two or three per CTA), 16384 rows
# (four units per CTA with SiLU*up; without it more than four, which the resident-slice
# kernel declines), a ragged last unit (6152 rows), long K (2048 x 8192)
SHAPES = [(2048, 2048), (6144, 2048), (16384, 1024), (6152, 1024), (2048, 8192)]


def _run(fmt, n, k, m, epi, norm, flags, seed=0):
    from breeze_b200 import _lib as L

    if fmt.startswith("int4") and n % 8:
        pytest.skip("int4 weights need N % 8 == 0")
    case = make_weight(fmt, n, k, seed=seed + n + k)
    g = torch.Generator().manual_seed(seed + m + 10 * epi + int(norm))
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16) if norm else None
    n_out = n // 2 if epi == 1 else n
    res = torch.randn(m, n_out, generator=g).to(torch.bfloat16) if epi == 2 else None
    scale = None if case["scale"] is None else case["scale"].to(DEV)
    out = L.gemv(x.to(DEV), case["w"].to(DEV), wfmt_code(fmt), n, scale=scale, group=case["group"],
                 gamma=None if gamma is None else gamma.to(DEV), epilogue=epi,
                 residual=None if res is None else res.to(DEV), flags=L.default_flags() | flags)
    ref = gemv.fused_reference(x, case["deq"], gamma, 1e-6, epi, res)
    return out, ref


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("epi,norm", [(0, True), (1, True), (2, False)])
@pytest.mark.parametrize("kernel", ["resident", "ring"])
def test_one_and_two_rows_match_oracle(fmt, m, epi, norm, kernel):
    from breeze_b200 import _lib as L

    flags = L.FLAG_RING_KERNEL if kernel == "ring" else 0
    for n, k in SHAPES:
        if epi == 1 and (n // 2) % 8:
            continue
        out, ref = _run(fmt, n, k, m, epi, norm, flags)
        err = gemv.max_rel_err(out.cpu().float(), ref)
        assert err < TOL, (fmt, m, epi, norm, kernel, n, k, err)
    assert L.device_status() == 0


@pytest.mark.parametrize("fmt", FORMATS)
def test_resident_slice_rerun_is_bit_identical(fmt):
    from breeze_b200 import _lib as L

    a, _ = _run(fmt, 6144, 2048, 1, 0, True, 0, seed=3)
    b, _ = _run(fmt, 6144, 2048, 1, 0, True, 0, seed=3)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert L.device_status() == 0


# (N, K) with fewer 16-row units than half the SMs: K split in two across a cluster of two
# CTAs per unit -- the depth decoder's down projection (1024 x 8192), the shortest K the
# split takes (eight k-blocks per CTA), a ragged last unit (1000 rows)
SPLIT_SHAPES = [(1024, 8192), (1024, 2048), (1000, 4096)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("epi,norm", [(0, True), (0, False), (2, False), (2, True)])
def test_k_split_matches_oracle(fmt, m, epi, norm):
    from breeze_b200 import _lib as L

    for n, k in SPLIT_SHAPES:
        out, ref = _run(fmt, n, k, m, epi, norm, 0)
        err = gemv.max_rel_err(out.cpu().float(), ref)
        assert err < TOL, (fmt, m, epi, norm, n, k, err)
    assert L.device_status() == 0


@pytest.mark.parametrize("fmt", ["int4_tinygemm", "int4_plain", "fp8", "bf16"])
def test_k_split_is_the_cluster_kernel_and_deterministic(fmt):
    """The few-unit shape runs the K-split instantiation (kernel names from the profiler),
    and a rerun gives bit-identical results (fixed rank order of the cluster sum)."""
    from torch.profiler import ProfilerActivity, profile

    from breeze_b200 import _lib as L

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        a, _ = _run(fmt, 1024, 8192, 1, 2, False, 0, seed=5)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if "gemv" in e.name]
    if not names:
        pytest.skip("the profiler recorded no kernels on this box")
    assert any("gemv_lean_kernel<" in nm and nm.split(">")[0].replace(" ", "").endswith(",2") for nm in names), names
    b, _ = _run(fmt, 1024, 8192, 1, 2, False, 0, seed=5)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert L.device_status() == 0
