"""The one-launch decode chain (bq_gemv_chain_*): failure handling and reuse.

A wait that nothing will satisfy -- the chain's start flag, a device word no
one sets -- must run out after its short bound, set BQ_DEVERR_WAIT_TIMEOUT,
and let the kernel return, leaving the context usable: the same chain,
prepared again with the flag set, and a fresh chain then compute the right
result. No GPU fault is involved; the flag is simply never written.

Also: repeated launches of one prepared chain (its per-op counters carry on
from launch to launch) give bit-identical results, and GEMVs of different
formats and epilogues share one chain.
"""

import pytest
import torch

from gpu_cases import make_weight, wfmt_code
from oracle import gemv as og

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda"


def _two_gemvs(m=2, k=1024, n=2048, seed=0):
    """x -> (RMSNorm, int4 tinygemm, SiLU*up) -> act -> (fp8, + x residual) -> y."""
    from breeze_b200 import _lib as L

    g = torch.Generator().manual_seed(seed)
    w1 = make_weight("int4_tinygemm", 2 * n, k, seed=seed + 1)
    w2 = make_weight("fp8", k, n, seed=seed + 2)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).to(DEV)
    act = torch.zeros(m, n, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros(m, k, dtype=torch.bfloat16, device=DEV)
    t = dict(w1=w1["w"].to(DEV), s1=w1["scale"].to(DEV), w2=w2["w"].to(DEV), s2=w2["scale"].to(DEV))
    descs = [L.gemv_desc(x, t["w1"], wfmt_code("int4_tinygemm"), 2 * n, out=act, scale=t["s1"], group=w1["group"],
                         gamma=gamma, epilogue=L.EPI_SILU_MUL, flags=L.default_flags()),
             L.gemv_desc(act, t["w2"], wfmt_code("fp8"), k, out=y, scale=t["s2"], epilogue=L.EPI_ADD_RESIDUAL,
                         residual=x, flags=L.default_flags())]
    keep = (x, gamma, act, y, t)

    def check():
        a_ref = og.fused_reference(x.cpu(), w1["deq"], gamma.cpu(), 1e-6, L.EPI_SILU_MUL)
        assert og.max_rel_err(act.cpu().float(), a_ref) <= TOL
        y_ref = og.fused_reference(act.cpu(), w2["deq"], None, 1e-6, L.EPI_ADD_RESIDUAL, x.cpu())
        assert og.max_rel_err(y.cpu().float(), y_ref) <= TOL

    return descs, keep, check, (act, y)


def test_chain_mixed_formats_and_repeated_launches():
    from breeze_b200 import _lib as L

    descs, keep, check, (act, y) = _two_gemvs()
    ch = L.GemvChain(descs, torch.device(DEV))
    ch.launch()
    torch.cuda.synchronize()
    check()
    first = y.clone()
    for _ in range(5):
        y.zero_()
        ch.launch()
    torch.cuda.synchronize()
    assert torch.equal(y, first)
    assert L.device_status(0) == 0


def test_chain_wait_runs_out_and_the_kernel_returns():
    from breeze_b200 import _lib as L

    L.device_status(0, clear=True)
    descs, keep, check, (act, y) = _two_gemvs(seed=5)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)  # nothing sets it
    ch = L.GemvChain(descs, torch.device(DEV), wait_cycles=400_000_000, start_flag=flag, start_target=1)  # ~0.2 s
    y.fill_(7.0)
    ch.launch()
    torch.cuda.synchronize()  # returns: every wait is bounded
    assert L.device_status(0) & L.BQ_DEVERR_WAIT_TIMEOUT
    assert bool((y == 7.0).all())  # the second GEMV never ran
    L.device_status(0, clear=True)
    # the context is still usable: the same chain with its flag set ...
    flag.fill_(1)
    ch.prepare()
    ch.launch()
    torch.cuda.synchronize()
    check()
    assert L.device_status(0) == 0
    # ... and a fresh chain without a flag
    descs2, keep2, check2, _ = _two_gemvs(seed=6)
    ch2 = L.GemvChain(descs2, torch.device(DEV))
    ch2.launch()
    torch.cuda.synchronize()
    check2()
    assert L.device_status(0) == 0
