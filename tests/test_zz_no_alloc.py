"""bq_gemv_noalloc against bq_gemv, through the C ABI.

bq_gemv_noalloc exists for callers that may not allocate device memory
(fixed VRAM budgets, hosts that own every allocation, real-time threads):
it runs the same GEMV but keeps its split-K scratch in an array built into
the library instead of a caller workspace. These checks call it twice in a
row (the array keeps the previous call's contents) and compare each result
with the allocating entry point's, within the suite's tolerance. This file
is collected last so that a failure here stops a -x run only after every
other test has run.
"""

import ctypes

import pytest
import torch

from gpu_cases import make_weight, wfmt_code
from oracle import gemv

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda"


def _call_noalloc(L, x, w, fmt, n, *, scale, group, gamma=None, epilogue=0, residual=None, out):
    d = L.make_desc(x, w, wfmt_code(fmt), n, scale=scale, group=group, gamma=gamma, epilogue=epilogue,
                    residual=residual, out=out, flags=L.default_flags())
    rc = L.load().bq_gemv_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    L.check(rc, "bq_gemv_noalloc")


@pytest.mark.parametrize("fmt,n,k,m,epi", [
    ("int4_tinygemm", 6144, 2048, 1, 0),   # config-1 shape, norm prologue
    ("fp8", 4096, 2048, 2, 1),             # SiLU*up epilogue
    ("int8", 2048, 2048, 9, 2),            # residual epilogue, two M tiles
])
def test_noalloc_matches_bq_gemv_on_two_calls(fmt, n, k, m, epi):
    from breeze_b200 import _lib as L

    case = make_weight(fmt, n, k, seed=n + m)
    g = torch.Generator().manual_seed(m + epi)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).to(DEV) if epi != 2 else None
    n_out = n // 2 if epi == 1 else n
    res = torch.randn(m, n_out, generator=g).to(torch.bfloat16).to(DEV) if epi == 2 else None
    w = case["w"].to(DEV)
    scale = None if case["scale"] is None else case["scale"].to(DEV)
    ref = L.gemv(x, w, wfmt_code(fmt), n, scale=scale, group=case["group"], gamma=gamma, epilogue=epi,
                 residual=res, flags=L.default_flags())
    outs = []
    for _ in range(2):
        out = torch.full((m, n_out), float("nan"), device=DEV, dtype=torch.bfloat16)
        _call_noalloc(L, x, w, fmt, n, scale=scale, group=case["group"], gamma=gamma, epilogue=epi,
                      residual=res, out=out)
        outs.append(out)
    torch.cuda.synchronize()
    for out in outs:
        assert not torch.isnan(out).any()
        assert gemv.max_rel_err(out.cpu().float(), ref.cpu().float()) < TOL
    assert L.device_status() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """A shape whose split-K scratch exceeds the fixed array is refused with
    a clear error before anything is launched."""
    from breeze_b200 import _lib as L

    lib = L.load()
    d = L.GemvDesc()
    d.M, d.N, d.K, d.wfmt, d.group = 16, 16384, 8192, L.W_BF16, 128
    d.x, d.w, d.out, d.ldx, d.ldo = 256, 256, 256, 8192, 16384
    rc = lib.bq_gemv_noalloc(ctypes.byref(d), None)
    assert rc == L.BQ_ERR_WORKSPACE
    assert "scratch" in L.last_error()
