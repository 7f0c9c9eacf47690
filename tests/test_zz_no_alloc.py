"""bq_gemv_noalloc, the entry point for callers that cannot allocate device memory.

Some callers of this library may not call cudaMalloc: a decode loop held to a
fixed VRAM budget, a host application that owns every device allocation
through its own allocator, or a real-time audio thread that must not take the
driver's allocation lock. bq_gemv_noalloc runs bq_gemv's kernel with the
split-K scratch kept in an array built into the library, so such a caller
passes only inputs and outputs.

Each case calls it twice in a row through the C ABI -- the array keeps what
the previous call left, so the second call checks that nothing stale leaks
in -- and compares both outputs with the CPU oracle and with the allocating
entry point (bq_gemv) at the suite's tolerance, max rel err 1e-2. The cases
cover every weight format and epilogue, a bias, a tinygemm group of 64, and
M above 16, where several row blocks run one after another on the shared
array. This file is collected last, so a failure here stops a -x run only
after every other test has run; it also passes alone in a fresh process.
"""

import ctypes

import pytest
import torch

from gpu_cases import make_weight, wfmt_code
from oracle import gemv

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda"
SCRATCH_BYTES = 4 << 20


def _lib():
    from breeze_b200 import _lib as L

    return L


def _noalloc(L, d):
    L.check(L.load().bq_gemv_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream), "bq_gemv_noalloc")


@pytest.mark.parametrize("fmt,n,k,m,epi,group,bias", [
    ("int4_tinygemm", 6144, 2048, 1, 0, 128, False),   # config-1 shape, norm prologue
    ("int4_tinygemm", 1024, 2048, 5, 2, 64, False),    # group 64, residual
    ("int4_plain", 2048, 2048, 2, 1, 128, False),      # fused-path layout, SiLU*up
    ("fp8", 4096, 2048, 2, 1, 128, False),             # SiLU*up
    ("int8", 2048, 2048, 9, 2, 128, True),             # residual and bias, two M tiles
    ("bf16", 1024, 1024, 3, 0, 128, True),             # bias, norm prologue
    ("int8", 2048, 8192, 40, 2, 128, False),           # several row blocks share the scratch
    ("int4_tinygemm", 16384, 2048, 33, 1, 128, False),  # gate+up at M = 33
])
def test_noalloc_matches_oracle_on_two_calls(fmt, n, k, m, epi, group, bias):
    L = _lib()
    case = make_weight(fmt, n, k, seed=n + m, group=group)
    g = torch.Generator().manual_seed(m + epi)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16) if epi != 2 else None
    n_out = n // 2 if epi == 1 else n
    res = torch.randn(m, n_out, generator=g).to(torch.bfloat16) if epi == 2 else None
    b = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16) if bias else None
    ref = gemv.fused_reference(x, case["deq"], gamma, 1e-6, epi, res, bias=b)
    dx, dgamma, dres, db = (None if t is None else t.to(DEV) for t in (x, gamma, res, b))
    w = case["w"].to(DEV)
    scale = None if case["scale"] is None else case["scale"].to(DEV)
    alloc = L.gemv(dx, w, wfmt_code(fmt), n, scale=scale, group=group, gamma=dgamma, epilogue=epi, residual=dres,
                   bias=db, flags=L.default_flags())
    outs = []
    for _ in range(2):
        out = torch.full((m, n_out), float("nan"), device=DEV, dtype=torch.bfloat16)
        d = L.make_desc(dx, w, wfmt_code(fmt), n, scale=scale, group=group, gamma=dgamma, epilogue=epi,
                        residual=dres, bias=db, out=out, flags=L.default_flags())
        _noalloc(L, d)
        outs.append(out)
    torch.cuda.synchronize()
    for out in outs:
        assert not torch.isnan(out).any()
        assert gemv.max_rel_err(out.cpu().float(), ref) < TOL
        assert gemv.max_rel_err(out.cpu().float(), alloc.cpu().float()) < TOL
    assert L.device_status() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """A shape whose split-K scratch exceeds the fixed array is refused with a
    clear error before anything is launched (the output keeps its canary)."""
    L = _lib()
    lib = L.load()
    over = None
    for n, k, m in ((16384, 8192, 16), (32768, 8192, 16), (65536, 8192, 16)):
        x = torch.zeros(m, k, dtype=torch.bfloat16, device=DEV)
        w = torch.zeros(n, k, dtype=torch.bfloat16, device=DEV)
        out = torch.full((m, n), 7.0, dtype=torch.bfloat16, device=DEV)
        d = L.make_desc(x, w, L.W_BF16, n, out=out, flags=L.default_flags())
        need = ctypes.c_size_t(0)
        L.check(lib.bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(need)), "bq_gemv_workspace_bytes")
        if need.value > SCRATCH_BYTES:
            over = (d, out)
            break
    assert over is not None, "no candidate shape needs more scratch than the fixed array"
    d, out = over
    rc = lib.bq_gemv_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    assert rc == L.BQ_ERR_WORKSPACE
    assert "scratch" in L.last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())


def test_noalloc_after_status_clear():
    """bq_device_status_clear (the recovery step after a device wait ran out)
    makes the next call clear the built-in array's counters again; the calls
    around it stay correct."""
    L = _lib()
    case = make_weight("int4_tinygemm", 2048, 2048, seed=3)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(1, 2048, generator=g).to(torch.bfloat16)
    ref = gemv.fused_reference(x, case["deq"], None, 1e-6, 0)
    dx, w, scale = x.to(DEV), case["w"].to(DEV), case["scale"].to(DEV)
    for clear in (False, True, False):
        if clear:
            torch.cuda.synchronize()
            L.device_status(0, clear=True)
        out = torch.full((1, 2048), float("nan"), device=DEV, dtype=torch.bfloat16)
        d = L.make_desc(dx, w, wfmt_code("int4_tinygemm"), 2048, scale=scale, group=128, out=out,
                        flags=L.default_flags())
        _noalloc(L, d)
        torch.cuda.synchronize()
        assert gemv.max_rel_err(out.cpu().float(), ref) < TOL
    assert L.device_status() == 0
