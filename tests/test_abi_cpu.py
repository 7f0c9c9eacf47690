"""The C-ABI library without a GPU: it loads, exports every function that
include/breeze_b200.h declares, and rejects bad descriptors on the host
(before touching a device), with the reference's exception types."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "breeze_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int32_t|const char\*)\s+(bq_\w+)\s*\(", text, re.M)))


def test_header_declares_the_api():
    names = declared_functions()
    for must in ("bq_gemv", "bq_gemv_workspace_bytes", "bq_dequant", "bq_int4_tinygemm_pack",
                 "bq_last_error_string", "bq_version"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_python_binding_covers_the_header():
    from breeze_b200 import _lib

    assert sorted(_lib.exported_symbols()) == declared_functions()


def test_version(lib):
    from breeze_b200 import _lib

    assert lib.bq_version() == 1
    assert isinstance(_lib.last_error(), str)


def test_desc_layout_matches_header():
    """The ctypes mirror has the C struct's size (12 x 4-byte fields + 10 x 8)."""
    from breeze_b200 import _lib

    assert ctypes.sizeof(_lib.GemvDesc) == 12 * 4 + 10 * 8
    assert _lib.GemvDesc.x.offset == 48


def _desc(**kw):
    from breeze_b200 import _lib

    d = _lib.GemvDesc()
    d.M, d.N, d.K, d.wfmt, d.group = 1, 64, 256, _lib.W_BF16, 128
    d.x, d.w, d.out, d.ldx, d.ldo = 16, 16, 16, 256, 64
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("field,value,code,pattern", [
    ("K", 200, -2, "multiple of 128"),
    ("M", 0, -2, "positive"),
    ("wfmt", 9, -4, "unknown weight format"),
    ("epilogue", 7, -1, "unknown epilogue"),
    ("x_dtype", 5, -1, "unknown dtype"),
    ("ldx", 100, -2, "ldx"),
])
def test_host_validation(lib, field, value, code, pattern):
    from breeze_b200 import _lib

    d = _desc(**{field: value})
    n = ctypes.c_size_t(0)
    rc = lib.bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(n))
    assert rc == code
    assert re.search(pattern, _lib.last_error())
    with pytest.raises(ValueError):
        _lib.check(rc, "bq_gemv_workspace_bytes")


def test_int4_geometry_rules(lib):
    from breeze_b200 import _lib

    n = ctypes.c_size_t(0)
    d = _desc(wfmt=_lib.W_INT4_TINYGEMM, N=60, scale=16)
    assert lib.bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(n)) == _lib.BQ_ERR_SHAPE
    d = _desc(wfmt=_lib.W_INT4_TINYGEMM, N=64, group=100, scale=16)
    assert lib.bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(n)) == _lib.BQ_ERR_SHAPE
    d = _desc(wfmt=_lib.W_INT4_PLAIN, N=64, group=64, scale=16)
    assert lib.bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(n)) == _lib.BQ_ERR_SHAPE
    d = _desc(wfmt=_lib.W_INT4_TINYGEMM, N=64, scale=0)
    assert lib.bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(n)) == _lib.BQ_ERR_INVALID_ARG
    d = _desc(w=8)  # misaligned weight pointer
    assert lib.bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(n)) == _lib.BQ_ERR_ALIGN


def test_pack_argument_checks(lib):
    from breeze_b200 import _lib

    assert lib.bq_int4_tinygemm_pack(None, None, 8, 256, 8, None) == _lib.BQ_ERR_INVALID_ARG
    assert lib.bq_int4_tinygemm_pack(16, 16, 12, 256, 8, None) == _lib.BQ_ERR_SHAPE
    assert lib.bq_int4_tinygemm_pack(16, 16, 8, 256, 3, None) == _lib.BQ_ERR_SHAPE


def test_no_cpu_fallback():
    """The product path refuses CPU tensors instead of computing elsewhere."""
    import torch

    from breeze_b200 import _lib

    x = torch.randn(1, 256, dtype=torch.bfloat16)
    w = torch.randn(64, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        _lib.gemv(x, w, _lib.W_BF16, 64)


def test_attention_desc_validation_without_gpu(lib):
    """Host-side validation of bq_attention_step needs no GPU."""
    import ctypes

    from breeze_b200 import _lib as L

    d = L.AttnDesc()
    need = ctypes.c_size_t(0)
    assert lib.bq_attention_workspace_bytes(ctypes.byref(d), ctypes.byref(need)) == L.BQ_ERR_SHAPE
    d.B, d.HQ, d.HKV, d.D, d.S = 1, 16, 16, 96, 64
    assert lib.bq_attention_workspace_bytes(ctypes.byref(d), ctypes.byref(need)) == L.BQ_ERR_SHAPE
    assert b"head dim" in lib.bq_last_error_string()
    d.D, d.HKV = 128, 3
    assert lib.bq_attention_workspace_bytes(ctypes.byref(d), ctypes.byref(need)) == L.BQ_ERR_SHAPE
    d.HKV = 16
    assert lib.bq_attention_step(ctypes.byref(d), None, 0, None) == L.BQ_ERR_INVALID_ARG


def test_attention_o_desc_validation_without_gpu(lib):
    """bq_attention_o_step (attention fused with the O projection): the
    descriptor mirrors the header (bq_attn_desc + 2 x 4 + 6 x 8 bytes) and
    its host-side checks need no GPU."""
    import ctypes

    from breeze_b200 import _lib as L

    assert ctypes.sizeof(L.AttnDesc) == 8 * 4 + 14 * 8
    assert ctypes.sizeof(L.AttnODesc) == ctypes.sizeof(L.AttnDesc) + 2 * 4 + 6 * 8
    assert L.AttnODesc.N.offset == ctypes.sizeof(L.AttnDesc)
    od = L.AttnODesc()
    a = od.attn
    a.B, a.HQ, a.HKV, a.D, a.S = 1, 8, 8, 128, 17
    a.qkv = a.cos = a.sin = a.pos = a.k_cache = a.v_cache = 256
    a.ldqkv = (8 + 16) * 128
    od.attn = a
    od.N, od.wo, od.ldw, od.residual, od.ldr, od.out, od.ldo = 1024, 256, 1024, 256, 1024, 256, 1024
    need = ctypes.c_size_t(0)
    assert lib.bq_attention_o_workspace_bytes(ctypes.byref(od), ctypes.byref(need)) == 0
    assert need.value > 0
    for field, value, code, text in [("N", 1000, L.BQ_ERR_SHAPE, b"multiple of 16"),
                                     ("ldw", 512, L.BQ_ERR_SHAPE, b"too small"),
                                     ("wo", 0, L.BQ_ERR_INVALID_ARG, b"non-NULL"),
                                     ("wo", 264, L.BQ_ERR_ALIGN, b"16-byte")]:
        bad = L.AttnODesc.from_buffer_copy(od)
        setattr(bad, field, value)
        assert lib.bq_attention_o_workspace_bytes(ctypes.byref(bad), ctypes.byref(need)) == code, field
        assert text in lib.bq_last_error_string()
    for field, value, text in [("B", 5, b"exceeds"), ("S", 300, b"cache length")]:
        bad = L.AttnODesc.from_buffer_copy(od)
        setattr(bad.attn, field, value)
        assert lib.bq_attention_o_workspace_bytes(ctypes.byref(bad), ctypes.byref(need)) == L.BQ_ERR_SHAPE, field
        assert text in lib.bq_last_error_string()
    bad = L.AttnODesc.from_buffer_copy(od)
    bad.attn.mask, bad.attn.mask_dtype = 256, 9
    assert lib.bq_attention_o_workspace_bytes(ctypes.byref(bad), ctypes.byref(need)) == L.BQ_ERR_INVALID_ARG
    assert lib.bq_attention_o_step(ctypes.byref(od), None, 0, None) != 0


def test_gemv_host_io_argument_checks(lib):
    """bq_gemv_host_io validates the descriptor and its host pointers before
    any copy or launch (no GPU needed)."""
    import ctypes

    from breeze_b200 import _lib as L

    d = _desc()
    assert lib.bq_gemv_host_io(ctypes.byref(d), None, None, None, 0, None) == L.BQ_ERR_INVALID_ARG
    assert b"x_host" in lib.bq_last_error_string()
    bad = _desc(K=200)
    assert lib.bq_gemv_host_io(ctypes.byref(bad), 16, 16, None, 0, None) == L.BQ_ERR_SHAPE
