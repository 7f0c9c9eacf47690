"""ctypes binding of libbreeze_b200.so (the C ABI in include/breeze_b200.h).

The library is the only compute path: if it is missing, or the tensors are
not on a CUDA device, calls raise -- there is no CPU or PyTorch fallback.
Status codes map to the exception types the reference raises for the same
conditions (ValueError for shape/format problems, RuntimeError otherwise).
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libbreeze_b200.so"

# ---- constants mirrored from include/breeze_b200.h ----------------------
BQ_OK = 0
BQ_ERR_INVALID_ARG, BQ_ERR_SHAPE, BQ_ERR_ALIGN, BQ_ERR_FORMAT = -1, -2, -3, -4
BQ_ERR_WORKSPACE, BQ_ERR_CUDA, BQ_ERR_DEVICE = -5, -6, -7
BQ_DEVERR_WAIT_TIMEOUT = 1

W_BF16, W_INT4_TINYGEMM, W_INT4_PLAIN, W_FP8_E4M3, W_INT8 = 0, 1, 2, 3, 4
EPI_NONE, EPI_SILU_MUL, EPI_ADD_RESIDUAL = 0, 1, 2
DT_BF16, DT_F16, DT_F32 = 0, 1, 2
FLAG_PDL, FLAG_SCALE_ROUND_BF16, FLAG_NO_TC, FLAG_RING_KERNEL = 1, 2, 4, 8

_DT = {torch.bfloat16: DT_BF16, torch.float16: DT_F16, torch.float32: DT_F32}


class GemvDesc(ctypes.Structure):
    """Mirror of ``bq_gemv_desc``."""

    _fields_ = [
        ("M", ctypes.c_int32), ("N", ctypes.c_int32), ("K", ctypes.c_int32),
        ("wfmt", ctypes.c_int32), ("group", ctypes.c_int32), ("epilogue", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32), ("res_dtype", ctypes.c_int32),
        ("flags", ctypes.c_uint32), ("eps", ctypes.c_float), ("reserved", ctypes.c_int32),
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("gamma", ctypes.c_void_p), ("w", ctypes.c_void_p), ("scale", ctypes.c_void_p),
        ("bias", ctypes.c_void_p), ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64),
        ("out", ctypes.c_void_p), ("ldo", ctypes.c_int64),
    ]


class AttnDesc(ctypes.Structure):
    """bq_attn_desc (include/breeze_b200.h)."""

    _fields_ = [
        ("B", ctypes.c_int32), ("HQ", ctypes.c_int32), ("HKV", ctypes.c_int32), ("D", ctypes.c_int32),
        ("S", ctypes.c_int32), ("mask_dtype", ctypes.c_int32), ("eps", ctypes.c_float), ("flags", ctypes.c_uint32),
        ("qkv", ctypes.c_void_p), ("ldqkv", ctypes.c_int64), ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p),
        ("ldcs", ctypes.c_int64), ("pos", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("mask", ctypes.c_void_p), ("ldm", ctypes.c_int64), ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
        ("out", ctypes.c_void_p), ("ldo", ctypes.c_int64),
    ]


class AttnODesc(ctypes.Structure):
    """bq_attn_o_desc (include/breeze_b200.h)."""

    _fields_ = [
        ("attn", AttnDesc), ("N", ctypes.c_int32), ("reserved", ctypes.c_int32), ("wo", ctypes.c_void_p),
        ("ldw", ctypes.c_int64), ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64), ("out", ctypes.c_void_p),
        ("ldo", ctypes.c_int64),
    ]


HEAD_NK = 0
HEAD_KN = 1
SAMPLE_TOPK_VALUE = 2
SAMPLE_APPEND_HISTORY = 4


class HeadDesc(ctypes.Structure):
    """bq_head_desc (include/breeze_b200.h)."""

    _fields_ = [
        ("M", ctypes.c_int32), ("N", ctypes.c_int32), ("K", ctypes.c_int32), ("layout", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32), ("flags", ctypes.c_uint32), ("eps", ctypes.c_float), ("reserved", ctypes.c_int32),
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64), ("gamma", ctypes.c_void_p), ("w", ctypes.c_void_p),
        ("ldw", ctypes.c_int64), ("out", ctypes.c_void_p), ("ldo", ctypes.c_int64),
    ]


class SampleDesc(ctypes.Structure):
    """bq_sample_desc (include/breeze_b200.h)."""

    _fields_ = [
        ("rows", ctypes.c_int32), ("V", ctypes.c_int32), ("cfg", ctypes.c_int32), ("max_k", ctypes.c_int32),
        ("mask_lo", ctypes.c_int32), ("mask_hi", ctypes.c_int32), ("clamp_hi", ctypes.c_int32),
        ("flags", ctypes.c_uint32), ("rep_penalty", ctypes.c_float), ("history_cap", ctypes.c_int32),
        ("logits", ctypes.c_void_p), ("ldl", ctypes.c_int64), ("guidance", ctypes.c_void_p),
        ("temperature", ctypes.c_void_p), ("top_k", ctypes.c_void_p), ("top_p", ctypes.c_void_p),
        ("do_sample", ctypes.c_void_p), ("history", ctypes.c_void_p), ("history_len", ctypes.c_void_p),
        ("suppress", ctypes.c_void_p), ("uniform", ctypes.c_void_p), ("rng", ctypes.c_void_p),
        ("cfg_out", ctypes.c_void_p), ("ldc", ctypes.c_int64), ("tokens", ctypes.c_void_p), ("ldt", ctypes.c_int64),
        ("tokens2", ctypes.c_void_p), ("ldt2", ctypes.c_int64), ("eos_id", ctypes.c_int64),
        ("eos_flag", ctypes.c_void_p),
    ]


class ChainOptions(ctypes.Structure):
    """bq_chain_options (include/breeze_b200.h)."""

    _fields_ = [("wait_cycles", ctypes.c_uint64), ("start_flag", ctypes.c_void_p), ("start_target", ctypes.c_uint32)]


_lib = None
_lock = threading.Lock()

_SIGS = {
    "bq_version": (ctypes.c_int32, []),
    "bq_last_error_string": (ctypes.c_char_p, []),
    "bq_device_status": (ctypes.c_int32, [ctypes.c_int32, ctypes.POINTER(ctypes.c_uint32)]),
    "bq_device_status_clear": (ctypes.c_int32, [ctypes.c_int32]),
    "bq_gemv_workspace_bytes": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.POINTER(ctypes.c_size_t)]),
    "bq_gemv": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "bq_gemv_noalloc": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.c_void_p]),
    "bq_gemv_chain_workspace_bytes": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.c_int32,
                                                       ctypes.POINTER(ctypes.c_size_t)]),
    "bq_gemv_chain_prepare": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.c_int32, ctypes.c_void_p,
                                               ctypes.c_size_t]),
    "bq_gemv_chain_prepare_ex": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.c_int32,
                                                  ctypes.POINTER(ChainOptions), ctypes.c_void_p, ctypes.c_size_t]),
    "bq_gemv_chain_launch": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.c_int32, ctypes.c_void_p,
                                              ctypes.c_size_t, ctypes.c_void_p]),
    "bq_attention_workspace_bytes": (ctypes.c_int32, [ctypes.POINTER(AttnDesc), ctypes.POINTER(ctypes.c_size_t)]),
    "bq_gemv_host_io": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_size_t, ctypes.c_void_p]),
    "bq_attention_step": (ctypes.c_int32, [ctypes.POINTER(AttnDesc), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "bq_attention_o_workspace_bytes": (ctypes.c_int32, [ctypes.POINTER(AttnODesc), ctypes.POINTER(ctypes.c_size_t)]),
    "bq_attention_o_step": (ctypes.c_int32, [ctypes.POINTER(AttnODesc), ctypes.c_void_p, ctypes.c_size_t,
                                              ctypes.c_void_p]),
    "bq_head_workspace_bytes": (ctypes.c_int32, [ctypes.POINTER(HeadDesc), ctypes.POINTER(ctypes.c_size_t)]),
    "bq_head_gemv": (ctypes.c_int32, [ctypes.POINTER(HeadDesc), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "bq_sample_workspace_bytes": (ctypes.c_int32, [ctypes.POINTER(SampleDesc), ctypes.POINTER(ctypes.c_size_t)]),
    "bq_sample": (ctypes.c_int32, [ctypes.POINTER(SampleDesc), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "bq_embed_rows": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_uint32, ctypes.c_void_p]),
    "bq_int4_tinygemm_pack": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                               ctypes.c_int32, ctypes.c_void_p]),
    "bq_int4_tinygemm_unpack": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                                 ctypes.c_int32, ctypes.c_void_p]),
    "bq_dequant": (ctypes.c_int32, [ctypes.POINTER(GemvDesc), ctypes.c_void_p, ctypes.c_void_p]),
    "bq_rmsnorm": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                    ctypes.c_void_p]),
    "bq_silu_mul": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                     ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_void_p]),
}


def default_flags() -> int:
    """Programmatic dependent launch is on unless BREEZE_B200_PDL=0: each
    GEMV starts streaming its (static) weights while the previous kernel in
    the stream finishes, and waits for it before reading activations."""
    return 0 if os.environ.get("BREEZE_B200_PDL", "1") == "0" else FLAG_PDL


def exported_symbols() -> list[str]:
    return list(_SIGS)


def load() -> ctypes.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = os.environ.get("BREEZE_B200_LIB", str(LIB_PATH))
            if not Path(path).exists():
                raise RuntimeError(
                    f"{path} is missing: build it with `python breeze-tts-2_b200/build.py` "
                    "(breeze_b200 has no fallback path)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in _SIGS.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    return load().bq_last_error_string().decode()


def check(rc: int, what: str) -> None:
    if rc == BQ_OK:
        return
    msg = f"{what}: {last_error()} (status {rc})"
    if rc in (BQ_ERR_SHAPE, BQ_ERR_FORMAT, BQ_ERR_ALIGN, BQ_ERR_INVALID_ARG, BQ_ERR_WORKSPACE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("breeze_b200 kernels need CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no tensor given")
    if dev.index != torch.cuda.current_device():
        torch.cuda.set_device(dev)
    return dev


# ---- workspace ---------------------------------------------------------------
class Workspace:
    """Per-device scratch for split-K partial sums and arrival counters.

    Zero-filled when (re)allocated; the kernels leave the counters at zero
    after every call, so the buffer is reused as is. It only grows outside
    stream capture: capture a CUDA graph after one warm-up call per shape,
    as the reference does before capturing its decode graphs.
    """

    def __init__(self):
        self._bufs: dict[int, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        idx = device.index
        buf = self._bufs.get(idx)
        if buf is None or buf.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    f"breeze_b200 workspace must grow to {nbytes} bytes during CUDA graph capture; "
                    "run the shape once before capturing")
            size = max(nbytes, 1 << 20, 0 if buf is None else 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            self._bufs[idx] = buf
        return buf

    def reset(self) -> None:
        for b in self._bufs.values():
            b.zero_()


WORKSPACE = Workspace()
# bq_attention_step keeps its own counters at the start of its workspace;
# bq_gemv's arrival counters (also at the start) must stay zero at rest, so
# the two never share a buffer.
ATTN_WORKSPACE = Workspace()
# bq_head_gemv (K-major layout) and bq_sample keep arrival counters the same way.
HEAD_WORKSPACE = Workspace()
SAMPLE_WORKSPACE = Workspace()


def make_desc(x: torch.Tensor, w: torch.Tensor, wfmt: int, n: int, *, scale=None, group: int = 128, gamma=None,
              eps: float = 1e-6, epilogue: int = EPI_NONE, residual=None, bias=None, out: torch.Tensor,
              flags: int = 0) -> GemvDesc:
    m, k = x.shape
    d = GemvDesc()
    d.M, d.N, d.K = m, n, k
    d.wfmt, d.group, d.epilogue = wfmt, group, epilogue
    d.x_dtype = _DT[x.dtype]
    d.out_dtype = _DT[out.dtype]
    d.res_dtype = _DT[residual.dtype] if residual is not None else DT_BF16
    d.flags = flags
    d.eps = eps
    d.x, d.ldx = x.data_ptr(), x.stride(0)
    d.gamma = _ptr(gamma)
    d.w = w.data_ptr()
    d.scale = _ptr(scale)
    d.bias = _ptr(bias)
    d.residual = _ptr(residual)
    d.ldr = residual.stride(0) if residual is not None else 0
    d.out, d.ldo = out.data_ptr(), out.stride(0)
    return d


def _rowmajor(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with unit stride in the last dimension")
    return t


# Descriptors of calls that name their output buffer, keyed by every pointer,
# shape, stride and dtype the descriptor holds: a repeated call (a decode loop
# over static buffers) skips validation, descriptor construction and the
# workspace query and goes straight to bq_gemv.
_GEMV_CACHE: dict = {}
_GEMV_CACHE_MAX = 4096


def _gemv_key(x, w, wfmt, n, scale, group, gamma, eps, epilogue, residual, bias, out, flags):
    return (x.data_ptr(), x.shape, x.stride(), x.dtype, x.device, w.data_ptr(), wfmt, n,
            None if scale is None else scale.data_ptr(), group,
            None if gamma is None else (gamma.data_ptr(), gamma.dtype), eps, epilogue,
            None if residual is None else (residual.data_ptr(), residual.shape, residual.stride(), residual.dtype),
            None if bias is None else (bias.data_ptr(), bias.dtype),
            out.data_ptr(), out.shape, out.stride(), out.dtype, flags)


def _gemv_prepared(x, w, wfmt, n, scale, group, gamma, eps, epilogue, residual, bias, out, out_dtype, flags):
    """(descriptor, workspace, out) of one GEMV; descriptors over the caller's
    own tensors are cached by the tensors' addresses, shapes and options."""
    key = None
    if out is not None and x.is_cuda:
        key = _gemv_key(x, w, wfmt, n, scale, group, gamma, eps, epilogue, residual, bias, out, flags)
        hit = _GEMV_CACHE.get(key)
        if hit is not None:
            return hit[0], hit[1], out
    dev = _require_cuda(x, w, scale, gamma, residual, bias, out)
    own = (_ptr(gamma), _ptr(bias))  # the caller's own tensors, before any dtype conversion
    x = _rowmajor(x, "x")
    if x.dtype not in _DT:
        raise ValueError(f"unsupported activation dtype {x.dtype}")
    m = x.shape[0]
    n_out = n // 2 if epilogue == EPI_SILU_MUL else n
    if residual is not None:
        residual = _rowmajor(residual, "residual")
    if out is None:
        dt = out_dtype or (residual.dtype if residual is not None else torch.bfloat16)
        out = torch.empty(m, n_out, device=dev, dtype=dt)
    else:
        out = _rowmajor(out, "out")
    if gamma is not None and gamma.dtype != torch.bfloat16:
        gamma = gamma.to(torch.bfloat16)
    if bias is not None and bias.dtype != out.dtype:
        bias = bias.to(out.dtype)
    lib = load()
    d = make_desc(x, w, wfmt, n, scale=scale, group=group, gamma=gamma, eps=eps, epilogue=epilogue,
                  residual=residual, bias=bias, out=out, flags=flags)
    need = ctypes.c_size_t(0)
    check(lib.bq_gemv_workspace_bytes(ctypes.byref(d), ctypes.byref(need)), "bq_gemv_workspace_bytes")
    ws = WORKSPACE.get(dev, need.value)
    # cache only descriptors that point at the caller's own tensors (no converted copies)
    if key is not None and (d.gamma, d.bias) == own:
        if len(_GEMV_CACHE) >= _GEMV_CACHE_MAX:
            _GEMV_CACHE.clear()
        _GEMV_CACHE[key] = (d, ws)
    return d, ws, out


def gemv(x: torch.Tensor, w: torch.Tensor, wfmt: int, n: int, *, scale=None, group: int = 128, gamma=None,
         eps: float = 1e-6, epilogue: int = EPI_NONE, residual=None, bias=None, out: torch.Tensor | None = None,
         out_dtype: torch.dtype | None = None, flags: int = 0) -> torch.Tensor:
    """out = epilogue(rmsnorm(x) @ dequant(w)^T) on the current stream."""
    d, ws, out = _gemv_prepared(x, w, wfmt, n, scale, group, gamma, eps, epilogue, residual, bias, out, out_dtype,
                                flags)
    check(_lib.bq_gemv(ctypes.byref(d), ws.data_ptr(), ws.numel(), torch.cuda.current_stream(x.device).cuda_stream),
          "bq_gemv")
    return out


def gemv_host_io(x_host: torch.Tensor, x: torch.Tensor, w: torch.Tensor, wfmt: int, n: int, *, out: torch.Tensor,
                 out_host: torch.Tensor, scale=None, group: int = 128, gamma=None, eps: float = 1e-6,
                 epilogue: int = EPI_NONE, residual=None, bias=None, flags: int = 0) -> torch.Tensor:
    """gemv with host-side input and output in one call (bq_gemv_host_io):
    x_host -> x, the GEMV into out, out -> out_host, enqueued on the current
    stream without waiting. x_host / out_host: dense CPU tensors shaped like x
    and out (pinned for asynchronous copies). Returns out_host."""
    if x_host.is_cuda or out_host.is_cuda:
        raise ValueError("x_host and out_host must be CPU tensors")
    if x_host.shape != x.shape or x_host.dtype != x.dtype or not x_host.is_contiguous():
        raise ValueError("x_host must be a dense CPU copy of x's shape and dtype")
    d, ws, out = _gemv_prepared(x, w, wfmt, n, scale, group, gamma, eps, epilogue, residual, bias, out, None, flags)
    if out_host.shape != out.shape or out_host.dtype != out.dtype or not out_host.is_contiguous():
        raise ValueError("out_host must be a dense CPU tensor of out's shape and dtype")
    check(_lib.bq_gemv_host_io(ctypes.byref(d), x_host.data_ptr(), out_host.data_ptr(), ws.data_ptr(), ws.numel(),
                               torch.cuda.current_stream(x.device).cuda_stream), "bq_gemv_host_io")
    return out_host


def gemv_desc(x: torch.Tensor, w: torch.Tensor, wfmt: int, n: int, *, out: torch.Tensor, scale=None,
              group: int = 128, gamma=None, eps: float = 1e-6, epilogue: int = EPI_NONE, residual=None,
              bias=None, flags: int = 0) -> GemvDesc:
    """Descriptor of one GEMV over existing device tensors (for chains)."""
    _require_cuda(x, w, scale, gamma, residual, bias, out)
    _rowmajor(x, "x")
    _rowmajor(out, "out")
    if residual is not None:
        _rowmajor(residual, "residual")
    if gamma is not None and gamma.dtype != torch.bfloat16:
        raise ValueError("chain descriptors need a bf16 gamma")
    return make_desc(x, w, wfmt, n, scale=scale, group=group, gamma=gamma, eps=eps, epilogue=epilogue,
                     residual=residual, bias=bias, out=out, flags=flags)


class GemvChain:
    """A list of GEMVs run as one persistent launch (bq_gemv_chain_*).

    The descriptors' tensors must stay alive and in place; ``launch()`` is
    capture-safe once the chain is built (``prepare`` runs here, outside any
    capture). ``wait_cycles`` bounds every device-side wait (0: the library's
    default, ~2 s); ``start_flag`` (an int32 device tensor written by the host
    or by earlier work, never by a kernel running at the same time) makes the
    first GEMV also wait until it reaches ``start_target``. ``prepare()``
    rewrites the workspace: call it again after a launch that set a device
    error bit.
    """

    def __init__(self, descs: list[GemvDesc], device: torch.device, wait_cycles: int = 0,
                 start_flag: torch.Tensor | None = None, start_target: int = 0):
        lib = load()
        self.n = len(descs)
        self._arr = (GemvDesc * self.n)(*descs)
        need = ctypes.c_size_t(0)
        check(lib.bq_gemv_chain_workspace_bytes(self._arr, self.n, ctypes.byref(need)), "bq_gemv_chain_workspace_bytes")
        self.ws = torch.zeros(max(int(need.value), 256), dtype=torch.uint8, device=device)
        self._opts = ChainOptions(wait_cycles, _ptr(start_flag), start_target)
        self._flag = start_flag
        self.device = device
        self.prepare()

    def prepare(self) -> None:
        check(load().bq_gemv_chain_prepare_ex(self._arr, self.n, ctypes.byref(self._opts), self.ws.data_ptr(),
                                              self.ws.numel()), "bq_gemv_chain_prepare_ex")

    def launch(self) -> None:
        check(load().bq_gemv_chain_launch(self._arr, self.n, self.ws.data_ptr(), self.ws.numel(), _stream(self.device)),
              "bq_gemv_chain_launch")


_MASKS: dict = {}


def additive_mask(mask: torch.Tensor, b: int, s: int) -> torch.Tensor:
    """(B, 1, Q, S) additive float or bool mask -> (B, S) additive, as the
    reference's _additive_mask (models/fused/kernels.py:492-502): bool masks
    become 0 / -1e30 fp32 once per static buffer."""
    if mask.dtype != torch.bool:
        m = mask.reshape(b, -1)
        return m[:, :s] if m.shape[1] != s else m
    key = (mask.data_ptr(), tuple(mask.shape), str(mask.device))
    m2 = _MASKS.get(key)
    if m2 is None:
        m2 = torch.where(mask.reshape(b, -1)[:, :s], 0.0, -1e30).float().contiguous()
        _MASKS[key] = m2
    return m2


def _attn_desc(qkv, cos, sin, cache_position, keys, values, mask, q_norm_w, k_norm_w, eps, flags):
    """bq_attn_desc of one attention step (out / ldo left unset), and the
    temporaries it points into (keep them alive until the launch)."""
    b = qkv.shape[0]
    _, hkv, s, d = keys.shape
    hq = (qkv.shape[1] - 2 * hkv * d) // d
    for t, name in ((qkv, "qkv"), (keys, "keys"), (values, "values")):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bf16")
    if not keys.is_contiguous() or not values.is_contiguous():
        raise ValueError("the KV caches must be contiguous (B, HKV, S, D)")
    qkv = _rowmajor(qkv, "qkv")
    cos2 = cos.reshape(cos.shape[0], -1).to(torch.bfloat16)
    sin2 = sin.reshape(sin.shape[0], -1).to(torch.bfloat16)
    if cos2.stride(1) != 1 or sin2.stride(1) != 1 or cos2.stride(0) != sin2.stride(0):
        raise ValueError("cos / sin rows must be contiguous with equal strides")
    if cache_position.dtype != torch.int64:
        raise ValueError("cache_position must be int64")
    ad = AttnDesc()
    ad.B, ad.HQ, ad.HKV, ad.D, ad.S = b, hq, hkv, d, s
    ad.eps, ad.flags = eps, flags
    ad.qkv, ad.ldqkv = qkv.data_ptr(), qkv.stride(0)
    ad.cos, ad.sin = cos2.data_ptr(), sin2.data_ptr()
    ad.ldcs = cos2.stride(0) if cos2.shape[0] == b else 0
    ad.pos = cache_position.data_ptr()
    ad.k_cache, ad.v_cache = keys.data_ptr(), values.data_ptr()
    keep = [qkv, cos2, sin2]
    if mask is not None:
        m2 = additive_mask(mask, b, s)
        if m2.dtype not in (torch.bfloat16, torch.float32):
            m2 = m2.float()
        if m2.stride(1) != 1:
            m2 = m2.contiguous()
        ad.mask, ad.ldm = m2.data_ptr(), m2.stride(0)
        ad.mask_dtype = _DT[m2.dtype]
        keep.append(m2)
    if q_norm_w is not None:
        qn, kn = q_norm_w.to(torch.bfloat16), k_norm_w.to(torch.bfloat16)
        ad.q_norm, ad.k_norm = qn.data_ptr(), kn.data_ptr()
        keep += [qn, kn]
    return ad, keep


def attention_step(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, cache_position: torch.Tensor,
                   keys: torch.Tensor, values: torch.Tensor, mask: torch.Tensor | None, q_norm_w=None, k_norm_w=None,
                   eps: float = 1e-6, out: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
    """One decode-attention step through bq_attention_step (see the header)."""
    dev = _require_cuda(qkv, cos, sin, cache_position, keys, values, mask, q_norm_w, k_norm_w, out)
    ad, keep = _attn_desc(qkv, cos, sin, cache_position, keys, values, mask, q_norm_w, k_norm_w, eps, flags)
    if out is None:
        out = torch.empty(ad.B, ad.HQ * ad.D, device=dev, dtype=torch.bfloat16)
    out = _rowmajor(out, "out")
    ad.out, ad.ldo = out.data_ptr(), out.stride(0)
    lib = load()
    need = ctypes.c_size_t(0)
    check(lib.bq_attention_workspace_bytes(ctypes.byref(ad), ctypes.byref(need)), "bq_attention_workspace_bytes")
    ws = ATTN_WORKSPACE.get(dev, need.value)
    check(lib.bq_attention_step(ctypes.byref(ad), ws.data_ptr(), ws.numel(), _stream(dev)), "bq_attention_step")
    del keep
    return out


def attention_o_step(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, cache_position: torch.Tensor,
                     keys: torch.Tensor, values: torch.Tensor, q_norm_w, k_norm_w, eps: float, wo: torch.Tensor,
                     residual: torch.Tensor, out: torch.Tensor | None = None, flags: int = 0,
                     mask: torch.Tensor | None = None) -> torch.Tensor:
    """The attention step fused with the output projection and residual add,
    through bq_attention_o_step: out = residual + attention_step(...) @ wo^T
    (wo bf16 [N, HQ D]); caches written as by attention_step; ``mask`` as
    attention_step takes it. Short caches only (see the header)."""
    dev = _require_cuda(qkv, cos, sin, cache_position, keys, values, q_norm_w, k_norm_w, wo, residual, out, mask)
    ad, keep = _attn_desc(qkv, cos, sin, cache_position, keys, values, mask, q_norm_w, k_norm_w, eps, flags)
    if wo.dtype != torch.bfloat16 or residual.dtype != torch.bfloat16:
        raise ValueError("wo and residual must be bf16")
    wo = _rowmajor(wo, "wo")
    residual = _rowmajor(residual, "residual")
    n = wo.shape[0]
    if out is None:
        out = torch.empty(ad.B, n, device=dev, dtype=torch.bfloat16)
    out = _rowmajor(out, "out")
    od = AttnODesc()
    od.attn = ad
    od.N = n
    od.wo, od.ldw = wo.data_ptr(), wo.stride(0)
    od.residual, od.ldr = residual.data_ptr(), residual.stride(0)
    od.out, od.ldo = out.data_ptr(), out.stride(0)
    lib = load()
    need = ctypes.c_size_t(0)
    check(lib.bq_attention_o_workspace_bytes(ctypes.byref(od), ctypes.byref(need)), "bq_attention_o_workspace_bytes")
    ws = ATTN_WORKSPACE.get(dev, need.value)
    check(lib.bq_attention_o_step(ctypes.byref(od), ws.data_ptr(), ws.numel(), _stream(dev)), "bq_attention_o_step")
    del keep
    return out


def head_gemv(x: torch.Tensor, w: torch.Tensor, layout: int, *, gamma: torch.Tensor | None = None, eps: float = 1e-6,
              out: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
    """fp32 output head through bq_head_gemv: out (M, N) fp32 = y @ W, with y = x
    or the reference's BreezeRMSNorm of x when gamma is given. layout HEAD_NK:
    w is an nn.Linear weight (N, K); HEAD_KN: w is one codebook slice (K, N)."""
    dev = _require_cuda(x, w, gamma, out)
    if w.dtype != torch.float32 or w.stride(1) != 1:
        raise ValueError("head weights must be fp32 with contiguous rows")
    x = _rowmajor(x, "x")
    m, k = x.shape
    n = w.shape[0] if layout == HEAD_NK else w.shape[1]
    if (w.shape[1] if layout == HEAD_NK else w.shape[0]) != k:
        raise ValueError(f"weight shape {tuple(w.shape)} does not match K={k}")
    if gamma is not None and (gamma.dtype != torch.bfloat16 or not gamma.is_contiguous()):
        raise ValueError("gamma must be a contiguous bf16 vector")
    if out is None:
        out = torch.empty(m, n, device=dev, dtype=torch.float32)
    out = _rowmajor(out, "out")
    d = HeadDesc()
    d.M, d.N, d.K, d.layout, d.x_dtype, d.flags, d.eps = m, n, k, layout, _DT[x.dtype], flags, eps
    d.x, d.ldx, d.gamma = x.data_ptr(), x.stride(0), _ptr(gamma)
    d.w, d.ldw, d.out, d.ldo = w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0)
    lib = load()
    need = ctypes.c_size_t(0)
    check(lib.bq_head_workspace_bytes(ctypes.byref(d), ctypes.byref(need)), "bq_head_workspace_bytes")
    ws = HEAD_WORKSPACE.get(dev, need.value) if need.value else None
    check(lib.bq_head_gemv(ctypes.byref(d), _ptr(ws), 0 if ws is None else ws.numel(), _stream(dev)), "bq_head_gemv")
    return out


def sample(logits: torch.Tensor, rows: int, *, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           do_sample: torch.Tensor, tokens: torch.Tensor, guidance: torch.Tensor | None = None, max_k: int | None = None,
           mask: tuple[int, int] = (0, 0), clamp_hi: int | None = None, topk_by_value: bool = False,
           rep_penalty: float = 1.0, history: torch.Tensor | None = None, history_len: torch.Tensor | None = None,
           suppress: torch.Tensor | None = None, uniform: torch.Tensor | None = None, rng: torch.Tensor | None = None,
           cfg_out: torch.Tensor | None = None, tokens2: torch.Tensor | None = None, append_history: bool = False,
           eos_id: int = -1, eos_flag: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
    """CFG mix + sampling through bq_sample (see the header). logits (rows or
    2 rows when guidance is given, V) fp32; per-row parameter buffers on the
    device; tokens (and tokens2) int64 with row stride given by stride(0)."""
    dev = _require_cuda(logits, temperature, top_k, top_p, do_sample, tokens, guidance, history, history_len,
                        suppress, uniform, rng, cfg_out, tokens2, eos_flag)
    if logits.dtype != torch.float32 or logits.stride(1) != 1:
        raise ValueError("logits must be fp32 with contiguous rows")
    v = logits.shape[1]
    cfg = guidance is not None
    if logits.shape[0] < (2 * rows if cfg else rows):
        raise ValueError("logits has too few rows")
    checks = ((temperature, torch.float32), (top_k, torch.int64), (top_p, torch.float32), (do_sample, torch.int64),
              (guidance, torch.float32), (uniform, torch.float32), (rng, torch.int64), (history, torch.int64),
              (history_len, torch.int32), (tokens, torch.int64), (tokens2, torch.int64))
    for t, dt in checks:
        if t is not None and t.dtype != dt:
            raise ValueError(f"sampling buffer of dtype {t.dtype}, expected {dt}")
    for t in (temperature, top_k, top_p, do_sample, guidance, uniform, rng, history_len, suppress):
        if t is not None and not t.is_contiguous():
            raise ValueError("per-row sampling buffers must be contiguous")
    d = SampleDesc()
    d.rows, d.V, d.cfg = rows, v, int(cfg)
    d.max_k = v if max_k is None else max_k
    d.mask_lo, d.mask_hi = mask
    d.clamp_hi = v - 1 if clamp_hi is None else clamp_hi
    d.flags = flags | (SAMPLE_TOPK_VALUE if topk_by_value else 0) | (SAMPLE_APPEND_HISTORY if append_history else 0)
    if eos_flag is not None and eos_flag.dtype != torch.int32:
        raise ValueError("eos_flag must be int32")
    d.eos_id, d.eos_flag = eos_id, _ptr(eos_flag)
    d.rep_penalty = rep_penalty
    d.logits, d.ldl = logits.data_ptr(), logits.stride(0)
    d.guidance, d.temperature, d.top_k, d.top_p = _ptr(guidance), temperature.data_ptr(), top_k.data_ptr(), top_p.data_ptr()
    d.do_sample = do_sample.data_ptr()
    if history is not None:
        if history.stride(1) != 1:
            raise ValueError("history rows must be contiguous")
        d.history, d.history_cap, d.history_len = history.data_ptr(), history.stride(0), _ptr(history_len)
    d.suppress, d.uniform, d.rng = _ptr(suppress), _ptr(uniform), _ptr(rng)
    if cfg_out is not None:
        d.cfg_out, d.ldc = cfg_out.data_ptr(), cfg_out.stride(0)
    d.tokens, d.ldt = tokens.data_ptr(), tokens.stride(0)
    if tokens2 is not None:
        d.tokens2, d.ldt2 = tokens2.data_ptr(), tokens2.stride(0)
    lib = load()
    need = ctypes.c_size_t(0)
    check(lib.bq_sample_workspace_bytes(ctypes.byref(d), ctypes.byref(need)), "bq_sample_workspace_bytes")
    ws = SAMPLE_WORKSPACE.get(dev, need.value)
    check(lib.bq_sample(ctypes.byref(d), ws.data_ptr(), ws.numel(), _stream(dev)), "bq_sample")
    return tokens


def embed_rows(table: torch.Tensor, ids: torch.Tensor, offset: int, out: torch.Tensor, flags: int = 0) -> torch.Tensor:
    """out[r] = table[clamp(ids[r] + offset, 0, rows - 1)] through bq_embed_rows
    (bf16 rows; ids int64, any row stride)."""
    dev = _require_cuda(table, ids, out)
    if table.dtype != torch.bfloat16 or out.dtype != torch.bfloat16 or ids.dtype != torch.int64:
        raise ValueError("embedding rows must be bf16 and ids int64")
    if table.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("embedding rows must be contiguous")
    n = out.shape[0]
    check(load().bq_embed_rows(table.data_ptr(), table.stride(0), table.shape[0], ids.data_ptr(), ids.stride(0), offset,
                               n, table.shape[1], out.data_ptr(), out.stride(0), flags, _stream(dev)), "bq_embed_rows")
    return out


def dequant(w: torch.Tensor, wfmt: int, n: int, k: int, *, scale=None, group: int = 128) -> torch.Tensor:
    """fp32 [N, K] dequantized weights, bit-exact with the reference."""
    dev = _require_cuda(w, scale)
    d = GemvDesc()
    d.N, d.K, d.wfmt, d.group = n, k, wfmt, group
    d.w, d.scale = w.data_ptr(), _ptr(scale)
    out = torch.empty(n, k, device=dev, dtype=torch.float32)
    check(load().bq_dequant(ctypes.byref(d), out.data_ptr(), _stream(dev)), "bq_dequant")
    return out


def tinygemm_pack(packed_u8: torch.Tensor, inner_k_tiles: int = 8) -> torch.Tensor:
    """(N, K/2) uint8 (odd k low) -> tinygemm int32 tiles, on the GPU."""
    dev = _require_cuda(packed_u8)
    packed_u8 = packed_u8.contiguous()
    n, kh = packed_u8.shape
    k = 2 * kh
    out = torch.empty(n // 8, k // (16 * inner_k_tiles), 32, inner_k_tiles // 2, device=dev, dtype=torch.int32)
    check(load().bq_int4_tinygemm_pack(packed_u8.data_ptr(), out.data_ptr(), n, k, inner_k_tiles, _stream(dev)),
          "bq_int4_tinygemm_pack")
    return out


def tinygemm_unpack(w: torch.Tensor) -> torch.Tensor:
    """tinygemm int32 tiles -> (N, K/2) uint8 (odd k low), on the GPU."""
    dev = _require_cuda(w)
    nt, kt, _, half = w.shape
    n, ikt = nt * 8, half * 2
    k = kt * 16 * ikt
    out = torch.empty(n, k // 2, device=dev, dtype=torch.uint8)
    check(load().bq_int4_tinygemm_unpack(w.contiguous().data_ptr(), out.data_ptr(), n, k, ikt, _stream(dev)),
          "bq_int4_tinygemm_unpack")
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out=None) -> torch.Tensor:
    dev = _require_cuda(x, w)
    m, k = x.shape
    if out is None:
        out = torch.empty_like(x)
    check(load().bq_rmsnorm(x.data_ptr(), x.stride(0), w.data_ptr(), out.data_ptr(), out.stride(0), m, k, eps,
                            _stream(dev)), "bq_rmsnorm")
    return out


def silu_mul(g: torch.Tensor, u: torch.Tensor, out=None) -> torch.Tensor:
    dev = _require_cuda(g, u)
    m, n = g.shape
    if out is None:
        out = torch.empty_like(g)
    check(load().bq_silu_mul(g.data_ptr(), g.stride(0), u.data_ptr(), u.stride(0), out.data_ptr(), out.stride(0),
                             m, n, _stream(dev)), "bq_silu_mul")
    return out


def device_status(device: int | None = None, clear: bool = False) -> int:
    """Device-side error bits (BQ_DEVERR_*) accumulated by the kernels."""
    lib = load()
    dev = torch.cuda.current_device() if device is None else device
    bits = ctypes.c_uint32(0)
    check(lib.bq_device_status(dev, ctypes.byref(bits)), "bq_device_status")
    if clear:
        check(lib.bq_device_status_clear(dev), "bq_device_status_clear")
    return bits.value
