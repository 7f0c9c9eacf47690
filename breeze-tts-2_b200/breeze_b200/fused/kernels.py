"""Fused decode GEMV API, drop-in for models/fused/kernels.py.

rms_gemv: out = epilogue( rmsnorm(x) @ W^T )
  W is bf16 (N, K); int4 (N, K/2) packed with per-group scale/min; or fp8
  e4m3 (N, K) with a per-row scale -- the reference's FusedWeight formats
  (models/fused/kernels.py:141-176). epilogue 0: none; 1: silu(gate) * up
  over a [gate | up] weight, output N/2; 2: add residual.

The reference runs two Triton kernels per call (split-K partial GEMV, then
an epilogue kernel) chosen by a per-GPU autotuner. Here each call is one
sm_100a kernel (bq_gemv): the norm prologue, the dequantization, the
split-K reduction and the epilogue all happen in that launch, and the
launch shape is computed from the device, so there is nothing to tune.
"""

from __future__ import annotations

import torch

from .. import _lib

GROUP = 128


def pack_int4(weight: torch.Tensor, group: int = GROUP):
    """(N, K) float -> packed (N, K/2) uint8, scale (N, K/group) bf16,
    min (N, K/group) bf16; w ~= q * scale + min, even k in the low nibble
    (models/fused/kernels.py:141-150)."""
    n, k = weight.shape
    g = weight.float().reshape(n, k // group, group)
    lo = g.amin(-1, keepdim=True)
    scale = ((g.amax(-1, keepdim=True) - lo) / 15).clamp_min(1e-8)
    q = ((g - lo) / scale).round().clamp(0, 15).to(torch.uint8).reshape(n, k)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()
    return (packed, scale.squeeze(-1).to(torch.bfloat16).contiguous(),
            lo.squeeze(-1).to(torch.bfloat16).contiguous())


def pack_fp8(weight: torch.Tensor):
    """(N, K) float -> fp8 e4m3 (N, K) with a per-row fp32 scale
    (models/fused/kernels.py:153-158)."""
    amax = weight.float().abs().amax(-1, keepdim=True).clamp_min(1e-8)
    scale = amax / 448.0
    q = (weight.float() / scale).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.contiguous(), scale.squeeze(-1).float().contiguous()


class FusedWeight:
    """A weight in one of the three formats, ready for rms_gemv.

    Attributes follow the reference (bits, N, K, w, s, z). For bits=4 the
    kernel reads scale and min interleaved per group as ``sz`` [K/128, N, 2]
    bf16; ``s`` and ``z`` are (N, K/128) views of it.
    """

    def __init__(self, weight: torch.Tensor, bits: int = 16):
        self.bits = bits
        self.N, self.K = weight.shape
        self.sz = None
        if bits == 16:
            self.w = weight.to(torch.bfloat16).contiguous()
            self._s = None
        elif bits == 8:
            self.w, self._s = pack_fp8(weight)
        elif bits == 4:
            self.w, s, z = pack_int4(weight)
            self.sz = torch.stack([s.t(), z.t()], dim=-1).contiguous()
            self._s = None
        else:
            raise ValueError(bits)

    @classmethod
    def from_parts(cls, bits: int, w: torch.Tensor, s: torch.Tensor | None = None, z: torch.Tensor | None = None):
        """Adopt already-packed tensors (e.g. Fp8Linear buffers, as the
        reference's models/fused/layer.py:20-29 does)."""
        fw = cls.__new__(cls)
        fw.bits, fw.w = bits, w.contiguous()
        fw.N = w.shape[0]
        fw.K = w.shape[1] * (2 if bits == 4 else 1)
        fw._s, fw.sz = None, None
        if bits == 8:
            fw._s = s.reshape(-1).float().contiguous()
        elif bits == 4:
            fw.sz = torch.stack([s.t(), z.t()], dim=-1).to(torch.bfloat16).contiguous()
        return fw

    @property
    def s(self):
        return self.sz[..., 0].t() if self.bits == 4 else self._s

    @property
    def z(self):
        return self.sz[..., 1].t() if self.bits == 4 else None

    def clone(self) -> "FusedWeight":
        c = FusedWeight.__new__(FusedWeight)
        c.bits, c.N, c.K = self.bits, self.N, self.K
        c.w = self.w.clone()
        c._s = None if self._s is None else self._s.clone()
        c.sz = None if self.sz is None else self.sz.clone()
        return c

    def gemv_args(self) -> dict:
        if self.bits == 16:
            return {"wfmt": _lib.W_BF16, "scale": None}
        if self.bits == 8:
            return {"wfmt": _lib.W_FP8_E4M3, "scale": self._s}
        return {"wfmt": _lib.W_INT4_PLAIN, "scale": self.sz}


def rms_gemv(x, fw: FusedWeight, norm_weight=None, eps: float = 1e-6, epilogue: int = 0, residual=None, out=None):
    """out = epilogue(rmsnorm(x) @ W^T) in one bq_gemv launch.

    Same signature and output dtype rule as models/fused/kernels.py:334-351
    (bf16, or residual.dtype when a residual is given). Any M works; the
    reference's Triton kernel is limited to M <= 2.
    """
    m, k = x.shape
    if k != fw.K:
        raise ValueError(f"x has K={k}, weight has K={fw.K}")
    a = fw.gemv_args()
    return _lib.gemv(x, fw.w, a["wfmt"], fw.N, scale=a["scale"], group=GROUP, gamma=norm_weight, eps=eps,
                     epilogue=epilogue, residual=residual, out=out,
                     out_dtype=torch.bfloat16 if residual is None else residual.dtype, flags=_lib.default_flags())


def rms_gemv_host_io(x_host, fw: FusedWeight, norm_weight=None, eps: float = 1e-6, epilogue: int = 0, residual=None,
                     *, x, out, out_host):
    """rms_gemv on host data in one call: x_host (dense CPU, pinned for an
    asynchronous copy) is copied into the device buffer ``x``, the GEMV writes
    ``out``, and ``out`` is copied into ``out_host``; everything is enqueued on
    the current stream (bq_gemv_host_io). Returns out_host, valid once the
    stream reaches it."""
    if x.shape[1] != fw.K:
        raise ValueError(f"x has K={x.shape[1]}, weight has K={fw.K}")
    a = fw.gemv_args()
    return _lib.gemv_host_io(x_host, x, fw.w, a["wfmt"], fw.N, out=out, out_host=out_host, scale=a["scale"],
                             group=GROUP, gamma=norm_weight, eps=eps, epilogue=epilogue, residual=residual,
                             flags=_lib.default_flags())


def attention_step(qkv, cos, sin, cache_position, keys, values, mask, q_norm_w=None, k_norm_w=None, eps=1e-6,
                   out=None, q_buf=None):  # noqa: ARG001 - q_buf: API parity (the kernel keeps q on chip)
    """qkv (B, (HQ+2HKV)*D) bf16 -> attention output (B, HQ*D) bf16, with the
    new k/v written into the static cache (B, HKV, S, D); same signature as
    models/fused/kernels.py:505-536. One bq_attention_step launch replaces the
    reference's three Triton kernels."""
    return _lib.attention_step(qkv, cos, sin, cache_position, keys, values, mask, q_norm_w, k_norm_w, eps, out,
                               flags=_lib.default_flags())


def rmsnorm(x, w, eps=1e-6, out=None):
    """Standalone RMSNorm (models/fused/kernels.py:552-557)."""
    return _lib.rmsnorm(x, w, eps, out)


def silu_mul(g, u, out=None):
    """silu(g) * u (models/fused/kernels.py:570-575)."""
    return _lib.silu_mul(g, u, out)


def load_tuning(device) -> None:  # noqa: ARG001 - API parity: launch shapes need no tuning
    """No-op: bq_gemv derives its launch shape from the device."""


def graph_time_us(fn, iters: int = 20, replays: int = 7) -> float:
    """Device time per call of ``fn`` in microseconds, the way the decode
    graphs pay for it: ``iters`` calls are recorded into one CUDA graph, the
    graph is replayed ``replays`` times with CUDA events around each replay,
    and the median replay is divided by ``iters``. Same name, arguments and
    unit as the reference's helper (models/fused/kernels.py:222-243)."""
    fn()  # outside capture: workspaces reach their size, descriptors are cached
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
        for _ in range(iters):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(replays + 1)]
    marks[0].record()
    for i in range(replays):
        graph.replay()
        marks[i + 1].record()
    torch.cuda.synchronize()
    per_replay = sorted(a.elapsed_time(b) for a, b in zip(marks, marks[1:]))
    return per_replay[len(per_replay) // 2] * 1e3 / iters


def cold_copies(fw: FusedWeight, budget_bytes: int | None = None) -> list:
    """Copies of a weight to rotate through so timing streams from DRAM.
    The budget defaults to 4x this device's L2 (the reference's fixed
    160 MB is below B200's 126 MB L2 plus headroom)."""
    if budget_bytes is None:
        l2 = torch.cuda.get_device_properties(fw.w.device).L2_cache_size
        budget_bytes = 4 * l2
    nbytes = fw.w.numel() * fw.w.element_size()
    n = max(2, min(64, budget_bytes // max(nbytes, 1)))
    return [fw.clone() for _ in range(n)]
