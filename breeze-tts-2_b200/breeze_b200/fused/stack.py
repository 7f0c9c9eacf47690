"""The projection chain of a decode step, as one CUDA graph of bq_gemv launches.

Per decoder layer, in the order of the reference's FusedDecoderLayer.forward
(models/fused/layer.py:87-98):

    qkv = rms_gemv(x, Wqkv, ln1)                      # fused RMSNorm prologue
    h   = gemv(attn, Wo) + x                          # residual epilogue
    act = silu(gate) * up, [gate|up] = rms_gemv(h, Wgu, ln2)
    x'  = gemv(act, Wd) + h

then the output head ``logits = rms_gemv(x, Whead, ln_f)`` in fp32 (the
reference keeps its output heads in fp32, cudagraph/backbone_graph.py:70).
``attn`` is the attention output: with ``attention=True`` each layer runs the
decode attention step (bq_attention_step: q/k RMSNorm, RoPE, KV-cache write,
flash-decode over the cache) between QKV and O, as FusedDecoderLayer does
(layer.py:89-90); otherwise the first ``attn_cols`` columns of ``qkv`` (the
query block) stand in for it, which keeps the QKV -> O data dependency.

Every projection is one bq_gemv launch (int4 tinygemm / plain, fp8 or int8
weight-only, bf16), launched with programmatic dependent launch so each
kernel's weight prefetch overlaps the previous kernel. The whole chain is
captured once and replayed; static buffers hold every intermediate.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _lib


@dataclass
class QWeight:
    """A quantized (or bf16) weight in one of the bq_gemv formats.

    w / scale follow the reference's buffers: Int4Linear ``weight_int4`` and
    ``scales_zeros`` [K/g, N, 2]; Fp8Linear ``weight_fp8`` and ``weight_scale``;
    Int8Linear ``weight_int8`` and ``weight_scale``; FusedWeight ``w`` and its
    scale/min pair.
    """

    wfmt: int
    w: torch.Tensor
    scale: torch.Tensor | None
    N: int
    K: int
    group: int = 128

    @property
    def nbytes(self) -> int:
        b = self.w.numel() * self.w.element_size()
        if self.scale is not None:
            b += self.scale.numel() * self.scale.element_size()
        return b

    @classmethod
    def from_module(cls, mod) -> "QWeight":
        """Adopt the buffers of an Int4Linear / Fp8Linear / Int8Linear."""
        name = type(mod).__name__
        if name == "Int4Linear":
            return cls(_lib.W_INT4_TINYGEMM, mod.weight_int4, mod.scales_zeros, mod.out_features, mod.in_features,
                       mod.group_size)
        if name == "Fp8Linear":
            return cls(_lib.W_FP8_E4M3, mod.weight_fp8, mod.weight_scale.reshape(-1).float().contiguous(),
                       mod.out_features, mod.in_features)
        if name == "Int8Linear":
            if mod.bias is not None:
                raise ValueError("DecodeStack projections carry no bias")
            return cls(_lib.W_INT8, mod.weight_int8, mod.weight_scale.reshape(-1).float().contiguous(),
                       mod.out_features, mod.in_features)
        raise TypeError(f"cannot adopt a {name}")

    @classmethod
    def from_fused(cls, fw) -> "QWeight":
        """Adopt a FusedWeight (bits 16 / 8 / 4)."""
        a = fw.gemv_args()
        return cls(a["wfmt"], fw.w, a["scale"], fw.N, fw.K)


def synthetic_weight(fmt: str, n: int, k: int, device, gen: torch.Generator, group: int = 128) -> QWeight:
    """Seeded random weight for the decode-stack benchmark, generated on
    ``device``: int4 codes uniform 0..15 (tinygemm tiles) with bf16 scales
    |N(0, 0.02)| / 7 and zero point 8; fp8 codes from N(0, 64) clamped to
    +-448 (the spread of a row scaled by absmax / 448) with per-row fp32
    scales; int8 codes uniform in -127..127 with per-row fp32 scales."""
    if fmt == "int4":
        # tinygemm tiles: every nibble of the int32 words is one code
        w = torch.randint(-(2 ** 31), 2 ** 31 - 1, (n // 8, k // 128, 32, 4), device=device, generator=gen,
                          dtype=torch.int64).to(torch.int32)
        s = (torch.randn(k // group, n, device=device, generator=gen).abs() * 0.02 / 7).to(torch.bfloat16)
        sz = torch.stack([s, torch.zeros_like(s)], dim=-1).contiguous()
        return QWeight(_lib.W_INT4_TINYGEMM, w, sz, n, k, group)
    if fmt == "fp8":
        q = (torch.randn(n, k, device=device, generator=gen, dtype=torch.bfloat16) * 64).clamp(-448, 448)
        q = q.to(torch.float8_e4m3fn)
        scale = torch.rand(n, device=device, generator=gen) * (0.08 / 448) + 1e-6
        return QWeight(_lib.W_FP8_E4M3, q, scale, n, k)
    if fmt == "int8":
        q = torch.randint(-127, 128, (n, k), device=device, generator=gen, dtype=torch.int8)
        scale = torch.rand(n, device=device, generator=gen) * (0.08 / 127) + 1e-6
        return QWeight(_lib.W_INT8, q, scale, n, k)
    if fmt == "bf16":
        w = (torch.randn(n, k, device=device, generator=gen) * 0.02).to(torch.bfloat16)
        return QWeight(_lib.W_BF16, w, None, n, k)
    raise ValueError(f"unknown format {fmt!r}")


@dataclass
class DecodeLayer:
    wqkv: QWeight
    wo: QWeight
    wgu: QWeight
    wd: QWeight
    ln1: torch.Tensor
    ln2: torch.Tensor
    q_norm: torch.Tensor | None = None  # per-head RMSNorm weights (head_dim), as Qwen3 attention
    k_norm: torch.Tensor | None = None


def synthetic_stack(fmt: str, n_layers: int, device, seed: int = 0, hidden: int = 2048, qkv: int = 6144,
                    inter: int = 8192, head: int = 8192):
    """Layers of the decode-stack benchmark: QKV hidden->qkv, O hidden->hidden,
    gate+up hidden->2*inter, down inter->hidden, plus the output head."""
    gen = torch.Generator(device=device).manual_seed(seed)

    def norm_w(n=hidden):
        return (1 + 0.1 * torch.randn(n, device=device, generator=gen)).to(torch.bfloat16)

    layers = []
    for _ in range(n_layers):
        layers.append(DecodeLayer(synthetic_weight(fmt, qkv, hidden, device, gen),
                                  synthetic_weight(fmt, hidden, hidden, device, gen),
                                  synthetic_weight(fmt, 2 * inter, hidden, device, gen),
                                  synthetic_weight(fmt, hidden, inter, device, gen), norm_w(), norm_w(),
                                  norm_w(128), norm_w(128)))
    return layers, synthetic_weight(fmt, head, hidden, device, gen), norm_w()


class DecodeStack:
    """Static-buffer decode step over ``layers`` plus an output head.

    ``x`` (rows, hidden) bf16 is the input of the step, ``logits`` (rows,
    head N) fp32 its output. ``run()`` enqueues the launches on the current
    stream; ``capture()`` records them into a CUDA graph that ``replay()``
    launches.
    """

    def __init__(self, layers: list[DecodeLayer], head: QWeight | None, ln_f: torch.Tensor, rows: int,
                 eps: float = 1e-6, attn_cols: int | None = None, chain: bool = False, attention: bool = False,
                 head_dim: int = 128, kv_heads: int | None = None, kv_len: int = 256,
                 lm_head: torch.Tensor | None = None, sampling: dict | None = None):
        """``lm_head``: an fp32 nn.Linear weight (V, hidden) used instead of the
        quantized ``head``, as the backbone graph casts lm_head to fp32
        (backbone_graph.py:70, 272-273). ``sampling`` (needs ``lm_head``):
        the token is drawn in the graph (bq_sample) instead of on the host
        after a copy (fast_streaming.py:929-939): keys temperature, top_k,
        top_p, do_sample, guidance_scale (CFG when rows >= 2: cond rows, then
        uncond rows), repetition_penalty, history_cap, suppress (lo, hi),
        eos_id, seed. Each step first appends the current token to the
        history, then draws; ``eos_flag`` becomes 1 when EOS is drawn."""
        if not layers:
            raise ValueError("DecodeStack needs at least one layer")
        if head is None and lm_head is None:
            raise ValueError("DecodeStack needs a head or an fp32 lm_head")
        if sampling is not None and lm_head is None:
            raise ValueError("in-graph sampling needs the fp32 lm_head")
        if lm_head is not None and chain:
            raise ValueError("the decode chain runs GEMVs only; lm_head needs chain=False")
        dev = layers[0].wqkv.w.device
        hidden = layers[0].wqkv.K
        for i, l in enumerate(layers):
            if l.wqkv.K != hidden or l.wo.N != hidden or l.wgu.K != hidden or l.wd.N != hidden:
                raise ValueError(f"layer {i}: projections do not match hidden size {hidden}")
            if l.wgu.N != 2 * l.wd.K or l.wgu.N % 2:
                raise ValueError(f"layer {i}: gate+up N={l.wgu.N} does not match down K={l.wd.K}")
        if head is not None and head.K != hidden:
            raise ValueError("head K does not match the hidden size")
        if lm_head is not None and (lm_head.dtype != torch.float32 or lm_head.dim() != 2 or lm_head.shape[1] != hidden):
            raise ValueError("lm_head must be fp32 (V, hidden)")
        self.layers, self.head, self.ln_f = layers, head, ln_f
        self.rows, self.eps, self.hidden = rows, eps, hidden
        self.attn_cols = attn_cols or hidden
        if self.attn_cols != layers[0].wo.K or self.attn_cols > layers[0].wqkv.N:
            raise ValueError("attention width must equal O's K and fit inside QKV's N")
        bf = dict(device=dev, dtype=torch.bfloat16)
        self.x = torch.zeros(rows, hidden, **bf)
        self.qkv = torch.zeros(rows, max(l.wqkv.N for l in layers), **bf)
        self.h = torch.zeros(rows, hidden, **bf)
        self.act = torch.zeros(rows, max(l.wd.K for l in layers), **bf)
        self.res = [torch.zeros(rows, hidden, **bf), torch.zeros(rows, hidden, **bf)]
        self.lm_head = lm_head
        self.logits = torch.zeros(rows, lm_head.shape[0] if lm_head is not None else head.N, device=dev,
                                  dtype=torch.float32)
        self.sampling = None
        if sampling is not None:
            sp = dict(temperature=0.9, top_k=50, top_p=0.95, do_sample=True, guidance_scale=3.0,
                      repetition_penalty=1.1, history_cap=2048, suppress=(0, 0), eos_id=-1, seed=0)
            unknown = set(sampling) - set(sp)
            if unknown:
                raise ValueError(f"unknown sampling keys {sorted(unknown)}")
            sp.update(sampling)
            half = rows // 2 if rows >= 2 else rows
            f = lambda v, dt: torch.full((half,), v, device=dev, dtype=dt)  # noqa: E731
            self.sampling = sp
            self.half, self.cfg = half, rows >= 2
            self.temperature_buf = f(sp["temperature"], torch.float32)
            self.top_k_buf = f(sp["top_k"], torch.int64)
            self.top_p_buf = f(sp["top_p"], torch.float32)
            self.do_sample_buf = f(1 if sp["do_sample"] else 0, torch.int64)
            self.guidance_scale = f(sp["guidance_scale"], torch.float32)
            self.history = torch.zeros(half, sp["history_cap"], device=dev, dtype=torch.int64)
            self.history_len = torch.zeros(half, device=dev, dtype=torch.int32)
            self.token = torch.zeros(rows, device=dev, dtype=torch.int64)
            self.eos_flag = torch.zeros(1, device=dev, dtype=torch.int32)
            self.rng = torch.tensor([sp["seed"], 0], device=dev, dtype=torch.int64)
        self.graph = None
        self.chain = None
        self.attention = attention
        if attention:
            if chain:
                raise ValueError("the decode chain runs GEMVs only; attention=True needs chain=False")
            hq = self.attn_cols // head_dim
            hkv = kv_heads or (layers[0].wqkv.N // head_dim - hq) // 2
            if (hq + 2 * hkv) * head_dim != layers[0].wqkv.N:
                raise ValueError("QKV width does not split into q / k / v heads of head_dim")
            self.hq, self.hkv, self.head_dim, self.kv_len = hq, hkv, head_dim, kv_len
            cache = dict(device=dev, dtype=torch.bfloat16)
            self.k_cache = [torch.zeros(rows, hkv, kv_len, head_dim, **cache) for _ in layers]
            self.v_cache = [torch.zeros(rows, hkv, kv_len, head_dim, **cache) for _ in layers]
            self.cos = torch.ones(rows, 1, head_dim, **cache)
            self.sin = torch.zeros(rows, 1, head_dim, **cache)
            self.pos = torch.full((1,), kv_len - 1, device=dev, dtype=torch.int64)  # attend over the whole cache
            self.attn_out = torch.zeros(rows, hq * head_dim, **bf)
        if chain:
            descs = [_lib.gemv_desc(x, qw.w, qw.wfmt, qw.N, out=out, scale=qw.scale, group=qw.group, gamma=g,
                                    eps=eps, epilogue=epi, residual=res, flags=_lib.default_flags())
                     for x, qw, out, g, epi, res in self._ops()]
            self.chain = _lib.GemvChain(descs, dev)

    @property
    def weight_bytes(self) -> int:
        b = (self.head.nbytes if self.lm_head is None else self.lm_head.numel() * 4) + self.ln_f.numel() * 2
        for l in self.layers:
            b += l.wqkv.nbytes + l.wo.nbytes + l.wgu.nbytes + l.wd.nbytes + 2 * l.ln1.numel() * 2
        return b

    @property
    def kv_bytes(self) -> int:
        """KV-cache bytes the attention steps read per decode step."""
        if not self.attention:
            return 0
        return len(self.layers) * 2 * self.rows * self.hkv * (int(self.pos.item()) + 1) * self.head_dim * 2

    @property
    def launches(self) -> int:
        if self.chain is not None:
            return 1
        return (5 if self.attention else 4) * len(self.layers) + 1 + (1 if self.sampling is not None else 0)

    def _ops(self):
        """(x, weight, out, gamma, epilogue, residual) of every launch, in order."""
        ops = []
        x = self.x
        for i, l in enumerate(self.layers):
            qkv = self.qkv[:, : l.wqkv.N]
            ops.append((x, l.wqkv, qkv, l.ln1, _lib.EPI_NONE, None))
            ops.append((qkv[:, : self.attn_cols], l.wo, self.h, None, _lib.EPI_ADD_RESIDUAL, x))
            act = self.act[:, : l.wd.K]
            ops.append((self.h, l.wgu, act, l.ln2, _lib.EPI_SILU_MUL, None))
            y = self.res[i % 2]
            ops.append((act, l.wd, y, None, _lib.EPI_ADD_RESIDUAL, self.h))
            x = y
        if self.lm_head is None:
            ops.append((x, self.head, self.logits, self.ln_f, _lib.EPI_NONE, None))
        else:
            self._final = x
        return ops

    def run(self) -> torch.Tensor:
        """Enqueue the step: one bq_gemv launch per projection (and one
        bq_attention_step per layer with ``attention=True``), or the whole
        step as one decode-chain launch (``chain=True``)."""
        if self.chain is not None:
            self.chain.launch()
            return self.logits
        ops = self._ops()
        for k, (x, qw, out, gamma, epi, res) in enumerate(ops):
            if self.attention and k % 4 == 1 and k < 4 * len(self.layers):
                li = k // 4
                l = self.layers[li]
                _lib.attention_step(self.qkv[:, : l.wqkv.N], self.cos, self.sin, self.pos, self.k_cache[li],
                                    self.v_cache[li], None, l.q_norm, l.k_norm, self.eps, out=self.attn_out,
                                    flags=_lib.default_flags())
                x = self.attn_out
            _lib.gemv(x, qw.w, qw.wfmt, qw.N, scale=qw.scale, group=qw.group, gamma=gamma, eps=self.eps,
                      epilogue=epi, residual=res, out=out, flags=_lib.default_flags())
        if self.lm_head is not None:
            _lib.head_gemv(self._final, self.lm_head, _lib.HEAD_NK, gamma=self.ln_f, eps=self.eps, out=self.logits,
                           flags=_lib.default_flags())
        if self.sampling is not None:
            sp = self.sampling
            _lib.sample(self.logits, self.half, temperature=self.temperature_buf, top_k=self.top_k_buf,
                        top_p=self.top_p_buf, do_sample=self.do_sample_buf, tokens=self.token,
                        guidance=self.guidance_scale if self.cfg else None, max_k=self.logits.shape[1],
                        mask=sp["suppress"], topk_by_value=True, rep_penalty=sp["repetition_penalty"],
                        history=self.history, history_len=self.history_len, append_history=True, rng=self.rng,
                        eos_id=sp["eos_id"], eos_flag=self.eos_flag, flags=_lib.default_flags())
        return self.logits

    def capture(self) -> None:
        """Warm up once (sizes the shared workspace), then record the step."""
        self.run()
        torch.cuda.synchronize()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                self.run()
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        self.graph = g

    def replay(self) -> None:
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()
