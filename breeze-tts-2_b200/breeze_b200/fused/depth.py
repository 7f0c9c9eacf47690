"""One frame of the depth decoder as one CUDA graph of breeze_b200 kernels.

Follows DepthDecoderGraph._full_loop (models/cudagraph/depth_decoder_graph.py:
560-660) on static buffers:

  prefill (positions 0 and 1, one pass over the layers with 2B rows):
      e[0:B]  = backbone hidden (projected by backbone_hidden_state_projector
                when its width differs from the audio embedding, :569-576)
      e[B:2B] = embed_tokens[first codebook token]                  (:563-567)
      x = inputs_embeds_projector(e)                                (:578)
      layers (attention: rows [0:B] at position 0, rows [B:2B] at 1)
      logits = codebooks_head(norm(x[B:2B]), codebook 0), fp32     (:594-603)
      token = cfg_sample(logits); output_tokens[:, 0] = token       (:608-614)
  steps j = 1 .. n-1 (position j + 1):                              (:617-660)
      e = embed_tokens[clamp(token + j * vocab)]; x = inputs_embeds_projector(e)
      layers; logits = codebooks_head(norm(x), codebook j); sample.

Kernels per frame: bq_embed_rows, bq_gemv (every projection, RMSNorm and
SiLU / residual epilogues fused), bq_attention_step, bq_head_gemv (the fp32
codebook head with the final norm fused) and bq_sample (CFG mix, codec-token
mask, temperature / top-k / top-p, Philox draw, token written to the feedback
buffer and to output_tokens), all launched with programmatic dependent launch
and captured once. Sampling parameters live in device buffers, so they change
between replays without a recapture, as in the reference (:240-290).
"""

from __future__ import annotations

import torch

from .. import _lib
from .stack import DecodeLayer, QWeight


def rope_table(positions: int, head_dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin (positions, head_dim) bf16 of the default rotary embedding:
    inv_freq = theta^(-2i/D), angles duplicated over both halves, computed in
    fp32 and cast to the activation dtype."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    ang = torch.arange(positions, dtype=torch.float32)[:, None] * inv[None, :]
    emb = torch.cat([ang, ang], dim=-1)
    return emb.cos().to(torch.bfloat16).to(device), emb.sin().to(torch.bfloat16).to(device)


class DepthDecoderLoop:
    """Static-buffer depth-decoder frame (see the module docstring).

    ``batch_size`` is 1 (no CFG) or 2 * half (cond rows, then uncond rows),
    as in the reference. Inputs: ``backbone_hidden_buf`` (B, backbone width)
    bf16 and ``first_cb_token_buf`` (B,) int64. Output: ``output_tokens``
    (B, num_decode_codebooks) int64; ``step_logits`` keeps every step's fp32
    logits (B, vocab). With ``fuse_attention_o`` (default) the single-position
    steps run attention, O projection and residual add as one launch
    (bq_attention_o_step) when the O weight is bf16; the two-position prefill
    keeps the separate launches."""

    def __init__(self, layers: list[DecodeLayer], norm_w: torch.Tensor, codebooks_head: torch.Tensor,
                 embed: torch.Tensor, in_proj: QWeight, batch_size: int, *, codebook_size: int,
                 num_decode_codebooks: int | None = None, bb_proj: QWeight | None = None, head_dim: int = 128,
                 kv_heads: int | None = None, rope_theta: float = 10000.0, max_k: int = 1024, eps: float = 1e-6,
                 temperature: float = 0.9, top_k: int = 50, top_p: float = 0.95, do_sample: bool = True,
                 guidance_scale: float = 3.0, seed: int = 0, fuse_attention_o: bool = True):
        if not layers:
            raise ValueError("the depth loop needs at least one layer")
        dev = layers[0].wqkv.w.device
        hidden = layers[0].wqkv.K
        ncb1, h2, vocab = codebooks_head.shape
        if h2 != hidden or codebooks_head.dtype != torch.float32:
            raise ValueError("codebooks_head must be fp32 (num_codebooks - 1, hidden, vocab)")
        n_dec = num_decode_codebooks or ncb1
        if n_dec > ncb1:
            raise ValueError(f"{n_dec} decode codebooks but the head has {ncb1} slices")
        emb_w = embed.shape[1]
        if in_proj.K != emb_w or in_proj.N != hidden:
            raise ValueError("inputs_embeds_projector must map the embedding width to the hidden size")
        bb_w = bb_proj.K if bb_proj is not None else emb_w
        if bb_proj is not None and bb_proj.N != emb_w:
            raise ValueError("backbone_hidden_state_projector must map to the embedding width")
        for i, l in enumerate(layers):
            if l.wqkv.K != hidden or l.wo.N != hidden or l.wgu.K != hidden or l.wd.N != hidden:
                raise ValueError(f"layer {i}: projections do not match hidden size {hidden}")
        self.layers, self.norm_w, self.head_w, self.embed = layers, norm_w, codebooks_head, embed
        self.in_proj, self.bb_proj = in_proj, bb_proj
        self.B, self.vocab, self.n_dec, self.eps = batch_size, vocab, n_dec, eps
        self.half = batch_size // 2 if batch_size >= 2 else batch_size
        self.cfg = batch_size >= 2
        self.codebook_size, self.max_k = codebook_size, min(max_k, vocab)
        self.hq = layers[0].wo.K // head_dim
        self.hkv = kv_heads or (layers[0].wqkv.N // head_dim - self.hq) // 2
        if (self.hq + 2 * self.hkv) * head_dim != layers[0].wqkv.N:
            raise ValueError("QKV width does not split into q / k / v heads of head_dim")
        self.head_dim = head_dim
        B = batch_size
        bf = dict(device=dev, dtype=torch.bfloat16)
        # embedding rows: [0:B] position 0 (backbone hidden), [B:2B] position 1, [2B:3B] decode steps
        self.emb = torch.zeros(3 * B, emb_w, **bf)
        self.backbone_hidden_buf = torch.zeros(B, bb_w, **bf) if bb_proj is not None else self.emb[0:B]
        self.first_cb_token_buf = torch.zeros(B, device=dev, dtype=torch.int64)
        self.output_tokens = torch.zeros(B, n_dec, device=dev, dtype=torch.int64)
        self.tok_buf = torch.zeros(B, device=dev, dtype=torch.int64)
        rows2 = 2 * B
        self.x = torch.zeros(rows2, hidden, **bf)
        self.qkv = torch.zeros(rows2, max(l.wqkv.N for l in layers), **bf)
        self.attn_out = torch.zeros(rows2, self.hq * head_dim, **bf)
        self.h = torch.zeros(rows2, hidden, **bf)
        self.act = torch.zeros(rows2, max(l.wd.K for l in layers), **bf)
        self.res = [torch.zeros(rows2, hidden, **bf), torch.zeros(rows2, hidden, **bf)]
        self.step_logits = torch.zeros(n_dec, B, vocab, device=dev, dtype=torch.float32)
        s = 2 + n_dec
        self.kv_len = s
        self.k_cache = [torch.zeros(B, self.hkv, s, head_dim, **bf) for _ in layers]
        self.v_cache = [torch.zeros(B, self.hkv, s, head_dim, **bf) for _ in layers]
        self.cos, self.sin = rope_table(s, head_dim, rope_theta, dev)
        self.pos = [torch.full((1,), p, device=dev, dtype=torch.int64) for p in range(s)]
        f = lambda v, dt: torch.full((self.half,), v, device=dev, dtype=dt)  # noqa: E731
        self.temperature_buf = f(temperature, torch.float32)
        self.top_k_buf = f(top_k, torch.int64)
        self.top_p_buf = f(top_p, torch.float32)
        self.do_sample_buf = f(1 if do_sample else 0, torch.int64)
        self.guidance_scale = f(guidance_scale, torch.float32)
        self.rng = torch.tensor([seed, 0], device=dev, dtype=torch.int64)
        self.fuse_attention_o = fuse_attention_o
        self.graph = None

    # ---- setters (device buffers: no recapture), as the reference's set_* (:240-290)
    def set_temperature(self, v: float) -> None:
        self.temperature_buf.fill_(v)

    def set_top_k(self, v: int) -> None:
        if v > self.max_k:
            raise ValueError(f"top_k={v} exceeds max_k={self.max_k}")
        self.top_k_buf.fill_(v)

    def set_top_p(self, v: float) -> None:
        self.top_p_buf.fill_(v)

    def set_do_sample(self, v: bool) -> None:
        self.do_sample_buf.fill_(1 if v else 0)

    def set_guidance_scale(self, v: float) -> None:
        self.guidance_scale.fill_(v)

    @property
    def launches(self) -> int:
        n_l = len(self.layers)
        pre = 1 + (1 if self.bb_proj is not None else 0) + 1 + 6 * n_l + 2
        per_layer = 4 if any(self._fused_o(l, [(0, 0, 0)]) for l in self.layers[:1]) else 5
        return pre + (self.n_dec - 1) * (2 + per_layer * n_l + 2)

    @property
    def weight_bytes_per_frame(self) -> int:
        """Weight bytes the frame streams (layers and input projection once per
        step, one head slice per step)."""
        per = self.in_proj.nbytes + sum(l.wqkv.nbytes + l.wo.nbytes + l.wgu.nbytes + l.wd.nbytes for l in self.layers)
        head = self.head_w[0].numel() * 4
        return self.n_dec * (per + head) + (self.bb_proj.nbytes if self.bb_proj is not None else 0)

    def _gemv(self, x, qw: QWeight, out, gamma=None, epi=_lib.EPI_NONE, res=None):
        _lib.gemv(x, qw.w, qw.wfmt, qw.N, scale=qw.scale, group=qw.group, gamma=gamma, eps=self.eps, epilogue=epi,
                  residual=res, out=out, flags=_lib.default_flags())

    def _fused_o(self, l, positions) -> bool:
        return self.fuse_attention_o and len(positions) == 1 and l.wo.wfmt == _lib.W_BF16

    def _layers(self, r0: int, r1: int, positions: list[tuple[int, int, int]]) -> torch.Tensor:
        """Layer pass over rows [r0, r1) of the work buffers; positions lists
        (row offset, row count, cache position) blocks for attention."""
        x = self.x[r0:r1]
        for i, l in enumerate(self.layers):
            qkv = self.qkv[r0:r1, : l.wqkv.N]
            self._gemv(x, l.wqkv, qkv, gamma=l.ln1)
            h = self.h[r0:r1]
            if self._fused_o(l, positions):
                p = positions[0][2]
                _lib.attention_o_step(qkv, self.cos[p:p + 1], self.sin[p:p + 1], self.pos[p], self.k_cache[i],
                                      self.v_cache[i], l.q_norm, l.k_norm, self.eps, l.wo.w, x, out=h,
                                      flags=_lib.default_flags())
            else:
                for off, n, p in positions:
                    _lib.attention_step(self.qkv[off:off + n, : l.wqkv.N], self.cos[p:p + 1], self.sin[p:p + 1],
                                        self.pos[p], self.k_cache[i], self.v_cache[i], None, l.q_norm, l.k_norm,
                                        self.eps, out=self.attn_out[off:off + n], flags=_lib.default_flags())
                self._gemv(self.attn_out[r0:r1], l.wo, h, epi=_lib.EPI_ADD_RESIDUAL, res=x)
            act = self.act[r0:r1, : l.wd.K]
            self._gemv(h, l.wgu, act, gamma=l.ln2, epi=_lib.EPI_SILU_MUL)
            y = self.res[i % 2][r0:r1]
            self._gemv(act, l.wd, y, epi=_lib.EPI_ADD_RESIDUAL, res=h)
            x = y
        return x

    def _head_and_sample(self, x: torch.Tensor, j: int) -> None:
        logits = self.step_logits[j]
        _lib.head_gemv(x, self.head_w[j], _lib.HEAD_KN, gamma=self.norm_w, eps=self.eps, out=logits,
                       flags=_lib.default_flags())
        _lib.sample(logits, self.half, temperature=self.temperature_buf, top_k=self.top_k_buf, top_p=self.top_p_buf,
                    do_sample=self.do_sample_buf, tokens=self.tok_buf,
                    guidance=self.guidance_scale if self.cfg else None, max_k=self.max_k,
                    mask=(self.codebook_size, self.vocab), clamp_hi=self.vocab - 1, rng=self.rng,
                    tokens2=self.output_tokens[:, j], flags=_lib.default_flags())

    def run(self) -> torch.Tensor:
        """Enqueue one frame on the current stream; returns output_tokens."""
        B, fl = self.B, _lib.default_flags()
        if self.bb_proj is not None:
            self._gemv(self.backbone_hidden_buf, self.bb_proj, self.emb[0:B])
        _lib.embed_rows(self.embed, self.first_cb_token_buf, 0, self.emb[B:2 * B], flags=fl)
        self._gemv(self.emb[0:2 * B], self.in_proj, self.x[0:2 * B])
        x = self._layers(0, 2 * B, [(0, B, 0), (B, B, 1)])
        self._head_and_sample(x[B:2 * B], 0)
        for j in range(1, self.n_dec):
            # tok_buf holds codebook j's token; its embedding row is offset by j * vocab (:602-609)
            _lib.embed_rows(self.embed, self.tok_buf, j * self.vocab, self.emb[2 * B:3 * B], flags=fl)
            self._gemv(self.emb[2 * B:3 * B], self.in_proj, self.x[0:B])
            x = self._layers(0, B, [(0, B, j + 1)])
            self._head_and_sample(x, j)
        return self.output_tokens

    def capture(self) -> None:
        """Warm up once (sizes the workspaces), then record the frame."""
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

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()
        return self.output_tokens


def synthetic_depth(fmt: str, n_layers: int, device, seed: int = 0, hidden: int = 1024, inter: int = 8192,
                    q_heads: int = 8, kv_heads: int = 8, head_dim: int = 128, emb_width: int = 2048,
                    vocab: int = 2051, num_codebooks: int = 16, attn_fmt: str | None = None,
                    proj_fmt: str | None = None):
    """Seeded random depth decoder: layers (QKV hidden -> (q + 2 kv) heads, O,
    gate+up hidden -> 2 inter, down), final norm, fp32 codebooks head
    (num_codebooks - 1, hidden, vocab), bf16 embedding (num_codebooks * vocab,
    emb_width) and the inputs_embeds_projector emb_width -> hidden. ``fmt``
    is the MLP format; QKV / O use ``attn_fmt`` and the projector
    ``proj_fmt`` (both default to ``fmt``; the reference keeps them bf16,
    FusedDecoderLayer(attn_bits=16) and an unquantized projector)."""
    from .stack import synthetic_weight

    gen = torch.Generator(device=device).manual_seed(seed)

    def norm_w(n):
        return (1 + 0.1 * torch.randn(n, device=device, generator=gen)).to(torch.bfloat16)

    qkv = (q_heads + 2 * kv_heads) * head_dim
    af, pf = attn_fmt or fmt, proj_fmt or fmt
    layers = [DecodeLayer(synthetic_weight(af, qkv, hidden, device, gen),
                          synthetic_weight(af, hidden, q_heads * head_dim, device, gen),
                          synthetic_weight(fmt, 2 * inter, hidden, device, gen),
                          synthetic_weight(fmt, hidden, inter, device, gen), norm_w(hidden), norm_w(hidden),
                          norm_w(head_dim), norm_w(head_dim)) for _ in range(n_layers)]
    head = torch.randn(num_codebooks - 1, hidden, vocab, device=device, generator=gen) * 0.05
    embed = (torch.randn(num_codebooks * vocab, emb_width, device=device, generator=gen)).to(torch.bfloat16)
    in_proj = synthetic_weight(pf, hidden, emb_width, device, gen)
    return layers, norm_w(hidden), head, embed, in_proj
