"""Benchmark of the fused RMSNorm -> int4 decode GEMV on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (config 1): out = rmsnorm(x) @ W^T with M=1, K=2048, N=6144 (fused
QKV), W int4 group-128 in the fused path's plain layout (FusedWeight bits=4),
x = residual bf16 N(0,1), gamma = bf16(1 + N(0, 0.1)), eps 1e-6. Synthetic
seeded inputs with BASELINE.json's distributions (no dataset exists for this).

One step = one CUDA-graph replay of R back-to-back rms_gemv calls, each on a
different copy of the weights; the R copies total >= 4x the L2 size, so
every call streams its weights from HBM (inputs larger than L2, no flush
needed). value = algorithmic bytes moved per second (GB/s), summed over
GPUs; per GPU the replicas are independent (weak scaling, no collectives).

--impl reference times the reference's own CPU path (torch dequant +
F.linear on the host cores, all threads) on the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "breeze-tts-2_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

M, K, N = 1, 2048, 6144
GROUP = 128
EPS = 1e-6
# algorithmic bytes of one call: codes + scale + min + x + gamma + out
ALGO_BYTES = N * K // 2 + 2 * (N * K // GROUP) * 2 + M * K * 2 + K * 2 + M * N * 2
METRIC = "fused quant GEMV HBM GB/s (% of 8 TB/s) at M=1; decode-step µs/token"
CONFIG = {"workload": "config1: fused RMSNorm -> int4 g128 GEMV, M=1, K=2048, N=6144 (plain int4 layout)",
          "global_batch": M, "seq_len": 1, "parallelism": "replicas"}


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class Ranks:
    """Start / finish lines and the max of per-rank timings across the replica
    processes (breeze_b200.replicas: a TCP store with deadlines, no collective
    and no NCCL). A rank that misses a deadline is reported in
    ``replicas_failed`` and the others carry on."""

    def __init__(self, rank: int, world: int):
        self.rank, self.world, self.n, self.grp = rank, world, 0, None
        if world > 1:
            from breeze_b200.replicas import ReplicaGroup

            self.grp = ReplicaGroup(rank, world, os.environ.get("MASTER_ADDR", "127.0.0.1"), timeout_s=300.0)

    def meet(self) -> None:
        if self.grp is not None:
            self.n += 1
            self.grp.meet(f"meet{self.n}")

    def max(self, value: float) -> float:
        """Max over the ranks that arrived (rank 0); a rank's own value elsewhere."""
        if self.grp is None:
            return value
        self.n += 1
        got = self.grp.gather(f"max{self.n}", value)
        return value if got is None else max(got.values())

    @property
    def failed(self) -> list[int]:
        return sorted(self.grp.failed) if self.grp is not None else []

    def close(self) -> None:
        """Leave the group (the rank hosting the store waits for the others)."""
        if self.grp is not None:
            self.grp.close()


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# DRAM bytes (read + write) of one GEMV launch on this workload (the resident-slice
# kernel, gemv_lean_kernel), from an ncu capture of this workload
# (dram__bytes_read.sum + dram__bytes_write.sum); re-captured whenever the kernel changes.
NCU_TRAFFIC_BYTES = 6_742_528


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.t0 = gpu, None, 0.0

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_inputs(device, seed: int):
    """Config-1 tensors on the device (seeded; plain int4 layout)."""
    from breeze_b200.fused.kernels import FusedWeight

    g = torch.Generator(device=device).manual_seed(seed)
    codes = torch.randint(0, 16, (N, K), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    scale = ((torch.randn(N, K // GROUP, generator=g, device=device) * 0.02).abs() / 7).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(K, generator=g, device=device)).to(torch.bfloat16)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    mn = (-8.0 * scale.float()).to(torch.bfloat16)
    fw = FusedWeight.from_parts(4, packed, scale, mn)
    return fw, x, gamma


def run_ours(args, rank, local_rank, world):
    from breeze_b200 import _lib
    from breeze_b200.fused.kernels import rms_gemv, rms_gemv_host_io

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ranks = Ranks(rank, world)
    fw, x, gamma = make_inputs(device, seed=1234 + rank)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    R = max(8, -(-4 * l2 // fw.w.numel()))  # copies totalling >= 4x L2
    copies = [fw.clone() for _ in range(R)]
    out = torch.empty(M, N, device=device, dtype=torch.bfloat16)
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for c in copies[:2]:
            rms_gemv(x, c, gamma, EPS, out=out)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for c in copies:
                rms_gemv(x, c, gamma, EPS, out=out)
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize(device)

    barrier = ranks.meet

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize(device)
    cur = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(args.steps):
        graph.replay()
    e1.record(cur)
    torch.cuda.synchronize(device)
    barrier()
    clock = clocks.stop()
    ms_max = ranks.max(e0.elapsed_time(e1))

    # ---- end to end: every step copies its input in from pinned host memory,
    # replays the step's graph of rms_gemv calls and copies the step's result
    # back; host clock from the first copy to the result being on the host
    x_host = x.cpu().pin_memory()
    out_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(1, min(args.steps, 500))

    def e2e_step():
        x.copy_(x_host, non_blocking=True)
        graph.replay()
        out_host.copy_(out, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(device)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    torch.cuda.synchronize(device)
    e2e_ms = ranks.max((time.perf_counter() - t0) * 1e3)
    # the same calls one at a time through the host-buffer entry point (rms_gemv_host_io:
    # x copied in, the GEMV, out copied back, per call), for comparison
    xd = torch.empty_like(x)
    call_steps = max(1, min(args.steps, 50))

    def per_call_step():
        for c in copies:
            rms_gemv_host_io(x_host, c, gamma, EPS, x=xd, out=out, out_host=out_host)

    per_call_step()
    torch.cuda.synchronize(device)
    barrier()
    t0 = time.perf_counter()
    for _ in range(call_steps):
        per_call_step()
    torch.cuda.synchronize(device)
    per_call_ms = ranks.max((time.perf_counter() - t0) * 1e3)
    barrier()
    status = _lib.device_status(local_rank)

    if rank == 0:
        peak, peak_kind = measured_peak()
        per_launch_s = ms_max / 1e3 / (args.steps * R)
        achieved = ALGO_BYTES / per_launch_s / 1e9
        alive = world - len(ranks.failed)  # replicas that reached every meeting
        value = alive * ALGO_BYTES * R * args.steps / (ms_max / 1e3) / 1e9
        e2e_val = alive * ALGO_BYTES * R * e2e_steps / (e2e_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, bf16 activations, fp32 accumulate",
            "data": "synthetic (seeded, BASELINE config-1 distributions)",
            "config": {**CONFIG, "calls_per_step": R, "l2_policy": f"inputs > L2: {R} weight copies = "
                       f"{R * ALGO_BYTES / 2**20:.0f} MiB rotated per step"},
            "us_per_call": round(per_launch_s * 1e6, 3),
            "pct_of_8TBs": round(100 * achieved / 8000, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC_BYTES, "algorithmic_bytes_per_launch": ALGO_BYTES},
            "e2e": {"value": round(e2e_val, 1), "unit": "GB/s", "h2d_bytes_per_step": M * K * 2,
                    "d2h_bytes_per_step": M * N * 2, "steps": e2e_steps,
                    "how": "per step: H2D of x from pinned memory, the step's CUDA graph of rms_gemv calls, D2H of "
                           "out to pinned memory; host clock until the last result is on the host",
                    "per_call_copies": {"value": round(alive * ALGO_BYTES * R * call_steps / (per_call_ms / 1e3) / 1e9, 1),
                                        "unit": "GB/s", "h2d_bytes_per_call": M * K * 2, "d2h_bytes_per_call": M * N * 2,
                                        "how": "rms_gemv_host_io per call (H2D of x, the GEMV, D2H of out, each call), "
                                               "eager, host clock"}},
            "gpu_launches": R * args.steps,
            "clocks": clock,
            "device_error_bits": status,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(seconds=args.cpu_seconds)
    decode = None if args.no_decode_step else decode_step_bench(device, ranks)
    depth = None if args.no_decode_step else depth_frame_bench(device, ranks)
    if rank == 0:
        if decode is not None:
            line["decode_step"] = decode
        if depth is not None:
            line["depth_frame"] = depth
        if world == 1 and not args.no_reference_gpu:
            ours_ref = {"config1_us": per_launch_s * 1e6}
            for e in (decode or {}).get("results", []):
                step = e.get("per_op", {}).get("step_us")
                if step is not None:
                    ours_ref[f"{e['format']}_{e['rows']}"] = step
            try:
                line["reference_gpu"] = reference_gpu_bench(device, copies, x, gamma, ours_ref)
            except Exception as ex:  # noqa: BLE001 - reported, never hidden
                line["reference_gpu"] = {"unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"}
        if world > 1:
            line["replicas_failed"] = ranks.failed
        print(json.dumps(line), flush=True)
    ranks.close()


DECODE_FORMATS = ("int4", "fp8", "int8")
DECODE_ROWS = (1, 2, 4, 8, 16)
DECODE_ROWS_INT4 = (1, 2, 4, 8, 16, 32, 64)  # config 4 adds 32 and 64 concurrent streams per GPU
DECODE_LAYERS = 28


def decode_step_bench(device, ranks: Ranks, replays: int = 10, warmup: int = 3, formats=DECODE_FORMATS,
                      rows_list=None, modes=("per_op", "chain", "attn")):
    """Decode-step leg (the 28-layer projection stack + head as one CUDA graph,
    breeze_b200.fused.stack.DecodeStack) for each weight format and row count.
    The stack's weights (1.0 GB int4, 1.9 GB fp8/int8) exceed L2 by far, so
    every replay streams them from HBM. Device time per replay, max over ranks."""
    from breeze_b200.fused.stack import DecodeStack, synthetic_stack

    results = []
    cur = torch.cuda.current_stream(device)
    for fmt in formats:
        layers, head, ln_f = synthetic_stack(fmt, DECODE_LAYERS, device, seed=7)
        for rows in rows_list or (DECODE_ROWS_INT4 if fmt == "int4" else DECODE_ROWS):
            entry = {"format": fmt, "rows": rows}
            for mode in modes:
                if mode == "chain" and rows > 16:
                    entry[mode] = {"unavailable": "the chain takes at most 16 rows"}
                    continue
                try:
                    st = DecodeStack(layers, head, ln_f, rows=rows, chain=(mode == "chain"),
                                     attention=(mode == "attn"))
                except (RuntimeError, ValueError) as e:  # chain limits (rows per pass) are reported, not hidden
                    entry[mode] = {"unavailable": str(e)[:160]}
                    continue
                st.x.copy_(torch.randn(rows, st.hidden, device=device, generator=torch.Generator(device=device)
                                       .manual_seed(rows)).to(torch.bfloat16))
                st.capture()
                for _ in range(warmup):
                    st.replay()
                torch.cuda.synchronize(device)
                ranks.meet()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(cur)
                for _ in range(replays):
                    st.replay()
                e1.record(cur)
                torch.cuda.synchronize(device)
                step_us = ranks.max(e0.elapsed_time(e1) / replays) * 1e3
                world = ranks.world - len(ranks.failed)
                wb = st.weight_bytes
                entry[mode] = {"step_us": round(step_us, 1), "us_per_row": round(step_us / rows, 2),
                               "tokens_per_s_all_gpus": round(world * rows / step_us * 1e6, 1),
                               "GBps": round((wb + st.kv_bytes) / step_us / 1e3, 1), "launches": st.launches,
                               "finite": bool(torch.isfinite(st.logits).all().item())}
                entry["weight_bytes"] = wb
                del st
            results.append(entry)
        del layers, head, ln_f
        torch.cuda.empty_cache()
    return {"what": f"{DECODE_LAYERS} layers x (QKV 2048->6144 +RMSNorm, O 2048->2048 +residual, "
                    "gate+up 2048->16384 +RMSNorm +SiLU*up, down 8192->2048 +residual) + head 2048->8192 "
                    "+RMSNorm (fp32 logits); per_op = one CUDA graph of 113 bq_gemv launches with PDL, chain = "
                    "one cooperative bq_gemv_chain launch, attn = per_op plus the decode attention step per layer "
                    "(16 q / 16 kv heads of 128, kv_len 256; 141 launches)",
            "launches_per_step": 4 * DECODE_LAYERS + 1, "replays_timed": replays,
            "l2_policy": "weights 1-1.9 GB per step >> L2", "results": results}


DEPTH_LAYERS = 12


def depth_frame_bench(device, ranks: Ranks, replays: int = 10, warmup: int = 3):
    """Depth-decoder frame leg (breeze_b200.fused.depth.DepthDecoderLoop): one
    CUDA graph of a whole frame (2-position prefill + 14 single steps over 12
    layers, fp32 codebook head and CFG sampling per step) at the depth shapes
    (hidden 1024, MLP 8192, 8 q / 8 kv heads of 128, audio embedding 2048,
    vocab 2051, 16 codebooks), int4 MLP with bf16 attention projections as the
    reference's FusedDecoderLayer(attn_bits=16) over Int4Linear runs it. Device
    time per replay, max over ranks."""
    from breeze_b200.fused.depth import DepthDecoderLoop, synthetic_depth

    cur = torch.cuda.current_stream(device)
    out = []
    layers, norm_w, head, embed, in_proj = synthetic_depth("int4", DEPTH_LAYERS, device, seed=9, attn_fmt="bf16",
                                                           proj_fmt="bf16")
    for batch in (1, 2):
        loop = DepthDecoderLoop(layers, norm_w, head, embed, in_proj, batch, codebook_size=2048, kv_heads=8, seed=batch)
        loop.capture()
        for _ in range(warmup):
            loop.replay()
        torch.cuda.synchronize(device)
        ranks.meet()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        for _ in range(replays):
            loop.replay()
        e1.record(cur)
        torch.cuda.synchronize(device)
        us = ranks.max(e0.elapsed_time(e1) / replays) * 1e3
        out.append({"batch": batch, "frame_us": round(us, 1), "us_per_codebook_step": round(us / loop.n_dec, 1),
                    "launches": loop.launches, "weight_GBps": round(loop.weight_bytes_per_frame / us / 1e3, 1),
                    "tokens_valid": bool(((loop.output_tokens >= 0) & (loop.output_tokens < 2048)).all().item())})
        del loop
    del layers, head, embed
    torch.cuda.empty_cache()
    return {"what": f"depth-decoder frame: {DEPTH_LAYERS} layers, 15 codebooks (prefill at positions 0-1 + 14 steps), "
                    "int4 MLP / bf16 QKV+O / bf16 projector, fp32 codebook head, CFG sampling in the graph",
            "replays_timed": replays, "results": out}


def shape_bench(device, spec: str, steps: int, warmup: int):
    """One GEMV shape as a CUDA graph over rotated weight copies (> 4x L2), PDL
    between calls; device time per call. For per-shape numbers and targeted
    profiles."""
    from breeze_b200 import _lib
    from breeze_b200.fused.stack import synthetic_weight

    fmt, n, k, m, epi = spec.split(":")
    n, k, m, epi = int(n), int(k), int(m), int(epi)
    g = torch.Generator(device=device).manual_seed(0)
    w0 = synthetic_weight(fmt, n, k, device, g)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    r = max(8, (4 * l2) // w0.nbytes + 1)
    copies = [w0] + [synthetic_weight(fmt, n, k, device, g) for _ in range(r - 1)]
    x = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, device=device, generator=g)).to(torch.bfloat16) if epi != 2 else None
    res = torch.randn(m, n, device=device, generator=g).to(torch.bfloat16) if epi == 2 else None
    out = torch.empty(m, n // 2 if epi == 1 else n, device=device, dtype=torch.bfloat16)

    def step():
        for q in copies:
            _lib.gemv(x, q.w, q.wfmt, q.N, scale=q.scale, group=q.group, gamma=gamma, epilogue=epi, residual=res,
                      out=out, flags=_lib.default_flags())

    step()
    torch.cuda.synchronize(device)
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step()
    torch.cuda.current_stream(device).wait_stream(s)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(device)
    us = e0.elapsed_time(e1) * 1e3 / (steps * r)
    algo = w0.nbytes + m * k * 2 + out.numel() * 2 + (0 if gamma is None else k * 2) + (0 if res is None else res.numel() * 2)
    return {"shape": spec, "us_per_call": round(us, 2), "GBps": round(algo / us / 1e3, 1), "calls_per_replay": r,
            "algorithmic_bytes_per_call": algo}


REF_DIR = ROOT / "baseline" / "_ref"
# The reference's own rms_gemv autotune results on this pool's B200 (its
# BREEZE_FUSED_TUNE file format, written by its unmodified tuner); the bench
# hands the reference a copy so its first call does not re-tune for minutes.
REF_TUNE = ROOT / "reference_tune_b200.json"


def _reference_modules():
    """The unmodified reference's fused kernels and Int4Linear from
    baseline/_ref (None when the reference is not installed there)."""
    if not (REF_DIR / "models" / "fused" / "kernels.py").exists():
        return None
    import shutil
    import tempfile

    tune = Path(tempfile.gettempdir()) / "bq_reference_fused_tune.json"
    if REF_TUNE.exists():
        shutil.copyfile(REF_TUNE, tune)
    os.environ["BREEZE_FUSED_TUNE"] = str(tune)  # read when models.fused.kernels is imported
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import models.fused.kernels as rk  # noqa: PLC0415 - the reference package
    import models.int4_linear as ri4  # noqa: PLC0415

    return rk, ri4


def _graph_us_per_replay(fn, device, replays: int = 10, warmup: int = 3) -> float:
    """fn recorded once into a CUDA graph; device time per replay (us)."""
    fn()
    torch.cuda.synchronize(device)
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
        fn()
    torch.cuda.current_stream(device).wait_stream(side)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(device)
    del graph
    return e0.elapsed_time(e1) * 1e3 / replays


def reference_gpu_bench(device, copies, x, gamma, ours: dict) -> dict:
    """The reference's own GPU path on this B200, timed like ours (CUDA-graph
    replays, cold rotated weight copies, CUDA events), next to ours:

      config 1: Triton rms_gemv over FusedWeight(W, 4) (the same plain int4
        codes, scales and mins as ours) and tinygemm Int4Linear alone (no
        norm), models/fused/kernels.py:334-351, models/int4_linear.py:99-109;
      config 3 int4 decode step (28 layers + head, M = 1, 2, 16): Int4Linear
        (tinygemm) projections with the reference's Triton rmsnorm / silu_mul
        around them, as its FusedDecoderLayer runs an int4 MLP
        (models/fused/layer.py:92-96), the attention projections in int4 too;
      config 3 fp8 decode step (M = 1, 2): Triton rms_gemv over FusedWeight(W,
        8) for every projection (layer.py:87-98 with mlp_bits=8, attn_bits=8).
    ``ours`` holds this build's figures for the same cases (us)."""
    mods = _reference_modules()
    if mods is None:
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    if not REF_TUNE.exists():
        return {"unavailable": "no B200 tune file for the reference's Triton kernels (reference_tune_b200.json)"}
    rk, ri4 = mods
    out = {"source": "unmodified reference modules from baseline/_ref, same box and run", "cases": []}
    for case in (_ref_config1_triton, _ref_config1_tinygemm, _ref_int4_stack, _ref_fp8_stack):
        try:
            case(rk, ri4, device, copies, x, gamma, ours, out)
        except Exception as ex:  # noqa: BLE001 - reported per case, never hidden
            out["cases"].append({"case": case.__name__, "unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"})
        torch.cuda.empty_cache()
    return out


def _ref_add(out, case, ref_us, ours_us, weight_bytes):
    e = {"case": case, "reference_us": round(ref_us, 2), "ours_us": None if ours_us is None else round(ours_us, 2),
         "reference_weight_GBps": round(weight_bytes / ref_us / 1e3, 1)}
    if ours_us:
        e["ours_over_reference_speedup"] = round(ref_us / ours_us, 3)
    out["cases"].append(e)


def _ref_config1_triton(rk, ri4, device, copies, x, gamma, ours, out):
    """config 1: Triton rms_gemv (plain int4) over the same rotated copies."""
    rf = []
    for c in copies:
        f = rk.FusedWeight.__new__(rk.FusedWeight)
        f.bits, f.N, f.K = 4, c.N, c.K
        f.w, f.s, f.z = c.w, c.s.contiguous(), c.z.contiguous()
        rf.append(f)
    y = torch.empty(M, N, device=device, dtype=torch.bfloat16)

    def triton_calls():
        for f in rf:
            rk.rms_gemv(x, f, gamma, EPS, out=y)

    us = _graph_us_per_replay(triton_calls, device) / len(rf)
    _ref_add(out, "config 1: fused RMSNorm -> int4 GEMV (Triton rms_gemv, bits=4), per call", us, ours.get("config1_us"),
             ALGO_BYTES)


def _ref_config1_tinygemm(rk, ri4, device, copies, x, gamma, ours, out):
    """config 1 shape: tinygemm Int4Linear alone (no norm), same rotation."""
    lin = torch.nn.Linear(K, N, bias=False, device=device, dtype=torch.bfloat16)
    base = ri4.Int4Linear(lin, group_size=GROUP)
    del lin
    mods4 = [base]
    for _ in range(len(copies) - 1):
        m = ri4.Int4Linear.__new__(ri4.Int4Linear)
        torch.nn.Module.__init__(m)
        m.in_features, m.out_features, m.group_size = base.in_features, base.out_features, base.group_size
        m.register_buffer("weight_int4", base.weight_int4.clone())
        m.register_buffer("scales_zeros", base.scales_zeros.clone())
        mods4.append(m)
    xs = x.clone()

    def tinygemm_calls():
        for m in mods4:
            m(xs)

    us = _graph_us_per_replay(tinygemm_calls, device) / len(mods4)
    wb = base.weight_int4.numel() * 4 + base.scales_zeros.numel() * 2
    _ref_add(out, "config 1 shape 2048->6144: tinygemm Int4Linear alone (no norm), per call", us, None, wb)


_REF_H, _REF_QKV, _REF_INTER, _REF_HEAD = 2048, 6144, 8192, 8192


def _ref_int4_stack(rk, ri4, device, copies, x, gamma, ours, out):
    """config 3 int4 step: Int4Linear (tinygemm) projections, Triton rmsnorm /
    silu_mul around them; O reads a static attention-output buffer (attention
    is not part of config 3; the reference's O input is always contiguous)."""
    H, QKV, INTER, HEAD, L = _REF_H, _REF_QKV, _REF_INTER, _REF_HEAD, DECODE_LAYERS
    gen = torch.Generator(device=device).manual_seed(5)

    def rand_linear(n, k):
        lin = torch.nn.Linear(k, n, bias=False, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(n, k, device=device, generator=gen) * 0.02)
        return lin

    def norm_w(n=H):
        return (1 + 0.1 * torch.randn(n, device=device, generator=gen)).to(torch.bfloat16)

    layers = []
    for _ in range(L):
        layers.append({name: ri4.Int4Linear(rand_linear(n, k), group_size=GROUP) for name, n, k in
                       (("qkv", QKV, H), ("o", H, H), ("gate", INTER, H), ("up", INTER, H), ("down", H, INTER))})
        layers[-1]["ln1"], layers[-1]["ln2"] = norm_w(), norm_w()
    head = ri4.Int4Linear(rand_linear(HEAD, H), group_size=GROUP)
    ln_f = norm_w()
    wb4 = sum(m.weight_int4.numel() * 4 + m.scales_zeros.numel() * 2 for l in layers for m in l.values()
              if isinstance(m, ri4.Int4Linear)) + head.weight_int4.numel() * 4 + head.scales_zeros.numel() * 2
    for rows in (1, 2, 16):
        x0 = torch.randn(rows, H, device=device, generator=gen).to(torch.bfloat16)
        attn = torch.randn(rows, H, device=device, generator=gen).to(torch.bfloat16)

        def step4():
            h = x0
            for l in layers:
                l["qkv"](rk.rmsnorm(h, l["ln1"], EPS))
                hh = l["o"](attn) + h
                n2 = rk.rmsnorm(hh, l["ln2"], EPS)
                h = l["down"](rk.silu_mul(l["gate"](n2), l["up"](n2))) + hh
            return head(rk.rmsnorm(h, ln_f, EPS)).float()

        us = _graph_us_per_replay(step4, device)
        _ref_add(out, f"config 3 int4 decode step M={rows} (tinygemm + Triton rmsnorm/silu_mul)", us,
                 ours.get(f"int4_{rows}"), wb4)


def _ref_fp8_stack(rk, ri4, device, copies, x, gamma, ours, out):
    """config 3 fp8 step: Triton rms_gemv over FusedWeight(W, 8) everywhere."""
    H, QKV, INTER, HEAD, L = _REF_H, _REF_QKV, _REF_INTER, _REF_HEAD, DECODE_LAYERS
    gen = torch.Generator(device=device).manual_seed(6)

    def norm_w(n=H):
        return (1 + 0.1 * torch.randn(n, device=device, generator=gen)).to(torch.bfloat16)

    layers8 = []
    for _ in range(L):
        wq = torch.randn(QKV, H, device=device, generator=gen) * 0.02
        wo = torch.randn(H, H, device=device, generator=gen) * 0.02
        wgu = torch.randn(2 * INTER, H, device=device, generator=gen) * 0.02
        wd = torch.randn(H, INTER, device=device, generator=gen) * 0.02
        layers8.append({"qkv": rk.FusedWeight(wq, 8), "o": rk.FusedWeight(wo, 8), "gu": rk.FusedWeight(wgu, 8),
                        "down": rk.FusedWeight(wd, 8), "ln1": norm_w(), "ln2": norm_w()})
    head8 = rk.FusedWeight(torch.randn(HEAD, H, device=device, generator=gen) * 0.02, 8)
    ln_f = norm_w()
    wb8 = sum(f.w.numel() + f.s.numel() * 4 for l in layers8 for f in l.values() if isinstance(f, rk.FusedWeight))
    wb8 += head8.w.numel() + head8.s.numel() * 4
    for rows in (1, 2):
        x0 = torch.randn(rows, H, device=device, generator=gen).to(torch.bfloat16)

        def step8():
            h = x0
            for l in layers8:
                qkv = rk.rms_gemv(h, l["qkv"], l["ln1"], EPS)
                hh = rk.rms_gemv(qkv[:, :H], l["o"], None, EPS, epilogue=2, residual=h)
                act = rk.rms_gemv(hh, l["gu"], l["ln2"], EPS, epilogue=1)
                h = rk.rms_gemv(act, l["down"], None, EPS, epilogue=2, residual=hh)
            return rk.rms_gemv(h, head8, ln_f, EPS).float()

        us = _graph_us_per_replay(step8, device)
        _ref_add(out, f"config 3 fp8 decode step M={rows} (Triton rms_gemv bits=8)", us, ours.get(f"fp8_{rows}"), wb8)


def _cpu_inputs():
    g = torch.Generator().manual_seed(1234)
    codes = torch.randint(0, 16, (N, K), generator=g, dtype=torch.int32).to(torch.uint8)
    scale = ((torch.randn(N, K // GROUP, generator=g) * 0.02).abs() / 7).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    mn = (-8.0 * scale.float()).to(torch.bfloat16)
    return x, packed, scale, mn, gamma


def cpu_baseline(seconds: float = 10.0):
    """The reference's CPU path (torch dequant + F.linear) on a bounded sample."""
    from oracle import cpu_path

    x, packed, scale, mn, gamma = _cpu_inputs()
    cpu_path.rms_gemv_int4_plain(x, packed, scale, mn, gamma, EPS)
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_path.rms_gemv_int4_plain(x, packed, scale, mn, gamma, EPS)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": round(ALGO_BYTES / dt / 1e9, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{n} calls of the full config-1 GEMV (M=1, K=2048, N=6144), "
            f"{dt * 1e3:.1f} ms per call"}


def run_reference(args, rank):
    if rank != 0:
        return
    from oracle import cpu_path

    # rank 0 alone runs the CPU path: every host core this process may use (torchrun
    # sets OMP_NUM_THREADS=1 for its ranks)
    torch.set_num_threads(len(os.sched_getaffinity(0)))

    x, packed, scale, mn, gamma = _cpu_inputs()
    for _ in range(args.warmup):
        cpu_path.rms_gemv_int4_plain(x, packed, scale, mn, gamma, EPS)
    steps = args.steps
    t0 = time.perf_counter()
    deadline = t0 + args.cpu_seconds * 6
    done = 0
    for _ in range(steps):
        cpu_path.rms_gemv_int4_plain(x, packed, scale, mn, gamma, EPS)
        done += 1
        if time.perf_counter() > deadline:
            break
    dt = time.perf_counter() - t0
    value = ALGO_BYTES * done / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": 0,
        "steps": done, "warmup": args.warmup, "ms_per_step": round(dt / done * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, fp32 dequant + F.linear (CPU)",
        "data": "synthetic (seeded, BASELINE config-1 distributions)", "config": CONFIG,
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": f"{done} calls of the full config-1 GEMV on the host"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode-step", action="store_true", help="skip the 28-layer decode-step leg")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU kernels (baseline/_ref) on the same device")
    ap.add_argument("--shape", default=None, metavar="FMT:N:K:M:EPI",
                    help="time one GEMV shape (fmt int4|fp8|int8|bf16, epilogue 0 none / 1 SiLU*up / 2 residual; "
                         "RMSNorm unless EPI is 2) over rotated weight copies > 4x L2 and print its JSON")
    ap.add_argument("--depth-only", action="store_true",
                    help="run only the depth-decoder frame leg (one GPU; for profiling) and print its JSON")
    ap.add_argument("--decode-only", default=None, metavar="FMT:ROWS[:MODE]",
                    help="run only one decode-step configuration (one GPU; for profiling): MODE per_op (default), "
                         "chain or attn")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank, local_rank, world = dist_env()
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.shape:
        device = torch.device("cuda", local_rank)
        torch.cuda.set_device(device)
        print(json.dumps(shape_bench(device, args.shape, args.steps, args.warmup)), flush=True)
        return
    if args.decode_only:
        device = torch.device("cuda", local_rank)
        torch.cuda.set_device(device)
        fmt, rows, *mode = args.decode_only.split(":")
        print(json.dumps({"decode_step": decode_step_bench(device, Ranks(0, 1), formats=(fmt,), rows_list=(int(rows),),
                                                           modes=tuple(mode) or ("per_op",))}), flush=True)
        return
    if args.depth_only:
        device = torch.device("cuda", local_rank)
        torch.cuda.set_device(device)
        print(json.dumps({"depth_frame": depth_frame_bench(device, Ranks(0, 1))}), flush=True)
        return
    run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    main()
