"""CFG mix + token sampling (bq_sample) and the fp32 output heads (bq_head_gemv).

CPU: the sampling oracle against the reference's own `_cfg_sample` and
`sample_logits` (tests/golden/sampling.npz, made by make_sampling_golden.py:
the probability vector handed to torch.multinomial, and greedy tokens), and
Philox4x32-10 against the published known-answer vectors. GPU (through the C
ABI): tokens identical to the oracle for the same u (rows whose draw sits
within 1e-5 of a cumulative boundary are skipped: fp32 summation order may
legitimately flip them), greedy exact, Philox u identical, the counter
advancing once per launch and per graph replay; heads within 1e-5 (2e-3 with
the bf16 norm roundings) of the float64 oracle, and deterministic.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import sampling as osm

GOLD = Path(__file__).resolve().parent / "golden" / "sampling.npz"


def test_philox_known_answers():
    # Random123 known-answer vectors for philox4x32, 10 rounds
    assert osm.philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    f = 0xFFFFFFFF
    assert osm.philox4x32_10((f, f, f, f), (f, f)) == (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert osm.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == (
        0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


def _depth_cases(z):
    i = 0
    while f"depth{i}_case" in z:
        yield i, z[f"depth{i}_case"]
        i += 1


def test_sampling_oracle_matches_reference_depth_graph():
    z = np.load(GOLD)
    n = 0
    for i, c in _depth_cases(z):
        rows, cfg, v, cb, max_k, temp, top_k, top_p, do_sample, g, _ = c
        rows, v, cb, max_k, top_k = int(rows), int(v), int(cb), int(max_k), int(top_k)
        logits = torch.from_numpy(z[f"depth{i}_logits"])
        mixed = osm.mixed_logits(logits, rows, torch.full((rows,), g) if cfg else None, mask=(cb, v))
        ref_probs = torch.from_numpy(z[f"depth{i}_probs"])
        for r in range(rows):
            p = osm.sample_probs(mixed[r], float(temp), top_k, float(top_p), max_k)
            assert torch.equal(p > 0, ref_probs[r] > 0), f"case {i} row {r}: kept set differs"
            assert float((p - ref_probs[r]).abs().max()) < 1e-6, f"case {i} row {r}"
            if not do_sample:
                assert int(z[f"depth{i}_tokens"][r]) == int(torch.argmax(mixed[r]))
            n += 1
    assert n >= 8


def test_sampling_oracle_matches_reference_sample_logits():
    z = np.load(GOLD)
    i = 0
    while f"bb{i}_case" in z:
        v, temp, top_k, top_p, do_sample, pen, hl, _, _ = z[f"bb{i}_case"]
        v, top_k, hl = int(v), int(top_k), int(hl)
        logits = torch.from_numpy(z[f"bb{i}_logits"])
        hist = torch.from_numpy(z[f"bb{i}_history"]).reshape(1, -1)
        sup = torch.from_numpy(z[f"bb{i}_suppress"])
        mixed = osm.mixed_logits(logits, 1, None, rep_penalty=float(pen), history=hist if hl else None,
                                 history_len=torch.tensor([hl]), suppress=sup if bool(sup.any()) else None)
        if do_sample:
            p = osm.sample_probs(mixed[0], float(temp), top_k, float(top_p) if top_p < 1.0 else 2.0, v,
                                 topk_by_value=True)
            ref = torch.from_numpy(z[f"bb{i}_probs"]).reshape(-1)
            assert torch.equal(p > 0, ref > 0), f"case {i}: kept set differs"
            assert float((p - ref).abs().max()) < 1e-6, f"case {i}"
        else:
            assert int(z[f"bb{i}_token"][0]) == int(torch.argmax(mixed[0]))
        i += 1
    assert i >= 4


# ---------------------------------------------------------------- GPU
def _params(rows, dev, temp, top_k, top_p, do_sample, g=None):
    f = lambda v, dt: torch.full((rows,), v, device=dev, dtype=dt)  # noqa: E731
    out = dict(temperature=f(temp, torch.float32), top_k=f(top_k, torch.int64), top_p=f(top_p, torch.float32),
               do_sample=f(do_sample, torch.int64))
    if g is not None:
        out["guidance"] = f(g, torch.float32)
    return out


CASES = [  # rows, cfg, V, mask (lo, hi), max_k, temperature, top_k, top_p
    (1, False, 2051, (2048, 2051), 1024, 0.9, 50, 0.95),
    (2, True, 2051, (2048, 2051), 1024, 0.7, 0, 0.9),
    (4, True, 2051, (2048, 2051), 1024, 1.0, 8, 1.0),
    (1, True, 4099, (4096, 4099), 1024, 1.3, 300, 0.5),
    (3, False, 8192, (0, 0), 1024, 1.1, 1024, 0.99),
    (2, False, 1000, (0, 0), 1000, 0.8, 1, 0.9),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(len(CASES)))
def test_sample_matches_oracle(case):
    from breeze_b200 import _lib as L

    rows, cfg, v, mask, max_k, temp, top_k, top_p = CASES[case]
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(100 + case)
    checked = 0
    for trial in range(6):
        logits = torch.randn(2 * rows if cfg else rows, v, generator=g) * 3.0
        u = torch.rand(rows, generator=g)
        tokens = torch.full((2 * rows if cfg else rows,), -1, dtype=torch.int64, device=dev)
        prm = _params(rows, dev, temp, top_k, top_p, 1, 2.5 if cfg else None)
        L.sample(logits.to(dev), rows, tokens=tokens, max_k=max_k, mask=mask, uniform=u.to(dev), **prm)
        greedy = torch.full_like(tokens, -1)
        prm["do_sample"].zero_()
        L.sample(logits.to(dev), rows, tokens=greedy, max_k=max_k, mask=mask, uniform=u.to(dev), **prm)
        torch.cuda.synchronize()
        mixed = osm.mixed_logits(logits, rows, torch.full((rows,), 2.5) if cfg else None, mask=mask)
        for r in range(rows):
            assert int(greedy[r]) == int(torch.argmax(mixed[r]))
            if osm.draw_margin(mixed[r], temp, top_k, top_p, float(u[r]), max_k) < 1e-5:
                continue
            want = osm.sample_row(mixed[r], temp, top_k, top_p, True, float(u[r]), max_k)
            assert int(tokens[r]) == want, f"trial {trial} row {r}"
            if cfg:
                assert int(tokens[r + rows]) == want
            checked += 1
    assert checked >= 4 * rows


@pytest.mark.gpu
def test_sample_penalty_suppress_and_cfg_out():
    from breeze_b200 import _lib as L

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(7)
    rows, v = 2, 2049
    logits = torch.randn(rows, v, generator=g) * 3.0
    hist = torch.randint(0, v, (rows, 64), generator=g)
    hl = torch.tensor([40, 64], dtype=torch.int32)
    sup = torch.zeros(v, dtype=torch.bool)
    sup[[5, 2048]] = True
    u = torch.rand(rows, generator=g)
    tokens = torch.zeros(rows, dtype=torch.int64, device=dev)
    cfg_out = torch.zeros(rows, v, device=dev)
    prm = _params(rows, dev, 0.9, 50, 0.95, 1)
    L.sample(logits.to(dev), rows, tokens=tokens, max_k=v, topk_by_value=True, rep_penalty=1.3,
             history=hist.to(dev), history_len=hl.to(dev), suppress=sup.to(torch.uint8).to(dev), uniform=u.to(dev),
             cfg_out=cfg_out, **prm)
    torch.cuda.synchronize()
    mixed = osm.mixed_logits(logits, rows, None, rep_penalty=1.3, history=hist, history_len=hl, suppress=sup)
    assert torch.equal(cfg_out.cpu(), mixed)
    for r in range(rows):
        if osm.draw_margin(mixed[r], 0.9, 50, 0.95, float(u[r]), v, topk_by_value=True) < 1e-5:
            continue
        assert int(tokens[r]) == osm.sample_row(mixed[r], 0.9, 50, 0.95, True, float(u[r]), v, topk_by_value=True)


@pytest.mark.gpu
def test_sample_philox_counter_and_graph_replay():
    from breeze_b200 import _lib as L

    dev = torch.device("cuda", 0)
    rows, v = 2, 2051
    logits = (torch.randn(2 * rows, v, generator=torch.Generator().manual_seed(3)) * 3.0).to(dev)
    seed = 0x1234_5678_9ABC
    rng = torch.tensor([seed, 0], dtype=torch.int64, device=dev)
    tokens = torch.zeros(2 * rows, dtype=torch.int64, device=dev)
    out_tokens = torch.zeros(2 * rows, 16, dtype=torch.int64, device=dev)
    prm = _params(rows, dev, 1.0, 0, 1.0, 1, 3.0)

    def call():
        L.sample(logits, rows, tokens=tokens, max_k=1024, mask=(2048, 2051), rng=rng, tokens2=out_tokens[:, 5], **prm)

    mixed = osm.mixed_logits(logits.cpu(), rows, torch.full((rows,), 3.0), mask=(2048, 2051))
    call()
    torch.cuda.synchronize()
    assert int(rng[1]) == 1
    for r in range(rows):
        u = osm.philox_uniform(seed, 0, r)
        if osm.draw_margin(mixed[r], 1.0, 0, 1.0, u, 1024) >= 1e-5:
            want = osm.sample_row(mixed[r], 1.0, 0, 1.0, True, u, 1024)
            assert int(tokens[r]) == want and int(tokens[r + rows]) == want
            assert int(out_tokens[r, 5]) == want and int(out_tokens[r + rows, 5]) == want
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            call()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    start = int(rng[1])
    for i in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert int(rng[1]) == start + i + 1
        for r in range(rows):
            u = osm.philox_uniform(seed, start + i, r)
            if osm.draw_margin(mixed[r], 1.0, 0, 1.0, u, 1024) >= 1e-5:
                assert int(tokens[r]) == osm.sample_row(mixed[r], 1.0, 0, 1.0, True, u, 1024)
    del graph


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("m,n,k", [(1, 2051, 1024), (2, 2051, 1024), (3, 8193, 2048), (2, 130, 256)])
@pytest.mark.parametrize("norm", [False, True])
def test_head_matches_oracle(layout, m, n, k, norm):
    from breeze_b200 import _lib as L

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(m * 7 + n + k)
    x = (torch.randn(m, k, generator=g) * 2.0).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16) if norm else None
    w = torch.randn(k, n, generator=g) * 0.02 if layout == "kn" else torch.randn(n, k, generator=g) * 0.02
    lay = L.HEAD_KN if layout == "kn" else L.HEAD_NK
    out = L.head_gemv(x.to(dev), w.to(dev), lay, gamma=None if gamma is None else gamma.to(dev), eps=1e-6)
    out2 = L.head_gemv(x.to(dev), w.to(dev), lay, gamma=None if gamma is None else gamma.to(dev), eps=1e-6)
    torch.cuda.synchronize()
    ref = osm.head(x, w, layout == "kn", gamma, 1e-6)
    err = float((out.cpu() - ref).abs().max() / ref.abs().max())
    assert err <= (2e-3 if norm else 1e-5), err
    assert torch.equal(out, out2)


def test_sample_rejects_bad_args_cpu():
    from breeze_b200 import _lib as L

    lib = L.load()
    import ctypes

    d = L.SampleDesc()
    d.rows, d.V, d.max_k = 1, 10000, 10
    assert lib.bq_sample_workspace_bytes(ctypes.byref(d), ctypes.byref(ctypes.c_size_t())) != 0
    h = L.HeadDesc()
    h.M, h.N, h.K, h.layout = 17, 10, 10, L.HEAD_NK
    assert lib.bq_head_workspace_bytes(ctypes.byref(h), ctypes.byref(ctypes.c_size_t())) != 0


# The reference's own sampling tests (tests/test_logits_process.py), through bq_sample.
@pytest.mark.gpu
def test_reference_case_penalty_on_generated_history():
    from breeze_b200 import _lib as L

    dev = torch.device("cuda", 0)
    tokens = torch.zeros(1, dtype=torch.int64, device=dev)
    L.sample(torch.tensor([[1.0, 0.9, 0.1]], device=dev), 1, tokens=tokens, rep_penalty=2.0,
             history=torch.tensor([[0]], device=dev), history_len=torch.tensor([1], dtype=torch.int32, device=dev),
             uniform=torch.zeros(1, device=dev), **_params(1, dev, 1.0, 0, 1.0, 0))
    assert int(tokens[0]) == 1


@pytest.mark.gpu
@pytest.mark.parametrize("width", [2052, 2051])
def test_reference_case_codec_mask(width):
    from breeze_b200 import _lib as L

    dev = torch.device("cuda", 0)
    cfg_out = torch.zeros(1, width, device=dev)
    L.sample(torch.zeros(1, width, device=dev), 1, tokens=torch.zeros(1, dtype=torch.int64, device=dev),
             mask=(2048, 2051), cfg_out=cfg_out, uniform=torch.zeros(1, device=dev), **_params(1, dev, 1.0, 0, 1.0, 0))
    torch.cuda.synchronize()
    s = cfg_out.cpu()[0]
    assert torch.isfinite(s[2047]) and torch.isneginf(s[2048:2051]).all()
    if width > 2051:
        assert torch.isfinite(s[2051])  # the backbone EOS class stays
