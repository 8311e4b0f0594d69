"""The device sampler (cuq_sample, cuq_generate_sampled) against the CPU
oracle's restatement of cpu.sampleProfiled / cpu.applyPenalties
(src/cpu.zig:529-721) and of Session.generate's sampling loop
(src/generate.zig:166-250).

Bars:
  * penalised logits bit-exact (the penalties are plain fp32 operations);
  * the LCG state identical after every call (a draw advances it once, greedy
    and degenerate cases not at all);
  * with top-k active and k <= 4096 the device repeats the reference's fp32
    steps in the reference's order: the token equals the oracle's unless the
    oracle's draw lands within 1e-5 (relative to the kept mass) of a boundary
    between two tokens (an expf rounding apart);
  * otherwise the mass is summed in fixed point: the device token must own the
    draw position r * sum of the reference's order, computed exactly (float64
    cumulative sums), within 1e-5 of the kept mass.
"""
import ctypes
import zlib

import numpy as np
import pytest

from anedvd_b200 import engine as E
from anedvd_b200 import runtime as rt
from anedvd_b200 import synth
from oracle import oracle as orc

from .gpu_util import dev, empty, host, lib, ptr

pytestmark = pytest.mark.gpu

SP = rt.CuqSamplerParams


def _params_pair(**kw):
    return SP(**kw), orc.SamplerParams(**kw)


def device_sample(logits, params, recent, rng):
    """One cuq_sample call: (token, rng after, penalised logits)."""
    L = lib()
    lg = dev(np.asarray(logits, dtype=np.float32))
    rc = np.asarray(recent, dtype=np.uint32)
    rd = dev(rc) if rc.size else None
    st = dev(np.array([rng], dtype=np.uint32))
    tok = empty(1, np.uint32)
    rt.check(L.cuq_sample(ptr(lg), lg.numel(), ctypes.byref(params), ptr(rd) if rd is not None else None, rc.size,
                          ptr(st), ptr(tok), None))
    return int(host(tok, np.uint32)[0]), int(host(st, np.uint32)[0]), host(lg)


def exact_draw(pen, params, rng_after):
    """The reference's draw done in float64 over its own order: (order, cumulative
    mass, target, kept mass, top-p boundary slack, top-k boundary slack)."""
    v = np.asarray(pen, dtype=np.float32)
    T = np.float32(params.temperature)
    maxv = np.float32(v.max())
    cut = np.float32(maxv - np.float32(params.min_keep_delta) * T)
    cand = np.nonzero(v >= cut)[0]
    k = params.top_k
    topk = 0 < k < cand.size
    desc = cand[np.lexsort((cand, -v[cand].astype(np.float64)))]
    if topk:
        order = desc[:k]
        kslack = float(v[desc[k - 1]]) - float(v[desc[k]])
    else:
        order = cand
        kslack = np.inf
    p = np.exp((v[order] - maxv) / T).astype(np.float64)
    top_p = params.top_p if params.top_p > 0 else 1.0
    top_p = min(top_p, 1.0)
    pslack = np.inf
    if top_p < 1.0:
        if not topk:
            o = np.lexsort((order, -p))
            order, p = order[o], p[o]
        c = np.cumsum(p) / p.sum()
        j = int(np.searchsorted(c, top_p - 1e-12))
        j = min(j, p.size - 1)
        pslack = min(abs(c[j] - top_p), abs((c[j - 1] if j else 0.0) - top_p))
        order, p = order[:j + 1], p[:j + 1]
    S = p.sum()
    r = (rng_after >> 8) / 16777216.0
    return order, np.cumsum(p), r * S, S, pslack, kslack


LOGITS = {
    "model": lambda rng, n: (rng.standard_normal(n) * 2.0).astype(np.float32),
    "peaked": lambda rng, n: np.where(rng.random(n) < 1e-4, 15.0, rng.standard_normal(n) * 3.0).astype(np.float32),
    "ties": lambda rng, n: (rng.integers(0, 1001, size=n) * 0.01).astype(np.float32),
    "flat": lambda rng, n: (rng.standard_normal(n) * 0.05).astype(np.float32),
}

PARAMS = {
    "default": dict(temperature=0.7, top_k=40),
    "k1": dict(temperature=1.0, top_k=1),
    "k4096": dict(temperature=1.0, top_k=4096),
    "k5000": dict(temperature=1.0, top_k=5000),
    "pure": dict(temperature=1.0),
    "top_p": dict(temperature=1.0, top_p=0.9),
    "k_and_p": dict(temperature=0.8, top_k=40, top_p=0.9),
    "penalties": dict(temperature=0.7, top_k=40, repetition_penalty=1.3, presence_penalty=0.4,
                      frequency_penalty=0.25),
    "penalties_pure": dict(temperature=1.0, repetition_penalty=1.3, frequency_penalty=0.1),
    "greedy_penalised": dict(temperature=0.0, repetition_penalty=1.5),
    "delta2": dict(temperature=1.0, min_keep_delta=2.0),
}

CASES = [
    (151936, "model", "default"), (151936, "model", "pure"), (151936, "model", "top_p"),
    (151936, "flat", "top_p"), (151936, "flat", "pure"), (151936, "ties", "default"),
    (151936, "ties", "top_p"), (128256, "model", "k_and_p"), (128256, "peaked", "top_p"),
    (128256, "model", "k4096"), (128256, "model", "k5000"), (128256, "ties", "k5000"),
    (128256, "model", "penalties"), (49152, "model", "penalties_pure"), (49152, "model", "greedy_penalised"),
    (49152, "peaked", "k1"), (49152, "model", "delta2"), (1000, "model", "default"), (1000, "flat", "top_p"),
    (1000, "ties", "pure"), (327680, "model", "default"), (327680, "flat", "k_and_p"),
]


@pytest.mark.parametrize("vocab,dist,pname", CASES, ids=["%d-%s-%s" % c for c in CASES])
def test_sample_matches_reference(vocab, dist, pname):
    kw = PARAMS[pname]
    dp, op = _params_pair(**kw)
    rng = np.random.default_rng(zlib.crc32(("%d-%s-%s" % (vocab, dist, pname)).encode()))
    exact_path = 0 < kw.get("top_k", 0) <= 4096
    state = 0x12345678
    near = 0
    for trial in range(12):
        logits = LOGITS[dist](rng, vocab)
        window = rng.integers(0, vocab, size=64).astype(np.uint32)
        window[::3] = window[0]  # repeated ids
        if not any(kw.get(x, d) != d for x, d in (("repetition_penalty", 1.0), ("presence_penalty", 0.0),
                                                  ("frequency_penalty", 0.0))):
            window = window[:0]
        want, want_state, info, want_pen = orc.sample(logits, op, window, state)
        got, got_state, got_pen = device_sample(logits, dp, window, state)
        assert np.array_equal(got_pen.view(np.uint32), want_pen.view(np.uint32)), "penalties differ"
        assert got_state == want_state, (trial, got_state, want_state)
        if kw["temperature"] <= 0 or info.path != 3:
            assert got == want, (trial, got, want, info.path)
        elif exact_path:
            if got != want:
                assert info.draw_margin < 1e-5, (trial, got, want, info.draw_margin)
                near += 1
        else:
            order, C, target, S, pslack, kslack = exact_draw(want_pen, op, want_state)
            pos = np.nonzero(order == got)[0]
            if pos.size == 0:
                # outside the kept set: only next to an ambiguous top-p or top-k cut
                assert pslack < 1e-5 or kslack == 0.0, (trial, got, pslack, kslack)
                near += 1
            else:
                j = int(pos[0])
                lo = C[j - 1] if j else 0.0
                tol = 1e-5 * S
                assert lo - tol <= target <= C[j] + tol or pslack < 1e-5, (trial, got, lo, target, C[j])
        state = want_state
    assert near <= 2


def test_reference_unit_cases_on_device():
    """cpu.zig:1054-1119 through cuq_sample."""
    assert device_sample([0.1, 5.0, 0.2], SP(temperature=0), [], 1)[0] == 1
    s = 1
    for _ in range(16):
        t, s, _ = device_sample([0.1, 5.0, 4.9], SP(temperature=1.0, top_k=1), [], s)
        assert t == 1
    s = 7
    for _ in range(16):
        t, s, _ = device_sample([20.0, 0.0, 0.0], SP(temperature=1.0, top_p=0.1), [], s)
        assert t == 0
    s, counts = 12345, [0] * 4
    for _ in range(400):
        t, s, _ = device_sample([1.0] * 4, SP(temperature=1.0, top_p=0.9), [], s)
        counts[t] += 1
    assert all(c > 50 for c in counts)
    logits = np.array([i % 7 for i in range(64)], dtype=np.float32)
    for p in (SP(temperature=1.0, repetition_penalty=0.0, top_p=0.9),
              SP(temperature=1.0, repetition_penalty=-1.0, top_p=0.9),
              SP(temperature=1.0, repetition_penalty=0.0, top_p=0.0)):
        t, _, after = device_sample(logits, p, [1, 2, 3], 7)
        assert 0 <= t < 64 and np.all(np.isfinite(after))


def test_sample_rejects_oversized_inputs():
    L = lib()
    lg = empty(16)
    st = dev(np.array([1], dtype=np.uint32))
    tok = empty(1, np.uint32)
    p = SP()
    assert L.cuq_sample(ptr(lg), rt.SAMPLE_MAX_VOCAB + 32, ctypes.byref(p), None, 0, ptr(st), ptr(tok),
                        None) == rt.EINVAL
    rec = empty(16, np.uint32)
    assert L.cuq_sample(ptr(lg), 16, ctypes.byref(p), ptr(rec), rt.SAMPLE_MAX_WINDOW + 1, ptr(st), ptr(tok),
                        None) == rt.EINVAL


def _oracle_generate(ref, ids, n_decode, op, seed, window, forced=None, tol_margin=5e-3):
    """Session.generate's loop on the oracle, teacher-forced with `forced` (the
    device's tokens) so one near-boundary draw does not derail the rest: the
    list of (oracle token, whether a mismatch there is excusable)."""
    for p, t in enumerate(ids):
        logits = ref.forward(int(t), p)
    recent = list(ids[-window:]) if window else []
    st = seed
    out = []
    for s in range(n_decode):
        tok, st, info, _ = orc.sample(logits, op, np.array(recent, dtype=np.uint32), st)
        scale = float(np.max(np.abs(logits)))
        excuse = (info.path == 3 and (info.draw_margin < tol_margin or info.top_p_margin < tol_margin
                                      or info.topk_gap < 2e-3 * scale))
        out.append((tok, excuse))
        nxt = int(forced[s]) if forced is not None else tok
        if window:
            if len(recent) >= window:
                recent.pop(0)
            recent.append(nxt)
        if s + 1 < n_decode:
            logits = ref.forward(nxt, len(ids) + s)
    return out


@pytest.mark.parametrize("pname", ["default", "k_and_p", "penalties", "top_p"])
def test_generate_sampled_matches_oracle(pname):
    kw = PARAMS[pname]
    dp, op = _params_pair(**kw)
    m = synth.model("smollm2-135m", layers=2, vocab=1024)
    n_prompt, n_decode, seed, window = 12, 24, 0xC0FFEE, 16
    ids = np.random.default_rng(5).integers(0, 1024, size=n_prompt).astype(np.uint32)
    eng = E.Engine.from_synth(m, max_seq=64, device=0)
    sess = E.Session(eng, 64)
    got = sess.generate(ids, n_decode, sampler=dp, seed=seed, penalty_window=window)
    ref = orc.Model(m.cfg, threads=4, max_seq=64)
    ref.load(m)
    want = _oracle_generate(ref, ids, n_decode, op, seed, window, forced=got)
    bad = [(s, int(g), w) for s, (g, (w, ex)) in enumerate(zip(got, want)) if g != w and not ex]
    assert not bad, bad
    assert sum(int(g) == w for g, (w, _) in zip(got, want)) >= n_decode - 2
    # the same call again: same tokens (the seed restarts the LCG)
    sess.reset()
    again = sess.generate(ids, n_decode, sampler=dp, seed=seed, penalty_window=window)
    assert np.array_equal(got, again)
    eng.close()


def test_generate_sampled_graph_and_eager_agree():
    dp = SP(temperature=0.9, top_k=50, top_p=0.95, repetition_penalty=1.1)
    m = synth.model("qwen2.5-0.5b", layers=2, vocab=2048)
    ids = np.random.default_rng(9).integers(0, 2048, size=20).astype(np.uint32)
    outs = []
    for graphs in (True, False):
        eng = E.Engine.from_synth(m, max_seq=64, device=0, use_graphs=graphs)
        outs.append(E.Session(eng, 64).generate(ids, 30, sampler=dp, seed=77, penalty_window=32))
        eng.close()
    assert np.array_equal(outs[0], outs[1])


def test_generate_sampled_reuses_the_prefix():
    """A growing transcript prefills only its new suffix (generate.zig:187-192);
    the tokens match a fresh session's.  Greedy after a repetition penalty, so
    the draw goes through the device sampler and its window but has no random
    part that a last-bit difference between decode-written and prefill-written
    K/V rows could tip."""
    dp = SP(temperature=0.0, repetition_penalty=1.3)
    m = synth.model("smollm2-135m", layers=2, vocab=1024)
    rng = np.random.default_rng(3)
    first = rng.integers(0, 1024, size=10).astype(np.uint32)
    eng = E.Engine.from_synth(m, max_seq=96, device=0)
    sess = E.Session(eng, 96)
    out1 = sess.generate(first, 8, sampler=dp, seed=5)
    follow = np.concatenate([first, out1, rng.integers(0, 1024, size=6).astype(np.uint32)])
    out2 = sess.generate(follow, 8, sampler=dp, seed=6)
    assert sess.last["prefill_reused"] == first.size + out1.size - 1
    eng2 = E.Engine.from_synth(m, max_seq=96, device=0)
    fresh = E.Session(eng2, 96).generate(follow, 8, sampler=dp, seed=6)
    assert np.array_equal(out2, fresh)
    eng.close()
    eng2.close()


def test_sample_draw_time():
    """One draw over a 151936-entry vocabulary (the c3/c4 lm_head) with the
    default sampler, timed on the device: well under a decode step."""
    import torch
    L = lib()
    logits = dev((np.random.default_rng(0).standard_normal(151936) * 2).astype(np.float32))
    st = dev(np.array([1], dtype=np.uint32))
    tok = empty(1, np.uint32)
    p = SP(temperature=0.7, top_k=40)
    for _ in range(3):
        rt.check(L.cuq_sample(ptr(logits), 151936, ctypes.byref(p), None, 0, ptr(st), ptr(tok), None))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(50):
        L.cuq_sample(ptr(logits), 151936, ctypes.byref(p), None, 0, ptr(st), ptr(tok), None)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / 50
    print("sample draw: %.1f us" % us)
    assert us < 200
