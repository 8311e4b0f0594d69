"""Parity at the lengths the benchmark configs run, on the GPU.

The short model tests stop at a few dozen positions.  These follow the decode
attention past the point where one CTA per KV group stops walking the whole
context (128 positions) and the split / last-CTA merge path takes over, the
prefill in one 2048-token chunk and in two, the causal tensor-core attention
over hundreds and thousands of queries, and the full 32-layer c5 model at its
full context.  References: the CPU oracle's refForward (main.zig:334-541),
its attentionPrefill (cpu.zig:165-217), and the engine's own property that a
batched prefill and per-token decoding agree (engine.zig:1707-1782).

Where the oracle would need minutes (a 4096-token CPU prefill through wide
MLPs), the model keeps the config's attention geometry and hidden width and
narrows what the check does not depend on (layers, vocabulary, MLP width), as
each test says.  Forced tokens are seeded random ids rather than greedy ones
where the oracle's logits are not computed at every step: the check is the
same (both sides run the same inputs), without an lm_head per step on the CPU.
"""
import os

import numpy as np
import pytest

from anedvd_b200 import engine as E
from anedvd_b200 import synth
from oracle import oracle as orc

from .gpu_util import dev, empty, host, lib, ptr, rel_err

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-3
KERNEL_TOL = 1e-3
THREADS = os.cpu_count() or 8


def _ids(vocab, n, seed):
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.uint32)


def _margin_ok(logits, tol):
    top = np.sort(logits)[-2:]
    return (top[1] - top[0]) > tol * np.max(np.abs(logits))


def _run(model, n_prompt, n_decode, compare_every=1, max_chunk=2048, greedy=True, seed=0):
    """Prefill n_prompt tokens on the GPU (batched, chunks of max_chunk) and on
    the oracle (token by token), then n_decode teacher-forced steps; compare the
    last prompt position and every `compare_every`-th decode step.  Returns the
    largest logits error and the number of positions compared."""
    cfg = model.cfg
    ref = orc.Model(cfg, threads=THREADS, max_seq=n_prompt + n_decode + 1)
    ref.load(model)
    eng = E.Engine.from_synth(model, max_seq=n_prompt + n_decode + 1, max_chunk=max_chunk)
    ids = _ids(cfg.vocab, n_prompt, 1000 + seed)
    forced = _ids(cfg.vocab, n_decode, 2000 + seed)
    for p, t in enumerate(ids):
        want = ref.forward(int(t), p, want_logits=p == n_prompt - 1)
    got, am = eng.prefill(ids, 0)
    errs = [rel_err(got, want)]
    if _margin_ok(want, LOGIT_TOL):
        assert am == orc.argmax(want)
    tok = orc.argmax(want) if greedy else int(forced[0])
    for s in range(n_decode):
        pos = n_prompt + s
        check = greedy or (s + 1) % compare_every == 0 or s == n_decode - 1
        want = ref.forward(tok, pos, want_logits=check)
        got, am = eng.forward(tok, pos, want_logits=check)
        if check:
            errs.append(rel_err(got, want))
            if _margin_ok(want, LOGIT_TOL):
                assert am == orc.argmax(want), (s, am, orc.argmax(want))
        tok = orc.argmax(want) if greedy else int(forced[(s + 1) % n_decode])
    eng.close()
    return max(errs), len(errs)


def test_decode_crosses_the_direct_attention_limit():
    """100 prompt positions, then 60 greedy steps: decode attention runs one CTA
    per KV group up to 128 positions and splits with a merge after that; every
    step is compared."""
    e, n = _run(synth.model("smollm2-135m", layers=2, vocab=1024), 100, 60)
    assert n == 61 and e < LOGIT_TOL, e


def test_c3_prompt_203_and_256_decode_steps_every_step():
    """Qwen2.5-0.5B shape (c3) at full width and vocabulary, 2 layers: the
    203-token prompt in one tensor-core chunk, then 256 greedy steps, each
    compared (decode positions 203-458, all on the split path)."""
    e, n = _run(synth.model("qwen2.5-0.5b", layers=2, payload="tiled"), 203, 256)
    assert n == 257 and e < LOGIT_TOL, e


def test_c4_prompt_2048_in_one_chunk():
    """Qwen2.5-1.5B shape (c4): hidden 1536, 12/2 heads of 128, full MLP width,
    1 layer, vocabulary cut to 4096.  The 2048-token prompt is one prefill
    chunk; 256 decode steps follow, compared at the last prompt position and
    every 32nd step."""
    m = synth.model("qwen2.5-1.5b", layers=1, vocab=4096, payload="tiled")
    e, n = _run(m, 2048, 256, compare_every=32, greedy=False, seed=4)
    assert n == 9 and e < LOGIT_TOL, e


def test_c5_prompt_4096_in_two_chunks():
    """Llama-3-8B shape (c5): hidden 4096, 32/8 heads of 128, 1 layer, MLP width
    cut to 1024 and vocabulary to 4096 (the oracle's CPU prefill of 4096
    positions stays under a minute).  The prompt runs as two 2048-token chunks,
    the second attending to the first through the cache; 64 decode steps
    follow, compared at the last prompt position and every 16th step."""
    m = synth.model("llama3-8b", layers=1, vocab=4096, inter=1024, payload="tiled")
    e, n = _run(m, 4096, 64, compare_every=16, greedy=False, seed=5)
    assert n == 5 and e < LOGIT_TOL, e


def test_c5_full_depth_at_full_context():
    """The whole c5 model (32 layers, vocabulary 128256) decoding at positions
    4096-4099, every step compared.  Both sides start from the same KV cache:
    4096 seeded fp16 rows per layer written into the engine (cuq_kv_write) and
    into the oracle, so the oracle does not have to prefill 4096 positions
    through 32 layers; the prefill itself is checked by the tests above."""
    m = synth.model("llama3-8b", payload="tiled")
    cfg = m.cfg
    n_ctx, n_dec = 4096, 4
    ref = orc.Model(cfg, threads=THREADS, max_seq=n_ctx + n_dec + 1)
    ref.load(m)
    eng = E.Engine.from_synth(m, max_seq=n_ctx + n_dec + 1, max_chunk=512)
    kvd = cfg.kv_heads * cfg.head_dim
    rng = np.random.default_rng(77)
    for layer in range(cfg.layers):
        k = (rng.standard_normal((n_ctx, kvd), dtype=np.float32) * 2.0).astype(np.float16).view(np.uint16)
        v = rng.standard_normal((n_ctx, kvd), dtype=np.float32).astype(np.float16).view(np.uint16)
        ref.set_kv(layer, 0, k, v)
        eng.kv_write(layer, 0, k, v)
    back_k, back_v = eng.kv_read(cfg.layers - 1, 0, n_ctx)
    assert np.array_equal(back_k, k) and np.array_equal(back_v, v)
    tok, errs = 11, []
    for s in range(n_dec):
        want = ref.forward(tok, n_ctx + s)
        got, am = eng.forward(tok, n_ctx + s)
        errs.append(rel_err(got, want))
        if _margin_ok(want, LOGIT_TOL):
            assert am == orc.argmax(want)
        tok = orc.argmax(want)
    eng.close()
    assert max(errs) < LOGIT_TOL, errs


def test_prefill_equals_per_token_decode_over_320_positions():
    """engine.zig:1707-1782's property at a length where decode attention
    splits: the batched prefill of 320 tokens and 320 single decode steps give
    the same last-position logits and the same KV cache rows."""
    m = synth.model("qwen2.5-0.5b", layers=2, vocab=1024)
    ids = _ids(m.cfg.vocab, 320, 9)
    a = E.Engine.from_synth(m, max_seq=336, max_chunk=2048)
    b = E.Engine.from_synth(m, max_seq=336, max_chunk=2048)
    la, _ = a.prefill(ids, 0)
    for p, t in enumerate(ids):
        lb, _ = b.forward(int(t), p)
    assert rel_err(la, lb) < LOGIT_TOL
    for layer in range(m.cfg.layers):
        ka, va = a.kv_read(layer, 0, 320)
        kb, vb = b.kv_read(layer, 0, 320)
        fa = ka.view(np.float16).astype(np.float32)
        fb = kb.view(np.float16).astype(np.float32)
        assert rel_err(fa, fb) < KERNEL_TOL
        assert rel_err(va.view(np.float16).astype(np.float32), vb.view(np.float16).astype(np.float32)) < KERNEL_TOL
    a.close()
    b.close()


def test_kv_rows_match_reference_rope_and_cache():
    """Engine.ropeAndCache (engine.zig:952-970): the fp16 K/V rows the GPU
    writes at every prompt and decode position against the oracle's."""
    m = synth.model("smollm2-135m", layers=2, vocab=1024)
    ref = orc.Model(m.cfg, threads=THREADS, max_seq=200)
    ref.load(m)
    eng = E.Engine.from_synth(m, max_seq=200, max_chunk=2048)
    ids = _ids(m.cfg.vocab, 150, 12)
    for p, t in enumerate(ids):
        ref.forward(int(t), p, want_logits=False)
    eng.prefill(ids, 0)
    for s in range(20):  # decode rows too, past the direct limit
        ref.forward(5 + s, 150 + s, want_logits=False)
        eng.forward(5 + s, 150 + s, want_logits=False)
    for layer in range(m.cfg.layers):
        k, v = eng.kv_read(layer, 0, 170)
        for pos in range(170):
            rk, rv = ref.kv_row(layer, pos)
            f = lambda a: a.view(np.float16).astype(np.float32)
            assert rel_err(f(k[pos]), f(rk)) < KERNEL_TOL, (layer, pos)
            assert rel_err(f(v[pos]), f(rv)) < KERNEL_TOL, (layer, pos)
    eng.close()


@pytest.mark.parametrize("n,pos0,heads,kv_heads,hd", [
    (203, 0, 14, 2, 64),      # c3: the whole prompt in one chunk
    (2048, 0, 12, 2, 128),    # c4: one 2048 chunk
    (2048, 2048, 8, 2, 128),  # second chunk of a 4096 prompt (c5 group 4)
    (37, 5, 9, 3, 64),        # ragged tail after a short chunk (c2 group 3)
])
def test_attention_prefill_matches_reference(n, pos0, heads, kv_heads, hd):
    """The tensor-core causal attention (cuq_attention_prefill) against the
    restated cpu.attentionPrefill (cpu.zig:165-217), multi-tile causal masks."""
    L = lib()
    rng = np.random.default_rng(n + pos0 + heads)
    total = pos0 + n
    stride = total + 8
    q = rng.standard_normal((n, heads * hd), dtype=np.float32)
    k = (rng.standard_normal((total, kv_heads, hd), dtype=np.float32) * 0.5).astype(np.float16)
    v = rng.standard_normal((total, kv_heads, hd), dtype=np.float32).astype(np.float16)
    kd = np.zeros((kv_heads, stride, hd), np.float16)
    vd = np.zeros((kv_heads, stride, hd), np.float16)
    kd[:, :total] = k.transpose(1, 0, 2)
    vd[:, :total] = v.transpose(1, 0, 2)
    qd, kdd, vdd = dev(q), dev(kd.view(np.uint16)), dev(vd.view(np.uint16))
    out = empty(n * heads * hd)
    from anedvd_b200 import runtime as rt
    rt.check(L.cuq_attention_prefill(ptr(out), ptr(qd), ptr(kdd), ptr(vdd), n, pos0, stride, heads, kv_heads, hd,
                                     None))
    got = host(out).reshape(n, heads * hd)
    want = orc.attention_prefill(q, k.reshape(total, -1).view(np.uint16), v.reshape(total, -1).view(np.uint16),
                                 total, pos0, heads, kv_heads, hd, threads=THREADS)
    assert rel_err(got, want) < KERNEL_TOL
    # per query row too: a causal-mask error at one position would hide in the global max
    rows = np.max(np.abs(got - want), axis=1) / np.maximum(np.max(np.abs(want), axis=1), 1e-30)
    assert float(rows.max()) < 4 * KERNEL_TOL, int(rows.argmax())
