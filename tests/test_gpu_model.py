"""Whole-model parity on the GPU: the device-resident engine against the CPU
oracle's refForward (teacher-forced, every position compared).

Bars: logits within 2e-3 relative error
(rel = max|a-b| / max|b|, main.zig:1920-1930); greedy tokens identical wherever
the oracle's top-2 margin exceeds that tolerance.
"""
import zlib

import numpy as np
import pytest

from anedvd_b200 import engine as E
from anedvd_b200 import runtime as rt
from anedvd_b200 import synth
from oracle import oracle as orc

from .gpu_util import rel_err

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-3

SMALL = [("smollm2-135m", dict(layers=2, vocab=1024)), ("qwen2.5-0.5b", dict(layers=2, vocab=1024)),
         ("qwen2.5-1.5b", dict(layers=3, vocab=1024)), ("llama3-8b", dict(layers=1, vocab=1024))]


def _prompt(cfg, n, salt=0):
    rng = np.random.default_rng(1234 + salt)
    return rng.integers(0, cfg.vocab, size=n).astype(np.uint32)


def _margin_ok(logits, tol):
    top = np.sort(logits)[-2:]
    return (top[1] - top[0]) > tol * np.max(np.abs(logits))


def _compare(model, n_prompt, n_decode, threads=8, use_graphs=True, max_chunk=512, decode_kernel=rt.DECODE_AUTO):
    cfg = model.cfg
    ref = orc.Model(cfg, threads=threads, max_seq=n_prompt + n_decode + 1)
    ref.load(model)
    eng = E.Engine.from_synth(model, max_seq=n_prompt + n_decode + 1, use_graphs=use_graphs, max_chunk=max_chunk,
                              decode_kernel=decode_kernel)
    ids = _prompt(cfg, n_prompt)
    errs = []
    # prefill: the reference's CPU path feeds the prompt token by token (main.zig:1255-1262)
    for p, t in enumerate(ids):
        want = ref.forward(int(t), p)
    got, am = eng.prefill(ids, 0)
    errs.append(rel_err(got, want))
    if _margin_ok(want, LOGIT_TOL):
        assert am == orc.argmax(want)
    # decode, teacher-forced with the oracle's greedy tokens
    tok = orc.argmax(want)
    for s in range(n_decode):
        pos = n_prompt + s
        want = ref.forward(tok, pos)
        got, am = eng.forward(tok, pos)
        errs.append(rel_err(got, want))
        if _margin_ok(want, LOGIT_TOL):
            assert am == orc.argmax(want), (s, am, orc.argmax(want))
        tok = orc.argmax(want)
    eng.close()
    return max(errs)


DECODE = [("per_op", rt.DECODE_PER_OP), ("persistent", rt.DECODE_PERSISTENT)]


@pytest.mark.parametrize("dk", [d[1] for d in DECODE], ids=[d[0] for d in DECODE])
@pytest.mark.parametrize("name,kw", SMALL, ids=[s[0] for s in SMALL])
def test_small_models_match_reference(name, kw, dk):
    e = _compare(synth.model(name, **kw), n_prompt=9, n_decode=6, decode_kernel=dk)
    assert e < LOGIT_TOL, e


@pytest.mark.parametrize("name,kw", SMALL, ids=[s[0] for s in SMALL])
def test_persistent_generate_equals_single_steps(name, kw):
    """One persistent launch over many steps takes the same tokens as one launch
    per step, and as the per-op kernels wherever the oracle margin is clear."""
    m = synth.model(name, **kw)
    ids = _prompt(m.cfg, 6, salt=3)
    eng = E.Engine.from_synth(m, max_seq=64, decode_kernel=rt.DECODE_PERSISTENT)
    gen = list(E.Session(eng, 64).generate(ids, 20))
    eng.reset()
    _, am = eng.prefill(ids)
    steps = [am]
    for s in range(19):
        _, am = eng.forward(steps[-1], len(ids) + s)
        steps.append(am)
    assert gen == steps
    eng.close()
    per_op = E.Engine.from_synth(m, max_seq=64, decode_kernel=rt.DECODE_PER_OP)
    gen2 = list(E.Session(per_op, 64).generate(ids, 20))
    per_op.close()
    assert gen2 == gen


def test_smollm2_full_size_matches_reference():
    """SmolLM2-135M Q8_0 at full size (30 layers, vocab 49152), 16-token prompt."""
    e = _compare(synth.model("smollm2-135m"), n_prompt=16, n_decode=8)
    assert e < LOGIT_TOL, e


# Qwen2.5-0.5B Q8_0, Qwen2.5-1.5B and Llama-3-8B Q4_K_M at their full depth and vocabulary (Llama with 8 of
# its 32 layers, to keep the CPU oracle within a few GB of host memory).  The
# weights are "tiled" payloads: every block a real quantised block, the same
# bytes for the GPU and the oracle.
FULL = [("qwen2.5-0.5b", {}), ("qwen2.5-1.5b", {}), ("llama3-8b", dict(layers=8))]


@pytest.mark.parametrize("name,kw", FULL, ids=[f[0] for f in FULL])
def test_full_size_configs_match_reference(name, kw):
    import os
    m = synth.model(name, payload="tiled", **kw)
    e = _compare(m, n_prompt=12, n_decode=4, threads=os.cpu_count() or 8)
    assert e < LOGIT_TOL, e


@pytest.mark.parametrize("chunk", [1, 4, 7])
def test_chunked_prefill_matches_reference(chunk):
    """The prompt split into several tensor-core chunks (the last one ragged)."""
    e = _compare(synth.model("qwen2.5-0.5b", layers=2, vocab=1024), n_prompt=11, n_decode=3, max_chunk=chunk)
    assert e < LOGIT_TOL, e


def test_batched_prefill_cache_feeds_decode():
    """A prefill at start_pos > 0 after an earlier one: the KV cache rows written by
    the batched path are the ones the decode step reads."""
    m = synth.model("smollm2-135m", layers=2, vocab=1024)
    ref = orc.Model(m.cfg, threads=8, max_seq=32)
    ref.load(m)
    eng = E.Engine.from_synth(m, max_seq=32, max_chunk=8)
    a, b = _prompt(m.cfg, 6, 1), _prompt(m.cfg, 9, 2)
    eng.prefill(a, 0)
    got, _ = eng.prefill(b, len(a))
    for p, t in enumerate(np.concatenate([a, b])):
        want = ref.forward(int(t), p)
    assert rel_err(got, want) < LOGIT_TOL
    got, _ = eng.forward(7, len(a) + len(b))
    want = ref.forward(7, len(a) + len(b))
    assert rel_err(got, want) < LOGIT_TOL
    eng.close()


def test_graph_and_eager_agree():
    m = synth.model("qwen2.5-0.5b", layers=2, vocab=1024)
    ids = _prompt(m.cfg, 7)
    a = E.Engine.from_synth(m, max_seq=32, use_graphs=True)
    b = E.Engine.from_synth(m, max_seq=32, use_graphs=False)
    la, _ = a.prefill(ids)
    lb, _ = b.prefill(ids)
    assert np.array_equal(la, lb)


def test_device_generate_equals_step_by_step():
    m = synth.model("smollm2-135m", layers=2, vocab=1024)
    ids = _prompt(m.cfg, 5)
    eng = E.Engine.from_synth(m, max_seq=64)
    gen = E.Session(eng, 64).generate(ids, 12)
    eng.reset()
    _, am = eng.prefill(ids)
    steps = [am]
    for s in range(11):
        _, am = eng.forward(steps[-1], len(ids) + s)
        steps.append(am)
    assert list(gen) == steps


def test_gguf_loader_matches_upload(tmp_path):
    m = synth.model("qwen2.5-0.5b", layers=2, vocab=1024)
    path = str(tmp_path / "m.gguf")
    m.write_gguf(path)
    ids = _prompt(m.cfg, 6)
    a = E.Engine.from_gguf(path, max_seq=16)
    b = E.Engine.from_synth(m, max_seq=16)
    la, _ = a.prefill(ids)
    lb, _ = b.prefill(ids)
    assert np.array_equal(la, lb)
    assert a.cfg.rope_adjacent == 0 and a.cfg.tie_embeddings == 1 and a.cfg.vocab == 1024


def test_context_overflow_and_bad_token():
    m = synth.model("smollm2-135m", layers=1, vocab=1024)
    eng = E.Engine.from_synth(m, max_seq=8)
    with pytest.raises(rt.CuqError) as ei:
        eng.forward(1, 8)
    assert ei.value.code == rt.ECONTEXT  # error.ContextOverflow, engine.zig:549
    with pytest.raises(rt.CuqError) as ei:
        eng.prefill(np.arange(9, dtype=np.uint32))
    assert ei.value.code == rt.ECONTEXT  # engine.zig:981
    with pytest.raises(rt.CuqError) as ei:
        eng.forward(5000, 0)
    assert ei.value.code == rt.EINVAL
    # still usable afterwards
    lg, am = eng.forward(3, 0)
    assert np.isfinite(lg).all()


def test_missing_tensor_is_reported():
    L = rt.load()
    rt.init(0)
    import ctypes
    c = synth.CONFIGS["smollm2-135m"]
    cfg = rt.CuqConfig(hidden=c.hidden, layers=1, heads=c.heads, kv_heads=c.kv_heads, head_dim=c.head_dim,
                       inter=c.inter, vocab=1024, eps=c.eps, rope_theta=c.rope_theta, rope_adjacent=1,
                       tie_embeddings=1)
    opts = rt.CuqOptions(max_seq=8, max_chunk=8, use_graphs=1, tp_rank=0, tp_size=1)
    h = L.cuq_model_create(ctypes.byref(cfg), ctypes.byref(opts))
    assert h
    assert L.cuq_model_finalize(h) == rt.EINVAL
    assert "MissingTensor" in rt.last_error()
    L.cuq_model_free(h)


def test_profile_decode_table():
    """cuq_profile_decode (the per-kernel table): every node of every step is
    timed once per launch, the bytes follow the weights and the cached rows, and
    the decode state advances as with cuq_forward."""
    m = synth.model("qwen2.5-0.5b", layers=2, vocab=1024)
    ref = orc.Model(m.cfg, threads=8, max_seq=32)
    ref.load(m)
    eng = E.Engine.from_synth(m, max_seq=32)
    ids = _prompt(m.cfg, 5)
    for p, t in enumerate(ids):
        ref.forward(int(t), p)
    eng.prefill(ids)
    n = 3
    tab = eng.profile_decode(7, len(ids), n)
    c = m.cfg
    assert tab["qkv"][0] >= n * c.layers and tab["attention"][0] == n * c.layers
    assert tab["o"][0] == n * c.layers and tab["down"][0] == n * c.layers and tab["lm_head"][0] == n
    # norms that run as kernels of their own: none when every GEMV computes its
    # own input norm, or only the final one before the lm_head (TMA-fed GEMVs)
    assert tab["norm"][0] in (0, n)
    assert all(v[1] > 0 for k, v in tab.items() if v[0])
    kvd = c.kv_heads * c.head_dim
    want_kv = sum(2 * 2 * kvd * c.layers * (len(ids) + i + 1) for i in range(n))
    assert tab["attention"][2] == want_kv
    # the three profiled steps decoded tokens 7, then the greedy argmax: the next
    # forward continues from there like the oracle does
    tok = 7
    for i in range(n):
        tok = orc.argmax(ref.forward(tok, len(ids) + i))
    got, _ = eng.forward(tok, len(ids) + n)
    want = ref.forward(tok, len(ids) + n)
    assert rel_err(got, want) < LOGIT_TOL
    eng.close()


def test_session_reuses_the_kv_prefix_of_a_growing_transcript():
    """generate.zig:187-192: a second turn whose prompt extends the first turn's
    prompt and answer prefills only the new suffix, and decodes the same tokens
    as a fresh engine given the whole second prompt."""
    m = synth.model("smollm2-135m", layers=2, vocab=1024)
    eng = E.Engine.from_synth(m, max_seq=96)
    sess = E.Session(eng, 96)
    p1 = _prompt(m.cfg, 12, salt=7)
    t1 = sess.generate(p1, 8)
    assert sess.last["prefill_reused"] == 0
    p2 = np.concatenate([p1, t1, _prompt(m.cfg, 5, salt=8)])
    t2 = sess.generate(p2, 10)
    assert sess.last["prefill_reused"] == p1.size + t1.size - 1
    fresh = E.Engine.from_synth(m, max_seq=96)
    want = E.Session(fresh, 96).generate(p2, 10)
    assert list(t2) == list(want)
    # a prompt that does not cover the cache starts over
    t3 = sess.generate(p2[:10], 4)
    assert sess.last["prefill_reused"] == 0
    assert list(t3) == list(E.Session(fresh, 96).generate(p2[:10], 4))
    eng.close()
    fresh.close()


def test_model_with_raw_block_types_matches_reference():
    """A Llama-shaped model whose projections use the block types kept raw on
    the device (Q5_K, Q3_K, Q2_K, Q8_K, Q8_1): decode GEMVs through the element
    dequantiser, prefill GEMMs through the fp16 expansion, against refForward."""
    from .test_gpu_kernels import golden_blocks
    m = synth.model("llama3-8b", layers=2, vocab=1024, hidden=512, heads=4, kv_heads=2, inter=1024)
    mix = {"q": 13, "k": 11, "v": 10, "o": 15, "gate": 9, "up": 9, "down": 13}
    for t in m.tensors():
        if t.role in mix:
            t.ggml_type = mix[t.role]
            t.data = golden_blocks(t.ggml_type, t.rows * t.cols, zlib.crc32(t.name.encode()) % 1000, model_scale=True)
    e = _compare(m, n_prompt=9, n_decode=5)
    assert e < LOGIT_TOL, e


@pytest.mark.parametrize("linear_type", [1, 30], ids=["f16", "bf16"])
def test_hf_directory_matches_reference(linear_type, tmp_path):
    """load_hf.zig's path (config.json + sharded safetensors + index) uploaded raw:
    F16 / BF16 weights as on disk, rounded by the kernels as readF16 does,
    against refForward on the same weights."""
    from .hf_util import to_hf_types, write_hf_dir
    m = to_hf_types(synth.model("qwen2.5-0.5b", layers=2, vocab=1024), linear_type)
    path = write_hf_dir(m, str(tmp_path / "hf"), shards=3)
    ref = orc.Model(m.cfg, threads=8, max_seq=32)
    ref.load(m)
    eng = E.Engine.from_hf(path, max_seq=32)
    assert eng.cfg.rope_adjacent == 0 and eng.cfg.tie_embeddings == 1
    ids = _prompt(m.cfg, 7)
    for p, t in enumerate(ids):
        want = ref.forward(int(t), p)
    got, _ = eng.prefill(ids)
    assert rel_err(got, want) < LOGIT_TOL
    got, _ = eng.forward(3, len(ids))
    assert rel_err(got, ref.forward(3, len(ids))) < LOGIT_TOL
    eng.close()
