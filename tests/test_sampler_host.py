"""The sampler's CPU restatement (oracle orc_sample / orc_apply_penalties)
pinned to the reference's own sampler tests (src/cpu.zig:1022-1119 and
:1470-1500), plus the properties the device sampler's tests rely on.  CPU only."""
import numpy as np

from oracle import oracle as orc

P = orc.SamplerParams


def test_temperature_zero_is_greedy():  # cpu.zig:1054-1059
    assert orc.sample([0.1, 5.0, 0.2], P(temperature=0), [], 1)[0] == 1


def test_top_k_one_picks_the_maximum():  # cpu.zig:1061-1068
    seed = 1
    for _ in range(16):
        tok, seed, _, _ = orc.sample([0.1, 5.0, 4.9], P(temperature=1.0, top_k=1), [], seed)
        assert tok == 1


def test_top_p_keeps_only_the_dominant_token():  # cpu.zig:1070-1077
    seed = 7
    for _ in range(16):
        tok, seed, _, _ = orc.sample([20.0, 0.0, 0.0], P(temperature=1.0, top_p=0.1), [], seed)
        assert tok == 0


def test_every_drawn_token_has_nonzero_probability():  # cpu.zig:1079-1090
    seed, counts = 12345, [0] * 4
    for _ in range(4000):
        tok, seed, _, _ = orc.sample([1.0] * 4, P(temperature=1.0, top_p=0.9), [], seed)
        counts[tok] += 1
    assert all(c > 500 for c in counts)


def test_invalid_parameters_give_a_usable_answer():  # cpu.zig:1092-1119
    logits = np.array([i % 7 for i in range(64)], dtype=np.float32)
    for params in (P(temperature=1.0, repetition_penalty=0.0, top_p=0.9),
                   P(temperature=1.0, repetition_penalty=-1.0, top_p=0.9),
                   P(temperature=1.0, repetition_penalty=0.0, top_p=0.0)):
        tok, _, _, after = orc.sample(logits, params, [1, 2, 3], 7)
        assert 0 <= tok < 64
        assert np.all(np.isfinite(after))


def test_penalties():  # cpu.zig:1121-1134
    v = orc.apply_penalties([5.0, 4.0], P(repetition_penalty=2.0), [0])
    assert abs(v[0] - 2.5) < 1e-6
    v = orc.apply_penalties([5.0, 4.0], P(presence_penalty=1.0, frequency_penalty=0.5), [0, 0])
    assert abs(v[0] - 3.0) < 1e-6  # presence once, frequency twice
    v = orc.apply_penalties([5.0, 4.0], P(repetition_penalty=2.0), [1])
    assert abs(v[0] - 5.0) < 1e-6


def test_top_k_draws_stay_at_or_above_the_kth_value():  # cpu.zig:1470-1500
    rng = np.random.default_rng(0)
    for _ in range(10):
        logits = (rng.integers(0, 1001, size=4000) * 0.01).astype(np.float32)  # many ties
        threshold = np.sort(logits)[::-1][7]
        seed = int(rng.integers(1, 2**32)) | 1
        for _ in range(20):
            tok, seed, _, _ = orc.sample(logits, P(temperature=1.0, top_k=8, top_p=1.0), [], seed)
            assert logits[tok] >= threshold


def test_penalties_depend_only_on_counts():
    """A token's penalised logit depends on how often it occurs in the window,
    not where: the device sampler applies them per distinct id."""
    rng = np.random.default_rng(1)
    logits = rng.normal(size=300).astype(np.float32)
    window = rng.integers(0, 300, size=200).astype(np.uint32)
    p = P(repetition_penalty=1.3, presence_penalty=0.4, frequency_penalty=0.25)
    a = orc.apply_penalties(logits, p, window)
    b = orc.apply_penalties(logits, p, rng.permutation(window))
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_rng_advances_once_per_draw_only():
    tok, st, info, _ = orc.sample([0.1, 5.0, 0.2], P(temperature=0.0), [], 99)
    assert st == 99 and info.path == 0
    tok, st, info, _ = orc.sample([0.1, 5.0, 0.2], P(temperature=1.0), [], 99)
    assert st == (99 * 1664525 + 1013904223) % 2**32 and info.path == 3
