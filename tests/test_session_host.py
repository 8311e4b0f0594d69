"""Host logic of Session.generate that needs no GPU: the KV prefix reuse rule
(generate.zig:456-460 reuseLength), checked on the reference's own cases
(generate.zig:491-514)."""
from anedvd_b200.engine import reuse_length


def test_reuse_length_reference_cases():
    cache = [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 50, 51, 52, 53, 54, 55, 56]
    prompt = [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13]
    # the prompt matches the cache's first 13 entries, but the cache holds more
    assert reuse_length(cache, prompt) == 0
    # a longer prompt that covers the whole cache reuses all of it
    assert reuse_length(cache, prompt + [50, 51, 52, 53, 54, 55, 56, 60, 61]) == 20
    # partial coverage is never safe
    assert reuse_length(cache, prompt + [50, 51]) == 0
    # divergence at the first token
    assert reuse_length(cache, [9, 9, 9]) == 0
    # an empty cache: everything is new
    assert reuse_length([], prompt) == 0
