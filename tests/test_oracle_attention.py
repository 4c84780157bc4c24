"""The oracle's cacheWrite and attention (restated from ops/CpuAttention.scala:
163-288) against a direct numpy statement of the same definition, and the
F32-to-F16 rounding against IEEE round-to-nearest-even (numpy's cast)."""

import math

import numpy as np

import oracle


def test_f16_rounding_is_ieee_nearest_even():
    rng = np.random.default_rng(3)
    scales = rng.choice([1e-8, 1e-6, 1e-3, 1.0, 100.0, 6e4], 50000)
    x = (rng.standard_normal(50000) * scales).astype(np.float32)
    x[:6] = [0.0, -0.0, 65504.0, 65520.0, 5.96e-8, 2.98e-8]
    with np.errstate(over="ignore"):
        np.testing.assert_array_equal(oracle.f32_to_f16(x), x.astype(np.float16).view(np.uint16))


def test_attention_is_the_softmax_of_the_definition():
    rng = np.random.default_rng(4)
    pages, page_size, kv_heads, dim, q_heads, key_count, tokens = 6, 16, 2, 64, 4, 70, 3
    table = rng.permutation(pages).astype(np.int32)
    keys = np.zeros((pages, page_size, kv_heads, dim), dtype=np.uint16)
    values = np.zeros((pages, kv_heads, dim, page_size), dtype=np.uint16)
    k = rng.standard_normal((key_count, kv_heads, dim)).astype(np.float32)
    v = rng.standard_normal((key_count, kv_heads, dim)).astype(np.float32)
    oracle.cache_write(k, v, keys, values, page_size, table, 0)
    # the layout: position p of head h lives at page table[p // 16], offset p % 16
    for p in (0, 15, 16, 69):
        page, offset = table[p // page_size], p % page_size
        np.testing.assert_array_equal(keys[page, offset], k[p].astype(np.float16).view(np.uint16))
        np.testing.assert_array_equal(values[page, :, :, offset],
                                      v[p].astype(np.float16).view(np.uint16))
    q = rng.standard_normal((tokens, q_heads, dim)).astype(np.float32)
    start, scale = key_count - tokens, 1 / math.sqrt(dim)
    got = oracle.attention(q, keys, values, page_size, kv_heads, table, start, key_count, scale)
    kf, vf = k.astype(np.float16).astype(np.float64), v.astype(np.float16).astype(np.float64)
    for t in range(tokens):
        for h in range(q_heads):
            g = h // (q_heads // kv_heads)
            seen = start + t + 1
            scores = kf[:seen, g] @ q[t, h].astype(np.float64) * np.float64(np.float32(scale))
            w = np.exp(scores - scores.max())
            expected = (w @ vf[:seen, g]) / w.sum()
            np.testing.assert_allclose(got[t, h], expected.astype(np.float32), rtol=1e-6, atol=1e-7)


# The known answers of the reference's AttentionReferenceTests.scala:47-111,
# held by the oracle (the GPU kernel holds them in test_gpu_attention.py).

def one_key_cache():
    """A cache of one page whose position 0 holds k = 0.5, v = d / 8 (exact
    in F16), 16 dimensions, one key head (AttentionReferenceTests.scala:47-58)."""
    keys = np.zeros((1, 16, 1, 16), dtype=np.uint16)
    values = np.zeros((1, 1, 16, 16), dtype=np.uint16)
    value = (np.arange(16) / 8).astype(np.float32)
    oracle.cache_write(np.full((1, 1, 16), 0.5, np.float32), value.reshape(1, 1, 16), keys,
                       values, 16, np.zeros(1, np.int32), 0)
    return keys, values, value


def test_one_visible_key_gives_its_value():
    keys, values, value = one_key_cache()
    q = np.ones((1, 1, 16), np.float32)
    out = oracle.attention(q, keys, values, 16, 1, np.zeros(1, np.int32), 0, 1, 0.25)
    np.testing.assert_array_equal(out.reshape(16), value)
    # a sink of the same logit as the key (q.k x scale = 2) takes half the weight
    out = oracle.attention(q, keys, values, 16, 1, np.zeros(1, np.int32), 0, 1, 0.25,
                           sinks=np.array([2.0], np.float32))
    np.testing.assert_array_equal(out.reshape(16), value / 2)


def plain_case(rng_seed=7, shuffled=False, tokens=5, window=0, queries=None):
    """AttentionReferenceTests' `plain` case: 5 tokens over 40 keys, 4 query
    heads over 2 key heads of 16, causal, pages of 16 (seeded here with
    numpy: the shapes and the invariants are the reference's, not its draws)."""
    rng = np.random.default_rng(rng_seed)
    key_count, q_heads, kv_heads, dim, page_size = 40, 4, 2, 16, 16
    pages = 3
    k = rng.standard_normal((key_count, kv_heads, dim)).astype(np.float32)
    v = rng.standard_normal((key_count, kv_heads, dim)).astype(np.float32)
    drawn = rng.standard_normal((5, q_heads, dim)).astype(np.float32)
    q = drawn if queries is None else queries
    table = np.array([2, 0, 1] if shuffled else [0, 1, 2], np.int32)
    keys = np.zeros((pages, page_size, kv_heads, dim), np.uint16)
    values = np.zeros((pages, kv_heads, dim, page_size), np.uint16)
    oracle.cache_write(k, v, keys, values, page_size, table, 0)
    q = q[-tokens:]
    return oracle.attention(q, keys, values, page_size, kv_heads, table, key_count - tokens,
                            key_count, 1 / math.sqrt(dim), True, window), q


def test_page_order_does_not_matter():
    plain, _ = plain_case()
    shuffled, _ = plain_case(shuffled=True)
    np.testing.assert_array_equal(plain, shuffled)


def test_prefill_then_decode_equals_one_longer_prefill():
    prefill, q = plain_case()
    decode, _ = plain_case(tokens=1, queries=q)
    np.testing.assert_array_equal(prefill[-1:], decode)


def test_a_whole_window_changes_nothing_and_a_narrow_one_does():
    full, _ = plain_case()
    np.testing.assert_array_equal(plain_case(window=40)[0], full)
    assert not np.array_equal(plain_case(window=8)[0], full)
