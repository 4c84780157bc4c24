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
