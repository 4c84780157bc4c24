"""Ops.cacheWrite and Ops.attention on the GPU against the oracle (the
reference's CpuAttention.cacheWrite/attention, ops/CpuAttention.scala:
181-288), over the reference's paged F16 cache layout.

cacheWrite is bit-exact (F32 to F16, nearest even). attention is held to
the benchmark's 1e-4 absolute + 1e-3 relative: the GPU sums in F32 where the CPU
sums in Double.
"""

import math

import numpy as np
import pytest
import torch

import oracle
from drift_b200.ops import Attention, CudaOps, KvCache
from tests.conftest import within

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    return CudaOps()


def filled_cache(rng, pages, page_size, kv_heads, dim, positions, table):
    """A cache whose first `positions` positions hold N(0, 1) keys and values,
    written by the oracle (numpy copies) and uploaded."""
    keys = np.zeros((pages, page_size, kv_heads, dim), dtype=np.uint16)
    values = np.zeros((pages, kv_heads, dim, page_size), dtype=np.uint16)
    k = rng.standard_normal((positions, kv_heads, dim)).astype(np.float32)
    v = rng.standard_normal((positions, kv_heads, dim)).astype(np.float32)
    oracle.cache_write(k, v, keys, values, page_size, table, 0)
    cache = KvCache(torch.from_numpy(keys.view(np.float16)).cuda(),
                    torch.from_numpy(values.view(np.float16)).cuda(), page_size)
    return keys, values, cache


@pytest.mark.parametrize("tokens,start,page_size,dim", [(1, 0, 16, 128), (1, 37, 16, 128),
                                                         (5, 30, 32, 64), (3, 100, 16, 256)])
def test_cache_write_is_bit_exact(ops, tokens, start, page_size, dim):
    rng = np.random.default_rng(tokens + start)
    kv_heads, pages = 4, 16
    table = rng.permutation(pages).astype(np.int32)
    keys = np.zeros((pages, page_size, kv_heads, dim), dtype=np.uint16)
    values = np.zeros((pages, kv_heads, dim, page_size), dtype=np.uint16)
    k = (rng.standard_normal((tokens, kv_heads, dim)) * 10).astype(np.float32)
    v = (rng.standard_normal((tokens, kv_heads, dim)) * 1e-3).astype(np.float32)
    cache = KvCache(torch.zeros(pages, page_size, kv_heads, dim, dtype=torch.float16).cuda(),
                    torch.zeros(pages, kv_heads, dim, page_size, dtype=torch.float16).cuda(),
                    page_size)
    ops.cache_write(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), cache,
                    torch.from_numpy(table).cuda(), start)
    oracle.cache_write(k, v, keys, values, page_size, table, start)
    np.testing.assert_array_equal(cache.keys.cpu().numpy().view(np.uint16), keys)
    np.testing.assert_array_equal(cache.values.cpu().numpy().view(np.uint16), values)


# (tokens, q_heads, kv_heads, dim, keys, page_size, causal, window, softcap, sinks)
CASES = [
    (1, 32, 8, 128, 1, 16, True, 0, None, False),       # first decode step
    (1, 32, 8, 128, 17, 16, True, 0, None, False),      # a partial page
    (1, 32, 8, 128, 300, 16, True, 0, None, False),     # several splits
    (1, 32, 8, 128, 4096, 16, True, 0, None, False),    # C4's context
    (1, 16, 2, 256, 1000, 32, True, 0, None, False),    # C5's full attention (group 8)
    (1, 16, 2, 256, 4096, 32, True, 0, None, False),    # C5's context: the separate join
    (1, 8, 8, 64, 129, 16, True, 0, None, False),
    (1, 10, 2, 80, 200, 16, True, 0, None, False),      # the 80-wide kernel
    (7, 32, 8, 128, 250, 16, True, 0, None, False),     # a prefill chunk, causal
    (4, 8, 2, 128, 300, 16, True, 64, None, False),     # sliding window
    (2, 8, 2, 128, 150, 16, True, 0, 30.0, True),       # softcap and sinks
    (3, 8, 4, 64, 40, 16, False, 0, None, False),       # not causal
]


@pytest.mark.parametrize("case", CASES, ids=[f"t{c[0]}h{c[1]}/{c[2]}d{c[3]}k{c[4]}" for c in CASES])
def test_attention_matches_the_oracle(ops, case):
    tokens, q_heads, kv_heads, dim, key_count, page_size, causal, window, softcap, sinks = case
    rng = np.random.default_rng(key_count * 7 + dim)
    table_pages = (key_count + page_size - 1) // page_size + 1
    pages = table_pages + 3
    table = rng.permutation(pages)[:table_pages].astype(np.int32)
    keys, values, cache = filled_cache(rng, pages, page_size, kv_heads, dim, key_count, table)
    q = rng.standard_normal((tokens, q_heads, dim)).astype(np.float32)
    sink_values = rng.standard_normal(q_heads).astype(np.float32) if sinks else None
    query_start = key_count - tokens if causal else 0
    scale = 1.0 / math.sqrt(dim)
    expected = oracle.attention(q, keys, values, page_size, kv_heads, table, query_start,
                                key_count, scale, causal, window, softcap, sink_values)
    out = torch.empty(tokens, q_heads, dim, device="cuda")
    ops.attention(torch.from_numpy(q).cuda(), cache, torch.from_numpy(table).cuda(), query_start,
                  key_count,
                  Attention(scale, causal, window or None, softcap,
                            None if sink_values is None else torch.from_numpy(sink_values).cuda()),
                  out)
    ok, _, _, summary = within(out.cpu().numpy(), expected, 1e-4, 1e-3)
    assert ok, summary


def test_attention_refuses_what_the_reference_refuses(ops):
    cache = KvCache.allocate(4, 16, 2, 128)
    table = torch.arange(4, dtype=torch.int32, device="cuda")
    q = torch.zeros(1, 6, 128, device="cuda")
    out = torch.empty_like(q)
    with pytest.raises(ValueError, match="query heads over"):
        ops.attention(q[:, :5], cache, table, 0, 1, Attention(1.0), out[:, :5])
    with pytest.raises(ValueError, match="past"):
        ops.attention(q, cache, table, 10, 5, Attention(1.0), out)
    with pytest.raises(ValueError, match="page table"):
        ops.attention(q, cache, table[:1], 0, 40, Attention(1.0), out)
    bad = KvCache(torch.zeros(4, 8, 2, 128, dtype=torch.float16, device="cuda"),
                  torch.zeros(4, 2, 128, 8, dtype=torch.float16, device="cuda"), 8)
    with pytest.raises(ValueError, match="multiple of 16"):
        ops.attention(q, bad, table, 0, 1, Attention(1.0), out)


@pytest.mark.parametrize("dim,q_heads,kv_heads", [(128, 32, 8), (256, 16, 2), (64, 8, 8)])
def test_batched_decode_is_each_sequence_alone(ops, dim, q_heads, kv_heads):
    """drift_attention_decode: every row bit for bit drift_attention of its
    sequence at its own length (sequences of different lengths in one launch)."""
    rng = np.random.default_rng(dim)
    batch, page_size, per_sequence = 4, 16, 20
    lengths = [1, 17, 130, 300]
    pages = batch * per_sequence
    tables = rng.permutation(pages).astype(np.int32).reshape(batch, per_sequence)
    keys = np.zeros((pages, page_size, kv_heads, dim), dtype=np.uint16)
    values = np.zeros((pages, kv_heads, dim, page_size), dtype=np.uint16)
    for i, n in enumerate(lengths):
        k = rng.standard_normal((n, kv_heads, dim)).astype(np.float32)
        v = rng.standard_normal((n, kv_heads, dim)).astype(np.float32)
        oracle.cache_write(k, v, keys, values, page_size, tables[i], 0)
    cache = KvCache(torch.from_numpy(keys.view(np.float16)).cuda(),
                    torch.from_numpy(values.view(np.float16)).cuda(), page_size)
    q = torch.from_numpy(rng.standard_normal((batch, q_heads, dim)).astype(np.float32)).cuda()
    table_dev = torch.from_numpy(tables).cuda()
    positions = torch.tensor([n - 1 for n in lengths], dtype=torch.int32, device="cuda")
    attention = Attention(1.0 / math.sqrt(dim))
    batched = torch.empty_like(q)
    ops.attention_decode(q, cache, table_dev, positions, per_sequence * page_size, attention,
                         batched)
    for i, n in enumerate(lengths):
        alone = torch.empty(1, q_heads, dim, device="cuda")
        ops.attention(q[i:i + 1], cache, table_dev[i], n - 1, n, attention, alone)
        assert torch.equal(batched[i:i + 1], alone), f"sequence {i}"


def test_separate_join_is_the_fused_join(ops):
    """C5's attention shape (16 query heads on 2 key heads of 256): decoded in a
    launch sized for 4096 positions (64 splits: the join is a launch of its
    own) and alone at their own lengths (the last split CTA joins): the same
    bits."""
    rng = np.random.default_rng(256)
    dim, q_heads, kv_heads, page_size = 256, 16, 2, 32
    lengths = [130, 300]
    per_sequence = 4096 // page_size
    batch = len(lengths)
    pages = batch * per_sequence
    tables = rng.permutation(pages).astype(np.int32).reshape(batch, per_sequence)
    keys = np.zeros((pages, page_size, kv_heads, dim), dtype=np.uint16)
    values = np.zeros((pages, kv_heads, dim, page_size), dtype=np.uint16)
    for i, n in enumerate(lengths):
        k = rng.standard_normal((n, kv_heads, dim)).astype(np.float32)
        v = rng.standard_normal((n, kv_heads, dim)).astype(np.float32)
        oracle.cache_write(k, v, keys, values, page_size, tables[i], 0)
    cache = KvCache(torch.from_numpy(keys.view(np.float16)).cuda(),
                    torch.from_numpy(values.view(np.float16)).cuda(), page_size)
    q = torch.from_numpy(rng.standard_normal((batch, q_heads, dim)).astype(np.float32)).cuda()
    table_dev = torch.from_numpy(tables).cuda()
    positions = torch.tensor([n - 1 for n in lengths], dtype=torch.int32, device="cuda")
    attention = Attention(1.0 / math.sqrt(dim))
    batched = torch.empty_like(q)
    ops.attention_decode(q, cache, table_dev, positions, 4096, attention, batched)
    for i, n in enumerate(lengths):
        alone = torch.empty(1, q_heads, dim, device="cuda")
        ops.attention(q[i:i + 1], cache, table_dev[i], n - 1, n, attention, alone)
        assert torch.equal(batched[i:i + 1], alone), f"sequence {i}"


def test_fused_attention_inputs_are_the_separate_ops(ops):
    """drift_attention_inputs_decode: the bits of rms_norm per head, rope and
    cache_write called in turn."""
    from drift_b200.ops import Rope

    rng = np.random.default_rng(8)
    batch, q_heads, kv_heads, dim, page_size, per_sequence = 3, 8, 2, 128, 16, 8
    pages = batch * per_sequence
    tables = torch.arange(pages, dtype=torch.int32, device="cuda").view(batch, per_sequence)
    q = torch.from_numpy(rng.standard_normal((batch, q_heads, dim)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal((batch, kv_heads, dim)).astype(np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal((batch, kv_heads, dim)).astype(np.float32)).cuda()
    q_norm = torch.from_numpy((1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)).cuda()
    k_norm = torch.from_numpy((1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)).cuda()
    positions = torch.tensor([5, 60, 100], dtype=torch.int32, device="cuda")
    rope = Rope(1e6, dim)
    fused_cache = KvCache.allocate(pages, page_size, kv_heads, dim)
    fused_q = torch.empty_like(q)
    ops.attention_inputs_decode(q, k, v, q_norm, k_norm, 1e-6, positions, rope, fused_q,
                                fused_cache, tables)
    cache = KvCache.allocate(pages, page_size, kv_heads, dim)
    qn, kn = torch.empty_like(q), torch.empty_like(k)
    ops.rms_norm(q, q_norm, 1e-6, 0.0, qn)
    ops.rms_norm(k, k_norm, 1e-6, 0.0, kn)
    q_turned = torch.empty_like(q)
    k_turned = torch.empty_like(k)
    for i in range(batch):
        ops.rope(qn[i:i + 1], positions[i:i + 1], rope, q_turned[i:i + 1])
        ops.rope(kn[i:i + 1], positions[i:i + 1], rope, k_turned[i:i + 1])
        ops.cache_write(k_turned[i:i + 1], v[i:i + 1], cache, tables[i], int(positions[i]))
    assert torch.equal(fused_q, q_turned)
    assert torch.equal(fused_cache.keys, cache.keys)
    assert torch.equal(fused_cache.values, cache.values)


# The known answers of the reference's AttentionReferenceTests.scala:47-111 on
# the GPU kernel (the oracle holds them in test_oracle_attention.py).

def test_one_visible_key_gives_its_value(ops):
    cache = KvCache.allocate(1, 16, 1, 16 * 4)
    table = torch.zeros(1, dtype=torch.int32, device="cuda")
    # heads of 64 (the kernels' narrowest): value d / 8 for d < 16, exact in F16
    dim = 64
    value = (torch.arange(dim, device="cuda") % 16 / 8).float().view(1, 1, dim)
    ops.cache_write(torch.full((1, 1, dim), 0.5, device="cuda"), value, cache, table, 0)
    q = torch.ones(1, 1, dim, device="cuda")
    out = torch.empty_like(q)
    ops.attention(q, cache, table, 0, 1, Attention(0.25 / 4), out)  # q.k x scale = 2
    assert torch.equal(out, value)
    ops.attention(q, cache, table, 0, 1,
                  Attention(0.25 / 4, sinks=torch.tensor([2.0], device="cuda")), out)
    assert torch.equal(out, value / 2)


def plain_gpu(ops, shuffled=False, tokens=5, window=None, queries=None):
    rng = np.random.default_rng(7)
    key_count, q_heads, kv_heads, dim, page_size = 40, 4, 2, 64, 16
    k = rng.standard_normal((key_count, kv_heads, dim)).astype(np.float32)
    v = rng.standard_normal((key_count, kv_heads, dim)).astype(np.float32)
    drawn = rng.standard_normal((5, q_heads, dim)).astype(np.float32)
    q = drawn if queries is None else queries
    table = torch.tensor([2, 0, 1] if shuffled else [0, 1, 2], dtype=torch.int32, device="cuda")
    cache = KvCache.allocate(3, page_size, kv_heads, dim)
    ops.cache_write(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), cache, table, 0)
    q = q[-tokens:]
    out = torch.empty(tokens, q_heads, dim, device="cuda")
    ops.attention(torch.from_numpy(q).cuda(), cache, table, key_count - tokens, key_count,
                  Attention(1 / math.sqrt(dim), True, window), out)
    return out, q


def test_page_order_does_not_matter(ops):
    assert torch.equal(plain_gpu(ops)[0], plain_gpu(ops, shuffled=True)[0])


def test_prefill_then_decode_equals_one_longer_prefill(ops):
    prefill, q = plain_gpu(ops)
    decode, _ = plain_gpu(ops, tokens=1, queries=q)
    assert torch.equal(prefill[-1:], decode)


def test_a_whole_window_changes_nothing_and_a_narrow_one_does(ops):
    full, _ = plain_gpu(ops)
    assert torch.equal(plain_gpu(ops, window=40)[0], full)
    assert not torch.equal(plain_gpu(ops, window=8)[0], full)
