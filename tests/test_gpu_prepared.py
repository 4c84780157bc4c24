"""Prepared x: the producers of a product's x (add_rms_norm, gated, the decode
attention) writing its records themselves, as the reference's rms_norm_f32 and
gated_f32 write xq/xd/xs for the product that follows (runner/kernels/
norm.hip:34-35, elementwise.hip:58-59). Products over prepared records are
bit for bit the products that prepare x themselves."""

import math

import numpy as np
import pytest
import torch

import oracle
from drift_b200 import synthetic
from drift_b200.ops import SILU, Attention, CudaOps, KvCache, RowNorm, SharedExpert, Stored

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    return CudaOps()


def weights(rng, shapes, k, dtype=oracle.Q4_1):
    return [Stored.upload(dtype, (n, k), synthetic.quantized(rng, dtype, n, k)) for n in shapes]


@pytest.mark.parametrize("m", [1, 2, 5])
@pytest.mark.parametrize("k", [1024, 4096, 6144])
def test_norm_records_feed_linears(ops, m, k):
    rng = np.random.default_rng(m * 7 + k)
    ws = weights(rng, [384, 96, 96], k)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    y = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    weight = torch.from_numpy((1 + 0.02 * rng.standard_normal(k)).astype(np.float32)).cuda()
    prepared = ops.prepared_x(m, k)
    x1, normed1 = x.clone(), torch.empty_like(x)
    ops.add_rms_norm(x1, y, RowNorm(weight, 1e-6, 0.0, normed1), prepared)
    fused = [torch.empty(m, w.shape[0], device="cuda") for w in ws]
    ops.linears(normed1, ws, fused, prepared)
    x2, normed2 = x.clone(), torch.empty_like(x)
    ops.add_rms_norm(x2, y, RowNorm(weight, 1e-6, 0.0, normed2))
    assert torch.equal(x1, x2) and torch.equal(normed1, normed2)
    for w, f in zip(ws, fused):
        alone = torch.empty_like(f)
        ops.linear(normed2, w, alone)
        assert torch.equal(f, alone)


def test_norm_alone_records(ops):
    """y None: the plain rmsNorm, with records."""
    rng = np.random.default_rng(3)
    m, k = 3, 2048
    (w,) = weights(rng, [200], k)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    weight = torch.from_numpy((1 + 0.02 * rng.standard_normal(k)).astype(np.float32)).cuda()
    prepared = ops.prepared_x(m, k)
    normed = torch.empty_like(x)
    ops.add_rms_norm(x, None, RowNorm(weight, 1e-6, 0.0, normed), prepared)
    fused = torch.empty(m, 200, device="cuda")
    ops.linears(normed, [w], [fused], prepared)
    expected = torch.empty_like(normed)
    ops.rms_norm(x, weight, 1e-6, 0.0, expected)
    assert torch.equal(normed, expected)
    alone = torch.empty_like(fused)
    ops.linear(expected, w, alone)
    assert torch.equal(fused, alone)


@pytest.mark.parametrize("m", [1, 3, 16])
def test_gated_records_feed_linear(ops, m):
    rng = np.random.default_rng(m)
    ffn, hidden = 1536, 512
    (down,) = weights(rng, [hidden], ffn)
    gate = torch.from_numpy(rng.standard_normal((m, ffn)).astype(np.float32)).cuda()
    up = torch.from_numpy(rng.standard_normal((m, ffn)).astype(np.float32)).cuda()
    prepared = ops.prepared_x(m, ffn)
    hidden1 = torch.empty_like(gate)
    ops.gated(SILU, gate, up, hidden1, prepared)
    fused = torch.empty(m, hidden, device="cuda")
    ops.linears(hidden1, [down], [fused], prepared)
    hidden2 = torch.empty_like(gate)
    ops.gated(SILU, gate, up, hidden2)
    assert torch.equal(hidden1, hidden2)
    alone = torch.empty_like(fused)
    ops.linear(hidden2, down, alone)
    assert torch.equal(fused, alone)


@pytest.mark.parametrize("dim,q_heads,kv_heads", [(128, 8, 2), (64, 4, 4), (256, 4, 1)])
def test_attention_records_feed_linear(ops, dim, q_heads, kv_heads):
    rng = np.random.default_rng(dim)
    batch, page_size, per_sequence = 3, 16, 8
    pages = batch * per_sequence
    cache = KvCache(torch.from_numpy(rng.standard_normal((pages, page_size, kv_heads, dim))
                                     .astype(np.float16)).cuda(),
                    torch.from_numpy(rng.standard_normal((pages, kv_heads, dim, page_size))
                                     .astype(np.float16)).cuda(), page_size)
    tables = torch.arange(pages, dtype=torch.int32, device="cuda").view(batch, per_sequence)
    positions = torch.tensor([3, 40, 100], dtype=torch.int32, device="cuda")
    q = torch.from_numpy(rng.standard_normal((batch, q_heads, dim)).astype(np.float32)).cuda()
    attention = Attention(1.0 / math.sqrt(dim))
    (o,) = weights(rng, [256], q_heads * dim)
    prepared = ops.prepared_x(batch, q_heads * dim)
    out1 = torch.empty_like(q)
    ops.attention_decode(q, cache, tables, positions, per_sequence * page_size, attention, out1,
                         prepared)
    fused = torch.empty(batch, 256, device="cuda")
    ops.linears(out1.view(batch, -1), [o], [fused], prepared)
    out2 = torch.empty_like(q)
    ops.attention_decode(q, cache, tables, positions, per_sequence * page_size, attention, out2)
    assert torch.equal(out1, out2)
    alone = torch.empty_like(fused)
    ops.linear(out2.view(batch, -1), o, alone)
    assert torch.equal(fused, alone)


@pytest.mark.parametrize("dtype", [oracle.Q8_0, oracle.Q4_0, oracle.Q4_1],
                         ids=lambda t: oracle.NAMES[t])
@pytest.mark.parametrize("tokens", [1, 3, 9])
def test_norm_records_feed_experts(ops, dtype, tokens):
    """The post norm's records feeding the router, the experts' gate and up
    products and a plain expert product (9 tokens: rows past the first
    8-row record): bit for bit the products that prepare x themselves."""
    rng = np.random.default_rng(90 + 7 * dtype + tokens)
    experts, ffn, hidden, used = 16, 256, 2048, 4
    gate = Stored.upload(dtype, (experts, ffn, hidden),
                         synthetic.quantized(rng, dtype, experts * ffn, hidden))
    up = Stored.upload(dtype, (experts, ffn, hidden),
                       synthetic.quantized(rng, dtype, experts * ffn, hidden))
    (router,) = weights(rng, [experts], hidden, dtype)
    x = torch.from_numpy(rng.standard_normal((tokens, hidden)).astype(np.float32)).cuda()
    weight = torch.from_numpy((1 + 0.02 * rng.standard_normal(hidden)).astype(np.float32)).cuda()
    prepared = ops.prepared_x(tokens, hidden)
    normed = torch.empty_like(x)
    ops.add_rms_norm(x, None, RowNorm(weight, 1e-6, 0.0, normed), prepared)
    ids = torch.from_numpy(np.stack([rng.permutation(experts)[:used] for _ in range(tokens)])
                           .astype(np.int32).reshape(-1)).cuda()
    logits = [torch.empty(tokens, experts, device="cuda") for _ in range(2)]
    route_ids = [torch.empty(tokens, used, dtype=torch.int32, device="cuda") for _ in range(2)]
    route_weights = [torch.empty(tokens, used, device="cuda") for _ in range(2)]
    ops.route_linear(normed, router, logits[0], route_ids[0], route_weights[0], prepared)
    ops.route_linear(normed, router, logits[1], route_ids[1], route_weights[1])
    assert torch.equal(logits[0], logits[1]) and torch.equal(route_ids[0], route_ids[1])
    gated = [torch.empty(tokens * used, ffn, device="cuda") for _ in range(2)]
    ops.experts_gated_linear(normed, gate, up, ids, gated[0], first_expert=0, prepared=prepared)
    ops.experts_gated_linear(normed, gate, up, ids, gated[1])
    assert torch.equal(gated[0], gated[1])
    plain = [torch.empty(tokens * used, ffn, device="cuda") for _ in range(2)]
    ops.experts_linear(normed, gate, ids, plain[0], first_expert=0, prepared=prepared)
    ops.experts_linear(normed, gate, ids, plain[1])
    assert torch.equal(plain[0], plain[1])
    # and the product itself against the oracle
    expected = oracle.experts_linear(dtype, normed.cpu().numpy(), gate.data.cpu().numpy(), experts,
                                     ffn, hidden, ids.cpu().numpy().reshape(tokens, used))
    assert np.allclose(plain[0].cpu().numpy(), expected, rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("tokens", [1, 3, 9])
def test_combine_norm_records_feed_linears(ops, tokens):
    """moe_combine_norm writing the next layer's records (shared expert on):
    the residual, the norm and the products over them bit for bit those of
    the unprepared calls."""
    rng = np.random.default_rng(120 + tokens)
    k, hidden = 10, 2048
    (w,) = weights(rng, [512], hidden)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    expert_out = dev(rng.standard_normal((tokens * k, hidden)))
    route = dev(rng.random((tokens, k)))
    shared = SharedExpert(dev(rng.standard_normal((tokens, hidden))),
                          dev(rng.standard_normal((tokens, hidden))),
                          dev(0.02 * rng.standard_normal(hidden)))
    residual = dev(rng.standard_normal((tokens, hidden)))
    norm_weight = dev(1 + 0.02 * rng.standard_normal(hidden))
    prepared = ops.prepared_x(tokens, hidden)
    r1, n1 = residual.clone(), torch.empty_like(residual)
    ops.moe_combine_norm(expert_out, route, shared, r1, RowNorm(norm_weight, 1e-6, 0.0, n1),
                         prepared)
    r2, n2 = residual.clone(), torch.empty_like(residual)
    ops.moe_combine_norm(expert_out, route, shared, r2, RowNorm(norm_weight, 1e-6, 0.0, n2))
    assert torch.equal(r1, r2) and torch.equal(n1, n2)
    fused, alone = torch.empty(tokens, 512, device="cuda"), torch.empty(tokens, 512, device="cuda")
    ops.linears(n1, [w], [fused], prepared)
    ops.linear(n2, w, alone)
    assert torch.equal(fused, alone)


def test_prepared_refusals(ops):
    x = torch.zeros(2, 100, device="cuda")
    w = torch.ones(100, device="cuda")
    buffer = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError, match="32-value blocks"):
        ops.add_rms_norm(x, None, RowNorm(w, 1e-6, 0.0, torch.empty_like(x)), buffer)
    with pytest.raises(ValueError, match="32-value blocks"):
        ops.gated(SILU, x, x, torch.empty_like(x), buffer)
