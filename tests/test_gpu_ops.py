"""The layer operations and the mixture of experts on the GPU against the CPU
oracle (the reference's SmallOpsTests and FusedOpsTests,
runner/gpuTest/src/drift/runner/SmallOpsTests.scala, FusedOpsTests.scala)."""

import numpy as np
import pytest
import torch

import oracle
from drift_b200 import synthetic
from drift_b200.ops import (CudaOps, Rope, RowNorm, SharedExpert, Stored, NEOX, INTERLEAVED,
                            SILU, SIGMOID, GELU_ERF, GELU_TANH, SITU)
from tests.conftest import within

pytestmark = pytest.mark.gpu

# SmallOpsTests' awkward shapes (L22-29) and the benchmark config C3 ones.
SHAPES = [(1, 1), (3, 7), (2, 255), (5, 4097), (17, 2560), (1, 2048), (1, 4096), (64, 4096)]


@pytest.fixture(scope="module")
def ops():
    return CudaOps()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---- embedding (bit-exact) -------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [oracle.Q8_0, oracle.Q4_0, oracle.Q4_1],
                         ids=lambda t: oracle.NAMES[t])
def test_embedding_is_bit_exact(ops, dtype):
    rng = np.random.default_rng(21)
    vocab, cols = 1000, 4096
    table = synthetic.random_blocks(rng, dtype, vocab, cols)
    ids = np.concatenate([[0, vocab - 1], rng.integers(0, vocab, 62)]).astype(np.int32)
    out = torch.empty(ids.size, cols, device="cuda")
    ops.embedding(Stored.upload(dtype, (vocab, cols), table), dev(ids), out)
    expected = oracle.embedding(dtype, table, vocab, cols, ids)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), expected.view(np.uint32))


def test_embedding_full_vocabulary_q8_0(ops):
    """benchmark config C3: a Q8_0 table 151936 x 4096, random ids, b in {1, 8, 16, 64}."""
    rng = np.random.default_rng(22)
    vocab, cols = 151936, 4096
    table = synthetic.quantized(rng, oracle.Q8_0, vocab, cols)
    stored = Stored.upload(oracle.Q8_0, (vocab, cols), table)
    for b in (1, 8, 16, 64):
        ids = rng.integers(0, vocab, b).astype(np.int32)
        ids[0] = vocab - 1
        out = torch.empty(b, cols, device="cuda")
        ops.embedding(stored, dev(ids), out)
        expected = oracle.embedding(oracle.Q8_0, table, vocab, cols, ids)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), expected.view(np.uint32))


def test_embedding_id_outside_the_table_is_flagged(ops):
    """The CPU reference refuses it ("token id ... outside the table",
    ops/CpuLinear.scala:19-23); here the row comes out NaN and the device
    error word says so -- no out-of-bounds read."""
    vocab, cols = 4, 64
    table = Stored.upload(oracle.Q8_0, (vocab, cols), np.zeros(vocab * 68, np.uint8))
    ops.take_device_error()
    out = torch.zeros(3, cols, device="cuda")
    ops.embedding(table, dev(np.array([0, 4, -1], np.int32)), out)
    assert ops.take_device_error() == 1
    result = out.cpu().numpy()
    assert (result[0] == 0).all() and np.isnan(result[1:]).all()
    assert ops.take_device_error() == 0


# ---- norms and elementwise ------------------------------------------------------------------------
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_rms_norm(ops, shape):
    rng = np.random.default_rng(sum(shape))
    x = synthetic.gaussian(rng, *shape)
    w = (1 + rng.standard_normal(shape[1]) * 0.02).astype(np.float32)
    out = torch.empty(shape, device="cuda")
    ops.rms_norm(dev(x), dev(w), 1e-6, 0.0, out)
    expected = oracle.rms_norm(x, w, 1e-6)
    ok, _, _, summary = within(out.cpu().numpy(), expected, 1e-5, 1e-5)  # SmallOpsTests L115-127
    assert ok, summary


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_add_rms_norm(ops, shape):
    rng = np.random.default_rng(sum(shape) + 1)
    x = synthetic.gaussian(rng, *shape)
    y = synthetic.gaussian(rng, *shape)
    w = (1 + rng.standard_normal(shape[1]) * 0.02).astype(np.float32)
    xd = dev(x)
    out = torch.empty(shape, device="cuda")
    ops.add_rms_norm(xd, dev(y), RowNorm(dev(w), 1e-6, 0.0, out))
    sum_expected, norm_expected = oracle.add_rms_norm(x, y, w, 1e-6)
    assert np.array_equal(xd.cpu().numpy(), sum_expected)
    ok, _, _, summary = within(out.cpu().numpy(), norm_expected, 1e-5, 1e-5)
    assert ok, summary


def test_rms_norm_weight_offset_and_zero_row(ops):
    x = np.zeros((2, 8), np.float32)
    x[1] = np.arange(8)
    w = np.full(8, 0.5, np.float32)
    out = torch.empty(2, 8, device="cuda")
    ops.rms_norm(dev(x), dev(w), 1e-6, 1.0, out)
    ok, _, _, summary = within(out.cpu().numpy(), oracle.rms_norm(x, w, 1e-6, 1.0), 1e-6, 1e-6)
    assert ok, summary
    assert (out[0] == 0).all()


@pytest.mark.parametrize("kind", [SILU, GELU_TANH, GELU_ERF, SIGMOID, SITU])
def test_gated(ops, kind):
    rng = np.random.default_rng(30 + kind)
    for shape in [(1, 1), (3, 7), (64, 12288)]:
        g = synthetic.gaussian(rng, *shape) * 3
        u = synthetic.gaussian(rng, *shape)
        out = torch.empty(shape, device="cuda")
        ops.gated(kind, dev(g), dev(u), out)
        ok, _, _, summary = within(out.cpu().numpy(), oracle.gated(kind, g, u), 1e-6, 1e-5)
        assert ok, summary  # SmallOpsTests L66, 95-103


def test_add_and_gated_in_place(ops):
    rng = np.random.default_rng(31)
    a, b = synthetic.gaussian(rng, 1000), synthetic.gaussian(rng, 1000)
    ad = dev(a)
    ops.add(ad, dev(b), ad)  # out may be an input
    assert np.array_equal(ad.cpu().numpy(), (a + b).astype(np.float32))


# ---- rotary embedding --------------------------------------------------------------------------
@pytest.mark.parametrize("layout", [NEOX, INTERLEAVED], ids=["neox", "interleaved"])
def test_rope_matches_the_cpu_angle(ops, layout):
    """benchmark config C3: theta 1e6, head_dim 128, positions up to 8191, q [b, 32,
    128] and k [b, 8, 128]. The reference holds its own kernel to 1e-2
    (SmallOpsTests L450-500); this one computes the CPU's angle bit for bit
    and lands within about an ulp."""
    rng = np.random.default_rng(40 + layout)
    for tokens, heads in [(1, 32), (16, 8), (64, 32)]:
        x = synthetic.gaussian(rng, tokens, heads, 128)
        positions = ((np.arange(tokens) * 131) % 4096).astype(np.int32)
        positions[-1] = 8191
        out = torch.empty(x.shape, device="cuda")
        ops.rope(dev(x), dev(positions), Rope(1e6, 128, layout), out)
        expected = oracle.rope(x, positions, 1e6, 128, layout)
        ok, _, max_abs, summary = within(out.cpu().numpy(), expected, 1e-6, 1e-6)
        assert ok, summary


def test_rope_partial_and_known_turns(ops):
    """ReferenceOpsTests' hand-worked turns, on the GPU."""
    x = np.array([1, 1, 0, 0], np.float32).reshape(1, 1, 4)
    out = torch.empty(1, 1, 4, device="cuda")
    ops.rope(dev(x), dev(np.array([1], np.int32)), Rope(100.0, 4, NEOX), out)
    expected = [np.cos(1.0), np.cos(0.1), np.sin(1.0), np.sin(0.1)]
    assert within(out.cpu().numpy(), expected, 1e-6, 0)[0]
    values = np.arange(1, 7, dtype=np.float32).reshape(1, 1, 6)
    out = torch.empty(1, 1, 6, device="cuda")
    ops.rope(dev(values), dev(np.array([7], np.int32)), Rope(1e4, 2, NEOX), out)
    assert np.array_equal(out.cpu().numpy()[0, 0, 2:], values[0, 0, 2:])


# ---- mixture of experts -------------------------------------------------------------------------
def test_route_matches_oracle(ops):
    """benchmark config C5: 512 experts, top-10, logits ~ N(0, 1)."""
    rng = np.random.default_rng(50)
    for tokens in (1, 16, 64):
        logits = synthetic.gaussian(rng, tokens, 512)
        ids = torch.empty(tokens, 10, dtype=torch.int32, device="cuda")
        weights = torch.empty(tokens, 10, device="cuda")
        ops.route(dev(logits), ids, weights)
        e_ids, e_weights = oracle.route(logits, 10)
        assert np.array_equal(ids.cpu().numpy(), e_ids)
        assert within(weights.cpu().numpy(), e_weights, 1e-7, 1e-6)[0]


def test_route_ties_take_the_lower_expert(ops):
    logits = np.array([[0.5, 2.0, 2.0, -1.0, 2.0, 0.5]], np.float32)
    ids = torch.empty(1, 4, dtype=torch.int32, device="cuda")
    weights = torch.empty(1, 4, device="cuda")
    ops.route(dev(logits), ids, weights)
    assert ids.cpu().numpy().tolist() == [[1, 2, 4, 0]]


def test_route_ties_across_lanes(ops):
    """Equal logits in one lane's experts and in different lanes' (5, 37 and
    6; the four zeros, two of them -0.0), then -inf ones: value first, the
    lower expert among equals, -0.0 equal to 0.0."""
    logits = np.full((1, 64), -np.inf, np.float32)
    for e in (5, 37, 6):
        logits[0, e] = 3.0
    logits[0, [0, 33]] = -0.0
    logits[0, [32, 1]] = 0.0
    ids = torch.empty(1, 8, dtype=torch.int32, device="cuda")
    weights = torch.empty(1, 8, device="cuda")
    ops.route(dev(logits), ids, weights)
    assert ids.cpu().numpy().tolist() == [[5, 6, 37, 0, 1, 32, 33, 2]]
    e_ids, e_weights = oracle.route(logits, 8)
    assert np.array_equal(ids.cpu().numpy(), e_ids)
    assert within(weights.cpu().numpy(), e_weights, 1e-7, 1e-6)[0]


@pytest.mark.parametrize("dtype", [oracle.Q8_0, oracle.Q4_1], ids=lambda t: oracle.NAMES[t])
def test_experts_linear_and_gated(ops, dtype):
    """C5 shapes with fewer experts: gate/up [E, 512, 2048], down [E, 2048, 512];
    b tokens of 10 slots."""
    rng = np.random.default_rng(60 + dtype)
    experts, ffn, hidden = 24, 512, 2048
    gate = synthetic.quantized(rng, dtype, experts * ffn, hidden)
    up = synthetic.quantized(rng, dtype, experts * ffn, hidden)
    down = synthetic.quantized(rng, dtype, experts * hidden, ffn)
    sg = Stored.upload(dtype, (experts, ffn, hidden), gate)
    su = Stored.upload(dtype, (experts, ffn, hidden), up)
    sd = Stored.upload(dtype, (experts, hidden, ffn), down)
    # x scaled so the gate pre-activations are O(1), as a normed layer input
    # makes them: at the raw law's scale (sigma ~ 36 for Q8_0 at K = 2048)
    # silu'(g) * up amplifies any float32 rounding of g near g = 0 past 1e-4
    w_rms = np.sqrt(np.mean(oracle.decode(dtype, gate[:ffn * hidden // 32 * synthetic.BLOCK_BYTES[dtype]],
                                          ffn * hidden) ** 2))
    x_scale = 1.0 / (np.sqrt(hidden) * w_rms)
    for tokens in (1, 4):
        x = synthetic.gaussian(rng, tokens, hidden)
        ids = np.stack([rng.permutation(experts)[:10] for _ in range(tokens)]).astype(np.int32)
        # the plain products at the raw scale: fp32-accumulated outputs
        g_out = torch.empty(tokens * 10, ffn, device="cuda")
        ops.experts_linear(dev(x), sg, dev(ids.reshape(-1)), g_out)
        e_g = oracle.experts_linear(dtype, x, gate, experts, ffn, hidden, ids)
        ok, _, _, summary = within(g_out.cpu().numpy(), e_g, 1e-4, 1e-3)
        assert ok, summary
        # the gated product (one launch) at a unit pre-activation scale
        xs = (x * x_scale).astype(np.float32)
        gated = torch.empty(tokens * 10, ffn, device="cuda")
        ops.experts_gated_linear(dev(xs), sg, su, dev(ids.reshape(-1)), gated)
        e_gated = oracle.experts_gated_linear(dtype, xs, gate, up, experts, ffn, hidden, ids)
        ok, _, _, summary = within(gated.cpu().numpy(), e_gated, 1e-4, 1e-3)
        assert ok, summary
        # down over every slot's own row (divisor 1), fed unit-scale activations
        # as a layer's normalised input is (the gated values above reach ~10^3,
        # where outputs that nearly cancel are beyond any float32 sum's 1e-4)
        act = (e_gated / e_gated.std()).astype(np.float32)
        out = torch.empty(tokens * 10, hidden, device="cuda")
        ops.experts_linear(dev(act), sd, dev(ids.reshape(-1)), out)
        e_out = oracle.experts_linear(dtype, act, down, experts, hidden, ffn, ids)
        ok, _, _, summary = within(out.cpu().numpy(), e_out, 1e-4, 1e-3)
        assert ok, summary
        # and at the raw scale, the reference's own float bar: 1e-5 of max|y|
        # (LinearTests.scala:154-157)
        ops.experts_linear(dev(e_gated), sd, dev(ids.reshape(-1)), out)
        e_raw = oracle.experts_linear(dtype, e_gated, down, experts, hidden, ffn, ids)
        ok, _, _, summary = within(out.cpu().numpy(), e_raw, 1e-5 * np.abs(e_raw).max(), 0)
        assert ok, summary


def _shifted(w: Stored) -> Stored:
    """The same blocks 4 bytes into a buffer: rows no longer start on 16-byte
    boundaries, so the products take the direct-load kernel."""
    data = torch.zeros(w.data.numel() + 4, dtype=torch.uint8, device="cuda")
    data[4:] = w.data
    return Stored(w.dtype, w.shape, data[4:])


@pytest.mark.parametrize("dtype", [oracle.Q8_0, oracle.Q4_0, oracle.Q4_1],
                         ids=lambda t: oracle.NAMES[t])
@pytest.mark.parametrize("tokens", [16, 40])
def test_streamed_experts_are_the_direct_kernel(ops, dtype, tokens):
    """Weights of whole 16-byte rows stream through shared memory
    (experts_stream_kernel, at a unit an SM or more: 16 tokens of 10 slots
    are) -- the gated products, and plain products of rows of at most
    16 blocks (the down product, x prepared in the kernel, a row to each
    half-warp); the same weights 4 bytes off take the direct-load kernel
    (experts_x22_kernel). Bit for bit, and for expert-parallel products whose
    other ranks' slots are zeros; the plain gate product (direct either way)
    alongside."""
    rng = np.random.default_rng(70 + dtype + tokens)
    experts, ffn, hidden = 24, 512, 2048
    gate = Stored.upload(dtype, (experts, ffn, hidden),
                         synthetic.quantized(rng, dtype, experts * ffn, hidden))
    up = Stored.upload(dtype, (experts, ffn, hidden),
                       synthetic.quantized(rng, dtype, experts * ffn, hidden))
    down = Stored.upload(dtype, (experts, hidden, ffn),
                         synthetic.quantized(rng, dtype, experts * hidden, ffn))
    x = dev((synthetic.gaussian(rng, tokens, hidden) * 0.02).astype(np.float32))
    ids = dev(np.stack([rng.permutation(experts)[:10] for _ in range(tokens)])
              .astype(np.int32).reshape(-1))
    slots = tokens * 10

    def both(run, n):
        a = torch.full((slots, n), float("nan"), device="cuda")
        b = torch.full((slots, n), float("nan"), device="cuda")
        run(False, a)
        run(True, b)
        assert torch.equal(a, b)
        return a

    gated = both(lambda shift, out: ops.experts_gated_linear(
        x, _shifted(gate) if shift else gate, _shifted(up) if shift else up, ids, out), ffn)
    both(lambda shift, out: ops.experts_linear(x, _shifted(gate) if shift else gate, ids, out),
         ffn)
    act = (gated / gated.std()).contiguous()
    full = both(lambda shift, out: ops.experts_linear(act, _shifted(down) if shift else down,
                                                       ids, out), hidden)
    # expert parallelism: this rank holds experts 8..15; the other slots are zeros
    per_expert = ffn * hidden // 32 * synthetic.BLOCK_BYTES[dtype]
    lg = Stored(dtype, (8, ffn, hidden), gate.data[8 * per_expert:16 * per_expert].contiguous())
    lu = Stored(dtype, (8, ffn, hidden), up.data[8 * per_expert:16 * per_expert].contiguous())
    part = both(lambda shift, out: ops.experts_gated_linear(
        x, _shifted(lg) if shift else lg, _shifted(lu) if shift else lu, ids, out,
        first_expert=8), ffn)
    outside = ((ids < 8) | (ids >= 16)).cpu().numpy()
    assert (part.cpu().numpy()[outside] == 0).all()
    inside = torch.from_numpy(~outside).cuda()
    assert torch.equal(part[inside], gated[inside])
    ld = Stored(dtype, (8, hidden, ffn), down.data[8 * per_expert:16 * per_expert].contiguous())
    part = both(lambda shift, out: ops.experts_linear(act, _shifted(ld) if shift else ld, ids,
                                                       out, first_expert=8), hidden)
    assert (part.cpu().numpy()[outside] == 0).all()
    assert torch.equal(part[inside], full[inside])


def test_shared_expert_rides_in_the_routed_launch(ops):
    """A shared tail: the routed slots, then one slot per row of x for the
    shared expert (one more expert of the weights), in one launch -- bit for
    bit the routed launch and the shared expert's launch apart."""
    rng = np.random.default_rng(62)
    experts, ffn, hidden, used, tokens = 8, 128, 1024, 3, 5
    dtype = oracle.Q4_1
    sg = Stored.upload(dtype, (experts + 1, ffn, hidden),
                       synthetic.quantized(rng, dtype, (experts + 1) * ffn, hidden))
    su = Stored.upload(dtype, (experts + 1, ffn, hidden),
                       synthetic.quantized(rng, dtype, (experts + 1) * ffn, hidden))
    x = dev((0.05 * synthetic.gaussian(rng, tokens, hidden)).astype(np.float32))
    routed_ids = rng.integers(0, experts, tokens * used).astype(np.int32)
    ids = np.concatenate([routed_ids, np.full(tokens, experts, np.int32)])
    together = torch.empty(tokens * (used + 1), ffn, device="cuda")
    ops.experts_gated_linear(x, sg, su, dev(ids), together, first_expert=0, shared_tail=True)
    routed = torch.empty(tokens * used, ffn, device="cuda")
    ops.experts_gated_linear(x, sg, su, dev(routed_ids), routed)
    shared = torch.empty(tokens, ffn, device="cuda")
    ops.experts_gated_linear(x, sg, su, dev(np.full(tokens, experts, np.int32)), shared)
    assert torch.equal(together[:tokens * used], routed)
    assert torch.equal(together[tokens * used:], shared)
    assert ops.take_device_error() == 0


@pytest.mark.parametrize("dtype", [oracle.Q8_0, oracle.Q4_0, oracle.Q4_1],
                         ids=lambda t: oracle.NAMES[t])
def test_down_product_prepares_x_in_the_kernel(ops, dtype):
    """expertsLinear with one F32 x row a slot (a down product) prepares x in
    the experts kernel; the same rows shared two slots each go through the
    preparation launch: bit for bit the same outputs, on two calls in a row."""
    rng = np.random.default_rng(63 + dtype)
    experts, hidden, ffn, slots = 12, 256, 512, 10
    down = Stored.upload(dtype, (experts, hidden, ffn),
                         synthetic.quantized(rng, dtype, experts * hidden, ffn))
    for call in range(2):
        rows = synthetic.gaussian(rng, slots // 2, ffn)
        ids = dev(rng.integers(0, experts, slots).astype(np.int32))
        alone = torch.empty(slots, hidden, device="cuda")
        ops.experts_linear(dev(np.repeat(rows, 2, axis=0)), down, ids, alone)
        shared = torch.empty(slots, hidden, device="cuda")
        ops.experts_linear(dev(rows), down, ids, shared)
        assert torch.equal(alone, shared), call
        expected = oracle.experts_linear(dtype, np.repeat(rows, 2, axis=0), down.data.cpu().numpy(),
                                         experts, hidden, ffn, ids.cpu().numpy())
        ok, _, _, summary = within(alone.cpu().numpy(), expected, 1e-4, 1e-3)
        assert ok, summary
    assert ops.take_device_error() == 0


def test_experts_bad_id_is_flagged(ops):
    rng = np.random.default_rng(61)
    w = Stored.upload(oracle.Q4_1, (2, 64, 64), synthetic.quantized(rng, oracle.Q4_1, 128, 64))
    ops.take_device_error()
    out = torch.zeros(2, 64, device="cuda")
    ops.experts_linear(dev(synthetic.gaussian(rng, 1, 64)), w, dev(np.array([1, 7], np.int32)),
                       out)
    assert ops.take_device_error() == 1
    result = out.cpu().numpy()
    assert np.isfinite(result[0]).all() and np.isnan(result[1]).all()


def test_moe_combine_and_norm(ops):
    rng = np.random.default_rng(70)
    tokens, k, hidden = 4, 10, 2048
    expert_out = synthetic.gaussian(rng, tokens * k, hidden)
    weights = rng.random((tokens, k)).astype(np.float32)
    weights /= weights.sum(axis=1, keepdims=True)
    residual = synthetic.gaussian(rng, tokens, hidden)
    shared_out = synthetic.gaussian(rng, tokens, hidden)
    shared_in = synthetic.gaussian(rng, tokens, hidden)
    router = (synthetic.gaussian(rng, hidden) * 0.05).astype(np.float32)
    norm_w = (1 + rng.standard_normal(hidden) * 0.02).astype(np.float32)
    shared = SharedExpert(dev(shared_out), dev(shared_in), dev(router))
    out = torch.empty(tokens, hidden, device="cuda")
    ops.moe_combine(dev(expert_out), dev(weights), shared, dev(residual), out)
    expected = oracle.moe_combine(expert_out, weights, hidden, shared_out, shared_in, router,
                                  residual)
    ok, _, _, summary = within(out.cpu().numpy(), expected, 1e-5, 1e-5)
    assert ok, summary
    res = dev(residual)
    normed = torch.empty(tokens, hidden, device="cuda")
    ops.moe_combine_norm(dev(expert_out), dev(weights), shared, res,
                         RowNorm(dev(norm_w), 1e-6, 0.0, normed))
    e_res, e_norm = oracle.moe_combine_norm(expert_out, weights, hidden, residual, norm_w, 1e-6,
                                            0.0, shared_out, shared_in, router)
    assert within(res.cpu().numpy(), e_res, 1e-5, 1e-5)[0]
    ok, _, _, summary = within(normed.cpu().numpy(), e_norm, 1e-5, 1e-5)
    assert ok, summary
    # no shared expert, no residual
    ops.moe_combine(dev(expert_out), dev(weights), None, None, out)
    expected = oracle.moe_combine(expert_out, weights, hidden)
    assert within(out.cpu().numpy(), expected, 1e-5, 1e-5)[0]
