"""Gated DeltaNet on the GPU (drift_causal_conv, drift_gated_delta_rule,
drift_gated_rms_norm) against the oracle (CpuSequence.causalConv /
gatedDeltaRule, CpuNormalisation.gatedRmsNorm, which sum in Double), held to
the 1e-4 absolute + 1e-3 relative bar; states too, after several decode steps."""

import numpy as np
import pytest
import torch

import oracle
from drift_b200.ops import SIGMOID, SILU, CudaOps
from tests.conftest import within

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    return CudaOps()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("tokens,channels,taps,dilation", [(1, 8192, 4, 1), (3, 1000, 4, 1),
                                                           (5, 64, 3, 2), (2, 33, 1, 1),
                                                           (4, 128, 9, 2)])
def test_causal_conv(ops, tokens, channels, taps, dilation):
    rng = np.random.default_rng(tokens * 100 + channels)
    span = (taps - 1) * dilation
    x = rng.standard_normal((tokens, channels)).astype(np.float32)
    w = (0.5 * rng.standard_normal((channels, taps))).astype(np.float32)
    state = rng.standard_normal((span, channels)).astype(np.float32)
    expected_state = state.copy()
    expected, expected_history = oracle.causal_conv(x, w, expected_state, dilation, keep_history=True)
    gpu_state = dev(state)
    history = torch.empty(tokens, span, channels, device="cuda")
    out = torch.empty(tokens, channels, device="cuda")
    ops.causal_conv(dev(x), dev(w), dilation, gpu_state, history, out)
    ok, _, _, summary = within(out.cpu().numpy(), expected, 1e-4, 1e-3)
    assert ok, summary
    # the state and the history are moved inputs: exact
    np.testing.assert_array_equal(gpu_state.cpu().numpy(), expected_state)
    np.testing.assert_array_equal(history.cpu().numpy(), expected_history)


RULES = [(16, 32, 128, False), (2, 4, 128, False), (2, 4, 64, True), (4, 4, 32, False),
         (1, 8, 128, True)]


@pytest.mark.parametrize("rule", RULES, ids=[f"k{r[0]}v{r[1]}d{r[2]}{'t' if r[3] else ''}" for r in RULES])
@pytest.mark.parametrize("tokens", [1, 3])
def test_gated_delta_rule(ops, rule, tokens):
    key_heads, value_heads, d, tiled = rule
    rng = np.random.default_rng(d + tokens + value_heads)
    width = (2 * key_heads + value_heads) * d
    qkv = rng.standard_normal((tokens, width)).astype(np.float32)
    a = rng.standard_normal((tokens, value_heads)).astype(np.float32)
    b = rng.standard_normal((tokens, value_heads)).astype(np.float32)
    decay = (-np.exp(rng.uniform(-1, 1.5, value_heads))).astype(np.float32)
    dt_bias = rng.standard_normal(value_heads).astype(np.float32)
    state = (0.05 * rng.standard_normal((value_heads, d, d))).astype(np.float32)
    expected_state = state.copy()
    expected, expected_history = oracle.gated_delta_rule(qkv, a, b, decay, dt_bias, expected_state,
                                                          key_heads, value_heads, tiled,
                                                          keep_history=True)
    gpu_state = dev(state)
    history = torch.empty(tokens, value_heads, d, d, device="cuda")
    out = torch.empty(tokens, value_heads, d, device="cuda")
    ops.gated_delta_rule(dev(qkv), dev(a), dev(b), dev(decay), dev(dt_bias), gpu_state,
                         (key_heads, value_heads, d, tiled), history, out)
    for got, want, name in ((out, expected, "out"), (gpu_state, expected_state, "state"),
                            (history, expected_history, "history")):
        ok, _, _, summary = within(got.cpu().numpy(), want, 1e-4, 1e-3)
        assert ok, f"{name}: {summary}"


def test_decode_steps_carry_the_state(ops):
    """Ten single-token steps (the decode loop) stay within the bar of the
    oracle's ten steps."""
    rng = np.random.default_rng(10)
    key_heads, value_heads, d = 2, 4, 128
    width = (2 * key_heads + value_heads) * d
    decay = (-np.exp(rng.uniform(-1, 1.5, value_heads))).astype(np.float32)
    dt_bias = rng.standard_normal(value_heads).astype(np.float32)
    state = np.zeros((value_heads, d, d), np.float32)
    gpu_state = dev(state)
    out = torch.empty(1, value_heads, d, device="cuda")
    for step in range(10):
        qkv = rng.standard_normal((1, width)).astype(np.float32)
        a = rng.standard_normal((1, value_heads)).astype(np.float32)
        b = rng.standard_normal((1, value_heads)).astype(np.float32)
        expected = oracle.gated_delta_rule(qkv, a, b, decay, dt_bias, state, key_heads, value_heads)
        ops.gated_delta_rule(dev(qkv), dev(a), dev(b), dev(decay), dev(dt_bias), gpu_state,
                             (key_heads, value_heads, d, False), None, out)
        ok, _, _, summary = within(out.cpu().numpy(), expected, 1e-4, 1e-3)
        assert ok, f"step {step}: {summary}"
        # carry the oracle's own state forward (each step is checked on its own)
        gpu_state.copy_(dev(state))


@pytest.mark.parametrize("kind", [SILU, SIGMOID])
@pytest.mark.parametrize("rows,cols", [(16, 128), (3, 64), (5, 256), (2, 500)])
def test_gated_rms_norm(ops, kind, rows, cols):
    rng = np.random.default_rng(rows * cols + kind)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    gate = rng.standard_normal((rows, cols)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    expected = oracle.gated_rms_norm(x, w, gate, kind, 1e-6)
    out = torch.empty(rows, cols, device="cuda")
    ops.gated_rms_norm(dev(x), dev(w), dev(gate), kind, 1e-6, out)
    ok, _, _, summary = within(out.cpu().numpy(), expected, 1e-4, 1e-3)
    assert ok, summary


def test_gated_rms_norm_records_feed_the_out_projection(ops):
    from drift_b200 import synthetic
    from drift_b200.ops import Stored
    rng = np.random.default_rng(12)
    tokens, heads, d = 2, 16, 128
    x = dev(rng.standard_normal((tokens * heads, d)).astype(np.float32))
    gate = dev(rng.standard_normal((tokens * heads, d)).astype(np.float32))
    w = dev((1 + 0.1 * rng.standard_normal(d)).astype(np.float32))
    weight = Stored.upload(oracle.Q4_1, (256, heads * d),
                           synthetic.quantized(rng, oracle.Q4_1, 256, heads * d))
    prepared = ops.prepared_x(tokens, heads * d)
    out = torch.empty_like(x)
    ops.gated_rms_norm(x, w, gate, SILU, 1e-6, out, prepared, heads)
    fused = torch.empty(tokens, 256, device="cuda")
    ops.linears(out.view(tokens, heads * d), [weight], [fused], prepared)
    alone = torch.empty_like(fused)
    ops.linear(out.view(tokens, heads * d), weight, alone)
    assert torch.equal(fused, alone)


@pytest.mark.parametrize("sequences", [1, 3, 16])
@pytest.mark.parametrize("key_heads,value_heads,dim,taps", [(4, 4, 128, 4), (16, 16, 128, 4),
                                                             (2, 4, 128, 4), (4, 4, 64, 3)])
def test_delta_decode_step_is_the_three_launches(ops, sequences, key_heads, value_heads, dim,
                                                 taps):
    """The fused decode step (one launch when each value head has its own key
    head and heads are 128 wide) against causal_conv_decode, then
    gated_delta_rule_decode, then the SiLU-gated rms norm with records: the
    same outputs, states, convolution states and records, bit for bit."""
    g = torch.Generator(device="cuda").manual_seed(sequences * 31 + key_heads + dim)
    channels = (2 * key_heads + value_heads) * dim
    f = lambda *shape, s=1.0: s * torch.randn(*shape, generator=g, device="cuda")
    qkv, z = f(sequences, channels), f(sequences, value_heads, dim)
    conv = f(channels, taps, s=0.5)
    conv_states = f(sequences, taps - 1, channels)
    a, b = f(sequences, value_heads), f(sequences, value_heads)
    decay = -torch.exp(torch.rand(value_heads, generator=g, device="cuda") * 2.5 - 1.0)
    dt_bias = f(value_heads)
    states = f(sequences, value_heads, dim, dim, s=0.02)
    norm = 1.0 + 0.02 * f(dim)
    rule = (key_heads, value_heads, dim, False)
    conv1, states1 = conv_states.clone(), states.clone()
    out1 = torch.empty(sequences, value_heads, dim, device="cuda")
    prepared1 = ops.prepared_x(sequences, value_heads * dim)
    prepared1.fill_(0xA5)  # the slots past the sequences are left as they were
    ops.delta_decode_step(qkv, z, conv, conv1, torch.empty_like(qkv), a, b, decay, dt_bias,
                          states1, rule, norm, 1e-6, out1, prepared1)
    conv2, states2 = conv_states.clone(), states.clone()
    convolved = torch.empty_like(qkv)
    ops.causal_conv_decode(qkv, conv, 1, conv2, convolved)
    out2 = torch.empty_like(out1)
    ops.gated_delta_rule_decode(convolved, a, b, decay, dt_bias, states2, rule, out2)
    prepared2 = ops.prepared_x(sequences, value_heads * dim)
    prepared2.fill_(0xA5)
    core = out2.view(sequences * value_heads, dim)
    ops.gated_rms_norm(core, norm, z.view(sequences * value_heads, dim), SILU, 1e-6, core,
                       prepared2, value_heads)
    torch.cuda.synchronize()
    assert torch.equal(conv1, conv2)
    assert torch.equal(states1, states2)
    assert torch.equal(out1, out2)
    assert torch.equal(prepared1, prepared2)


def test_refusals(ops):
    x = torch.zeros(1, 64, device="cuda")
    with pytest.raises(ValueError, match="state"):
        ops.causal_conv(x, torch.zeros(64, 4, device="cuda"), 1, torch.zeros(2, 64, device="cuda"),
                        None, torch.empty_like(x))
    with pytest.raises(ValueError, match="heads of 48"):
        ops.gated_delta_rule(torch.zeros(1, 4 * 48, device="cuda"), torch.zeros(1, 2, device="cuda"),
                             torch.zeros(1, 2, device="cuda"), torch.zeros(2, device="cuda"),
                             torch.zeros(2, device="cuda"), torch.zeros(2, 48, 48, device="cuda"),
                             (1, 2, 48, False), None, torch.zeros(1, 2, 48, device="cuda"))
    with pytest.raises(ValueError, match="SiLU or sigmoid"):
        ops.gated_rms_norm(x, torch.ones(64, device="cuda"), x, 1, 1e-6, torch.empty_like(x))
