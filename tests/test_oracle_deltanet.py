"""The oracle's Gated DeltaNet ops (restated from ops/CpuSequence.scala:29-158,
CpuNormalisation.scala:167-178) against the golden vectors of transformers'
implementation, which the reference restates (tests/golden/
make_deltanet_golden.py; transformers computes in F32, so the bar is F32
rounding), and their structural properties."""

import os

import numpy as np

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "deltanet.npz")


def test_causal_conv_matches_transformers():
    z = np.load(GOLDEN)
    state = z["conv_state"].copy()
    out = oracle.causal_conv(z["x"], z["weight"], state)
    np.testing.assert_allclose(out, z["convolved"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(state, z["conv_state_after"])


def test_gated_delta_rule_matches_transformers():
    z = np.load(GOLDEN)
    tokens, key_heads, value_heads, d, _ = (int(v) for v in z["shape"])
    state = z["state"].copy()
    out = oracle.gated_delta_rule(z["convolved"], z["a"], z["b"], z["decay"], z["dt_bias"], state,
                                  key_heads, value_heads)
    np.testing.assert_allclose(out, z["out"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(state, z["state_after"], rtol=1e-4, atol=1e-6)


def test_token_by_token_equals_all_at_once():
    """Decode steps one token at a time end where the three-token call ends
    (the state carries everything), and the history holds each step's state."""
    z = np.load(GOLDEN)
    tokens, key_heads, value_heads, d, _ = (int(v) for v in z["shape"])
    whole = z["state"].copy()
    out, history = oracle.gated_delta_rule(z["convolved"], z["a"], z["b"], z["decay"],
                                           z["dt_bias"], whole, key_heads, value_heads,
                                           keep_history=True)
    step = z["state"].copy()
    for t in range(tokens):
        one = oracle.gated_delta_rule(z["convolved"][t:t + 1], z["a"][t:t + 1], z["b"][t:t + 1],
                                      z["decay"], z["dt_bias"], step, key_heads, value_heads)
        np.testing.assert_allclose(one[0], out[t], rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(step, history[t], rtol=1e-6, atol=1e-7)
    conv_whole = z["conv_state"].copy()
    conv_out, conv_history = oracle.causal_conv(z["x"], z["weight"], conv_whole, keep_history=True)
    conv_step = z["conv_state"].copy()
    for t in range(tokens):
        np.testing.assert_array_equal(oracle.causal_conv(z["x"][t:t + 1], z["weight"], conv_step)[0],
                                      conv_out[t])
        np.testing.assert_array_equal(conv_step, conv_history[t])


def test_tiled_heads_read_key_head_h_mod_key_heads():
    """DeltaRule.keyHeadOf (ops/DeltaRule.scala:18-20): with tiled heads, value
    head h reads key head h % key_heads; swapping the key heads' q and k then
    swaps the results of value heads 0 and 1 (2 key heads, 4 value heads)."""
    rng = np.random.default_rng(5)
    key_heads, value_heads, d = 2, 4, 16
    qkv = rng.standard_normal((1, (2 * key_heads + value_heads) * d)).astype(np.float32)
    a = rng.standard_normal((1, value_heads)).astype(np.float32)
    b = rng.standard_normal((1, value_heads)).astype(np.float32)
    decay = np.full(value_heads, -1.0, np.float32)
    bias = np.zeros(value_heads, np.float32)
    tiled = oracle.gated_delta_rule(qkv, a, b, decay, bias, np.zeros((4, d, d), np.float32),
                                    key_heads, value_heads, tiled=True)
    grouped = oracle.gated_delta_rule(qkv, a, b, decay, bias, np.zeros((4, d, d), np.float32),
                                      key_heads, value_heads, tiled=False)
    # value head 1 reads key head 1 when tiled, key head 0 when grouped
    assert not np.allclose(tiled[0, 1], grouped[0, 1])
    np.testing.assert_array_equal(tiled[0, 0], grouped[0, 0])


def test_gated_rms_norm_is_the_norm_times_the_gate():
    rng = np.random.default_rng(6)
    x = rng.standard_normal((4, 128)).astype(np.float32)
    gate = rng.standard_normal((4, 128)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    for kind in (0, 3):
        got = oracle.gated_rms_norm(x, w, gate, kind, 1e-6)
        np.testing.assert_array_equal(got, oracle.gated(kind, gate, oracle.rms_norm(x, w, 1e-6)))
