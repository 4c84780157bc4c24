"""The hybrid MoE decode step (drift_b200/hybrid.py: HybridBlocks' op order,
runner/src/drift/runner/models/HybridBlocks.scala:403-588) on a small model
against the same step composed from the oracle's ops (the reference's
CpuOps: CpuSequence's convolution and delta rule, CpuAttention, CpuExperts),
weights, caches and states downloaded from the GPU. Held to the benchmark's
1e-4 absolute + 1e-3 relative on the logits after four layers (three DeltaNet,
one gated full attention, each with a mixture of experts)."""

import dataclasses
import math

import numpy as np
import pytest
import torch

import oracle
from drift_b200.hybrid import FullLayer, HybridConfig, HybridDecoder, HybridWeights
from drift_b200.ops import CudaOps
from tests.conftest import within

pytestmark = pytest.mark.gpu

SMALL = HybridConfig(layers=4, hidden=256, delta_key_heads=2, delta_value_heads=4, delta_dim=32,
                     q_heads=4, kv_heads=2, head_dim=64, rotary=16, theta=1e6, experts=16,
                     used=4, expert_ffn=64, shared_ffn=64, vocab=500)
# a shared expert of another width: its own launches (SMALL's rides in the
# routed experts' launches, as one more expert of their weights)
APART = dataclasses.replace(SMALL, shared_ffn=128)


def host(t):
    return t.cpu().numpy()


def reference_step(c, w, d, ids, positions):
    """The decode step of HybridBlocks, op for op, on the oracle; `d` holds
    the decoder's caches and states as they were before the step (numpy)."""
    b = len(ids)
    x = oracle.embedding(w.embedding.dtype, host(w.embedding.data), c.vocab, c.hidden, ids)
    normed = oracle.rms_norm(x, host(w.layers[0].input_norm), c.epsilon)
    for index, layer in enumerate(w.layers):
        m = layer.mixer
        if isinstance(m, FullLayer):
            qg = oracle.linear(m.q.dtype, normed, host(m.q.data), c.q_heads * 2 * c.head_dim, c.hidden)
            k = oracle.linear(m.k.dtype, normed, host(m.k.data), c.kv_heads * c.head_dim, c.hidden)
            v = oracle.linear(m.v.dtype, normed, host(m.v.data), c.kv_heads * c.head_dim, c.hidden)
            qg = qg.reshape(b, c.q_heads, 2 * c.head_dim)
            q, gate = qg[:, :, :c.head_dim], qg[:, :, c.head_dim:]
            q = oracle.rms_norm(q.reshape(b, c.q_heads, c.head_dim), host(m.q_norm), c.epsilon)
            k = oracle.rms_norm(k.reshape(b, c.kv_heads, c.head_dim), host(m.k_norm), c.epsilon)
            pos = np.array(positions, np.int32)
            q = oracle.rope(q, pos, c.theta, c.rotary, 0)
            k = oracle.rope(k, pos, c.theta, c.rotary, 0)
            v = v.reshape(b, c.kv_heads, c.head_dim)
            keys, values = d["caches"][index]
            attended = np.empty((b, c.q_heads, c.head_dim), np.float32)
            for i in range(b):
                oracle.cache_write(k[i:i + 1], v[i:i + 1], keys, values, c.page_size, d["tables"][i],
                                   positions[i])
                attended[i:i + 1] = oracle.attention(q[i:i + 1], keys, values, c.page_size,
                                                     c.kv_heads, d["tables"][i], positions[i],
                                                     positions[i] + 1, 1 / math.sqrt(c.head_dim))
            attended = oracle.gated(3, gate, attended)  # sigmoid(gate) x attended
            out = oracle.linear(m.o.dtype, attended.reshape(b, -1), host(m.o.data), c.hidden,
                                c.q_heads * c.head_dim)
        else:
            channels = (2 * c.delta_key_heads + c.delta_value_heads) * c.delta_dim
            width = c.delta_value_heads * c.delta_dim
            qkv = oracle.linear(m.qkv.dtype, normed, host(m.qkv.data), channels, c.hidden)
            z = oracle.linear(m.z.dtype, normed, host(m.z.data), width, c.hidden)
            a = normed.astype(np.float64) @ host(m.a).astype(np.float64).T
            bb = normed.astype(np.float64) @ host(m.b).astype(np.float64).T
            a, bb = a.astype(np.float32), bb.astype(np.float32)
            core = np.empty((b, c.delta_value_heads, c.delta_dim), np.float32)
            for i in range(b):
                conv = oracle.causal_conv(qkv[i:i + 1], host(m.conv), d["conv"][index][i])
                core[i:i + 1] = oracle.gated_delta_rule(conv, a[i:i + 1], bb[i:i + 1],
                                                        host(m.decay), host(m.dt_bias),
                                                        d["delta"][index][i], c.delta_key_heads,
                                                        c.delta_value_heads)
            core = oracle.gated_rms_norm(core.reshape(-1, c.delta_dim), host(m.norm),
                                         z.reshape(-1, c.delta_dim), 0, c.epsilon)
            out = oracle.linear(m.out.dtype, core.reshape(b, -1), host(m.out.data), c.hidden, width)
        x, normed = oracle.add_rms_norm(x, out, host(layer.post_norm), c.epsilon)
        mix = layer.mixture
        logits = (normed.astype(np.float64) @ host(mix.router).astype(np.float64).T).astype(np.float32)
        ids_k, weights_k = oracle.route(logits, c.used)
        gated = oracle.experts_gated_linear(mix.gate.dtype, normed, host(mix.gate.data),
                                            host(mix.up.data), c.experts, c.expert_ffn, c.hidden,
                                            ids_k)
        shared_gated = oracle.experts_gated_linear(mix.shared_gate.dtype, normed,
                                                   host(mix.shared_gate.data),
                                                   host(mix.shared_up.data), 1, c.shared_ffn,
                                                   c.hidden, np.zeros(b, np.int32))
        expert_out = oracle.experts_linear(mix.down.dtype, gated, host(mix.down.data), c.experts,
                                           c.hidden, c.expert_ffn, ids_k)
        shared_out = oracle.linear(mix.shared_down.dtype, shared_gated, host(mix.shared_down.data),
                                   c.hidden, c.shared_ffn)
        following = (w.layers[index + 1].input_norm if index + 1 < len(w.layers) else w.final_norm)
        x, normed = oracle.moe_combine_norm(expert_out, weights_k, c.hidden, x, host(following),
                                            c.epsilon, 0.0, shared_out, normed, host(mix.shared_router))
    return oracle.linear(w.lm_head.dtype, normed, host(w.lm_head.data), c.vocab, c.hidden)


@pytest.mark.parametrize("c", [SMALL, APART], ids=["shared-in-experts", "shared-apart"])
@pytest.mark.parametrize("batch", [1, 3])
def test_hybrid_step_matches_the_oracle(c, batch):
    ops = CudaOps()
    weights = HybridWeights.random(c, seed=7)
    decoder = HybridDecoder(ops, c, weights, batch=batch, context=64)
    decoder.prefill_random(30)
    positions = [30 - 2 * i for i in range(batch)]
    rng = np.random.default_rng(batch)
    ids = rng.integers(0, c.vocab, batch).astype(np.int32)
    decoder.ids.copy_(torch.from_numpy(ids))
    decoder.positions.copy_(torch.tensor(positions, dtype=torch.int32))
    before = {
        "caches": {i: (cache.keys.cpu().numpy().view(np.uint16).copy(),
                       cache.values.cpu().numpy().view(np.uint16).copy())
                   for i, cache in decoder.caches.items()},
        "conv": {i: s.cpu().numpy().copy() for i, s in decoder.conv_states.items()},
        "delta": {i: s.cpu().numpy().copy() for i, s in decoder.delta_states.items()},
        "tables": [t.cpu().numpy() for t in decoder.page_tables],
    }
    logits = decoder.step().cpu().numpy()
    expected = reference_step(c, weights, before, ids, positions)
    ok, _, _, summary = within(logits, expected, 1e-4, 1e-3)
    assert ok, summary
    # the step's greedy choice: the CPU argmax of its own logits, bit for bit
    assert list(decoder.next_ids.cpu().numpy()) == [oracle.argmax(row) for row in logits]
    # the recurrent states moved as the oracle's did
    for i, state in decoder.delta_states.items():
        ok, _, _, summary = within(state.cpu().numpy(), before["delta"][i], 1e-4, 1e-3)
        assert ok, f"delta state {i}: {summary}"
    for i, state in decoder.conv_states.items():
        ok, _, _, summary = within(state.cpu().numpy(), before["conv"][i], 1e-4, 1e-3)
        assert ok, f"conv state {i}: {summary}"


def test_captured_hybrid_step_replays_the_eager_step():
    c = SMALL
    ops = CudaOps()
    weights = HybridWeights.random(c, seed=8)
    decoder = HybridDecoder(ops, c, weights, batch=2, context=64)
    decoder.prefill_random(20)
    decoder.ids.copy_(torch.tensor([3, 9], dtype=torch.int32))
    decoder.positions.copy_(torch.tensor([20, 15], dtype=torch.int32))
    conv = {i: s.clone() for i, s in decoder.conv_states.items()}
    delta = {i: s.clone() for i, s in decoder.delta_states.items()}
    eager = decoder.step().clone()
    eager_delta = {i: s.clone() for i, s in decoder.delta_states.items()}
    for i in conv:
        decoder.conv_states[i].copy_(conv[i])
    for i in delta:
        decoder.delta_states[i].copy_(delta[i])
    decoder.capture()
    decoder.replay()
    torch.cuda.synchronize()
    assert torch.equal(decoder.logits, eager)
    for i in delta:
        assert torch.equal(decoder.delta_states[i], eager_delta[i])
    decoder.release()
