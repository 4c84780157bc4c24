"""The dense decode step (drift_b200/decoder.py, DenseDecoder.run's op order)
on a small model against the same step composed from the oracle's ops (the
reference's CpuOps), weights and caches downloaded from the GPU.

Held to the benchmark's 1e-4 absolute + 1e-3 relative on the logits after two
layers: each op is within its own bar, and the step compounds them.
"""

import math

import numpy as np
import pytest
import torch

import oracle
from drift_b200.decoder import DenseConfig, DenseDecoder, DenseWeights
from drift_b200.ops import CudaOps
from tests.conftest import within

pytestmark = pytest.mark.gpu

SMALL = DenseConfig(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000)


def host(stored):
    return stored.data.cpu().numpy()


def reference_step(c, w, caches, tables, ids, positions):
    """The decode step of DenseDecoder.run, op for op, on the oracle."""
    b, hd = len(ids), c.head_dim
    x = oracle.embedding(w.embedding.dtype, host(w.embedding), c.vocab, c.hidden, ids)
    normed = oracle.rms_norm(x, w.layers[0].attention_norm.cpu().numpy(), c.epsilon)
    for index, (layer, (keys, values)) in enumerate(zip(w.layers, caches)):
        q = oracle.linear(layer.q.dtype, normed, host(layer.q), c.q_heads * hd, c.hidden)
        k = oracle.linear(layer.k.dtype, normed, host(layer.k), c.kv_heads * hd, c.hidden)
        v = oracle.linear(layer.v.dtype, normed, host(layer.v), c.kv_heads * hd, c.hidden)
        q = oracle.rms_norm(q.reshape(b, c.q_heads, hd), layer.q_norm.cpu().numpy(), c.epsilon)
        k = oracle.rms_norm(k.reshape(b, c.kv_heads, hd), layer.k_norm.cpu().numpy(), c.epsilon)
        pos = np.array(positions, dtype=np.int32)
        q = oracle.rope(q, pos, c.theta, hd, 0)
        k = oracle.rope(k, pos, c.theta, hd, 0)
        v = v.reshape(b, c.kv_heads, hd)
        attended = np.empty((b, c.q_heads, hd), dtype=np.float32)
        for i in range(b):
            oracle.cache_write(k[i:i + 1], v[i:i + 1], keys, values, c.page_size, tables[i],
                               positions[i])
            attended[i:i + 1] = oracle.attention(q[i:i + 1], keys, values, c.page_size,
                                                 c.kv_heads, tables[i], positions[i],
                                                 positions[i] + 1, 1.0 / math.sqrt(hd))
        projected = oracle.linear(layer.o.dtype, attended.reshape(b, -1), host(layer.o), c.hidden,
                                  c.q_heads * hd)
        x, normed = oracle.add_rms_norm(x, projected, layer.mlp_norm.cpu().numpy(), c.epsilon)
        gate = oracle.linear(layer.gate.dtype, normed, host(layer.gate), c.ffn, c.hidden)
        up = oracle.linear(layer.up.dtype, normed, host(layer.up), c.ffn, c.hidden)
        hidden = oracle.gated(0, gate, up)
        down = oracle.linear(layer.down.dtype, hidden, host(layer.down), c.hidden, c.ffn)
        following = (w.layers[index + 1].attention_norm if index + 1 < len(w.layers)
                     else w.final_norm)
        x, normed = oracle.add_rms_norm(x, down, following.cpu().numpy(), c.epsilon)
    return oracle.linear(w.lm_head.dtype, normed, host(w.lm_head), c.vocab, c.hidden)


@pytest.mark.parametrize("batch", [1, 3])
def test_decode_step_matches_the_oracle(batch):
    c = SMALL
    ops = CudaOps()
    weights = DenseWeights.random(c, seed=3)
    decoder = DenseDecoder(ops, c, weights, batch=batch, context=96)
    decoder.prefill_random(40)
    positions = [40 - i for i in range(batch)]  # sequences at different lengths
    rng = np.random.default_rng(batch)
    ids = rng.integers(0, c.vocab, batch).astype(np.int32)
    decoder.ids.copy_(torch.from_numpy(ids))
    decoder.positions.copy_(torch.tensor(positions, dtype=torch.int32))
    caches = [(cache.keys.cpu().numpy().view(np.uint16).copy(),
               cache.values.cpu().numpy().view(np.uint16).copy()) for cache in decoder.caches]
    tables = [t.cpu().numpy() for t in decoder.tables]
    logits = decoder.step(positions).cpu().numpy()
    expected = reference_step(c, weights, caches, tables, ids, positions)
    ok, _, _, summary = within(logits, expected, 1e-4, 1e-3)
    assert ok, summary
    # the step's greedy choice: the CPU argmax of its own logits, bit for bit
    assert list(decoder.next_ids.cpu().numpy()) == [oracle.argmax(row) for row in logits]
    # the caches took the new keys and values: the same F16 values, give or
    # take the rounding of inputs that differ in their last F32 bits (the
    # write itself is bit-exact, test_gpu_attention.py)
    for (keys, values), cache in zip(caches, decoder.caches):
        for got, want in ((cache.keys, keys), (cache.values, values)):
            ok, _, _, summary = within(got.float().cpu().numpy(),
                                       want.view(np.float16).astype(np.float32), 1e-4, 1e-3)
            assert ok, summary


def test_captured_step_replays_the_eager_step():
    c = SMALL
    ops = CudaOps()
    weights = DenseWeights.random(c, seed=4)
    decoder = DenseDecoder(ops, c, weights, batch=2, context=64)
    decoder.prefill_random(30)
    decoder.ids.copy_(torch.tensor([5, 7], dtype=torch.int32))
    decoder.positions.copy_(torch.tensor([30, 30], dtype=torch.int32))
    eager = decoder.step([30, 30]).clone()
    decoder.capture([30, 30])
    decoder.replay()
    torch.cuda.synchronize()
    assert torch.equal(decoder.logits, eager)
    assert list(decoder.next_ids.cpu().numpy()) == [oracle.argmax(r) for r in eager.cpu().numpy()]
    decoder.release()
