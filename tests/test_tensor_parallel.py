"""The tensor-parallel split of the products (drift_b200/tensor_parallel.py)
on the CPU: the shard arithmetic, and two gloo ranks running a column-split
product into a row-split one with the all-reduce, each rank's products
computed by the oracle (CpuLinear.linear) standing in for the GPU's.

The products themselves are checked on the GPU elsewhere; here the question
is whether the shards and the exchange reassemble the unsplit result.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from drift_b200 import synthetic
from drift_b200.tensor_parallel import (ColumnParallelLinear, RowParallelLinear, column_range,
                                        max_over_ranks, row_range, shard_columns, shard_rows)
from tests.conftest import within

TYPES = [oracle.Q8_0, oracle.Q4_0, oracle.Q4_1]


@pytest.mark.parametrize("rows,world", [(4096, 2), (4096, 8), (151936, 8), (7, 3), (12288, 4)])
def test_row_ranges_tile_the_rows(rows, world):
    spans = [row_range(rows, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == rows
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1


@pytest.mark.parametrize("cols,world", [(4096, 2), (4096, 8), (12288, 8), (2560, 3)])
def test_column_ranges_are_whole_blocks(cols, world):
    spans = [column_range(cols, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == cols
    assert all(l % 32 == 0 and h % 32 == 0 for l, h in spans)
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_column_ranges_refuse_partial_blocks():
    with pytest.raises(ValueError):
        column_range(100, 0, 2)
    with pytest.raises(ValueError):
        column_range(64, 0, 3)  # two blocks, three ranks


@pytest.mark.parametrize("dtype", TYPES)
def test_shards_decode_to_the_slices(dtype):
    rng = np.random.default_rng(5)
    n, k, world = 24, 320, 3
    w = synthetic.random_blocks(rng, dtype, n, k)
    full = oracle.decode(dtype, w, n * k).reshape(n, k)
    for rank in range(world):
        part, count = shard_rows(w, dtype, n, k, rank, world)
        lo, hi = row_range(n, rank, world)
        assert count == hi - lo
        np.testing.assert_array_equal(oracle.decode(dtype, part, count * k).reshape(count, k),
                                      full[lo:hi])
        part, k0, k1 = shard_columns(w, dtype, n, k, rank, world)
        np.testing.assert_array_equal(
            oracle.decode(dtype, part, n * (k1 - k0)).reshape(n, k1 - k0), full[:, k0:k1])


class OracleWeight:
    def __init__(self, dtype, shape, data):
        self.dtype, self.shape, self.data = dtype, shape, data


class OracleOps:
    """`ops.linear` on the CPU: the oracle's CpuLinear.linear."""

    def linear(self, x, weight, out):
        n, k = weight.shape
        out.copy_(torch.from_numpy(oracle.linear(weight.dtype, x.numpy(), weight.data, n, k)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, dtype, m, n_mid, k, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        rng = np.random.default_rng(11)  # every rank draws the same weights and x
        up = synthetic.random_blocks(rng, dtype, n_mid, k)    # [n_mid, k]: column-split
        down = synthetic.random_blocks(rng, dtype, k, n_mid)  # [k, n_mid]: row-split
        x = rng.standard_normal((m, k)).astype(np.float32)
        upload = lambda t, shape, data: OracleWeight(t, shape, data)
        col = ColumnParallelLinear.from_blocks(up, dtype, n_mid, k, rank, world, upload)
        row = RowParallelLinear.from_blocks(down, dtype, k, n_mid, rank, world, upload)
        assert (col.lo, col.hi) == (row.k0, row.k1), "the shards of the two products must meet"
        ops = OracleOps()
        hidden = torch.empty(m, col.hi - col.lo)
        col(ops, torch.from_numpy(x), hidden)
        out = torch.empty(m, k)
        row(ops, hidden, out)
        slowest = max_over_ranks(float(rank + 1))
        results.put((rank, out.numpy(), hidden.numpy(), col.lo, col.hi, slowest))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype", TYPES)
def test_two_gloo_ranks_reassemble_the_product(dtype):
    """Column-split up (n_mid = 256 rows, 128 per rank) then row-split down
    with the all-reduce: every rank ends with the unsplit down . (up . x)."""
    m, n_mid, k, world = 3, 256, 512, 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, dtype, m, n_mid, k, results))
             for r in range(world)]
    for p in procs:
        p.start()
    got = [results.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(11)
    up = synthetic.random_blocks(rng, dtype, n_mid, k)
    down = synthetic.random_blocks(rng, dtype, k, n_mid)
    x = rng.standard_normal((m, k)).astype(np.float32)
    hidden = oracle.linear(dtype, x, up, n_mid, k)
    expected = oracle.linear(dtype, hidden, down, k, n_mid)
    for rank, out, part, lo, hi, slowest in got:
        # the column split is the unsplit rows, bit for bit
        np.testing.assert_array_equal(part, hidden[:, lo:hi])
        # the row split sums two float partials: the benchmark's bar
        ok, _, _, summary = within(out, expected, 1e-4, 1e-3)
        assert ok, summary
        assert slowest == float(world)


# ---- the greedy choice over vocabulary shards (VocabSampler) ------------------------------------
class KeyedArgmax:
    """The device argmax's order on the host (numpy): the value's order bits
    (a NaN lowest, except at id 0, which is highest) above the id, lower ids
    first -- so a shard's local choice and the merge pick what
    CpuSequence.argmax picks over the whole row."""

    @staticmethod
    def _keys(values, ids):
        bits = values.astype(np.float32).copy()
        bits[bits == 0] = 0.0
        u = bits.view(np.uint32).astype(np.uint64)
        order = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
        nan = np.isnan(values)
        order = np.where(nan, np.where(ids == 0, 0xFFFFFFFF, 0), order).astype(np.uint64)
        return (order << np.uint64(32)) | ((~ids.astype(np.uint64)) & np.uint64(0xFFFFFFFF))

    def argmax(self, values, ids, out_values, id_offset):
        v = values.numpy()
        rows, width = v.shape
        index = np.arange(width, dtype=np.int64) + id_offset
        best = self._keys(v, np.broadcast_to(index, v.shape)).argmax(axis=1)
        ids.copy_(torch.from_numpy((best + id_offset).astype(np.int32)))
        if out_values is not None:
            out_values.copy_(torch.from_numpy(v[np.arange(rows), best]))

    def argmax_merge(self, values, ids_in, ids, out_values):
        v, g = values.numpy(), ids_in.numpy().astype(np.int64)
        best = self._keys(v, g).argmax(axis=1)
        ids.copy_(torch.from_numpy(g[np.arange(v.shape[0]), best].astype(np.int32)))


def _sampler_rank(rank, world, port, results):
    from drift_b200.tensor_parallel import VocabSampler, row_range
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        rng = np.random.default_rng(3)  # every rank draws the same logits
        rows, vocab = 4, 1003
        logits = rng.standard_normal((rows, vocab)).astype(np.float32)
        logits[0, 17] = logits[0, 900] = 9.0   # a tie across shards: the lower id
        logits[1, 0] = np.nan                  # a NaN at id 0: id 0, whatever follows
        logits[2, 5] = np.nan                  # a NaN elsewhere never wins
        lo, hi = row_range(vocab, rank, world)
        sampler = VocabSampler(KeyedArgmax(), rows, lo, dist.group.WORLD)
        ids = torch.empty(rows, dtype=torch.int32)
        sampler(torch.from_numpy(np.ascontiguousarray(logits[:, lo:hi])), ids)
        results.put((rank, ids.numpy().copy(), logits))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_vocabulary_shards_choose_the_whole_rows_argmax(world):
    """Each gloo rank holds a vocabulary shard; after the sampler's gather and
    merge every rank holds CpuSequence.argmax of the whole rows."""
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sampler_rank, args=(r, world, port, results))
             for r in range(world)]
    for p in procs:
        p.start()
    got = [results.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ids, logits in got:
        assert list(ids) == [oracle.argmax(row) for row in logits], rank
