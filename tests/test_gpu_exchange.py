"""The tensor-parallel exchange over NVLink peer memory (drift_comm_*,
drift_add_rms_norm_allreduce) on two GPUs, one process each: the fused
exchange + residual add + RMSNorm equals the sum in rank order followed by
addRmsNorm, bit for bit; and a two-rank decode step over the peer exchange
equals the same step over NCCL's all-reduce (for two ranks both sums are
p0 + p1); and the expert-parallel hybrid MoE step (DeltaNet and query heads,
experts and vocabulary split over two ranks) equals the whole model's step on
one GPU within the benchmark's bar; in both, every rank's greedy next token
is the argmax of the whole vocabulary's gathered row. Skipped with fewer
than two GPUs."""

import os
import socket
from datetime import timedelta

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs two GPUs")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int):
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return dist


def _exchange_ranks(rank: int, world: int, port: int):
    dist = _init(rank, world, port)
    from drift_b200.ops import CudaOps, RowNorm
    from drift_b200.tensor_parallel import PeerExchange
    try:
        ops = CudaOps()
        for rows, cols in ((1, 4096), (5, 4096), (16, 2048), (3, 512)):
            g = torch.Generator(device="cuda").manual_seed(1)
            x0 = torch.randn(rows, cols, device="cuda", generator=g)          # the same on every rank
            weight = 1 + 0.02 * torch.randn(cols, device="cuda", generator=g)
            parts = [torch.randn(rows, cols, device="cuda", generator=g) for _ in range(world)]
            exchange = PeerExchange(ops, dist.group.WORLD, rows, cols)
            prepared = ops.prepared_x(rows, cols)
            for step in range(3):  # the slots alternate; the counts advance
                slot = step % 2
                exchange.slots[slot].copy_(parts[rank] * (step + 1))
                x = x0.clone()
                normed = torch.empty_like(x)
                exchange.add_rms_norm(slot, x, RowNorm(weight, 1e-6, 0.0, normed), prepared)
                total = torch.zeros_like(x0)
                for p in range(world):
                    total = total + parts[p] * (step + 1)
                expected_x = x0.clone()
                expected = torch.empty_like(x)
                ops.add_rms_norm(expected_x, total, RowNorm(weight, 1e-6, 0.0, expected))
                torch.cuda.synchronize()
                assert torch.equal(x, expected_x), (rows, cols, step)
                assert torch.equal(normed, expected), (rows, cols, step)
            torch.cuda.synchronize()
            dist.barrier()
            exchange.close()
        assert ops.take_device_error() == 0
    finally:
        dist.destroy_process_group()


def _decode_ranks(rank: int, world: int, port: int):
    dist = _init(rank, world, port)
    from drift_b200.decoder import DenseConfig, DenseDecoder, DenseWeights
    from drift_b200.ops import CudaOps
    try:
        ops = CudaOps()
        c = DenseConfig(layers=2, hidden=512, q_heads=4, kv_heads=2, head_dim=64, ffn=1024,
                        vocab=1000)
        weights = DenseWeights.random(c, seed=5, rank=rank, world=world)
        logits = {}
        for exchange in ("nccl", "peer"):
            decoder = DenseDecoder(ops, c, weights, batch=3, context=64, group=dist.group.WORLD,
                                   exchange=exchange)
            decoder.prefill_random(20)
            decoder.ids.copy_(torch.tensor([1, 2, 3], dtype=torch.int32))
            decoder.positions.copy_(torch.tensor([20, 18, 7], dtype=torch.int32))
            logits[exchange] = decoder.step().clone()
            # the greedy choice over both ranks' vocabulary rows: every rank
            # picks the argmax of the whole gathered row
            gathered = [torch.empty_like(logits[exchange]) for _ in range(world)]
            dist.all_gather(gathered, logits[exchange])
            whole = torch.cat(gathered, dim=1).cpu().numpy()
            assert list(decoder.next_ids.cpu().numpy()) == [oracle.argmax(r) for r in whole]
            # and captured: the replay equals the eager step
            decoder.capture([20, 18, 7])
            decoder.replay()
            torch.cuda.synchronize()
            assert torch.equal(decoder.logits, logits[exchange]), exchange
            decoder.release()
        assert torch.equal(logits["peer"], logits["nccl"])
        assert ops.take_device_error() == 0
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _timeout_ranks(rank: int, world: int, port: int):
    """Rank 1 skips one exchange; rank 0's rows give up after the comm's 10 ms
    limit, device error 3, x and out untouched; both ranks then close the
    comm, and a new one works (the context is still usable)."""
    dist = _init(rank, world, port)
    try:
        # the one-CTA exchange (rows of up to 1024) and the clustered one
        for cols in (1024, 4096):
            _timeout_case(rank, world, dist, 4, cols)
    finally:
        dist.destroy_process_group()


def _timeout_case(rank, world, dist, rows, cols):
    """One skipped exchange under a 10 ms limit, then a fresh comm."""
    import time

    from drift_b200.ops import CudaOps, RowNorm
    from drift_b200.tensor_parallel import PeerExchange
    ops = CudaOps()
    g = torch.Generator(device="cuda").manual_seed(2)
    x0 = torch.randn(rows, cols, device="cuda", generator=g)
    weight = 1 + 0.02 * torch.randn(cols, device="cuda", generator=g)
    parts = [torch.randn(rows, cols, device="cuda", generator=g) for _ in range(world)]
    exchange = PeerExchange(ops, dist.group.WORLD, rows, cols, wait_limit_ns=10_000_000)
    exchange.slots[0].copy_(parts[rank])
    torch.cuda.synchronize()
    dist.barrier()
    assert ops.take_device_error() == 0
    if rank == 0:
        x = x0.clone()
        normed = torch.full_like(x, 7.0)
        start = time.perf_counter()
        exchange.add_rms_norm(0, x, RowNorm(weight, 1e-6, 0.0, normed))
        torch.cuda.synchronize()
        waited = time.perf_counter() - start
        assert waited < 2.0, waited
        assert ops.take_device_error() == 3
        assert torch.equal(x, x0)
        assert bool((normed == 7.0).all())
    torch.cuda.synchronize()
    dist.barrier()  # rank 0's pushes into rank 1's buffer have ended
    exchange.close()
    dist.barrier()
    # a fresh exchange on the same context sums as before
    exchange = PeerExchange(ops, dist.group.WORLD, rows, cols)
    exchange.slots[0].copy_(parts[rank])
    x = x0.clone()
    normed = torch.empty_like(x)
    exchange.add_rms_norm(0, x, RowNorm(weight, 1e-6, 0.0, normed))
    expected_x = x0.clone()
    expected = torch.empty_like(x)
    ops.add_rms_norm(expected_x, parts[0] + parts[1], RowNorm(weight, 1e-6, 0.0, expected))
    torch.cuda.synchronize()
    assert torch.equal(x, expected_x)
    assert torch.equal(normed, expected)
    assert ops.take_device_error() == 0
    dist.barrier()
    exchange.close()


@needs_two
def test_exchange_wait_runs_out_when_a_rank_skips():
    torch.multiprocessing.spawn(_timeout_ranks, args=(2, free_port()), nprocs=2, join=True)


@needs_two
def test_exchange_sums_in_rank_order_then_norms():
    torch.multiprocessing.spawn(_exchange_ranks, args=(2, free_port()), nprocs=2, join=True)


@needs_two
def test_decode_step_over_peer_memory_equals_nccl():
    torch.multiprocessing.spawn(_decode_ranks, args=(2, free_port()), nprocs=2, join=True)


def _hybrid_ranks(rank: int, world: int, port: int):
    dist = _init(rank, world, port)
    from drift_b200.hybrid import HybridConfig, HybridDecoder, HybridWeights
    from drift_b200.ops import CudaOps
    try:
        ops = CudaOps()
        c = HybridConfig(layers=4, hidden=256, delta_key_heads=2, delta_value_heads=4,
                         delta_dim=32, q_heads=4, kv_heads=2, head_dim=64, rotary=16, theta=1e6,
                         experts=16, used=4, expert_ffn=64, shared_ffn=64, vocab=500)
        full = HybridWeights.random(c, seed=5)          # the same on every rank
        whole = HybridDecoder(ops, c, full, batch=2, context=64)
        whole.prefill_random(25)
        part = full.shard(c, rank, world)
        split = HybridDecoder(ops, c, part, batch=2, context=64, group=dist.group.WORLD)
        p = part.part
        # the same caches and states, sliced to this rank's heads and channels
        d = c.delta_dim
        keys = c.delta_key_heads * d
        ranges = [(p.delta_key_heads[0] * d, p.delta_key_heads[1] * d),
                  (keys + p.delta_key_heads[0] * d, keys + p.delta_key_heads[1] * d),
                  (2 * keys + p.delta_value_heads[0] * d, 2 * keys + p.delta_value_heads[1] * d)]
        for i, cache in split.caches.items():
            k0, k1 = p.kv_heads
            cache.keys.copy_(whole.caches[i].keys[:, :, k0:k1])
            cache.values.copy_(whole.caches[i].values[:, k0:k1])
        for i, state in split.delta_states.items():
            state.copy_(whole.delta_states[i][:, p.delta_value_heads[0]:p.delta_value_heads[1]])
        for i, state in split.conv_states.items():
            state.copy_(torch.cat([whole.conv_states[i][:, :, lo:hi] for lo, hi in ranges], dim=2))
        for decoder in (whole, split):
            decoder.ids.copy_(torch.tensor([7, 11], dtype=torch.int32))
            decoder.positions.copy_(torch.tensor([25, 19], dtype=torch.int32))
        expected = whole.step()[:, p.vocab[0]:p.vocab[1]].clone()
        got = split.step().clone()
        torch.cuda.synchronize()
        # the greedy choice over the split vocabulary: the argmax of the
        # gathered rows on every rank
        gathered = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(gathered, got)
        rows = torch.cat(gathered, dim=1).cpu().numpy()
        assert list(split.next_ids.cpu().numpy()) == [oracle.argmax(r) for r in rows]
        bound = 1e-4 + 1e-3 * expected.abs()
        assert ((got - expected).abs() <= bound).all(), float((got - expected).abs().max())
        # the recurrent state moved as the whole model's did
        for i, state in split.delta_states.items():
            want = whole.delta_states[i][:, p.delta_value_heads[0]:p.delta_value_heads[1]]
            assert ((state - want).abs() <= 1e-4 + 1e-3 * want.abs()).all()
        split.capture()
        split.release()
        assert ops.take_device_error() == 0
        dist.barrier()
    finally:
        dist.destroy_process_group()


@needs_two
def test_expert_parallel_hybrid_step_equals_the_whole_model():
    torch.multiprocessing.spawn(_hybrid_ranks, args=(2, free_port()), nprocs=2, join=True)
