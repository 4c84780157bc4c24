"""The dense decoder's decode step on this library's ops: the op order of the
runner's DenseDecoder.run (runner/src/drift/runner/models/DenseDecoder.scala:
778-939), for a batch of sequences, on one GPU or tensor-parallel across the
GPUs of one box (drift_b200/tensor_parallel.py).

Per token and layer: RMSNorm (writing the products' x records); q, k, v
products in one launch; per-head
q/k RMSNorm (Qwen3), RoPE of q and k and the new k, v into each sequence's
paged F16 cache (one fused launch for the batch); attention over the caches
(one launch for the batch); o product; residual add + RMSNorm; gate and up
products; SwiGLU; down product; residual add. Then the final RMSNorm and the
lm-head product. With tensor parallelism a rank holds its share of
the query and key heads and of the FFN rows (column-split q/k/v/gate/up),
the matching columns of o and down (row-split, one all-reduce each), and its
share of the vocabulary rows of the lm-head; the embedding and the norms are
replicated.

This is the harness the benchmark's decode tok/s is measured on: weights are
random-init (the benchmark laws), the caches prefilled with N(0, 1) keys and
values; a step is captured once as a CUDA graph and replayed.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from . import synthetic
from ._lib import Q4_1, Q8_0
from .ops import SILU, Attention, CudaOps, KvCache, Rope, RowNorm, Stored
from .tensor_parallel import row_range


@dataclass(frozen=True)
class DenseConfig:
    """A dense decoder's shape (benchmark config C4: Qwen3-8B-like)."""
    layers: int = 36
    hidden: int = 4096
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 12288
    vocab: int = 151936
    epsilon: float = 1e-6
    theta: float = 1e6
    qk_norm: bool = True
    page_size: int = 16


@dataclass
class DenseLayer:
    attention_norm: torch.Tensor
    q: Stored
    k: Stored
    v: Stored
    q_norm: Optional[torch.Tensor]
    k_norm: Optional[torch.Tensor]
    o: Stored
    mlp_norm: torch.Tensor
    gate: Stored
    up: Stored
    down: Stored


@dataclass
class DenseWeights:
    """One rank's weights: its heads and FFN rows of the column-split
    products, the matching columns of o and down, its vocabulary rows of the
    lm-head; the embedding and norms whole."""
    embedding: Stored
    layers: list
    final_norm: torch.Tensor
    lm_head: Stored
    rank: int = 0
    world: int = 1

    @staticmethod
    def random(config: DenseConfig, dtype: int = Q4_1, embedding_dtype: int = Q8_0,
               seed: int = 0, rank: int = 0, world: int = 1) -> "DenseWeights":
        """Random-init weights by the benchmark laws, drawn on the device: this
        rank's shards only (different ranks draw different numbers -- a
        timing harness, not a model)."""
        c = config
        g = torch.Generator(device="cuda")
        g.manual_seed(seed * 1000 + rank)
        q_heads, kv_heads = c.q_heads // world, c.kv_heads // world
        ffn = row_range(c.ffn, rank, world)
        ffn_rows = ffn[1] - ffn[0]
        vocab = row_range(c.vocab, rank, world)

        def stored(t, n, k):
            return Stored(t, (n, k), synthetic.quantized_device(t, n, k, g))

        def norm(width):
            return 1.0 + 0.02 * torch.randn(width, generator=g, device="cuda")

        layers = []
        for _ in range(c.layers):
            layers.append(DenseLayer(
                attention_norm=norm(c.hidden),
                q=stored(dtype, q_heads * c.head_dim, c.hidden),
                k=stored(dtype, kv_heads * c.head_dim, c.hidden),
                v=stored(dtype, kv_heads * c.head_dim, c.hidden),
                q_norm=norm(c.head_dim) if c.qk_norm else None,
                k_norm=norm(c.head_dim) if c.qk_norm else None,
                o=stored(dtype, c.hidden, q_heads * c.head_dim),
                mlp_norm=norm(c.hidden),
                gate=stored(dtype, ffn_rows, c.hidden),
                up=stored(dtype, ffn_rows, c.hidden),
                down=stored(dtype, c.hidden, ffn_rows)))
        return DenseWeights(stored(embedding_dtype, c.vocab, c.hidden), layers, norm(c.hidden),
                            stored(dtype, vocab[1] - vocab[0], c.hidden), rank, world)

    def nbytes(self) -> int:
        """Bytes of weights one decode step streams on this rank (all but the
        embedding, of which a step reads only the batch's rows)."""
        total = self.final_norm.numel() * 4 + self.lm_head.data.numel()
        for layer in self.layers:
            for w in (layer.q, layer.k, layer.v, layer.o, layer.gate, layer.up, layer.down):
                total += w.data.numel()
            total += (layer.attention_norm.numel() + layer.mlp_norm.numel()) * 4
        return total


class DenseDecoder:
    """Decode steps for `batch` sequences of up to `context` positions each,
    on this rank's weights. `group`: the tensor-parallel process group (NCCL),
    or None for one GPU."""

    def __init__(self, ops: CudaOps, config: DenseConfig, weights: DenseWeights, batch: int,
                 context: int, group=None, exchange: str = "peer"):
        c = self.config = config
        self.ops, self.weights, self.batch, self.context, self.group = ops, weights, batch, context, group
        world = weights.world
        self.q_heads, self.kv_heads = c.q_heads // world, c.kv_heads // world
        self.ffn = weights.layers[0].gate.shape[0] if weights.layers else 0
        self.vocab_rows = weights.lm_head.shape[0]
        pages_per_sequence = (context + c.page_size - 1) // c.page_size
        self.pages_per_sequence = pages_per_sequence
        pages = pages_per_sequence * batch
        self.caches = [KvCache.allocate(pages, c.page_size, self.kv_heads, c.head_dim)
                       for _ in weights.layers]
        # sequence i's pages: [i P, (i + 1) P); one row of the page table each
        self.page_tables = torch.arange(pages, dtype=torch.int32,
                                        device="cuda").view(batch, pages_per_sequence)
        self.tables = [self.page_tables[i] for i in range(batch)]
        self.rope = Rope(c.theta, c.head_dim)
        self.attention = Attention(1.0 / math.sqrt(c.head_dim))
        b, hd = batch, c.head_dim
        f32 = dict(dtype=torch.float32, device="cuda")
        self.ids = torch.zeros(b, dtype=torch.int32, device="cuda")
        self.positions = torch.zeros(b, dtype=torch.int32, device="cuda")
        self.x = torch.zeros(b, c.hidden, **f32)
        self.normed = torch.zeros(b, c.hidden, **f32)
        self.q = torch.zeros(b, self.q_heads * hd, **f32)
        self.k = torch.zeros(b, self.kv_heads * hd, **f32)
        self.v = torch.zeros(b, self.kv_heads * hd, **f32)
        self.q_turned = torch.zeros(b, self.q_heads, hd, **f32)
        self.k_turned = torch.zeros(b, self.kv_heads, hd, **f32)
        self.attended = torch.zeros(b, self.q_heads, hd, **f32)
        self.projected = torch.zeros(b, c.hidden, **f32)
        self.gate = torch.zeros(b, self.ffn, **f32)
        self.up = torch.zeros(b, self.ffn, **f32)
        self.logits = torch.zeros(b, self.vocab_rows, **f32)
        # the greedy choice of each sequence's next token over the whole
        # vocabulary (this rank's rows, gathered and merged across ranks)
        self.next_ids = torch.zeros(b, dtype=torch.int32, device="cuda")
        vocab_lo, _ = row_range(c.vocab, weights.rank, weights.world)
        from .tensor_parallel import VocabSampler
        self.sampler = VocabSampler(ops, b, vocab_lo, group, device="cuda")
        # x's records for the products, written by the kernel that makes x
        # (the norms, the attention join, SwiGLU): one buffer, each product
        # reading it before the next producer writes it
        self.prepared = ops.prepared_x(b, max(c.hidden, self.q_heads * hd, self.ffn))
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        # the row-split products' exchange: peer memory over NVLink, fused
        # with the residual add and the norm ("peer"), or NCCL ("nccl")
        self.exchange = None
        if group is not None and exchange == "peer":
            from .tensor_parallel import PeerExchange
            self.exchange = PeerExchange(ops, group, b, c.hidden)
        self._positions_host: list[int] = [0] * b
        # (name, CUDA event) after each op group of an eager step, when a
        # profiler sets it to a list
        self.marks: Optional[list] = None

    def _mark(self, name: str) -> None:
        if self.marks is not None:
            # (an event record node when the step is captured in a graph)
            event = torch.cuda.Event(enable_timing=True, external=True)
            event.record()
            self.marks.append((name, event))

    def prefill_random(self, positions: int, seed: int = 1) -> None:
        """Every sequence's cache holds `positions` positions of N(0, 1) keys
        and values (benchmark config C4's prefilled cache), as F16."""
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        used = (positions + self.config.page_size - 1) // self.config.page_size
        for cache in self.caches:
            for i in range(self.batch):
                pages = slice(i * self.pages_per_sequence, i * self.pages_per_sequence + used)
                cache.keys[pages].normal_(generator=g)
                cache.values[pages].normal_(generator=g)

    def _all_reduce(self, t: torch.Tensor) -> None:
        if self.group is not None:
            torch.distributed.all_reduce(t, group=self.group)

    def step(self, positions: Optional[list[int]] = None) -> torch.Tensor:
        """One decode step: self.ids at self.positions (device, one per
        sequence, set by the caller) -> self.logits [batch, this rank's
        vocabulary rows] and self.next_ids [batch], each sequence's greedy
        next token (the argmax over the whole vocabulary; a generation loop
        copies it into self.ids). `positions` is not needed: the kernels read
        the device copy (so a captured step replays at new positions)."""
        ops, c, w = self.ops, self.config, self.weights
        b, hd = self.batch, c.head_dim
        prepared = self.prepared
        mark = self._mark
        mark("start")
        ops.embedding(w.embedding, self.ids, self.x)
        ops.add_rms_norm(self.x, None, RowNorm(w.layers[0].attention_norm, c.epsilon, 0.0,
                                               self.normed), prepared)
        mark("embed")
        for index, (layer, cache) in enumerate(zip(w.layers, self.caches)):
            ops.linears(self.normed, [layer.q, layer.k, layer.v], [self.q, self.k, self.v], prepared)
            mark("qkv")
            # per-head q/k norms, rope, cache write: one launch for the batch;
            # then every sequence's attention in one launch
            ops.attention_inputs_decode(
                self.q.view(b, self.q_heads, hd), self.k.view(b, self.kv_heads, hd),
                self.v.view(b, self.kv_heads, hd), layer.q_norm, layer.k_norm, c.epsilon,
                self.positions, self.rope, self.q_turned, cache, self.page_tables)
            ops.attention_decode(self.q_turned, cache, self.page_tables, self.positions,
                                 self.context, self.attention, self.attended, prepared)
            mark("attention")
            following = w.layers[index + 1].attention_norm if index + 1 < len(w.layers) else w.final_norm
            mlp_norm = RowNorm(layer.mlp_norm, c.epsilon, 0.0, self.normed)
            next_norm = RowNorm(following, c.epsilon, 0.0, self.normed)
            attended = self.attended.view(b, self.q_heads * hd)
            if self.exchange is not None:
                # partials into the exchange's slots; every rank sums them
                ops.linears(attended, [layer.o], [self.exchange.slots[0]], prepared)
                mark("o")
                self.exchange.add_rms_norm(0, self.x, mlp_norm, prepared)
                mark("exchange")
                ops.linears(self.normed, [layer.gate, layer.up], [self.gate, self.up], prepared)
                mark("gate_up")
                ops.gated(SILU, self.gate, self.up, self.gate, prepared)
                mark("swiglu")
                ops.linears(self.gate, [layer.down], [self.exchange.slots[1]], prepared)
                mark("down")
                self.exchange.add_rms_norm(1, self.x, next_norm, prepared)
                mark("exchange")
                continue
            ops.linears(attended, [layer.o], [self.projected], prepared)
            mark("o")
            self._all_reduce(self.projected)
            ops.add_rms_norm(self.x, self.projected, mlp_norm, prepared)
            mark("add_norm" if self.group is None else "exchange")
            # SwiGLU stays a launch of its own: fused into the gate/up
            # launch's epilogue it held that launch's SMs to its end, and the
            # down product's weight copies, which start during the short
            # SwiGLU launch, lost more than the launch cost
            ops.linears(self.normed, [layer.gate, layer.up], [self.gate, self.up], prepared)
            mark("gate_up")
            ops.gated(SILU, self.gate, self.up, self.gate, prepared)
            mark("swiglu")
            ops.linears(self.gate, [layer.down], [self.projected], prepared)
            mark("down")
            self._all_reduce(self.projected)
            ops.add_rms_norm(self.x, self.projected, next_norm, prepared)
            mark("add_norm" if self.group is None else "exchange")
        ops.linears(self.normed, [w.lm_head], [self.logits], prepared)
        mark("lm_head")
        self.sampler(self.logits, self.next_ids)
        mark("sample")
        return self.logits

    def reserve(self) -> None:
        """Sizes the library's scratch for every product and attention of a
        step, so a capture allocates nothing."""
        c = self.config
        widest = max(c.hidden, self.q_heads * c.head_dim, self.ffn)
        self.ops.reserve_workspace(self.batch, widest)
        lib = self.ops.lib
        attention_bytes = lib.drift_attention_workspace_bytes(self.batch, self.q_heads, c.head_dim,
                                                              self.context)
        from ._lib import check
        check("drift_workspace_reserve", lib.drift_workspace_reserve(
            max(attention_bytes, lib.drift_linear_workspace_bytes(self.batch, widest))))

    def capture(self, positions: list[int], stream: Optional[torch.cuda.Stream] = None) -> None:
        """Records one step at `positions` as a CUDA graph (replayed by
        `replay`): the positions are fixed in the graph's launches."""
        self.positions.copy_(torch.tensor(positions, dtype=torch.int32))
        self.reserve()
        stream = stream or torch.cuda.Stream()
        with torch.cuda.stream(stream):
            self.step(positions)  # first calls resolve lazy state outside the capture
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.step(positions)
        torch.cuda.synchronize()

    def replay(self) -> None:
        self.graph.replay()

    def release(self) -> None:
        """Drops the graph (it must go before an NCCL group is destroyed) and
        the exchange's buffers."""
        self.graph = None
        if self.exchange is not None:
            torch.cuda.synchronize()
            self.exchange.close()
            self.exchange = None
