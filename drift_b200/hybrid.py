"""The hybrid MoE decoder's decode step on this library's ops: the op order of
the runner's HybridBlocks (runner/src/drift/runner/models/HybridBlocks.scala:
403-588) and Qwen35.decoderLayer (models/Qwen35.scala:356-410), for a batch
of sequences, on one GPU or expert-parallel across the GPUs of a box.

A layer is either Gated DeltaNet (three of every four) or gated full
attention, then a mixture of experts:

- DeltaNet: q/k/v (one matrix), z, a, b products of the normed input in one
  call; the causal convolution + SiLU of q/k/v; the gated delta rule (every
  sequence its own state); the gated RMSNorm by z (writing the out
  projection's x records); the out projection.
- Full attention: q-and-gate, k, v products; per-head q/k norms, partial RoPE
  and the cache write (queryAndGate split in halves, one launch); attention
  over the paged F16 cache with the output gate sigmoid(gate) applied in the
  join (writing o's records); o.
- Then x += the block's output and the RMSNorm of x; the F32 router and
  top-k; the routed experts' gate/up (SwiGLU, one launch for every slot), the
  shared expert's; the experts' down products and the shared one's; the
  combine (weights, the shared expert by sigmoid(x . shared router), the
  residual) and the next norm, one launch.

With a process group (one process per GPU), the layers are split as the
benchmark's expert-parallel configuration splits them (`Partition`): DeltaNet
heads and query heads by rank (the key heads a rank's query heads read are
its own), the out projections row-split, experts by id (routing replicated),
the shared expert on rank 0, the lm-head by vocabulary rows; the two
exchanges of a layer (the mixer's output, the mixture's) go through the
NVLink peer exchange fused with the residual add and the norm.

This is the harness of the benchmark's C5 decode tok/s: random-init weights
(the benchmark's Q4_1 law; F32 routers, a and b, convolution, decay and norm
weights), DeltaNet states N(0, 0.02), caches prefilled with N(0, 1); a step is
captured as a CUDA graph and replayed.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import synthetic
from ._lib import Q4_1, Q8_0
from .ops import SIGMOID, Attention, CudaOps, KvCache, Rope, RowNorm, SharedExpert, Stored


@dataclass(frozen=True)
class HybridConfig:
    """A hybrid MoE decoder's shape (the benchmark's C5: a Qwen3.5-MoE-like
    model)."""
    layers: int = 48
    hidden: int = 2048
    full_every: int = 4           # layer i is full attention when i % full_every == full_every - 1
    # Gated DeltaNet
    delta_key_heads: int = 16
    delta_value_heads: int = 16
    delta_dim: int = 128
    conv_taps: int = 4
    # gated full attention
    q_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 256
    rotary: int = 64
    theta: float = 1e7
    # mixture
    experts: int = 512
    used: int = 10
    expert_ffn: int = 512
    shared_ffn: int = 512
    vocab: int = 151936
    epsilon: float = 1e-6
    page_size: int = 16

    def is_full(self, layer: int) -> bool:
        return layer % self.full_every == self.full_every - 1


@dataclass
class DeltaLayer:
    qkv: Stored
    z: Stored
    a: torch.Tensor      # F32 [value heads, hidden]
    b: torch.Tensor
    conv: torch.Tensor   # F32 [channels, taps]
    decay: torch.Tensor  # F32 [value heads]: -exp(A_log)
    dt_bias: torch.Tensor
    norm: torch.Tensor   # F32 [delta_dim]
    out: Stored


@dataclass
class FullLayer:
    q: Stored            # [q_heads * 2 head_dim, hidden]: query and gate
    k: Stored
    v: Stored
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o: Stored


@dataclass
class MixtureLayer:
    router: torch.Tensor         # F32 [experts, hidden]
    gate: Stored                 # [experts, ffn, hidden]
    up: Stored
    down: Stored                 # [experts, hidden, ffn]
    shared_gate: Stored          # [1, shared ffn, hidden]
    shared_up: Stored
    shared_down: Stored          # [hidden, shared ffn]
    shared_router: torch.Tensor  # F32 [hidden]
    # (gate, up, down) of experts + 1 experts when the fields above are views
    # of them (one launch serves both): on one GPU the shared expert last (id
    # `experts`); under expert parallelism, on rank 0, first (id -1)
    fused: Optional[tuple] = None


def _expert_range(w: Stored, e0: int, e1: int) -> Stored:
    """Experts [e0, e1) of an [experts, n, k] weight, as a view."""
    per = w.data.numel() // w.shape[0]
    return Stored(w.dtype, (e1 - e0,) + tuple(w.shape[1:]), w.data[e0 * per:e1 * per])


@dataclass
class HybridLayer:
    input_norm: torch.Tensor
    mixer: object                # DeltaLayer or FullLayer
    post_norm: torch.Tensor
    mixture: MixtureLayer


@dataclass(frozen=True)
class Partition:
    """What rank `rank` of `world` holds (expert and tensor parallelism over
    the GPUs of a box): its DeltaNet key and value heads, its query heads and
    the key heads they read, its experts, its vocabulary rows."""
    rank: int
    world: int
    delta_key_heads: tuple
    delta_value_heads: tuple
    q_heads: tuple
    kv_heads: tuple
    experts: tuple
    vocab: tuple

    @staticmethod
    def of(c: "HybridConfig", rank: int = 0, world: int = 1) -> "Partition":
        def even(total):
            if total % world:
                raise ValueError(f"{total} does not split {world} ways")
            return (total * rank // world, total * (rank + 1) // world)

        q = even(c.q_heads)
        group = c.q_heads // c.kv_heads
        kv = (q[0] // group, (q[1] - 1) // group + 1)  # the key heads of the rank's query heads
        return Partition(rank, world, even(c.delta_key_heads), even(c.delta_value_heads), q, kv,
                         even(c.experts), (c.vocab * rank // world, c.vocab * (rank + 1) // world))


def _shared_first(router, gate: Stored, up: Stored, down: Stored, experts: int, c, dtype: int,
                  shared_router) -> "MixtureLayer":
    """A mixture whose (gate, up, down) hold the shared expert first, then
    `experts` routed experts (expert parallelism's rank 0)."""
    first = _expert_range(down, 0, 1)
    return MixtureLayer(router, _expert_range(gate, 1, experts + 1),
                        _expert_range(up, 1, experts + 1), _expert_range(down, 1, experts + 1),
                        _expert_range(gate, 0, 1), _expert_range(up, 0, 1),
                        Stored(dtype, (c.hidden, c.shared_ffn), first.data), shared_router,
                        (gate, up, down))


def _rows(w: Stored, ranges, width: int) -> Stored:
    """The listed row ranges of w [N, K], concatenated."""
    row = w.data.numel() // w.shape[0]
    parts = [w.data[lo * row:hi * row] for lo, hi in ranges]
    return Stored(w.dtype, (sum(hi - lo for lo, hi in ranges), width), torch.cat(parts).contiguous())


def _columns(w: Stored, lo: int, hi: int) -> Stored:
    """Columns [lo, hi) (whole 32-value blocks) of every row of w [N, K]."""
    n, k = w.shape
    row = w.data.numel() // n
    per = row // (k // 32)
    data = w.data.view(n, row)[:, lo // 32 * per:hi // 32 * per].contiguous().view(-1)
    return Stored(w.dtype, (n, hi - lo), data)


@dataclass
class HybridWeights:
    embedding: Stored
    layers: list
    final_norm: torch.Tensor
    lm_head: Stored
    part: Optional[Partition] = None

    @staticmethod
    def random(c: HybridConfig, dtype: int = Q4_1, seed: int = 0, rank: int = 0,
               world: int = 1) -> "HybridWeights":
        """Random-init weights by the benchmark laws, drawn on the device: this
        rank's shards only (different ranks draw different numbers -- a timing
        harness, not a model)."""
        part = Partition.of(c, rank, world)
        g = torch.Generator(device="cuda")
        g.manual_seed(seed * 1000 + rank)
        span = lambda r: r[1] - r[0]

        def stored(n, k, experts: int = 0):
            rows = n * max(1, experts)
            shape = (experts, n, k) if experts else (n, k)
            return Stored(dtype, shape, synthetic.quantized_device(dtype, rows, k, g))

        def f32(*shape, scale=1.0):
            return scale * torch.randn(*shape, generator=g, device="cuda")

        def norm(width):
            return 1.0 + 0.02 * torch.randn(width, generator=g, device="cuda")

        dk, dv = span(part.delta_key_heads), span(part.delta_value_heads)
        channels = (2 * dk + dv) * c.delta_dim
        value_width = dv * c.delta_dim
        qh, kvh, experts = span(part.q_heads), span(part.kv_heads), span(part.experts)
        layers = []
        for i in range(c.layers):
            if c.is_full(i):
                mixer = FullLayer(stored(qh * 2 * c.head_dim, c.hidden),
                                  stored(kvh * c.head_dim, c.hidden),
                                  stored(kvh * c.head_dim, c.hidden),
                                  norm(c.head_dim), norm(c.head_dim),
                                  stored(c.hidden, qh * c.head_dim))
            else:
                mixer = DeltaLayer(stored(channels, c.hidden), stored(value_width, c.hidden),
                                   f32(dv, c.hidden, scale=0.02), f32(dv, c.hidden, scale=0.02),
                                   f32(channels, c.conv_taps, scale=0.5),
                                   -torch.exp(torch.rand(dv, generator=g, device="cuda") * 2.5 - 1.0),
                                   f32(dv), norm(c.delta_dim), stored(c.hidden, value_width))
            if world > 1 and rank == 0 and c.shared_ffn == c.expert_ffn:
                # expert parallelism: the shared expert on rank 0, as expert
                # 0 (id -1) of its weights, before its routed experts
                router = f32(c.experts, c.hidden, scale=0.02)
                gate, up, down = (stored(c.expert_ffn, c.hidden, experts + 1),
                                  stored(c.expert_ffn, c.hidden, experts + 1),
                                  stored(c.hidden, c.expert_ffn, experts + 1))
                mixture = _shared_first(router, gate, up, down, experts, c, dtype,
                                        f32(c.hidden, scale=0.02))
            elif world == 1 and c.shared_ffn == c.expert_ffn:
                # the shared expert as expert `experts` of the routed weights
                router = f32(c.experts, c.hidden, scale=0.02)
                gate, up, down = (stored(c.expert_ffn, c.hidden, experts + 1),
                                  stored(c.expert_ffn, c.hidden, experts + 1),
                                  stored(c.hidden, c.expert_ffn, experts + 1))
                last = _expert_range(down, experts, experts + 1)
                mixture = MixtureLayer(router, _expert_range(gate, 0, experts),
                                       _expert_range(up, 0, experts),
                                       _expert_range(down, 0, experts),
                                       _expert_range(gate, experts, experts + 1),
                                       _expert_range(up, experts, experts + 1),
                                       Stored(dtype, (c.hidden, c.shared_ffn), last.data),
                                       f32(c.hidden, scale=0.02), (gate, up, down))
            else:
                mixture = MixtureLayer(f32(c.experts, c.hidden, scale=0.02),
                                       stored(c.expert_ffn, c.hidden, experts),
                                       stored(c.expert_ffn, c.hidden, experts),
                                       stored(c.hidden, c.expert_ffn, experts),
                                       stored(c.shared_ffn, c.hidden, 1),
                                       stored(c.shared_ffn, c.hidden, 1),
                                       stored(c.hidden, c.shared_ffn),
                                       f32(c.hidden, scale=0.02))
            layers.append(HybridLayer(norm(c.hidden), mixer, norm(c.hidden), mixture))
        return HybridWeights(Stored(Q8_0, (c.vocab, c.hidden),
                                    synthetic.quantized_device(Q8_0, c.vocab, c.hidden, g)),
                             layers, norm(c.hidden), stored(span(part.vocab), c.hidden), part)

    def shard(self, c: HybridConfig, rank: int, world: int) -> "HybridWeights":
        """Rank `rank`'s shards of these (whole-model) weights."""
        part = Partition.of(c, rank, world)
        d, hd = c.delta_dim, c.head_dim
        kh, vh = part.delta_key_heads, part.delta_value_heads
        layers = []
        for layer in self.layers:
            m = layer.mixer
            if isinstance(m, FullLayer):
                q0, q1 = part.q_heads
                k0, k1 = part.kv_heads
                mixer = FullLayer(_rows(m.q, [(q0 * 2 * hd, q1 * 2 * hd)], c.hidden),
                                  _rows(m.k, [(k0 * hd, k1 * hd)], c.hidden),
                                  _rows(m.v, [(k0 * hd, k1 * hd)], c.hidden),
                                  m.q_norm, m.k_norm, _columns(m.o, q0 * hd, q1 * hd))
            else:
                keys = c.delta_key_heads * d
                ranges = [(kh[0] * d, kh[1] * d), (keys + kh[0] * d, keys + kh[1] * d),
                          (2 * keys + vh[0] * d, 2 * keys + vh[1] * d)]
                conv = torch.cat([m.conv[lo:hi] for lo, hi in ranges]).contiguous()
                mixer = DeltaLayer(_rows(m.qkv, ranges, c.hidden),
                                   _rows(m.z, [(vh[0] * d, vh[1] * d)], c.hidden),
                                   m.a[vh[0]:vh[1]].contiguous(), m.b[vh[0]:vh[1]].contiguous(),
                                   conv, m.decay[vh[0]:vh[1]].contiguous(),
                                   m.dt_bias[vh[0]:vh[1]].contiguous(), m.norm,
                                   _columns(m.out, vh[0] * d, vh[1] * d))
            x = layer.mixture
            e0, e1 = part.experts
            if world > 1 and rank == 0 and c.shared_ffn == c.expert_ffn:
                # the shared expert first, then the rank's routed experts
                def joined(shared: Stored, routed: Stored) -> Stored:
                    part_ = _expert_range(routed, e0, e1)
                    data = torch.cat([shared.data.reshape(-1), part_.data.reshape(-1)])
                    return Stored(routed.dtype, (e1 - e0 + 1,) + tuple(routed.shape[1:]), data)
                shared_down = Stored(x.shared_down.dtype, (1,) + tuple(x.shared_down.shape),
                                     x.shared_down.data)
                mixture = _shared_first(x.router, joined(x.shared_gate, x.gate),
                                        joined(x.shared_up, x.up), joined(shared_down, x.down),
                                        e1 - e0, c, x.gate.dtype, x.shared_router)
            else:
                mixture = MixtureLayer(x.router, _expert_range(x.gate, e0, e1),
                                       _expert_range(x.up, e0, e1), _expert_range(x.down, e0, e1),
                                       x.shared_gate, x.shared_up, x.shared_down, x.shared_router)
            layers.append(HybridLayer(layer.input_norm, mixer, layer.post_norm, mixture))
        v0, v1 = part.vocab
        return HybridWeights(self.embedding, layers, self.final_norm,
                             _rows(self.lm_head, [(v0, v1)], c.hidden), part)

    def bytes_per_token(self, c: HybridConfig) -> int:
        """Weight bytes one sequence's decode step reads: every layer's
        mixer, router and shared expert, `used` experts' slices, the norms,
        the lm-head (the embedding: one row)."""
        total = self.lm_head.data.numel() + self.final_norm.numel() * 4
        expert = 3 * c.expert_ffn * c.hidden * 20 // 32  # one expert's gate, up and down (Q4_1)
        for layer in self.layers:
            m = layer.mixer
            if isinstance(m, FullLayer):
                total += sum(w.data.numel() for w in (m.q, m.k, m.v, m.o))
            else:
                total += m.qkv.data.numel() + m.z.data.numel() + m.out.data.numel()
                total += (m.a.numel() + m.b.numel() + m.conv.numel()) * 4
            x = layer.mixture
            total += x.router.numel() * 4 + c.used * expert
            total += sum(w.data.numel() for w in (x.shared_gate, x.shared_up, x.shared_down))
            total += (layer.input_norm.numel() + layer.post_norm.numel()) * 4
        return total


class HybridDecoder:
    """Decode steps for `batch` sequences of up to `context` positions."""

    def __init__(self, ops: CudaOps, config: HybridConfig, weights: HybridWeights, batch: int,
                 context: int, group=None):
        c = self.config = config
        self.ops, self.weights, self.batch, self.context = ops, weights, batch, context
        b = batch
        part = weights.part or Partition.of(c)
        self.part = part
        span = lambda r: r[1] - r[0]
        # this rank's heads (all of them on one GPU)
        self.delta_key_heads, self.delta_value_heads = (span(part.delta_key_heads),
                                                        span(part.delta_value_heads))
        self.q_heads, self.kv_heads = span(part.q_heads), span(part.kv_heads)
        self.exchange = None
        if group is not None and part.world > 1:
            from .tensor_parallel import PeerExchange
            self.exchange = PeerExchange(ops, group, b, c.hidden)
        f32 = dict(dtype=torch.float32, device="cuda")
        pages_per_sequence = (context + c.page_size - 1) // c.page_size
        self.page_tables = torch.arange(pages_per_sequence * b, dtype=torch.int32,
                                        device="cuda").view(b, pages_per_sequence)
        self.channels = (2 * self.delta_key_heads + self.delta_value_heads) * c.delta_dim
        self.value_width = self.delta_value_heads * c.delta_dim
        self.caches, self.conv_states, self.delta_states = {}, {}, {}
        for i, layer in enumerate(weights.layers):
            if isinstance(layer.mixer, FullLayer):
                self.caches[i] = KvCache.allocate(pages_per_sequence * b, c.page_size,
                                                  self.kv_heads, c.head_dim)
            else:
                self.conv_states[i] = torch.zeros(b, c.conv_taps - 1, self.channels, **f32)
                self.delta_states[i] = torch.zeros(b, self.delta_value_heads, c.delta_dim,
                                                   c.delta_dim, **f32)
        self.rope = Rope(c.theta, c.rotary)
        self.attention = Attention(1.0 / math.sqrt(c.head_dim))
        self.ids = torch.zeros(b, dtype=torch.int32, device="cuda")
        self.positions = torch.zeros(b, dtype=torch.int32, device="cuda")
        self.x = torch.zeros(b, c.hidden, **f32)
        self.normed = torch.zeros(b, c.hidden, **f32)
        self.block_out = torch.zeros(b, c.hidden, **f32)
        # DeltaNet
        self.qkv = torch.zeros(b, self.channels, **f32)
        self.convolved = torch.zeros(b, self.channels, **f32)
        self.z = torch.zeros(b, self.value_width, **f32)
        self.a = torch.zeros(b, self.delta_value_heads, **f32)
        self.b = torch.zeros(b, self.delta_value_heads, **f32)
        self.core = torch.zeros(b, self.delta_value_heads, c.delta_dim, **f32)
        # full attention
        self.query_gate = torch.zeros(b, self.q_heads, 2 * c.head_dim, **f32)
        self.k = torch.zeros(b, self.kv_heads, c.head_dim, **f32)
        self.v = torch.zeros(b, self.kv_heads, c.head_dim, **f32)
        self.q_turned = torch.zeros(b, self.q_heads, c.head_dim, **f32)
        self.attended = torch.zeros(b, self.q_heads, c.head_dim, **f32)
        # mixture
        self.logits_router = torch.zeros(b, c.experts, **f32)
        # the routed slots, then one shared slot per sequence: the ids (the
        # shared ones the shared expert's index in fused weights), the SwiGLU
        # outputs and the down outputs as one buffer each, viewed per part
        routed = b * c.used
        # the shared slots' id: `experts` on one GPU (the shared expert last
        # in fused weights); -1 under expert parallelism (first on rank 0,
        # another rank's -- zeros -- elsewhere)
        shared_id = c.experts if part.world == 1 else -1
        self.all_ids = torch.full((routed + b,), shared_id, dtype=torch.int32, device="cuda")
        self.route_ids = self.all_ids[:routed].view(b, c.used)
        self.route_weights = torch.zeros(b, c.used, **f32)
        self.all_gated = torch.zeros(routed + b, c.expert_ffn, **f32)
        self.expert_gated = self.all_gated[:routed]
        self.all_out = torch.zeros(routed + b, c.hidden, **f32)
        self.expert_out = self.all_out[:routed]
        self.shared_ids = torch.zeros(b, dtype=torch.int32, device="cuda")
        self.shared_gated = (self.all_gated[routed:] if c.shared_ffn == c.expert_ffn
                             else torch.zeros(b, c.shared_ffn, **f32))
        self.shared_out = self.all_out[routed:]
        self.logits = torch.zeros(b, span(part.vocab), **f32)
        # each sequence's greedy next token over the whole vocabulary
        self.next_ids = torch.zeros(b, dtype=torch.int32, device="cuda")
        from .tensor_parallel import VocabSampler
        self.sampler = VocabSampler(ops, b, part.vocab[0], group if part.world > 1 else None,
                                    device="cuda")
        widest = max(c.hidden, self.value_width, self.q_heads * c.head_dim, c.shared_ffn)
        self.prepared = ops.prepared_x(b, widest)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        # (name, CUDA event) after each op group of an eager step, when a
        # profiler sets it to a list
        self.marks: Optional[list] = None
        # one GPU: the mixture in one launch (drift_moe_decode) rather than
        # the router, top-k, experts and combine launches -- the same bits.
        # Off for the captured step: its four grid barriers cost more than
        # the four launches they replace (C5 batch 1: 4019 against 3181 us a
        # step), which a graph replays with programmatic dependent launch;
        # for a host launching every op itself the one launch saves four
        # launches' host time
        self.whole_mixture = False

    def _mark(self, name: str) -> None:
        if self.marks is not None:
            # (an event record node when the step is captured in a graph)
            event = torch.cuda.Event(enable_timing=True, external=True)
            event.record()
            self.marks.append((name, event))

    def prefill_random(self, positions: int, seed: int = 1) -> None:
        """Caches holding `positions` positions of N(0, 1) keys and values;
        DeltaNet states N(0, 0.02), convolution states N(0, 1)."""
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        c = self.config
        used = (positions + c.page_size - 1) // c.page_size
        per = self.page_tables.shape[1]
        for cache in self.caches.values():
            for i in range(self.batch):
                pages = slice(i * per, i * per + used)
                cache.keys[pages].normal_(generator=g)
                cache.values[pages].normal_(generator=g)
        for state in self.delta_states.values():
            state.normal_(generator=g).mul_(0.02)
        for state in self.conv_states.values():
            state.normal_(generator=g)

    def _delta(self, layer: DeltaLayer, index: int) -> None:
        ops, c, b, P = self.ops, self.config, self.batch, self.prepared
        # (the layer's input and its records come from the previous mixture's
        # combine + norm, or the first norm)
        ops.linears(self.normed, [layer.qkv, layer.z, layer.a, layer.b],
                    [self.qkv, self.z, self.a, self.b], P)
        self._mark("mixer_in")
        # the convolution, the delta rule and the gated norm (with the out
        # projection's records): one launch
        ops.delta_decode_step(self.qkv, self.z, layer.conv, self.conv_states[index],
                              self.convolved, self.a, self.b, layer.decay, layer.dt_bias,
                              self.delta_states[index],
                              (self.delta_key_heads, self.delta_value_heads, c.delta_dim, False),
                              layer.norm, c.epsilon, self.core, P)
        self._mark("delta_step")
        ops.linears(self.core.view(b, self.value_width), [layer.out], [self._block_out(0)], P)
        self._mark("mixer_out")

    def _full(self, layer: FullLayer, index: int) -> None:
        ops, c, b, P = self.ops, self.config, self.batch, self.prepared
        ops.linears(self.normed, [layer.q, layer.k, layer.v],
                    [self.query_gate.view(b, -1), self.k.view(b, -1), self.v.view(b, -1)], P)
        self._mark("mixer_in")
        ops.attention_inputs_decode(self.query_gate, self.k, self.v, layer.q_norm, layer.k_norm,
                                    c.epsilon, self.positions, self.rope, self.q_turned,
                                    self.caches[index], self.page_tables)
        ops.attention_decode(self.q_turned, self.caches[index], self.page_tables, self.positions,
                             self.context, self.attention, self.attended, P,
                             gate=self.query_gate[:, :, c.head_dim:])
        self._mark("attention")
        ops.linears(self.attended.view(b, -1), [layer.o], [self._block_out(0)], P)
        self._mark("mixer_out")

    def _block_out(self, slot: int) -> torch.Tensor:
        """Where a row-split output goes: the exchange's slot, or block_out."""
        return self.exchange.slots[slot] if self.exchange is not None else self.block_out

    def _mixture(self, mixture: MixtureLayer, following: torch.Tensor) -> None:
        ops, c, P = self.ops, self.config, self.prepared
        next_norm = RowNorm(following, c.epsilon, 0.0, self.normed)
        if self.exchange is None and mixture.fused is not None and self.whole_mixture:
            # the router, the top-k, the experts' SwiGLU and down products
            # (the shared expert as the last expert) and the combine with
            # the residual and the next norm: one launch
            gate, up, down = mixture.fused
            ops.moe_decode(self.normed, P, mixture.router, self.logits_router, self.all_ids,
                           self.route_weights, gate, up, down, self.all_gated, self.all_out,
                           mixture.shared_router, self.x, next_norm, P)
            self._mark("moe")
            return
        # routing is the same on every rank (the same x, the same router);
        # the post norm wrote normed's records into P for the router and the
        # gate and up products (the weights hold every expert from 0 on)
        ops.route_linear(self.normed, mixture.router, self.logits_router, self.route_ids,
                         self.route_weights, P)
        self._mark("route")
        if self.exchange is None and mixture.fused is not None:
            # routed and shared experts in one launch each: gate/up (the
            # shared slots last, one per sequence), then down
            gate, up, down = mixture.fused
            ops.experts_gated_linear(self.normed, gate, up, self.all_ids, self.all_gated, 0, P,
                                     shared_tail=True)
            self._mark("experts_gate_up")
            ops.experts_linear(self.all_gated, down, self.all_ids, self.all_out)
            self._mark("experts_down")
            ops.moe_combine_norm(self.expert_out, self.route_weights,
                                 SharedExpert(self.shared_out, self.normed, mixture.shared_router),
                                 self.x, next_norm, P)
            self._mark("combine_norm")
            return
        if self.exchange is None:
            ops.experts_gated_linear(self.normed, mixture.gate, mixture.up,
                                     self.route_ids.view(-1), self.expert_gated, 0, P)
            ops.experts_gated_linear(self.normed, mixture.shared_gate, mixture.shared_up,
                                     self.shared_ids, self.shared_gated, 0, P)
            ops.experts_linear(self.expert_gated, mixture.down, self.route_ids.view(-1),
                               self.expert_out)
            ops.linears(self.shared_gated, [mixture.shared_down], [self.shared_out])
            ops.moe_combine_norm(self.expert_out, self.route_weights,
                                 SharedExpert(self.shared_out, self.normed, mixture.shared_router),
                                 self.x, next_norm, P)
            return
        # expert parallelism: this rank's experts (other ranks' slots are
        # zeros), the shared expert on rank 0, the partial combine into the
        # exchange, summed over the ranks with the residual and normalised
        first = self.part.experts[0]
        if mixture.fused is not None:
            # rank 0: the shared expert (id -1) first in the fused weights,
            # its slots in the routed experts' launches -- no launches of its
            # own, so every rank runs the same ones
            gate, up, down = mixture.fused
            ops.experts_gated_linear(self.normed, gate, up, self.all_ids, self.all_gated,
                                     first_expert=first - 1, prepared=P, shared_tail=True)
            self._mark("experts_gate_up")
            ops.experts_linear(self.all_gated, down, self.all_ids, self.all_out,
                               first_expert=first - 1)
            self._mark("experts_down")
            shared = SharedExpert(self.shared_out, self.normed, mixture.shared_router)
            ops.moe_combine(self.expert_out, self.route_weights, shared, None,
                            self.exchange.slots[1])
            self._mark("combine")
            self.exchange.add_rms_norm(1, self.x, next_norm, P)
            self._mark("exchange")
            return
        ops.experts_gated_linear(self.normed, mixture.gate, mixture.up, self.route_ids.view(-1),
                                 self.expert_gated, first_expert=first, prepared=P)
        self._mark("experts_gate_up")
        ops.experts_linear(self.expert_gated, mixture.down, self.route_ids.view(-1),
                           self.expert_out, first_expert=first)
        self._mark("experts_down")
        shared = None
        if self.part.rank == 0:
            ops.experts_gated_linear(self.normed, mixture.shared_gate, mixture.shared_up,
                                     self.shared_ids, self.shared_gated, 0, P)
            ops.linears(self.shared_gated, [mixture.shared_down], [self.shared_out])
            shared = SharedExpert(self.shared_out, self.normed, mixture.shared_router)
        ops.moe_combine(self.expert_out, self.route_weights, shared, None, self.exchange.slots[1])
        self._mark("combine")
        self.exchange.add_rms_norm(1, self.x, next_norm, P)
        self._mark("exchange")

    def step(self) -> torch.Tensor:
        """One decode step: self.ids at self.positions -> self.logits (this
        rank's vocabulary rows) and self.next_ids (each sequence's greedy next
        token over the whole vocabulary)."""
        ops, c, w, P = self.ops, self.config, self.weights, self.prepared
        self._mark("start")
        ops.embedding(w.embedding, self.ids, self.x)
        ops.add_rms_norm(self.x, None, RowNorm(w.layers[0].input_norm, c.epsilon, 0.0, self.normed),
                         P)
        self._mark("embed")
        for index, layer in enumerate(w.layers):
            if isinstance(layer.mixer, FullLayer):
                self._full(layer.mixer, index)
            else:
                self._delta(layer.mixer, index)
            post = RowNorm(layer.post_norm, c.epsilon, 0.0, self.normed)
            if self.exchange is not None:
                self.exchange.add_rms_norm(0, self.x, post, P)
                self._mark("exchange")
            else:
                ops.add_rms_norm(self.x, self.block_out, post, P)
                self._mark("add_norm")
            following = (w.layers[index + 1].input_norm if index + 1 < len(w.layers)
                         else w.final_norm)
            self._mixture(layer.mixture, following)
        ops.linears(self.normed, [w.lm_head], [self.logits], P)
        self._mark("lm_head")
        self.sampler(self.logits, self.next_ids)
        self._mark("sample")
        return self.logits

    def reserve(self) -> None:
        c, lib = self.config, self.ops.lib
        from ._lib import check
        widest = max(c.hidden, self.value_width, self.q_heads * c.head_dim, c.shared_ffn,
                     c.expert_ffn)
        self.ops.reserve_workspace(self.batch * c.used, widest)
        need = max(lib.drift_attention_workspace_bytes(self.batch, self.q_heads, c.head_dim,
                                                       self.context),
                   lib.drift_linear_workspace_bytes(self.batch * c.used, widest))
        check("drift_workspace_reserve", lib.drift_workspace_reserve(need))

    def capture(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Records one step as a CUDA graph (positions read from the device)."""
        self.reserve()
        stream = stream or torch.cuda.Stream()
        # the first calls resolve lazy state outside the capture; the states
        # they advance are restored so the captured step starts where the
        # caller left them
        saved = ([s.clone() for s in self.conv_states.values()],
                 [s.clone() for s in self.delta_states.values()])
        with torch.cuda.stream(stream):
            self.step()
        torch.cuda.synchronize()
        for s, kept in zip(self.conv_states.values(), saved[0]):
            s.copy_(kept)
        for s, kept in zip(self.delta_states.values(), saved[1]):
            s.copy_(kept)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.step()
        torch.cuda.synchronize()

    def replay(self) -> None:
        self.graph.replay()

    def release(self) -> None:
        """Drops the graph and the exchange's buffers."""
        self.graph = None
        if self.exchange is not None:
            torch.cuda.synchronize()
            self.exchange.close()
            self.exchange = None
