"""The hybrid MoE decoder's decode step on this library's ops: the op order of
the runner's HybridBlocks (runner/src/drift/runner/models/HybridBlocks.scala:
403-588) and Qwen35.decoderLayer (models/Qwen35.scala:356-410), for a batch
of sequences on one GPU.

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
from .ops import SIGMOID, SILU, Attention, CudaOps, KvCache, Rope, RowNorm, SharedExpert, Stored


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


@dataclass
class HybridLayer:
    input_norm: torch.Tensor
    mixer: object                # DeltaLayer or FullLayer
    post_norm: torch.Tensor
    mixture: MixtureLayer


@dataclass
class HybridWeights:
    embedding: Stored
    layers: list
    final_norm: torch.Tensor
    lm_head: Stored

    @staticmethod
    def random(c: HybridConfig, dtype: int = Q4_1, seed: int = 0) -> "HybridWeights":
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)

        def stored(n, k, experts: int = 0):
            rows = n * max(1, experts)
            shape = (experts, n, k) if experts else (n, k)
            return Stored(dtype, shape, synthetic.quantized_device(dtype, rows, k, g))

        def f32(*shape, scale=1.0):
            return scale * torch.randn(*shape, generator=g, device="cuda")

        def norm(width):
            return 1.0 + 0.02 * torch.randn(width, generator=g, device="cuda")

        channels = (2 * c.delta_key_heads + c.delta_value_heads) * c.delta_dim
        value_width = c.delta_value_heads * c.delta_dim
        layers = []
        for i in range(c.layers):
            if c.is_full(i):
                mixer = FullLayer(stored(c.q_heads * 2 * c.head_dim, c.hidden),
                                  stored(c.kv_heads * c.head_dim, c.hidden),
                                  stored(c.kv_heads * c.head_dim, c.hidden),
                                  norm(c.head_dim), norm(c.head_dim),
                                  stored(c.hidden, c.q_heads * c.head_dim))
            else:
                mixer = DeltaLayer(stored(channels, c.hidden), stored(value_width, c.hidden),
                                   f32(c.delta_value_heads, c.hidden, scale=0.02),
                                   f32(c.delta_value_heads, c.hidden, scale=0.02),
                                   f32(channels, c.conv_taps, scale=0.5),
                                   -torch.exp(torch.rand(c.delta_value_heads, generator=g,
                                                         device="cuda") * 2.5 - 1.0),
                                   f32(c.delta_value_heads), norm(c.delta_dim),
                                   stored(c.hidden, value_width))
            mixture = MixtureLayer(f32(c.experts, c.hidden, scale=0.02),
                                   stored(c.expert_ffn, c.hidden, c.experts),
                                   stored(c.expert_ffn, c.hidden, c.experts),
                                   stored(c.hidden, c.expert_ffn, c.experts),
                                   stored(c.shared_ffn, c.hidden, 1),
                                   stored(c.shared_ffn, c.hidden, 1),
                                   stored(c.hidden, c.shared_ffn),
                                   f32(c.hidden, scale=0.02))
            layers.append(HybridLayer(norm(c.hidden), mixer, norm(c.hidden), mixture))
        return HybridWeights(Stored(Q8_0, (c.vocab, c.hidden),
                                    synthetic.quantized_device(Q8_0, c.vocab, c.hidden, g)),
                             layers, norm(c.hidden), stored(c.vocab, c.hidden))

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
                 context: int):
        c = self.config = config
        self.ops, self.weights, self.batch, self.context = ops, weights, batch, context
        b = batch
        f32 = dict(dtype=torch.float32, device="cuda")
        pages_per_sequence = (context + c.page_size - 1) // c.page_size
        self.page_tables = torch.arange(pages_per_sequence * b, dtype=torch.int32,
                                        device="cuda").view(b, pages_per_sequence)
        self.channels = (2 * c.delta_key_heads + c.delta_value_heads) * c.delta_dim
        self.value_width = c.delta_value_heads * c.delta_dim
        self.caches, self.conv_states, self.delta_states = {}, {}, {}
        for i, layer in enumerate(weights.layers):
            if isinstance(layer.mixer, FullLayer):
                self.caches[i] = KvCache.allocate(pages_per_sequence * b, c.page_size, c.kv_heads,
                                                  c.head_dim)
            else:
                self.conv_states[i] = torch.zeros(b, c.conv_taps - 1, self.channels, **f32)
                self.delta_states[i] = torch.zeros(b, c.delta_value_heads, c.delta_dim,
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
        self.a = torch.zeros(b, c.delta_value_heads, **f32)
        self.b = torch.zeros(b, c.delta_value_heads, **f32)
        self.core = torch.zeros(b, c.delta_value_heads, c.delta_dim, **f32)
        # full attention
        self.query_gate = torch.zeros(b, c.q_heads, 2 * c.head_dim, **f32)
        self.k = torch.zeros(b, c.kv_heads, c.head_dim, **f32)
        self.v = torch.zeros(b, c.kv_heads, c.head_dim, **f32)
        self.q_turned = torch.zeros(b, c.q_heads, c.head_dim, **f32)
        self.attended = torch.zeros(b, c.q_heads, c.head_dim, **f32)
        # mixture
        self.logits_router = torch.zeros(b, c.experts, **f32)
        self.route_ids = torch.zeros(b, c.used, dtype=torch.int32, device="cuda")
        self.route_weights = torch.zeros(b, c.used, **f32)
        self.expert_gated = torch.zeros(b * c.used, c.expert_ffn, **f32)
        self.expert_out = torch.zeros(b * c.used, c.hidden, **f32)
        self.shared_ids = torch.zeros(b, dtype=torch.int32, device="cuda")
        self.shared_gated = torch.zeros(b, c.shared_ffn, **f32)
        self.shared_out = torch.zeros(b, c.hidden, **f32)
        self.logits = torch.zeros(b, c.vocab, **f32)
        widest = max(c.hidden, self.value_width, c.q_heads * c.head_dim, c.shared_ffn)
        self.prepared = ops.prepared_x(b, widest)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

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
        # (the layer's input comes from the mixture's combine + norm, which
        # writes no records: the products prepare x themselves)
        ops.linears(self.normed, [layer.qkv, layer.z, layer.a, layer.b],
                    [self.qkv, self.z, self.a, self.b])
        ops.causal_conv_decode(self.qkv, layer.conv, 1, self.conv_states[index], self.convolved)
        ops.gated_delta_rule_decode(self.convolved, self.a, self.b, layer.decay, layer.dt_bias,
                                    self.delta_states[index],
                                    (c.delta_key_heads, c.delta_value_heads, c.delta_dim, False),
                                    self.core)
        core = self.core.view(b * c.delta_value_heads, c.delta_dim)
        ops.gated_rms_norm(core, layer.norm, self.z.view(b * c.delta_value_heads, c.delta_dim),
                           SILU, c.epsilon, core, P, c.delta_value_heads)
        ops.linears(self.core.view(b, self.value_width), [layer.out], [self.block_out], P)

    def _full(self, layer: FullLayer, index: int) -> None:
        ops, c, b, P = self.ops, self.config, self.batch, self.prepared
        ops.linears(self.normed, [layer.q, layer.k, layer.v],
                    [self.query_gate.view(b, -1), self.k.view(b, -1), self.v.view(b, -1)])
        ops.attention_inputs_decode(self.query_gate, self.k, self.v, layer.q_norm, layer.k_norm,
                                    c.epsilon, self.positions, self.rope, self.q_turned,
                                    self.caches[index], self.page_tables)
        ops.attention_decode(self.q_turned, self.caches[index], self.page_tables, self.positions,
                             self.context, self.attention, self.attended, P,
                             gate=self.query_gate[:, :, c.head_dim:])
        ops.linears(self.attended.view(b, -1), [layer.o], [self.block_out], P)

    def _mixture(self, mixture: MixtureLayer, following: torch.Tensor) -> None:
        ops, c, P = self.ops, self.config, self.prepared
        ops.route_linear(self.normed, mixture.router, self.logits_router, self.route_ids,
                         self.route_weights)
        ops.experts_gated_linear(self.normed, mixture.gate, mixture.up, self.route_ids.view(-1),
                                 self.expert_gated)
        ops.experts_gated_linear(self.normed, mixture.shared_gate, mixture.shared_up,
                                 self.shared_ids, self.shared_gated)
        ops.experts_linear(self.expert_gated, mixture.down, self.route_ids.view(-1),
                           self.expert_out)
        ops.linears(self.shared_gated, [mixture.shared_down], [self.shared_out])
        ops.moe_combine_norm(self.expert_out, self.route_weights,
                             SharedExpert(self.shared_out, self.normed, mixture.shared_router),
                             self.x, RowNorm(following, c.epsilon, 0.0, self.normed))

    def step(self) -> torch.Tensor:
        """One decode step: self.ids at self.positions -> self.logits."""
        ops, c, w, P = self.ops, self.config, self.weights, self.prepared
        ops.embedding(w.embedding, self.ids, self.x)
        ops.rms_norm(self.x, w.layers[0].input_norm, c.epsilon, 0.0, self.normed)
        for index, layer in enumerate(w.layers):
            if isinstance(layer.mixer, FullLayer):
                self._full(layer.mixer, index)
            else:
                self._delta(layer.mixer, index)
            ops.add_rms_norm(self.x, self.block_out,
                             RowNorm(layer.post_norm, c.epsilon, 0.0, self.normed))
            following = (w.layers[index + 1].input_norm if index + 1 < len(w.layers)
                         else w.final_norm)
            self._mixture(layer.mixture, following)
        ops.linears(self.normed, [w.lm_head], [self.logits])
        return self.logits

    def reserve(self) -> None:
        c, lib = self.config, self.ops.lib
        from ._lib import check
        widest = max(c.hidden, self.value_width, c.q_heads * c.head_dim, c.shared_ffn, c.expert_ffn)
        self.ops.reserve_workspace(self.batch * c.used, widest)
        need = max(lib.drift_attention_workspace_bytes(self.batch, c.q_heads, c.head_dim,
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
        self.graph = None
