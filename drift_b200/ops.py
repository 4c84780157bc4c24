"""The drift runner's `Ops` API for the quantized-inference hot path, on B200.

`CudaOps` mirrors the reference's operator interface (runner/src/drift/runner/
ops/Ops.scala and its LinearOps, NormalisationOps, ElementwiseOps,
AttentionOps.rope, ExpertsOps traits): the same operations, argument meanings
and shape rules, with `out` tensors written and never read. Each call goes
through libdrift_cuda's C ABI (include/drift_ops.h) -- the kernels, their
dispatch and their checks are native; PyTorch only owns device memory and
streams here. There is no CPU path: without the built library or a GPU the
calls raise.

Tensors: activations are torch CUDA tensors, F32 (and BF16 for a product's x);
a stored weight is a `Stored` (its GGML type, logical shape and raw block
bytes on the device), as the reference's Tensor(dtype, shape, storage) is.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import BF16, F32, Q4_0, Q4_1, Q8_0, check
from .dtypes import DTYPES, byte_size

# Activation codes (runner/src/drift/runner/ops/Activation.scala:5-19).
SILU, GELU_TANH, GELU_ERF, SIGMOID, SITU = 0, 1, 2, 3, 4
# RoPE layouts (ops/Rope.scala:7-10).
NEOX, INTERLEAVED = 0, 1


@dataclass
class Stored:
    """A weight in a storage type: `data` holds the raw blocks (uint8, on the
    device), `shape` the logical elements ([N, K], or [experts, N, K])."""
    dtype: int
    shape: tuple
    data: torch.Tensor

    def __post_init__(self):
        expected = byte_size(self.dtype, _count(self.shape))
        if self.data.dtype != torch.uint8 or self.data.numel() < expected:
            raise ValueError(f"{DTYPES[self.dtype].name} {list(self.shape)} needs {expected} "
                             f"bytes, not {self.data.numel()} {self.data.dtype}")

    @staticmethod
    def upload(dtype: int, shape: Sequence[int], blocks, device=None) -> "Stored":
        """Raw blocks (numpy uint8 or a tensor) copied to the device."""
        tensor = torch.as_tensor(blocks).to(torch.uint8).reshape(-1)
        return Stored(dtype, tuple(int(s) for s in shape),
                      tensor.to(device or torch.device("cuda")))


@dataclass
class Rope:
    """A rotary embedding (ops/Rope.scala:37-46), Single sections only."""
    theta: float
    rotary_dimensions: int
    layout: int = NEOX


@dataclass
class KvCache:
    """The reference's paged F16 key/value cache (ops/KvCache.scala:12-23):
    keys [pages, page_size, kv_heads, D], values [pages, kv_heads, D,
    page_size]; page_size a multiple of 16."""
    keys: torch.Tensor
    values: torch.Tensor
    page_size: int

    @property
    def pages(self) -> int:
        return int(self.keys.shape[0])

    @property
    def kv_heads(self) -> int:
        return int(self.keys.shape[2])

    @property
    def head_dim(self) -> int:
        return int(self.keys.shape[3])

    @staticmethod
    def allocate(pages: int, page_size: int, kv_heads: int, head_dim: int,
                 device=None) -> "KvCache":
        device = device or torch.device("cuda")
        return KvCache(torch.zeros(pages, page_size, kv_heads, head_dim, dtype=torch.float16,
                                   device=device),
                       torch.zeros(pages, kv_heads, head_dim, page_size, dtype=torch.float16,
                                   device=device), page_size)


@dataclass
class Attention:
    """An attention's parameters (ops/Attention.scala:11-17)."""
    scale: float
    causal: bool = True
    window: Optional[int] = None
    softcap: Optional[float] = None
    sinks: Optional[torch.Tensor] = None


@dataclass
class RowNorm:
    """An RMS norm taken of a result as it is written (ops/RowNorm.scala:20-25)."""
    weight: torch.Tensor
    epsilon: float
    weight_offset: float
    out: torch.Tensor


@dataclass
class SharedExpert:
    """A mixture's shared expert in moe_combine (ops/ExpertTensors.scala:8-12):
    its output [tokens, H] weighted by sigmoid(input . router)."""
    output: torch.Tensor
    input: torch.Tensor
    router: torch.Tensor


def _count(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _require(condition: bool, message: str) -> None:
    if not condition:
        raise ValueError(message)


def _f32(name: str, *tensors: torch.Tensor) -> None:
    for t in tensors:
        _require(t.dtype == torch.float32, f"{name} takes F32, not {t.dtype}")
        _require(t.is_cuda and t.is_contiguous(),
                 f"{name}: tensors are contiguous device memory")


def _same_shape(name: str, *tensors: torch.Tensor) -> None:
    shapes = {tuple(t.shape) for t in tensors}
    _require(len(shapes) == 1,
             f"{name} needs equal shapes, got {', '.join(str(list(t.shape)) for t in tensors)}")


def _x_dtype(name: str, x: torch.Tensor) -> int:
    _require(x.dtype in (torch.float32, torch.bfloat16),
             f"{name} takes F32 (or BF16) x, not {x.dtype}")
    _require(x.is_cuda and x.is_contiguous(), f"{name}: x is contiguous device memory")
    return F32 if x.dtype == torch.float32 else BF16


class CudaOps:
    """The B200 backend of the `Ops` operations on the hot path."""

    name = "cuda"

    def __init__(self, device: int | None = None):
        self.lib = _lib.load()
        if device is not None:
            torch.cuda.set_device(device)
        self.device = torch.cuda.current_device()

    # -- plumbing -------------------------------------------------------------------------
    @staticmethod
    def _stream():
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def synchronize(self) -> None:
        torch.cuda.current_stream().synchronize()

    def take_device_error(self) -> int:
        """The device error word, cleared: 0 none, 1 an id outside its table,
        2 a bounded wait inside a kernel gave up, 3 the tensor-parallel
        exchange's wait for a peer rank gave up."""
        code = ctypes.c_int(0)
        check("drift_device_error_take", self.lib.drift_device_error_take(ctypes.byref(code)))
        return code.value

    def reserve_workspace(self, m: int, k: int) -> None:
        """Sizes the library's scratch for products of m rows of k (call before
        capturing a CUDA graph)."""
        check("drift_workspace_reserve",
              self.lib.drift_workspace_reserve(self.lib.drift_linear_workspace_bytes(m, k)))

    # -- LinearOps (ops/LinearOps.scala) ------------------------------------------------------
    @staticmethod
    def _check_linear(x: torch.Tensor, weight, out: torch.Tensor):
        """Ops.checkLinear (ops/LinearOps.scala:227-249); returns (M, N, K)."""
        _x_dtype("linear", x)
        _f32("linear", out)
        wshape = weight.shape if isinstance(weight, Stored) else tuple(weight.shape)
        _require(x.dim() == 2 and len(wshape) == 2 and out.dim() == 2,
                 f"linear takes [M, K] · [N, K]ᵀ → [M, N], got {list(x.shape)}, "
                 f"{list(wshape)}, {list(out.shape)}")
        m, k = x.shape
        n, wk = wshape
        _require(wk == k, f"linear: x rows of {k} against weight rows of {wk}")
        _require(tuple(out.shape) == (m, n), f"linear: out {list(out.shape)} for [{m}, {n}]")
        return int(m), int(n), int(k)

    @staticmethod
    def _weight(weight):
        if isinstance(weight, Stored):
            return weight.dtype, weight.data
        _require(weight.dtype == torch.float32 and weight.is_cuda and weight.is_contiguous(),
                 f"no kernels for {weight.dtype} weights yet")
        return F32, weight

    def linear(self, x: torch.Tensor, weight, out: torch.Tensor) -> None:
        """out = x · weightᵀ (ops/LinearOps.scala:147-150)."""
        self.linears(x, [weight], [out])

    def prepared_x(self, m: int, k: int) -> torch.Tensor:
        """A buffer for the records of m rows of k values, which a producer
        (add_rms_norm, gated, attention_decode with `prepared=`) writes for
        the products that follow (linears with `prepared=`)."""
        size = self.lib.drift_prepared_x_bytes(m, k)
        _require(size > 0, f"no prepared x for [{m}, {k}]")
        return torch.empty(size, dtype=torch.uint8, device="cuda")

    def linears(self, x: torch.Tensor, weights: Sequence, outs: Sequence[torch.Tensor],
                prepared: Optional[torch.Tensor] = None) -> None:
        """Several products of the same x, x prepared once (LinearOps.scala:152-156);
        `prepared`: x's records, already written by the kernel that made x."""
        shapes = [self._check_linear(x, w, o) for w, o in zip(weights, outs)]
        _require(len(weights) == len(outs), "linears: as many outs as weights")
        if not shapes:
            return
        m, _, k = shapes[0]
        count = len(weights)
        dtypes = (ctypes.c_int * count)()
        wptrs = (ctypes.c_void_p * count)()
        optrs = (ctypes.c_void_p * count)()
        ns = (ctypes.c_int64 * count)()
        for i, (w, o, (_, n, _)) in enumerate(zip(weights, outs, shapes)):
            dtype, data = self._weight(w)
            dtypes[i], wptrs[i], optrs[i], ns[i] = dtype, data.data_ptr(), o.data_ptr(), n
        if prepared is None:
            status = self.lib.drift_linears(_x_dtype("linear", x), _ptr(x), count, dtypes, wptrs,
                                            optrs, ns, m, k, self._stream())
        else:
            status = self.lib.drift_linears_prepared(_x_dtype("linear", x), _ptr(x),
                                                     _ptr(prepared), count, dtypes, wptrs, optrs,
                                                     ns, m, k, self._stream())
        check("drift_linears", status)

    def embedding(self, table: Stored, ids: torch.Tensor, out: torch.Tensor) -> None:
        """out[t] = table[ids[t]] as F32 (LinearOps.scala:83-87; checks L163-177)."""
        _require(len(table.shape) == 2,
                 f"an embedding table is [vocabulary, D], not {list(table.shape)}")
        _require(ids.dtype == torch.int32 and ids.dim() == 1,
                 f"embedding ids are I32 [tokens], not {ids.dtype} {list(ids.shape)}")
        _f32("embedding", out)
        vocab, cols = table.shape
        _require(tuple(out.shape) == (ids.shape[0], cols),
                 f"embedding: out {list(out.shape)} for {ids.shape[0]} rows of {cols}")
        status = self.lib.drift_embedding(table.dtype, _ptr(table.data), vocab, cols, _ptr(ids),
                                          ids.shape[0], _ptr(out), self._stream())
        check("drift_embedding", status)

    # -- NormalisationOps (ops/NormalisationOps.scala) ---------------------------------------------
    @staticmethod
    def _check_row_wise(name: str, x, out, *vectors) -> int:
        """Ops.checkRowWise (ops/Ops.scala:76-92); returns the row count."""
        _f32(name, x, out)
        _same_shape(name, x, out)
        _require(x.dim() >= 1, f"{name} needs at least one dimension")
        for v in vectors:
            _f32(name, v)
            _require(tuple(v.shape) == (x.shape[-1],),
                     f"{name}: {list(v.shape)} for rows of {x.shape[-1]}")
        return x.numel() // max(1, x.shape[-1])

    def rms_norm(self, x, weight, epsilon: float, weight_offset: float, out) -> None:
        """out = x / sqrt(mean(x²) + eps) × (weight + offset) (NormalisationOps.scala:205-215)."""
        rows = self._check_row_wise("rmsNorm", x, out, weight)
        status = self.lib.drift_rms_norm(_ptr(x), _ptr(weight), epsilon, weight_offset, _ptr(out),
                                         rows, x.shape[-1], self._stream())
        check("drift_rms_norm", status)

    def add_rms_norm(self, x, y, norm: RowNorm, prepared: Optional[torch.Tensor] = None) -> None:
        """x += y, then norm's RMS norm of x into norm.out, one launch
        (NormalisationOps.scala:217-224); with `prepared`, norm.out's records
        too (y None: the norm alone)."""
        if y is not None:
            _f32("add", x, y)
            _same_shape("add", x, y)
        rows = self._check_row_wise("rmsNorm", x, norm.out, norm.weight)
        if prepared is None:
            _require(y is not None, "addRmsNorm: no y")
            status = self.lib.drift_add_rms_norm(_ptr(x), _ptr(y), _ptr(norm.weight), norm.epsilon,
                                                 norm.weight_offset, _ptr(norm.out), rows,
                                                 x.shape[-1], self._stream())
        else:
            status = self.lib.drift_add_rms_norm_prepared(
                _ptr(x), _ptr(y), _ptr(norm.weight), norm.epsilon, norm.weight_offset,
                _ptr(norm.out), rows, x.shape[-1], _ptr(prepared), self._stream())
        check("drift_add_rms_norm", status)

    def add(self, a, b, out) -> None:
        """out = a + b (ops/CpuElementwise.scala:9-13)."""
        _f32("add", a, b, out)
        _same_shape("add", a, b, out)
        check("drift_add", self.lib.drift_add(_ptr(a), _ptr(b), _ptr(out), a.numel(),
                                              self._stream()))

    def gated(self, kind: int, gate, up, out, prepared: Optional[torch.Tensor] = None) -> None:
        """out = kind(gate) × up: SwiGLU with SILU (NormalisationOps.scala:200-203);
        with `prepared`, out's records (rows of out's last dimension) too."""
        _f32("gated", gate, up, out)
        _same_shape("gated", gate, up, out)
        if prepared is None:
            status = self.lib.drift_gated(kind, _ptr(gate), _ptr(up), _ptr(out), gate.numel(),
                                          self._stream())
        else:
            cols = out.shape[-1]
            status = self.lib.drift_gated_prepared(kind, _ptr(gate), _ptr(up), _ptr(out),
                                                   out.numel() // max(1, cols), cols,
                                                   _ptr(prepared), self._stream())
        check("drift_gated", status)

    # -- AttentionOps.rope (ops/AttentionOps.scala:42-45) ---------------------------------------------
    def rope(self, x, positions, rope: Rope, out) -> None:
        """Rotary embedding of x [tokens, heads, D]; positions I32 [tokens]."""
        _f32("rope", x, out)
        _same_shape("rope", x, out)
        _require(x.dim() == 3, f"rope takes [tokens, heads, headDimension], got {list(x.shape)}")
        _require(positions.dtype == torch.int32,
                 f"rope positions are I32, not {positions.dtype}")
        tokens, heads, dim = x.shape
        _require(tuple(positions.shape) == (tokens,),
                 f"rope: positions {list(positions.shape)} for {tokens} tokens")
        status = self.lib.drift_rope(_ptr(x), _ptr(positions), _ptr(out), tokens, heads, dim,
                                     rope.theta, rope.rotary_dimensions, rope.layout,
                                     self._stream())
        check("drift_rope", status)

    def cache_write(self, k, v, cache: KvCache, page_table, start: int) -> None:
        """k, v [tokens, kv_heads, D] into the cache at positions start..
        (AttentionOps.scala:58-64; checks L225-257)."""
        _f32("cacheWrite", k, v)
        _require(k.shape == v.shape and k.dim() == 3 and
                 tuple(k.shape[1:]) == (cache.kv_heads, cache.head_dim),
                 f"cacheWrite: {list(k.shape)} into a cache of {cache.kv_heads} heads of "
                 f"{cache.head_dim}")
        _require(page_table.dtype == torch.int32 and page_table.dim() == 1,
                 f"a page table is I32 [pages], not {page_table.dtype} {list(page_table.shape)}")
        status = self.lib.drift_cache_write(
            _ptr(k), _ptr(v), int(k.shape[0]), cache.kv_heads, cache.head_dim, _ptr(cache.keys),
            _ptr(cache.values), cache.pages, cache.page_size, _ptr(page_table),
            int(page_table.numel()), start, self._stream())
        check("drift_cache_write", status)

    def attention(self, q, cache: KvCache, page_table, query_start: int, key_count: int,
                  attention: Attention, out) -> None:
        """Attention of q [tokens, q_heads, D] over the cache's first key_count
        positions (AttentionOps.scala:113-121; checks L259-294)."""
        _f32("attention", q, out)
        _same_shape("attention", q, out)
        _require(q.dim() == 3 and q.shape[2] == cache.head_dim,
                 f"attention: queries {list(q.shape)} against heads of {cache.head_dim}")
        _require(page_table.dtype == torch.int32 and page_table.dim() == 1,
                 f"a page table is I32 [pages], not {page_table.dtype} {list(page_table.shape)}")
        tokens, q_heads, _ = q.shape
        sinks = attention.sinks
        if sinks is not None:
            _f32("attention sinks", sinks)
            _require(tuple(sinks.shape) == (q_heads,),
                     f"attention: sinks {list(sinks.shape)} for {q_heads} heads")
        status = self.lib.drift_attention(
            _ptr(q), tokens, q_heads, _ptr(cache.keys), _ptr(cache.values), cache.pages,
            cache.page_size, cache.kv_heads, cache.head_dim, _ptr(page_table),
            int(page_table.numel()), query_start, key_count, attention.scale,
            int(attention.causal), int(attention.window or 0), float(attention.softcap or 0.0),
            _ptr(sinks), _ptr(out), self._stream())
        check("drift_attention", status)

    def attention_inputs_decode(self, q, k, v, q_norm, k_norm, epsilon: float, positions,
                                rope: Rope, q_out, cache: KvCache, page_tables,
                                weight_offset: float = 0.0) -> None:
        """A decode step's per-head q/k RMS norms, their rope and the cache
        write of k and v, for one token per sequence, in one launch.
        q [b, q_heads, D] -- or queryAndGate [b, q_heads, 2 D], whose first
        half per head is the query -- k, v [b, kv_heads, D]; positions I32
        [b]; page_tables I32 [b, pages per sequence]."""
        _f32("attentionInputs", q, k, v, q_out)
        _same_shape("attentionInputs", k, v)
        split = q.shape[-1] == 2 * q_out.shape[-1]
        _require(split or tuple(q.shape) == tuple(q_out.shape),
                 f"attentionInputs: q {list(q.shape)} for out {list(q_out.shape)}")
        b, q_heads, dim = q_out.shape
        _require(k.dim() == 3 and k.shape[0] == b and tuple(k.shape[1:]) ==
                 (cache.kv_heads, cache.head_dim) and dim == cache.head_dim,
                 f"attentionInputs: {list(q.shape)}, {list(k.shape)} for a cache of "
                 f"{cache.kv_heads} heads of {cache.head_dim}")
        _require(positions.dtype == torch.int32 and tuple(positions.shape) == (b,),
                 f"attentionInputs: positions {list(positions.shape)} for {b} sequences")
        _require(page_tables.dtype == torch.int32 and page_tables.dim() == 2 and
                 page_tables.shape[0] == b and page_tables.is_contiguous(),
                 f"attentionInputs: page tables {list(page_tables.shape)} for {b} sequences")
        call = (self.lib.drift_attention_inputs_decode_split if split
                else self.lib.drift_attention_inputs_decode)
        status = call(
            _ptr(q), _ptr(k), _ptr(v), b, q_heads, cache.kv_heads, dim, _ptr(q_norm),
            _ptr(k_norm), epsilon, weight_offset, _ptr(positions), rope.theta,
            rope.rotary_dimensions, rope.layout, _ptr(q_out), _ptr(cache.keys),
            _ptr(cache.values), cache.pages, cache.page_size, _ptr(page_tables),
            int(page_tables.shape[1]), self._stream())
        check("drift_attention_inputs_decode", status)

    def attention_decode(self, q, cache: KvCache, page_tables, positions, max_key_count: int,
                         attention: Attention, out, prepared: Optional[torch.Tensor] = None,
                         gate: Optional[torch.Tensor] = None) -> None:
        """Attention of one query per sequence, all sequences in one launch:
        row z of q [b, q_heads, D] at positions[z] over its keys 0..positions[z];
        with `prepared`, the records of out as [b, q_heads D] too."""
        _f32("attention", q, out)
        _same_shape("attention", q, out)
        b, q_heads, dim = q.shape
        _require(dim == cache.head_dim,
                 f"attention: queries {list(q.shape)} against heads of {cache.head_dim}")
        _require(page_tables.dtype == torch.int32 and page_tables.dim() == 2 and
                 page_tables.shape[0] == b and page_tables.is_contiguous(),
                 f"attention: page tables {list(page_tables.shape)} for {b} sequences")
        _require(positions.dtype == torch.int32 and tuple(positions.shape) == (b,),
                 f"attention: positions {list(positions.shape)} for {b} sequences")
        _require(attention.causal, "a decode step's attention is causal")
        args = (_ptr(q), b, q_heads, _ptr(cache.keys), _ptr(cache.values), cache.pages,
                cache.page_size, cache.kv_heads, dim, _ptr(page_tables), int(page_tables.shape[1]),
                _ptr(positions), max_key_count, attention.scale, int(attention.window or 0),
                float(attention.softcap or 0.0), _ptr(attention.sinks), _ptr(out))
        if gate is not None:
            # gate: [b, q_heads, stride] whose first D of each head gate the
            # output (the second half of queryAndGate, viewed from there)
            _require(gate.dtype == torch.float32 and gate.is_cuda and tuple(gate.shape) == (b, q_heads, dim),
                     f"attention: gate {list(gate.shape)} {gate.dtype} for {list(q.shape)}")
            stride = gate.stride(1)
            _require(gate.stride(0) == q_heads * stride and gate.stride(2) == 1,
                     "attention: the gate is rows of heads")
            status = self.lib.drift_attention_decode_gated(*args, _ptr(gate), stride, _ptr(prepared),
                                                           self._stream())
        elif prepared is None:
            status = self.lib.drift_attention_decode(*args, self._stream())
        else:
            status = self.lib.drift_attention_decode_prepared(*args, _ptr(prepared),
                                                              self._stream())
        check("drift_attention_decode", status)

    # -- SequenceOps: Gated DeltaNet (ops/SequenceOps.scala) --------------------------------------
    def causal_conv(self, x, weight, dilation: int, state, history, out) -> None:
        """SiLU of the causal depthwise convolution of x [tokens, channels] with
        weight [channels, taps]; state [span, channels] updated in place
        (SequenceOps.causalConv; CpuSequence.scala:29-80)."""
        _f32("causalConv", x, weight, state, out)
        _same_shape("causalConv", x, out)
        _require(x.dim() == 2, f"causalConv takes [tokens, channels], not {list(x.shape)}")
        tokens, channels = x.shape
        taps = weight.shape[-1]
        _require(tuple(weight.shape) == (channels, taps) and taps <= 9,
                 f"causalConv: weight {list(weight.shape)} for {channels} channels")
        span = (taps - 1) * dilation
        _require(dilation >= 1 and span <= 16 and tuple(state.shape) == (span, channels),
                 f"causalConv: state {list(state.shape)}, expected [{span}, {channels}]")
        status = self.lib.drift_causal_conv(_ptr(x), tokens, channels, _ptr(weight), taps, dilation,
                                            _ptr(state), _ptr(history), _ptr(out), self._stream())
        check("drift_causal_conv", status)

    def gated_delta_rule(self, qkv, a, b, decay, dt_bias, state, rule, history, out) -> None:
        """The gated delta rule of `rule` (key_heads, value_heads, dimension,
        tiled_heads) over qkv [tokens, qkv_width]; state [value_heads, D, D]
        updated in place; out [tokens, value_heads, D]
        (SequenceOps.gatedDeltaRule; CpuSequence.scala:82-158)."""
        key_heads, value_heads, d, tiled = rule
        _f32("gatedDeltaRule", qkv, a, b, decay, dt_bias, state, out)
        tokens = qkv.shape[0]
        width = (2 * key_heads + value_heads) * d
        _require(tuple(qkv.shape) == (tokens, width),
                 f"gatedDeltaRule: qkv {list(qkv.shape)}, expected [{tokens}, {width}]")
        _require(tuple(a.shape) == (tokens, value_heads) and tuple(b.shape) == tuple(a.shape),
                 f"gatedDeltaRule: a {list(a.shape)}, b {list(b.shape)}")
        _require(tuple(decay.shape) == (value_heads,) and tuple(dt_bias.shape) == (value_heads,),
                 f"gatedDeltaRule: decay {list(decay.shape)}, dtBias {list(dt_bias.shape)}")
        _require(tuple(state.shape) == (value_heads, d, d),
                 f"gatedDeltaRule: state {list(state.shape)}")
        _require(tuple(out.shape) == (tokens, value_heads, d),
                 f"gatedDeltaRule: out {list(out.shape)}")
        status = self.lib.drift_gated_delta_rule(
            _ptr(qkv), tokens, key_heads, value_heads, d, int(tiled), _ptr(a), _ptr(b),
            _ptr(decay), _ptr(dt_bias), _ptr(state), _ptr(history), _ptr(out), self._stream())
        check("drift_gated_delta_rule", status)

    def causal_conv_decode(self, x, weight, dilation: int, states, out) -> None:
        """One token per sequence: x [S, channels], states [S, span, channels]."""
        _f32("causalConv", x, weight, states, out)
        _same_shape("causalConv", x, out)
        sequences, channels = x.shape
        taps = weight.shape[-1]
        span = (taps - 1) * dilation
        _require(tuple(states.shape) == (sequences, span, channels),
                 f"causalConv: states {list(states.shape)}")
        status = self.lib.drift_causal_conv_decode(_ptr(x), sequences, channels, _ptr(weight), taps,
                                                   dilation, _ptr(states), _ptr(out), self._stream())
        check("drift_causal_conv_decode", status)

    def gated_delta_rule_decode(self, qkv, a, b, decay, dt_bias, states, rule, out) -> None:
        """One token per sequence: qkv [S, width], a, b [S, value_heads],
        states [S, value_heads, D, D], out [S, value_heads, D]."""
        key_heads, value_heads, d, tiled = rule
        _f32("gatedDeltaRule", qkv, a, b, decay, dt_bias, states, out)
        sequences = qkv.shape[0]
        _require(tuple(states.shape) == (sequences, value_heads, d, d),
                 f"gatedDeltaRule: states {list(states.shape)}")
        _require(tuple(out.shape) == (sequences, value_heads, d), f"gatedDeltaRule: out {list(out.shape)}")
        status = self.lib.drift_gated_delta_rule_decode(
            _ptr(qkv), sequences, key_heads, value_heads, d, int(tiled), _ptr(a), _ptr(b),
            _ptr(decay), _ptr(dt_bias), _ptr(states), _ptr(out), self._stream())
        check("drift_gated_delta_rule_decode", status)

    def delta_decode_step(self, qkv, z, conv_weight, conv_states, convolved, a, b, decay,
                          dt_bias, states, rule, norm_weight, epsilon: float, out,
                          prepared: Optional[torch.Tensor] = None) -> None:
        """causal_conv_decode (dilation 1), gated_delta_rule_decode and the
        SiLU-gated rms norm of the core by z, in one launch where it can
        (every value head with a key head of its own, heads of 128): out
        [S, value_heads, D]; `convolved` [S, channels] is used only when it
        falls back to the three launches."""
        key_heads, value_heads, d, tiled = rule
        _f32("deltaDecodeStep", qkv, z, conv_weight, conv_states, convolved, a, b, decay,
             dt_bias, states, norm_weight, out)
        sequences, channels = qkv.shape
        _require(channels == (2 * key_heads + value_heads) * d,
                 f"deltaDecodeStep: qkv {list(qkv.shape)}")
        taps = conv_weight.shape[-1]
        _require(tuple(conv_states.shape) == (sequences, taps - 1, channels),
                 f"deltaDecodeStep: conv states {list(conv_states.shape)}")
        _require(tuple(states.shape) == (sequences, value_heads, d, d),
                 f"deltaDecodeStep: states {list(states.shape)}")
        _require(tuple(out.shape) == (sequences, value_heads, d) and z.numel() == out.numel(),
                 f"deltaDecodeStep: out {list(out.shape)}")
        status = self.lib.drift_delta_decode_step(
            _ptr(qkv), _ptr(z), sequences, key_heads, value_heads, d, int(tiled),
            _ptr(conv_weight), taps, _ptr(conv_states), _ptr(convolved), _ptr(a), _ptr(b),
            _ptr(decay), _ptr(dt_bias), _ptr(states), _ptr(norm_weight), epsilon, _ptr(out),
            _ptr(prepared), self._stream())
        check("drift_delta_decode_step", status)

    def gated_rms_norm(self, x, weight, gate, kind: int, epsilon: float, out,
                       prepared: Optional[torch.Tensor] = None, heads: int = 0) -> None:
        """rmsNorm(x) × act(gate) per row (NormalisationOps.gatedRmsNorm); with
        `prepared`, the records of out as [rows / heads, heads × cols]."""
        rows = self._check_row_wise("gatedRmsNorm", x, out, weight)
        _f32("gatedRmsNorm", gate)
        _same_shape("gatedRmsNorm", x, gate)
        status = self.lib.drift_gated_rms_norm(_ptr(x), _ptr(weight), _ptr(gate), kind, epsilon,
                                               _ptr(out), rows, x.shape[-1], heads, _ptr(prepared),
                                               self._stream())
        check("drift_gated_rms_norm", status)

    # -- SequenceOps sampling (ops/SequenceOps.scala:14-20) ------------------------------------------
    def argmax(self, values, ids, out_values=None, id_offset: int = 0) -> None:
        """Each row's argmax (CpuSequence.argmax's order) into ids [rows]
        (int32), plus id_offset; its value into out_values when given."""
        _f32("argmax", values)
        width = values.shape[-1]
        rows = values.numel() // max(width, 1)
        _require(ids.dtype == torch.int32 and ids.numel() == rows, f"argmax: ids {list(ids.shape)}")
        check("drift_argmax", self.lib.drift_argmax(_ptr(values), rows, width, id_offset, _ptr(ids),
                                                    _ptr(out_values), self._stream()))

    def argmax_merge(self, values, ids_in, ids, out_values=None) -> None:
        """The argmax over gathered (value, id) pairs [rows, n]."""
        rows, n = values.shape
        check("drift_argmax_merge", self.lib.drift_argmax_merge(
            _ptr(values), _ptr(ids_in), rows, n, _ptr(ids), _ptr(out_values), self._stream()))

    def candidates(self, values, count: int, ids, out_values=None, id_offset: int = 0) -> None:
        """Each row's `count` largest (Candidates.of's order) into ids / out_values
        [rows, count], plus id_offset (SequenceOps.requireCandidates: 1 to 1024)."""
        _f32("candidates", values)
        _require(1 <= count <= 1024, f"{count} candidates, 1 to 1024")
        width = values.shape[-1]
        rows = values.numel() // max(width, 1)
        check("drift_candidates", self.lib.drift_candidates(
            _ptr(values), rows, width, id_offset, count, _ptr(ids), _ptr(out_values),
            self._stream()))

    def candidates_merge(self, values, ids_in, count: int, ids, out_values=None) -> None:
        """The `count` largest of gathered (value, id) pairs [rows, n]."""
        rows, n = values.shape
        check("drift_candidates_merge", self.lib.drift_candidates_merge(
            _ptr(values), _ptr(ids_in), rows, n, count, _ptr(ids), _ptr(out_values),
            self._stream()))

    # -- ExpertsOps (ops/ExpertsOps.scala) -------------------------------------------------------------
    def route(self, logits, ids, weights) -> None:
        """Top-k routing (ExpertsOps.scala:116-120; checks L252-269)."""
        _f32("route", logits, weights)
        _require(ids.dtype == torch.int32 and tuple(ids.shape) == tuple(weights.shape)
                 and logits.dim() == 2,
                 f"route: {list(logits.shape)}, {list(ids.shape)}, {list(weights.shape)}")
        tokens, experts = logits.shape
        k = weights.shape[-1]
        _require(tuple(weights.shape) == (tokens, k) and k <= 16 and experts <= 512,
                 f"route: top-{k} of {experts}")
        status = self.lib.drift_route(_ptr(logits), _ptr(ids), _ptr(weights), tokens, experts, k,
                                      self._stream())
        check("drift_route", status)

    def route_linear(self, x, router, logits, ids, weights,
                     prepared: Optional[torch.Tensor] = None) -> None:
        """A router's logits = x · routerᵀ, then route (ExpertsOps.scala:176-186);
        `prepared` as for linears."""
        self.linears(x, [router], [logits], prepared)
        self.route(logits, ids, weights)

    @staticmethod
    def _check_experts(x, weight: Stored, ids, out):
        """Ops.checkExperts (ExpertsOps.scala:271-295); returns (slots, N, K, rows)."""
        _x_dtype("expertsLinear", x)
        _f32("expertsLinear", out)
        _require(len(weight.shape) == 3 and ids.dtype == torch.int32,
                 f"expertsLinear: weight {list(weight.shape)}, ids {ids.dtype}")
        _, n, k = weight.shape
        slots = ids.numel()
        rows = x.shape[0]
        _require(x.dim() == 2 and x.shape[1] == k and rows > 0 and slots % rows == 0,
                 f"expertsLinear: x {list(x.shape)} for {slots} slots of {k}")
        _require(tuple(out.shape) == (slots, n),
                 f"expertsLinear: out {list(out.shape)}, expected [{slots}, {n}]")
        return slots, n, k, rows

    def experts_linear(self, x, weight: Stored, ids, out, first_expert: Optional[int] = None,
                       prepared: Optional[torch.Tensor] = None) -> None:
        """Slot s: expert ids[s] of weight [experts, N, K] times x row
        s / (slots / rows of x) (ExpertsOps.scala:122-126). `first_expert`:
        the weight holds the model's experts from there on (expert
        parallelism); other ranks' slots get zeros. `prepared` (with
        `first_expert`): x's records, already written by the kernel that
        made x."""
        slots, n, k, rows = self._check_experts(x, weight, ids, out)
        _require(prepared is None or first_expert is not None,
                 "expertsLinear: a prepared x goes with first_expert")
        if first_expert is None:
            status = self.lib.drift_experts_linear(
                _x_dtype("expertsLinear", x), _ptr(x), rows, weight.dtype, _ptr(weight.data),
                weight.shape[0], n, k, _ptr(ids), slots, _ptr(out), self._stream())
        else:
            status = self.lib.drift_experts_linear_local(
                _x_dtype("expertsLinear", x), _ptr(x), rows, weight.dtype, _ptr(weight.data),
                weight.shape[0], first_expert, n, k, _ptr(ids), slots, _ptr(out),
                _ptr(prepared), self._stream())
        check("drift_experts_linear", status)

    def experts_gated_linear(self, x, gate: Stored, up: Stored, ids, out,
                             first_expert: Optional[int] = None,
                             prepared: Optional[torch.Tensor] = None,
                             shared_tail: bool = False) -> None:
        """silu(gate · x) × (up · x) per slot, one launch (ExpertsOps.scala:188-198);
        `first_expert` and `prepared` as for experts_linear. `shared_tail`
        (with `first_expert`): the last rows-of-x slots are a shared expert's,
        one per row of x, the slots before them routed."""
        _require(tuple(gate.shape) == tuple(up.shape) and gate.dtype == up.dtype,
                 f"expertsGatedLinear needs equal shapes, got {list(gate.shape)}, "
                 f"{list(up.shape)}")
        slots, n, k, rows = self._check_experts(x, gate, ids, out)
        _require((prepared is None and not shared_tail) or first_expert is not None,
                 "expertsGatedLinear: a prepared x or a shared tail goes with first_expert")
        if first_expert is None:
            status = self.lib.drift_experts_gated_linear(
                _x_dtype("expertsGatedLinear", x), _ptr(x), rows, gate.dtype, _ptr(gate.data),
                _ptr(up.data), gate.shape[0], n, k, _ptr(ids), slots, _ptr(out), self._stream())
        else:
            status = self.lib.drift_experts_gated_linear_local(
                _x_dtype("expertsGatedLinear", x), _ptr(x), rows, gate.dtype, _ptr(gate.data),
                _ptr(up.data), gate.shape[0], first_expert, n, k, _ptr(ids), slots, _ptr(out),
                _ptr(prepared), int(shared_tail), self._stream())
        check("drift_experts_gated_linear", status)

    def moe_decode(self, x, x_prepared, router, logits, ids, route_weights, gate: Stored,
                   up: Stored, down: Stored, gated, out, shared_router, residual, norm: RowNorm,
                   prepared: Optional[torch.Tensor] = None) -> None:
        """The mixture of a decode step in one launch (route_linear,
        experts_gated_linear with the shared tail, experts_linear and
        moe_combine_norm): x [b, H] with its records; router F32 [E, H];
        gate/up [E + 1, F, H] and down [E + 1, H, F] with the shared expert
        last; ids [b k + b], route_weights [b, k], gated [b k + b, F], out
        [b k + b, H]; residual updated and norm.out (its records into
        `prepared`) written last."""
        _f32("moe", x, router, logits, route_weights, gated, out, shared_router, residual,
             norm.weight, norm.out)
        tokens, hidden = x.shape
        experts = router.shape[0]
        k = route_weights.shape[-1]
        ffn = gate.shape[1]
        _require(tuple(gate.shape) == (experts + 1, ffn, hidden) and tuple(up.shape) == tuple(gate.shape)
                 and tuple(down.shape) == (experts + 1, hidden, ffn)
                 and gate.dtype == up.dtype == down.dtype,
                 f"moe: weights {list(gate.shape)}, {list(up.shape)}, {list(down.shape)} for "
                 f"{experts} experts and a shared one")
        _require(ids.dtype == torch.int32 and ids.numel() == tokens * k + tokens
                 and tuple(gated.shape) == (tokens * k + tokens, ffn)
                 and tuple(out.shape) == (tokens * k + tokens, hidden)
                 and tuple(logits.shape) == (tokens, experts),
                 "moe: slot buffers")
        status = self.lib.drift_moe_decode(
            gate.dtype, _ptr(x), _ptr(x_prepared), _ptr(router), _ptr(logits), _ptr(ids),
            _ptr(route_weights), _ptr(gate.data), _ptr(up.data), _ptr(down.data), _ptr(gated),
            _ptr(out), _ptr(shared_router), _ptr(residual), _ptr(norm.weight), norm.epsilon,
            norm.weight_offset, _ptr(norm.out), _ptr(prepared), tokens, experts, k, hidden, ffn,
            self._stream())
        check("drift_moe_decode", status)

    @staticmethod
    def _check_combine(expert_out, weights, shared, residual, out):
        _f32("moeCombine", expert_out, weights, out)
        tokens, hidden = out.shape
        _require(weights.numel() % max(1, tokens) == 0, "moeCombine: weights per token")
        k = weights.numel() // max(1, tokens)
        _require(tuple(expert_out.shape) == (tokens * k, hidden),
                 f"moeCombine: expert outputs {list(expert_out.shape)} for [{tokens * k}, "
                 f"{hidden}]")
        if shared is not None:
            _f32("moeCombine", shared.output, shared.input, shared.router)
            _require(tuple(shared.output.shape) == (tokens, hidden)
                     and tuple(shared.input.shape) == (tokens, hidden)
                     and tuple(shared.router.shape) == (hidden,),
                     "moeCombine: shared expert shapes")
        if residual is not None:
            _f32("moeCombine", residual)
            _same_shape("moeCombine", residual, out)
        return tokens, k, hidden

    def moe_combine(self, expert_out, weights, shared: Optional[SharedExpert],
                    residual: Optional[torch.Tensor], out) -> None:
        """out[t] = residual[t] + Σ_j weights[t, j]·expertOut[t·k + j] (+ the
        shared expert by its gate) (ExpertsOps.scala:128-138)."""
        tokens, k, hidden = self._check_combine(expert_out, weights, shared, residual, out)
        status = self.lib.drift_moe_combine(
            _ptr(expert_out), _ptr(weights), tokens, k, hidden,
            _ptr(shared.output) if shared else None, _ptr(shared.input) if shared else None,
            _ptr(shared.router) if shared else None, _ptr(residual), _ptr(out), self._stream())
        check("drift_moe_combine", status)

    def moe_combine_norm(self, expert_out, weights, shared: Optional[SharedExpert], residual,
                         norm: RowNorm, prepared: Optional[torch.Tensor] = None) -> None:
        """moe_combine into the residual, then norm's RMS norm of it into
        norm.out, one launch (ExpertsOps.scala:140-152); with `prepared`,
        norm.out's records too."""
        tokens, k, hidden = self._check_combine(expert_out, weights, shared, residual, residual)
        self._check_row_wise("rmsNorm", residual, norm.out, norm.weight)
        status = self.lib.drift_moe_combine_norm_prepared(
            _ptr(expert_out), _ptr(weights), tokens, k, hidden,
            _ptr(shared.output) if shared else None, _ptr(shared.input) if shared else None,
            _ptr(shared.router) if shared else None, _ptr(residual), _ptr(norm.weight),
            norm.epsilon, norm.weight_offset, _ptr(norm.out), _ptr(prepared), self._stream())
        check("drift_moe_combine_norm", status)
