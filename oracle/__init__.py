"""CPU oracle for the quantized-inference hot path -- TEST INFRASTRUCTURE ONLY.

A ctypes front to ``oracle/liboracle.so``, the plain-C restatement of the drift
runner's CPU reference backend (``CpuOps``) for this path
(runner/src/drift/runner/ops/CpuLinear.scala, CpuNormalisation.scala,
CpuAttention.scala:92-146, CpuExperts.scala; tensor/GgmlQuants.scala).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker. The product path
(``drift_b200``) never imports it and has no CPU fallback.

Parity pin: the decoders reproduce the reference's committed golden quant
fixtures bit for bit (``tests/golden``), and the op functions reproduce the
hand-worked known answers of the reference's own CPU tests.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "liboracle.so")

# GGML type ids (runner/src/drift/runner/tensor/DType.scala:151-175).
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, BF16 = 0, 1, 2, 3, 6, 7, 8, 30
Q4_K, Q6_K = 12, 14  # tensor/KQuants.scala:99, 122
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20),
         Q5_0: (32, 22), Q5_1: (32, 24), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}
NAMES = {F32: "F32", F16: "F16", BF16: "BF16", Q4_0: "Q4_0", Q4_1: "Q4_1",
         Q5_0: "Q5_0", Q5_1: "Q5_1", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}


def build() -> str:
    """Compiles the restatement (oracle/Makefile) if it is missing or stale."""
    source = os.path.join(HERE, "drift_oracle.c")
    if (not os.path.exists(LIBRARY)
            or os.path.getmtime(LIBRARY) < os.path.getmtime(source)):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIBRARY


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIBRARY)
        p, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        sigs = {
            "oracle_f16_to_f32": (f32, [ctypes.c_uint16]),
            "oracle_f32_to_f16": (ctypes.c_uint16, [f32]),
            "oracle_cache_write": (None, [p, p, i32, i32, i32, p, p, i32, p, i32]),
            "oracle_attention": (None, [p, i32, i32, p, p, i32, i32, i32, p, i32, i32, f32, i32, i32,
                                        i32, f32, p, p]),
            "oracle_f32_to_bf16": (ctypes.c_uint16, [f32]),
            "oracle_decode": (i32, [i32, p, i64, p]),
            "oracle_linear": (i32, [i32, p, p, p, i64, i64, i64]),
            "oracle_linear_rows": (i32, [i32, p, p, p, i64, i64, i64, p, i64]),
            "oracle_linear_threads": (i32, [i32, p, p, p, i64, i64, i64, i32]),
            "oracle_max_threads": (i32, []),
            "oracle_embedding": (i64, [i32, p, i64, i64, p, i64, p]),
            "oracle_rms_norm": (None, [p, p, f32, f32, p, i64, i64]),
            "oracle_add_rms_norm": (None, [p, p, p, f32, f32, p, i64, i64]),
            "oracle_gated": (None, [i32, p, p, p, i64]),
            "oracle_activation": (None, [i32, f32, p, p, i64]),
            "oracle_inverse_frequency": (f32, [f32, i32, i32]),
            "oracle_rope": (None, [p, p, p, i32, i32, i32, f32, i32, i32]),
            "oracle_argmax": (ctypes.c_int64, [p, ctypes.c_int64]),
            "oracle_candidates": (i32, [p, ctypes.c_int64, ctypes.c_int64, i32, p, p]),
            "oracle_rope_sections": (None, [p, p, p, i32, i32, i32, f32, i32, i32, i32, i32, i32,
                                            i32, i32]),
            "oracle_route": (None, [p, i32, i32, i32, p, p]),
            "oracle_experts_linear": (i32, [i32, p, i64, p, i64, i64, i64, p, i64, p]),
            "oracle_experts_gated_linear": (i32, [i32, p, i64, p, p, i64, i64, i64, p, i64, p]),
            "oracle_moe_combine": (None, [p, p, i64, i64, i64, p, p, p, p, p]),
            "oracle_moe_combine_norm": (None, [p, p, i64, i64, i64, p, p, p, p, p, f32, f32, p]),
            "oracle_causal_conv": (None, [p, i32, i32, p, i32, i32, p, p, p]),
            "oracle_gated_delta_rule": (None, [p, i32, i32, i32, i32, i32, p, p, p, p, p, p, p]),
            "oracle_gated_rms_norm": (None, [p, p, p, i32, f32, p, i64, i64]),
        }
        for name, (restype, argtypes) in sigs.items():
            fn = getattr(_lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def row_bytes(dtype: int, k: int) -> int:
    per, size = BLOCK[dtype]
    if k % per:
        raise ValueError(f"{k} elements are not whole {NAMES[dtype]} blocks of {per}")
    return k // per * size


def bf16_widen(bits: np.ndarray) -> np.ndarray:
    """BF16 bit patterns as the F32 values they are (tensor/DType.scala:99-102)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(values: np.ndarray) -> np.ndarray:
    """F32 to BF16 bits, to nearest even (ops/CpuOps.scala:53-57)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(values, dtype=np.float32))
    rounded[nan] = ((bits[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def decode(dtype: int, data: np.ndarray, elements: int) -> np.ndarray:
    """DType.decode (tensor/DType.scala:49-63)."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(elements, dtype=np.float32)
    if lib().oracle_decode(dtype, _p(data), elements, _p(out)) != 0:
        raise ValueError(f"{elements} elements are not whole {NAMES[dtype]} blocks")
    return out


def linear(dtype: int, x: np.ndarray, weight: np.ndarray, n: int, k: int) -> np.ndarray:
    """CpuLinear.linear: x [m, k] F32 times weight [n, k] -> [m, n] F32."""
    x = _f32(x).reshape(-1, k)
    weight = np.ascontiguousarray(weight, dtype=np.uint8)
    assert weight.size >= n * row_bytes(dtype, k)
    out = np.empty((x.shape[0], n), dtype=np.float32)
    if lib().oracle_linear(dtype, _p(x), _p(weight), _p(out), x.shape[0], n, k) != 0:
        raise ValueError("oracle linear refused its shapes")
    return out


def linear_rows(dtype: int, x: np.ndarray, weight: np.ndarray, n: int, k: int,
                rows: np.ndarray) -> np.ndarray:
    """The sums of CpuLinear.linear for the listed rows only: [m, len(rows)]."""
    x = _f32(x).reshape(-1, k)
    weight = np.ascontiguousarray(weight, dtype=np.uint8)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    out = np.empty((x.shape[0], rows.size), dtype=np.float32)
    status = lib().oracle_linear_rows(dtype, _p(x), _p(weight), _p(out), x.shape[0], n, k,
                                      _p(rows), rows.size)
    if status != 0:
        raise ValueError("oracle linear_rows refused its arguments")
    return out


def linear_threads(dtype: int, x: np.ndarray, weight: np.ndarray, n: int, k: int,
                   threads: int) -> np.ndarray:
    x = _f32(x).reshape(-1, k)
    weight = np.ascontiguousarray(weight, dtype=np.uint8)
    out = np.empty((x.shape[0], n), dtype=np.float32)
    if lib().oracle_linear_threads(dtype, _p(x), _p(weight), _p(out), x.shape[0], n, k,
                                   threads) != 0:
        raise ValueError("oracle linear refused its shapes")
    return out


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def embedding(dtype: int, table: np.ndarray, vocab: int, cols: int,
              ids: np.ndarray) -> np.ndarray:
    """CpuLinear.embedding; an id outside the table raises as `require` does."""
    table = np.ascontiguousarray(table, dtype=np.uint8)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty((ids.size, cols), dtype=np.float32)
    status = lib().oracle_embedding(dtype, _p(table), vocab, cols, _p(ids), ids.size, _p(out))
    if status != 0:
        t = -status - 1
        raise ValueError(f"token id {int(ids[t])} outside the table")
    return out


def rms_norm(x, weight, epsilon: float, weight_offset: float = 0.0) -> np.ndarray:
    x = _f32(x)
    cols = x.shape[-1]
    out = np.empty_like(x)
    lib().oracle_rms_norm(_p(x), _p(_f32(weight)), epsilon, weight_offset, _p(out),
                          x.size // cols, cols)
    return out


def add_rms_norm(x, y, weight, epsilon: float, weight_offset: float = 0.0):
    """Returns (x + y, its RMS norm), as addRmsNorm leaves them."""
    x = _f32(x).copy()
    cols = x.shape[-1]
    out = np.empty_like(x)
    lib().oracle_add_rms_norm(_p(x), _p(_f32(y)), _p(_f32(weight)), epsilon, weight_offset,
                              _p(out), x.size // cols, cols)
    return x, out


def gated(kind: int, gate, up) -> np.ndarray:
    gate, up = _f32(gate), _f32(up)
    out = np.empty_like(gate)
    lib().oracle_gated(kind, _p(gate), _p(up), _p(out), gate.size)
    return out


def activation(kind: int, x, scale: float = 1.0) -> np.ndarray:
    x = _f32(x)
    out = np.empty_like(x)
    lib().oracle_activation(kind, scale, _p(x), _p(out), x.size)
    return out


def inverse_frequency(theta: float, pair: int, rotary: int) -> float:
    return float(lib().oracle_inverse_frequency(theta, pair, rotary))


def rope(x, positions, theta: float, rotary: int, layout: int) -> np.ndarray:
    """CpuAttention.rope, Single sections; x [tokens, heads, D]."""
    x = _f32(x)
    tokens, heads, dim = x.shape
    positions = np.ascontiguousarray(positions, dtype=np.int32)
    out = np.empty_like(x)
    lib().oracle_rope(_p(x), _p(positions), _p(out), tokens, heads, dim, theta, rotary, layout)
    return out


def rope_sections(x, positions, theta: float, rotary: int, layout: int, sections: int,
                  sizes=(0, 0, 0, 0)) -> np.ndarray:
    """CpuAttention.rope with mRoPE sections (codes of RopeSections); x
    [tokens, heads, D], positions [positions per token, tokens]."""
    x = _f32(x)
    tokens, heads, dim = x.shape
    positions = np.ascontiguousarray(positions, dtype=np.int32)
    out = np.empty_like(x)
    s0, s1, s2, s3 = (list(sizes) + [0, 0, 0, 0])[:4]
    lib().oracle_rope_sections(_p(x), _p(positions), _p(out), tokens, heads, dim, theta, rotary,
                               layout, sections, s0, s1, s2, s3)
    return out


def argmax(values) -> int:
    """CpuSequence.argmax over all the values: the first index of the largest
    by `>` from index 0 (a NaN never wins unless at index 0)."""
    values = _f32(values).reshape(-1)
    return int(lib().oracle_argmax(_p(values), values.size))


def candidates(values, count: int):
    """Candidates.of: each row's `count` largest (ids, values), largest first,
    the lower index first among equals (-0 ranks as 0; NaN above +inf)."""
    values = _f32(values)
    width = values.shape[-1]
    rows = values.size // width
    kept = min(count, width)
    ids = np.empty((rows, kept), np.int32)
    out = np.empty((rows, kept), np.float32)
    if lib().oracle_candidates(_p(values), rows, width, count, _p(ids), _p(out)) != 0:
        raise ValueError("oracle candidates refused its arguments")
    return ids, out


def route(logits, k: int):
    logits = _f32(logits)
    tokens, experts = logits.shape
    ids = np.empty((tokens, k), dtype=np.int32)
    weights = np.empty((tokens, k), dtype=np.float32)
    lib().oracle_route(_p(logits), tokens, experts, k, _p(ids), _p(weights))
    return ids, weights


def experts_linear(dtype: int, x, weight, experts: int, n: int, k: int, ids) -> np.ndarray:
    x = _f32(x).reshape(-1, k)
    weight = np.ascontiguousarray(weight, dtype=np.uint8)
    ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
    out = np.empty((ids.size, n), dtype=np.float32)
    if lib().oracle_experts_linear(dtype, _p(x), x.shape[0], _p(weight), experts, n, k, _p(ids),
                                   ids.size, _p(out)) != 0:
        raise ValueError("oracle experts_linear refused its arguments")
    return out


def experts_gated_linear(dtype: int, x, gate, up, experts: int, n: int, k: int, ids):
    x = _f32(x).reshape(-1, k)
    gate = np.ascontiguousarray(gate, dtype=np.uint8)
    up = np.ascontiguousarray(up, dtype=np.uint8)
    ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
    out = np.empty((ids.size, n), dtype=np.float32)
    if lib().oracle_experts_gated_linear(dtype, _p(x), x.shape[0], _p(gate), _p(up), experts, n,
                                         k, _p(ids), ids.size, _p(out)) != 0:
        raise ValueError("oracle experts_gated_linear refused its arguments")
    return out


def moe_combine(expert_out, weights, hidden: int, shared_out=None, shared_input=None,
                shared_router=None, residual=None) -> np.ndarray:
    weights = _f32(weights)
    tokens, k = weights.shape
    expert_out = _f32(expert_out)
    out = np.empty((tokens, hidden), dtype=np.float32)
    conv = lambda a: None if a is None else _f32(a)
    so, si, sr, res = conv(shared_out), conv(shared_input), conv(shared_router), conv(residual)
    lib().oracle_moe_combine(_p(expert_out), _p(weights), tokens, k, hidden, _p(so), _p(si),
                             _p(sr), _p(res), _p(out))
    return out


def moe_combine_norm(expert_out, weights, hidden: int, residual, norm_weight, epsilon: float,
                     weight_offset: float = 0.0, shared_out=None, shared_input=None,
                     shared_router=None):
    """Returns (the updated residual, its norm)."""
    weights = _f32(weights)
    tokens, k = weights.shape
    residual = _f32(residual).copy()
    normed = np.empty_like(residual)
    conv = lambda a: None if a is None else _f32(a)
    so, si, sr = conv(shared_out), conv(shared_input), conv(shared_router)
    lib().oracle_moe_combine_norm(_p(_f32(expert_out)), _p(weights), tokens, k, hidden, _p(so),
                                  _p(si), _p(sr), _p(residual), _p(_f32(norm_weight)), epsilon,
                                  weight_offset, _p(normed))
    return residual, normed


def f32_to_f16(values) -> np.ndarray:
    """Float.floatToFloat16 (round to nearest even) of each value, as bits."""
    flat = _f32(values).reshape(-1)
    out = np.empty(flat.size, dtype=np.uint16)
    fn = lib().oracle_f32_to_f16
    for i, v in enumerate(flat):
        out[i] = fn(float(v))
    return out.reshape(np.shape(values))


def cache_write(k, v, keys: np.ndarray, values: np.ndarray, page_size: int, page_table,
                start: int) -> None:
    """CpuAttention.cacheWrite: k, v [tokens, kvHeads, D] into the F16 cache
    (uint16 bits; keys [pages, page, kvHeads, D], values [pages, kvHeads, D,
    page]) in place."""
    k, v = _f32(k), _f32(v)
    tokens, kv_heads, dim = k.shape
    table = np.ascontiguousarray(page_table, dtype=np.int32)
    assert keys.dtype == np.uint16 and values.dtype == np.uint16
    assert keys.flags.c_contiguous and values.flags.c_contiguous
    lib().oracle_cache_write(_p(k), _p(v), tokens, kv_heads, dim, _p(keys), _p(values), page_size,
                             _p(table), start)


def attention(q, keys: np.ndarray, values: np.ndarray, page_size: int, kv_heads: int,
              page_table, query_start: int, key_count: int, scale: float, causal: bool = True,
              window: int = 0, softcap: float | None = None, sinks=None) -> np.ndarray:
    """CpuAttention.attention: q [tokens, qHeads, D] F32 over the F16 cache."""
    q = _f32(q)
    tokens, q_heads, dim = q.shape
    table = np.ascontiguousarray(page_table, dtype=np.int32)
    keys = np.ascontiguousarray(keys, dtype=np.uint16)
    values = np.ascontiguousarray(values, dtype=np.uint16)
    sinks_arr = None if sinks is None else _f32(sinks)
    out = np.empty_like(q)
    lib().oracle_attention(_p(q), tokens, q_heads, _p(keys), _p(values), page_size, kv_heads, dim,
                           _p(table), query_start, key_count, scale, int(causal), window,
                           int(softcap is not None), float(softcap or 0.0), _p(sinks_arr), _p(out))
    return out


# ---- Gated DeltaNet (ops/CpuSequence.scala:29-158) ---------------------------------------


def causal_conv(x, weight, state, dilation: int = 1, keep_history: bool = False):
    """CpuSequence.causalConv (SiLU included): x [tokens, channels], weight
    [channels, taps], state [span, channels] (updated in place). Returns out
    (and the history [tokens, span, channels] with keep_history)."""
    x, weight = _f32(x), _f32(weight)
    assert state.dtype == np.float32 and state.flags.c_contiguous
    tokens, channels = x.shape
    taps = weight.shape[1]
    span = (taps - 1) * dilation
    out = np.empty_like(x)
    history = np.empty((tokens, span, channels), np.float32) if keep_history else None
    lib().oracle_causal_conv(_p(x), tokens, channels, _p(weight), taps, dilation, _p(state),
                             _p(history), _p(out))
    return (out, history) if keep_history else out


def gated_delta_rule(qkv, a, b, decay, dt_bias, state, key_heads: int, value_heads: int,
                     tiled: bool = False, keep_history: bool = False):
    """CpuSequence.gatedDeltaRule: qkv [tokens, (2 key_heads + value_heads) D],
    a, b [tokens, value_heads], decay, dt_bias [value_heads], state
    [value_heads, D, D] (updated in place). Returns out [tokens, value_heads,
    D] (and the history [tokens, value_heads, D, D] with keep_history)."""
    qkv = _f32(qkv)
    tokens = qkv.shape[0]
    d = state.shape[-1]
    assert state.dtype == np.float32 and state.flags.c_contiguous
    assert qkv.shape[1] == (2 * key_heads + value_heads) * d
    out = np.empty((tokens, value_heads, d), np.float32)
    history = np.empty((tokens, value_heads, d, d), np.float32) if keep_history else None
    lib().oracle_gated_delta_rule(_p(qkv), tokens, key_heads, value_heads, d, int(tiled),
                                  _p(_f32(a)), _p(_f32(b)), _p(_f32(decay)), _p(_f32(dt_bias)),
                                  _p(state), _p(history), _p(out))
    return (out, history) if keep_history else out


def gated_rms_norm(x, weight, gate, kind: int, epsilon: float) -> np.ndarray:
    """CpuNormalisation.gatedRmsNorm: rmsNorm(x) * act(gate) per row."""
    x, gate = _f32(x), _f32(gate)
    cols = x.shape[-1]
    out = np.empty_like(x)
    lib().oracle_gated_rms_norm(_p(x), _p(_f32(weight)), _p(gate), kind, epsilon, _p(out),
                                x.size // cols, cols)
    return out

