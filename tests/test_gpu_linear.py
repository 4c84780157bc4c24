"""Quantized products on the GPU against the CPU oracle (the reference's
LinearTests, runner/gpuTest/src/drift/runner/LinearTests.scala, on this path).

Every case is held to the benchmark's bar: |gpu - oracle| <= 1e-4 + 1e-3
|oracle| (the oracle restates CpuLinear.linear: Double sums in column order).
On top of it:
- up to 31 rows of x (the reference's matrix-vector path, float x), the
  rigorous bound of the x preparation: x enters as exact integers 21 bits
  below each 32-value block's largest |x| (drift_b200/csrc/quant.cuh), so an
  output can move by at most sum_k |w_k| * max|x_block| * 2^-21, plus float
  rounding of the sums, 1e-5 of the output scale (the reference's own
  float-x tolerance, LinearTests.scala:154-157);
- from 32 rows on (the reference's GEMM path, ops/HipLinear.scala:389-469,
  here on the tcgen05 tensor cores with exact two-term F16 operands), also
  the reference's own bound for its F16 GEMM (LinearTests.scala:139-147):
  |gpu - oracle| <= (2 sum|w x| + |y|) 2^-11 1.01, which the benchmark's bar
  is far inside.
"""

import numpy as np
import pytest
import torch

import oracle
from drift_b200 import synthetic
from drift_b200.ops import CudaOps, Stored
from tests.conftest import within

pytestmark = pytest.mark.gpu

TYPES = [oracle.Q8_0, oracle.Q4_0, oracle.Q4_1]

# (M, N, K) as LinearTests.cases (L33-58): one row, odd row counts, rows
# shorter than a chunk, a model's width, several vectors, past 8 vectors.
CASES = [(1, 1, 64), (1, 7, 512), (1, 33, 640), (1, 64, 2560), (2, 9, 4096), (3, 20, 1024),
         (8, 16, 2560), (9, 24, 512), (40, 72, 2560), (1, 1030, 1024), (64, 130, 4096),
         (16, 300, 4096), (31, 70, 2048)]


@pytest.fixture(scope="module")
def ops():
    return CudaOps()


def bound(decoded: np.ndarray, x: np.ndarray) -> np.ndarray:
    """sum_k |w_k| * max|x_block(k)| * 2^-21 per output [m, n]."""
    m, k = x.shape
    block_max = np.abs(x.reshape(m, k // 32, 32)).max(axis=2)  # [m, k/32]
    per_block = np.abs(decoded.reshape(decoded.shape[0], k // 32, 32)).sum(axis=2)  # [n, k/32]
    return (block_max.astype(np.float64) @ per_block.T.astype(np.float64)) * 2.0 ** -21


def gemm_bound(decoded: np.ndarray, x: np.ndarray, expected: np.ndarray) -> np.ndarray:
    """(2 sum_k |w_k x_k| + |y|) 2^-11 1.01 per output [m, n]."""
    sums = np.abs(x.astype(np.float64)) @ np.abs(decoded.astype(np.float64)).T
    return (2 * sums + np.abs(expected)) * 2.0 ** -11 * 1.01


def run_case(ops, dtype, m, n, k, seed, x_bf16: bool, law: str):
    rng = np.random.default_rng(seed)
    if law == "tests":
        w = synthetic.random_blocks(rng, dtype, n, k)
    else:
        w = synthetic.quantized(rng, dtype, n, k)
    x32 = synthetic.gaussian(rng, m, k)
    if x_bf16:
        bits = synthetic.bf16_bits(x32)
        x_eff = synthetic.bf16_values(bits)
        x_dev = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    else:
        x_eff = x32
        x_dev = torch.from_numpy(x32).cuda()
    weight = Stored.upload(dtype, (n, k), w)
    out = torch.full((m, n), float("nan"), device="cuda")
    ops.linear(x_dev, weight, out)
    torch.cuda.synchronize()
    actual = out.cpu().numpy()
    expected = oracle.linear(dtype, x_eff, w, n, k)
    decoded = oracle.decode(dtype, w, n * k).reshape(n, k)
    return actual, expected, bound(decoded, x_eff)


@pytest.mark.parametrize("dtype", TYPES, ids=lambda t: oracle.NAMES[t])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c)))
@pytest.mark.parametrize("x_bf16", [False, True], ids=["x_f32", "x_bf16"])
def test_linear_matches_oracle(ops, dtype, case, x_bf16):
    m, n, k = case
    for law in ("tests", "bench"):
        actual, expected, limit = run_case(ops, dtype, m, n, k, seed=hash(case) % 1000,
                                           x_bf16=x_bf16, law=law)
        ok, _, _, summary = within(actual, expected, 1e-4, 1e-3)
        assert ok, f"{law} weights: {summary}"
        if m >= 32:
            rng = np.random.default_rng(hash(case) % 1000)
            w = (synthetic.random_blocks if law == "tests" else synthetic.quantized)(
                rng, dtype, n, k)
            x32 = synthetic.gaussian(rng, m, k)
            x_eff = synthetic.bf16_values(synthetic.bf16_bits(x32)) if x_bf16 else x32
            decoded = oracle.decode(dtype, w, n * k).reshape(n, k)
            err = np.abs(actual.astype(np.float64) - expected)
            bound = gemm_bound(decoded, x_eff, expected)
            assert (err <= bound).all(), \
                f"{law} weights: worst at {(err / bound).max():.2f} of the GEMM bound"
            continue
        scale = np.abs(expected).max()
        err = np.abs(actual.astype(np.float64) - expected)
        assert (err <= limit + 1e-5 * scale).all(), \
            f"{law} weights: worst at {(err / (limit + 1e-5 * scale)).max():.2f} of the bound"


@pytest.mark.parametrize("dtype", TYPES, ids=lambda t: oracle.NAMES[t])
def test_linears_share_one_preparation(ops, dtype):
    """linears (Q, K, V) equals separate linears, bit for bit."""
    rng = np.random.default_rng(11)
    k = 2048
    shapes = [512, 128, 128]
    ws = [synthetic.quantized(rng, dtype, n, k) for n in shapes]
    x = torch.from_numpy(synthetic.gaussian(rng, 3, k)).cuda()
    weights = [Stored.upload(dtype, (n, k), w) for n, w in zip(shapes, ws)]
    together = [torch.empty(3, n, device="cuda") for n in shapes]
    ops.linears(x, weights, together)
    for w, t in zip(weights, together):
        alone = torch.empty_like(t)
        ops.linear(x, w, alone)
        assert torch.equal(alone, t)


@pytest.mark.parametrize("m", [1, 2, 5])
def test_mixed_linears_share_launches(ops, m):
    """A list of two Q4_1, two F32 and one Q8_0 products of one x (a DeltaNet
    layer's qkv, z, a, b, plus another type): the Q4_1 pair shares a launch,
    the F32 pair another, and every output is bit for bit its product alone."""
    rng = np.random.default_rng(13 + m)
    k = 2048
    ws = [Stored.upload(oracle.Q4_1, (384, k), synthetic.quantized(rng, oracle.Q4_1, 384, k)),
          Stored.upload(oracle.Q4_1, (128, k), synthetic.quantized(rng, oracle.Q4_1, 128, k)),
          torch.from_numpy((0.02 * rng.standard_normal((16, k))).astype(np.float32)).cuda(),
          torch.from_numpy((0.02 * rng.standard_normal((16, k))).astype(np.float32)).cuda(),
          Stored.upload(oracle.Q8_0, (96, k), synthetic.quantized(rng, oracle.Q8_0, 96, k))]
    x = torch.from_numpy(synthetic.gaussian(rng, m, k)).cuda()
    together = [torch.empty(m, w.shape[0], device="cuda") for w in ws]
    ops.linears(x, ws, together)
    for w, t in zip(ws, together):
        alone = torch.empty_like(t)
        ops.linear(x, w, alone)
        assert torch.equal(alone, t)


def test_pipelined_host_copies(ops):
    """A host's pipeline through the C ABI: x copied in on one stream, the
    product on a second, y copied out on a third, ordered per buffer by
    events (drift_stream_wait_event), two steps in a row with new x each step
    and the same buffers: every host y is bit for bit the product of its step's
    x."""
    import ctypes
    lib = ops.lib
    rng = np.random.default_rng(14)
    k = 4096
    cases = [(1, 512), (8, 1024), (3, 256)]
    weights = {n: Stored.upload(oracle.Q4_1, (n, k), synthetic.quantized(rng, oracle.Q4_1, n, k))
               for _, n in cases}
    host_x = {c: torch.empty(c[0], k, dtype=torch.float32).pin_memory() for c in cases}
    host_y = {c: torch.empty(c[0], c[1], dtype=torch.float32).pin_memory() for c in cases}
    dev_x = {c: torch.empty(c[0], k, device="cuda") for c in cases}
    dev_y = {c: torch.empty(c[0], c[1], device="cuda") for c in cases}

    def created(call):
        handle = ctypes.c_void_p()
        assert call(ctypes.byref(handle)) == 0
        return handle

    streams = [created(lib.drift_stream_create) for _ in range(3)]
    s_in, s_run, s_out = streams
    events = {c: [created(lib.drift_event_create) for _ in range(3)] for c in cases}
    torch.cuda.synchronize()
    for step in range(2):
        xs = {c: synthetic.gaussian(rng, c[0], k) for c in cases}
        for c in cases:
            host_x[c].copy_(torch.from_numpy(xs[c]))
        for c in cases:
            m, n = c
            copied_in, computed, copied_out = events[c]
            assert lib.drift_stream_wait_event(s_in, computed) == 0
            assert lib.drift_memcpy_async(ctypes.c_void_p(dev_x[c].data_ptr()),
                                          ctypes.c_void_p(host_x[c].data_ptr()), m * k * 4, 1,
                                          s_in) == 0
            assert lib.drift_event_record(copied_in, s_in) == 0
            assert lib.drift_stream_wait_event(s_run, copied_in) == 0
            assert lib.drift_stream_wait_event(s_run, copied_out) == 0
            assert lib.drift_linear(0, ctypes.c_void_p(dev_x[c].data_ptr()), oracle.Q4_1,
                                    ctypes.c_void_p(weights[n].data.data_ptr()),
                                    ctypes.c_void_p(dev_y[c].data_ptr()), m, n, k, s_run) == 0
            assert lib.drift_event_record(computed, s_run) == 0
            assert lib.drift_stream_wait_event(s_out, computed) == 0
            assert lib.drift_memcpy_async(ctypes.c_void_p(host_y[c].data_ptr()),
                                          ctypes.c_void_p(dev_y[c].data_ptr()), m * n * 4, 2,
                                          s_out) == 0
            assert lib.drift_event_record(copied_out, s_out) == 0
        assert lib.drift_device_synchronize() == 0
        for c in cases:
            expected = torch.empty(c[0], c[1], device="cuda")
            ops.linear(torch.from_numpy(xs[c]).cuda(), weights[c[1]], expected)
            torch.cuda.synchronize()
            assert torch.equal(host_y[c], expected.cpu()), (step, c)
    for c in cases:
        for e in events[c]:
            assert lib.drift_event_destroy(e) == 0
    for handle in streams:
        assert lib.drift_stream_destroy(handle) == 0


@pytest.mark.parametrize("m", [8, 16])
def test_linear_rows_do_not_depend_on_batch(ops, m):
    """A row's sum is the same whether it comes alone or with 7 (or 15) others."""
    rng = np.random.default_rng(12)
    n, k = 300, 4096
    w = Stored.upload(oracle.Q4_1, (n, k), synthetic.quantized(rng, oracle.Q4_1, n, k))
    x = torch.from_numpy(synthetic.gaussian(rng, m, k)).cuda()
    batch = torch.empty(m, n, device="cuda")
    ops.linear(x, w, batch)
    for i in range(m):
        one = torch.empty(1, n, device="cuda")
        ops.linear(x[i:i + 1].contiguous(), w, one)
        assert torch.equal(one[0], batch[i])


# 9-16 vectors stream the weights once (the MMA16 mode): every schedule --
# the tile schedule with and without leftover tiles, the balanced one for
# long rows, and two 8-vector passes where the leftover sums would not fit
# (20000 x 8192) -- against passes of at most 8 vectors, bit for bit.
SIXTEEN_SHAPES = [(300, 4096), (20000, 4096), (4096, 12288), (20000, 8192)]


@pytest.mark.parametrize("dtype", TYPES, ids=lambda t: oracle.NAMES[t])
@pytest.mark.parametrize("shape", SIXTEEN_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_sixteen_vectors_are_two_passes(ops, dtype, shape):
    n, k = shape
    rng = np.random.default_rng(n + k + dtype)
    w = Stored.upload(dtype, (n, k), synthetic.quantized(rng, dtype, n, k))
    x = torch.from_numpy(synthetic.gaussian(rng, 31, k)).cuda()
    for m in (9, 16, 31):
        together = torch.empty(m, n, device="cuda")
        ops.linear(x[:m].contiguous(), w, together)
        for first in range(0, m, 8):
            count = min(8, m - first)
            part = torch.empty(count, n, device="cuda")
            ops.linear(x[first:first + count].contiguous(), w, part)
            assert torch.equal(part, together[first:first + count]), (m, first)


def test_sixteen_vectors_share_a_launch(ops):
    """Two Q4_1 products of 16 vectors in one balanced launch: each equals its
    8-vector passes alone."""
    rng = np.random.default_rng(15)
    k = 4096
    ws = [Stored.upload(oracle.Q4_1, (n, k), synthetic.quantized(rng, oracle.Q4_1, n, k))
          for n in (1024, 512)]
    x = torch.from_numpy(synthetic.gaussian(rng, 16, k)).cuda()
    together = [torch.empty(16, w.shape[0], device="cuda") for w in ws]
    ops.linears(x, ws, together)
    for w, t in zip(ws, together):
        for first in (0, 8):
            part = torch.empty(8, w.shape[0], device="cuda")
            ops.linear(x[first:first + 8].contiguous(), w, part)
            assert torch.equal(part, t[first:first + 8])


# The benchmark config C2 shapes at full size: sampled rows against the oracle,
# at the benchmark's bar for every batch; from 32 rows (the tensor-core path)
# for all three storage types, and the worst error is printed.
FULL = [(4096, 4096), (12288, 4096), (4096, 12288), (151936, 4096)]
FULL_CASES = ([(oracle.Q4_1, m) for m in (1, 8)]
              + [(t, m) for t in TYPES for m in (32, 64)])


@pytest.mark.parametrize("shape", FULL, ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("case", FULL_CASES, ids=lambda c: f"{oracle.NAMES[c[0]]}-m{c[1]}")
def test_full_size_sampled_rows(ops, shape, case):
    dtype, m = case
    n, k = shape
    rng = np.random.default_rng(n + k + m + dtype)
    generator = torch.Generator(device="cuda")
    generator.manual_seed(n + k + m + dtype)
    stored = synthetic.quantized_device(dtype, n, k, generator=generator)
    w = stored.cpu().numpy()
    bits = synthetic.bf16_bits(synthetic.gaussian(rng, m, k))
    x_eff = synthetic.bf16_values(bits)
    weight = Stored(dtype, (n, k), stored)
    out = torch.empty((m, n), device="cuda")
    ops.linear(torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16), weight, out)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, 200)]))
    expected = oracle.linear_rows(dtype, x_eff, w, n, k, rows)
    actual = out.cpu().numpy()[:, rows]
    ok, _, worst, summary = within(actual, expected, 1e-4, 1e-3)
    print(f"{oracle.NAMES[dtype]} [{m}, {k}] x [{n}, {k}]: max |gpu - oracle| {worst:.3g}")
    assert ok, summary
    if m >= 32:
        size = oracle.row_bytes(dtype, k)
        decoded = np.stack([oracle.decode(dtype, w[r * size:(r + 1) * size], k) for r in rows])
        err = np.abs(actual.astype(np.float64) - expected)
        bound = gemm_bound(decoded, x_eff, expected)
        assert (err <= bound).all(), f"worst at {(err / bound).max():.2f} of the GEMM bound"
    assert torch.isfinite(out).all()


def test_f32_router_weights(ops):
    """F32 weights (the MoE router, ops/ExpertTensors.scala:15) against the oracle."""
    rng = np.random.default_rng(13)
    n, k = 512, 2048
    w = synthetic.gaussian(rng, n, k) * 0.05
    x = synthetic.gaussian(rng, 4, k)
    out = torch.empty(4, n, device="cuda")
    ops.linear(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), out)
    expected = oracle.linear(oracle.F32, x, w.view(np.uint8), n, k)
    ok, _, _, summary = within(out.cpu().numpy(), expected, 1e-4, 1e-3)
    assert ok, summary


def test_linear_refuses_like_the_reference(ops):
    x = torch.zeros(1, 96, device="cuda")
    w = Stored.upload(oracle.Q8_0, (1, 96), np.zeros(102, np.uint8))
    with pytest.raises(ValueError, match="are not whole words"):
        ops.linear(x, w, torch.empty(1, 1, device="cuda"))
    with pytest.raises(ValueError, match="x rows of 64 against weight rows of 96"):
        ops.linear(torch.zeros(1, 64, device="cuda"), w, torch.empty(1, 1, device="cuda"))
