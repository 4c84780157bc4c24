"""The runner's kernels launched by name, as HipOps launches them: each kernel
is looked up with drift_module_get_function(&f, NULL, name) and launched with
drift_module_launch_kernel on exactly the argument list and the grid and block
the reference's dispatch builds (runner/src/drift/runner/ops/HipLinear.scala:
21-52, 187-273, 337-346; HipNormalisation.scala:25-50, 96-115, 266-281;
HipAttention.scala:81-103; HipExperts.scala:18-31, 254-273, 452-475;
HipSequence.scala:100-118), then compared with the CPU oracle: gathers bit
for bit, the rest at the benchmark's 1e-4 + 1e-3 |e| (rope within 1e-6).
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from drift_b200 import _lib, synthetic
from drift_b200.ops import CudaOps
from tests.conftest import within

pytestmark = pytest.mark.gpu

TYPES = {"q8_0": oracle.Q8_0, "q4_0": oracle.Q4_0, "q4_1": oracle.Q4_1}


@pytest.fixture(scope="module")
def lib():
    CudaOps()  # the library loaded and a context on cuda:0
    return _lib.load()


# device tensors made for a launch's arguments, kept alive until it is done
# (a pointer argument alone does not hold its tensor)
ALIVE = []


def P(t):  # a device pointer argument (NULL for None)
    if t is not None:
        ALIVE.append(t)
    return ctypes.c_void_p(None if t is None else t.data_ptr())


I32, I64, F32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float


def launch(lib, name, grid, block, *args):
    """drift_module_get_function + drift_module_launch_kernel with the
    argument slots HipRuntime.launch packs (one pointer per argument)."""
    function = ctypes.c_void_p()
    _lib.check("drift_module_get_function",
               lib.drift_module_get_function(ctypes.byref(function), None, name.encode()))
    slots = (ctypes.c_void_p * len(args))(*[ctypes.cast(ctypes.pointer(a), ctypes.c_void_p)
                                            for a in args])
    gx, gy = (grid, 1) if isinstance(grid, int) else grid
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(name, lib.drift_module_launch_kernel(function, gx, gy, 1, block, 1, 1, 0, stream,
                                                    slots, None))
    torch.cuda.synchronize()
    ALIVE.clear()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def good(actual, expected, absolute=1e-4, relative=1e-3):
    ok, _, _, summary = within(actual, expected, absolute, relative)
    assert ok, summary


@pytest.mark.parametrize("name", TYPES)
def test_gather(lib, name):
    dtype = TYPES[name]
    rng = np.random.default_rng(1)
    vocab, cols, count = 1000, 4096, 13
    table = synthetic.quantized(rng, dtype, vocab, cols)
    ids = rng.integers(0, vocab, count).astype(np.int32)
    out = torch.full((count, cols), float("nan"), device="cuda")
    launch(lib, f"gather_{name}", (count + 7) // 8, 256, P(dev(table)), P(dev(ids)), P(out),
           I32(count), I32(cols))
    assert np.array_equal(out.cpu().numpy(), oracle.embedding(dtype, table, vocab, cols, ids))


def test_gather_rows_f32(lib):
    rng = np.random.default_rng(2)
    table = rng.standard_normal((50, 37)).astype(np.float32)
    ids = rng.integers(0, 50, 9).astype(np.int32)
    out = torch.empty(9, 37, device="cuda")
    launch(lib, "gather_rows_f32", (9 * 37 + 255) // 256, 256, P(dev(table)), P(dev(ids)),
           P(out), I32(9), I32(37))
    assert np.array_equal(out.cpu().numpy(), table[ids])


def int8_format(values):
    """The runner's int8 x (kernels/quantize.h:6-25) of the values a kernel
    wrote: per 32, xd = max|x| / 127, xq = round half away (x / xd), xs = xd sum."""
    blocks = values.reshape(-1, 32).astype(np.float32)
    d = (np.abs(blocks).max(axis=1) / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = (blocks / d[:, None]).astype(np.float32)
    q = np.where(d[:, None] == 0, 0, np.sign(r) * np.floor(np.abs(r) + 0.5)).astype(np.int32)
    return q.astype(np.int8).reshape(-1), d, (d * q.sum(axis=1).astype(np.float32))


@pytest.mark.parametrize("rows,cols,added", [(3, 4096, False), (5, 4096, True), (2, 768, True)])
def test_rms_norm_f32(lib, rows, cols, added):
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    y = rng.standard_normal((rows, cols)).astype(np.float32)
    weight = (1 + 0.02 * rng.standard_normal(cols)).astype(np.float32)
    x_dev, out = dev(x), torch.empty(rows, cols, device="cuda")
    xq = torch.zeros(rows * cols, dtype=torch.int8, device="cuda")
    xd = torch.zeros(rows * cols // 32, device="cuda")
    xs = torch.zeros(rows * cols // 32, device="cuda")
    launch(lib, "rms_norm_f32", rows, 1024 if cols >= 1024 else 256, P(x_dev),
           P(dev(y) if added else None), P(dev(weight)), P(out), I32(cols), F32(1e-6),
           F32(0.0), I32(1), P(xq), P(xd), P(xs))
    if added:
        summed, expected = oracle.add_rms_norm(x, y, weight, 1e-6)
        assert np.array_equal(x_dev.cpu().numpy(), summed)
    else:
        expected = oracle.rms_norm(x, weight, 1e-6)
    got = out.cpu().numpy()
    good(got, expected)
    q, d, s = int8_format(got)
    assert np.array_equal(xq.cpu().numpy(), q)
    assert np.array_equal(xd.cpu().numpy(), d)
    good(xs.cpu().numpy(), s, 1e-6, 1e-6)


@pytest.mark.parametrize("kind", [0, 1, 2, 3, 4])
def test_gated_f32(lib, kind):
    rng = np.random.default_rng(10 + kind)
    n = 3 * 12288
    gate = rng.standard_normal(n).astype(np.float32)
    up = rng.standard_normal(n).astype(np.float32)
    out = torch.empty(n, device="cuda")
    null = ctypes.c_void_p(None)
    launch(lib, "gated_f32", min((n + 255) // 256, 1 << 20), 256, P(dev(gate)), P(dev(up)),
           P(out), I64(n), I32(kind), null, null, null)
    good(out.cpu().numpy(), oracle.gated(kind, gate, up))


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("sections,sizes,per_token",
                         [(0, (0, 0, 0, 0), 1), (1, (16, 24, 24, 0), 3),
                          (2, (24, 20, 20, 0), 3), (3, (16, 16, 24, 8), 4)])
def test_rope_f32(lib, layout, sections, sizes, per_token):
    rng = np.random.default_rng(20 + sections)
    tokens, heads, dim = 5, 8, 128
    x = rng.standard_normal((tokens, heads, dim)).astype(np.float32)
    positions = rng.integers(0, 8192, (per_token, tokens)).astype(np.int32)
    out = torch.empty(tokens, heads, dim, device="cuda")
    count = tokens * heads * dim
    launch(lib, "rope_f32", (count + 255) // 256, 256, P(dev(x)), P(dev(positions)), P(out),
           I32(tokens), I32(heads), I32(dim), I32(dim), F32(1e6), I32(layout), I32(sections),
           *[I32(s) for s in sizes])
    expected = oracle.rope_sections(x, positions, 1e6, dim, layout, sections, sizes)
    good(out.cpu().numpy(), expected, 1e-6, 1e-6)


def product_inputs(rng, dtype, n, k, m):
    w = synthetic.quantized(rng, dtype, n, k)
    x = synthetic.gaussian(rng, m, k)
    return w, x, oracle.linear(dtype, x, w, n, k)


@pytest.mark.parametrize("name", TYPES)
@pytest.mark.parametrize("m", [1, 3, 8])
def test_matvec_float_x(lib, name, m):
    dtype = TYPES[name]
    rng = np.random.default_rng(30 + m)
    n, k = 1100, 4096  # more rows than the split kernel's 1024
    w, x, expected = product_inputs(rng, dtype, n, k, m)
    for kernel in (f"matvec_float_x_{name}", f"matvec_float_x_narrow_{name}"):
        out = torch.full((m, n), float("nan"), device="cuda")
        launch(lib, kernel, (n + 7) // 8, 256, P(dev(w)), P(dev(x)), P(out), I32(n), I32(k),
               I32(m))
        good(out.cpu().numpy(), expected)


@pytest.mark.parametrize("name", TYPES)
def test_matvec_float_x_multi(lib, name):
    dtype = TYPES[name]
    rng = np.random.default_rng(40)
    k, m, shapes = 2048, 2, [512, 128, 96]
    ws = [synthetic.quantized(rng, dtype, n, k) for n in shapes]
    x = synthetic.gaussian(rng, m, k)
    outs = [torch.full((m, n), float("nan"), device="cuda") for n in shapes]
    args = []
    for i in range(4):
        if i < len(shapes):
            args += [P(dev(ws[i])), P(outs[i]), I32(shapes[i])]
        else:
            args += [ctypes.c_void_p(None), ctypes.c_void_p(None), I32(0)]
    launch(lib, f"matvec_float_x_multi_{name}", (sum(shapes) + 7) // 8, 256, *args, P(dev(x)),
           I32(k), I32(m))
    for w, out, n in zip(ws, outs, shapes):
        good(out.cpu().numpy(), oracle.linear(dtype, x, w, n, k))


@pytest.mark.parametrize("name", TYPES)
def test_matvec_split(lib, name):
    dtype = TYPES[name]
    rng = np.random.default_rng(50)
    n, k, m = 300, 4096, 2
    w, x, expected = product_inputs(rng, dtype, n, k, m)
    out = torch.full((m, n), float("nan"), device="cuda")
    launch(lib, f"matvec_split_{name}", (n, m), 256, P(dev(w)), P(dev(x)), P(out), I32(n), I32(k))
    good(out.cpu().numpy(), expected)


def test_matvec_rows_f32(lib):
    rng = np.random.default_rng(60)
    n, k, m = 512, 2048, 3
    w = (0.05 * rng.standard_normal((n, k))).astype(np.float32)
    x = synthetic.gaussian(rng, m, k)
    out = torch.empty(m, n, device="cuda")
    launch(lib, "matvec_rows_f32", (n + 3) // 4, 256, P(dev(w)), P(dev(x)), P(out), I32(n), I32(k),
           I32(m))
    good(out.cpu().numpy(), oracle.linear(oracle.F32, x, w.view(np.uint8), n, k))


def test_route_topk(lib):
    rng = np.random.default_rng(70)
    tokens, experts, k = 5, 512, 10
    logits = rng.standard_normal((tokens, experts)).astype(np.float32)
    logits[0, 7] = logits[0, 300] = 9.0  # a tie: the lower id first
    ids = torch.empty(tokens, k, dtype=torch.int32, device="cuda")
    weights = torch.empty(tokens, k, device="cuda")
    launch(lib, "route_topk", (tokens + 7) // 8, 256, P(dev(logits)), P(ids), P(weights),
           I32(tokens), I32(experts), I32(k))
    e_ids, e_weights = oracle.route(logits, k)
    assert np.array_equal(ids.cpu().numpy(), e_ids)
    good(weights.cpu().numpy(), e_weights)


def combine_inputs(rng, tokens, k, hidden):
    return (rng.standard_normal((tokens * k, hidden)).astype(np.float32),
            rng.random((tokens, k)).astype(np.float32),
            rng.standard_normal((tokens, hidden)).astype(np.float32),
            rng.standard_normal((tokens, hidden)).astype(np.float32),
            (0.02 * rng.standard_normal(hidden)).astype(np.float32),
            rng.standard_normal((tokens, hidden)).astype(np.float32))


@pytest.mark.parametrize("shared", [False, True])
def test_moe_combine(lib, shared):
    rng = np.random.default_rng(80)
    tokens, k, hidden = 3, 10, 2048
    eo, w, so, si, sr, res = combine_inputs(rng, tokens, k, hidden)
    out = torch.empty(tokens, hidden, device="cuda")
    launch(lib, "moe_combine", tokens * 8, 256, P(dev(eo)), P(dev(w)),
           P(dev(so) if shared else None), P(dev(si) if shared else None),
           P(dev(sr) if shared else None), P(dev(res)), P(out), I32(k), I32(hidden))
    expected = oracle.moe_combine(eo, w, hidden, so if shared else None,
                                  si if shared else None, sr if shared else None, res)
    good(out.cpu().numpy(), expected)


def test_moe_combine_norm(lib):
    rng = np.random.default_rng(81)
    tokens, k, hidden = 2, 10, 2048
    eo, w, so, si, sr, res = combine_inputs(rng, tokens, k, hidden)
    norm = (1 + 0.02 * rng.standard_normal(hidden)).astype(np.float32)
    residual, normed = dev(res), torch.empty(tokens, hidden, device="cuda")
    xq = torch.zeros(tokens * hidden, dtype=torch.int8, device="cuda")
    xd, xs = torch.zeros(tokens * hidden // 32, device="cuda"), torch.zeros(tokens * hidden // 32,
                                                                            device="cuda")
    launch(lib, "moe_combine_norm", tokens, 1024, P(dev(eo)), P(dev(w)), P(dev(so)), P(dev(si)),
           P(dev(sr)), P(residual), I32(k), I32(hidden), P(dev(norm)), P(normed), F32(1e-6),
           F32(0.0), P(xq), P(xd), P(xs))
    e_res, e_normed = oracle.moe_combine_norm(eo, w, hidden, res, norm, 1e-6, 0.0, so, si, sr)
    good(residual.cpu().numpy(), e_res)
    got = normed.cpu().numpy()
    good(got, e_normed)
    q, d, _ = int8_format(got)
    assert np.array_equal(xq.cpu().numpy(), q) and np.array_equal(xd.cpu().numpy(), d)


@pytest.mark.parametrize("history", [False, True])
def test_causal_conv_silu(lib, history):
    rng = np.random.default_rng(90)
    tokens, channels, taps = 3, 1000, 4
    x = rng.standard_normal((tokens, channels)).astype(np.float32)
    weight = (0.3 * rng.standard_normal((channels, taps))).astype(np.float32)
    state = rng.standard_normal((taps - 1, channels)).astype(np.float32)
    state_dev, out = dev(state), torch.empty(tokens, channels, device="cuda")
    hist = torch.empty(tokens, taps - 1, channels, device="cuda") if history else None
    launch(lib, "causal_conv_silu", (channels + 255) // 256, 256, P(dev(x)), P(dev(weight)),
           P(state_dev), P(out), I32(tokens), I32(channels), I32(taps), I32(1), P(hist))
    result = oracle.causal_conv(x, weight, state, 1, keep_history=history)
    expected = result[0] if history else result
    good(out.cpu().numpy(), expected)
    good(state_dev.cpu().numpy(), state, 0, 0)  # the last inputs, copied
    if history:
        good(hist.cpu().numpy(), result[1], 0, 0)


@pytest.mark.parametrize("sigmoid", [0, 1])
def test_gated_rms_norm_f32(lib, sigmoid):
    rng = np.random.default_rng(95 + sigmoid)
    rows, cols = 16, 128
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    gate = rng.standard_normal((rows, cols)).astype(np.float32)
    weight = (1 + 0.02 * rng.standard_normal(cols)).astype(np.float32)
    out = torch.empty(rows, cols, device="cuda")
    null = ctypes.c_void_p(None)
    launch(lib, "gated_rms_norm_f32", rows, 256, P(dev(x)), P(dev(weight)), P(dev(gate)), P(out),
           I32(cols), F32(1e-6), I32(sigmoid), null, null, null)
    good(out.cpu().numpy(), oracle.gated_rms_norm(x, weight, gate, 3 if sigmoid else 0, 1e-6))


def test_add_f32(lib):
    rng = np.random.default_rng(99)
    a, b = rng.standard_normal(5000).astype(np.float32), rng.standard_normal(5000).astype(np.float32)
    out = torch.empty(5000, device="cuda")
    launch(lib, "add_f32", (5000 + 255) // 256, 256, P(dev(a)), P(dev(b)), P(out), I64(5000))
    assert np.array_equal(out.cpu().numpy(), a + b)


def test_read_sum_f32x4(lib):
    """The bandwidth probe (bandwidth.hip:5-20): one partial sum per block of
    a grid-stride read; the partials add up to the data's sum."""
    rng = np.random.default_rng(100)
    n4 = 1 << 20
    data = rng.integers(-8, 8, 4 * n4).astype(np.float32)  # sums exact in F32
    partials = torch.empty(96, device="cuda")
    launch(lib, "read_sum_f32x4", 96, 256, P(dev(data)), I64(n4), P(partials))
    assert float(partials.double().sum()) == float(data.astype(np.float64).sum())
