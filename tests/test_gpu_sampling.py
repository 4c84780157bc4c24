"""Sampling on the GPU (SequenceOps.argmax / candidates) against the CPU
oracle (CpuSequence.argmax, Candidates.of): ids bit for bit, values bit for
bit -- over the C4/C5 vocabulary of 151,936, with ties, NaNs, signed zeros,
rows narrower than the candidate count; then split into vocabulary shards
(each shard's selection with its id offset, the pairs gathered, one merge)
as tensor parallelism runs it: the same ids as the whole row's. And the
runner's argmax_f32 / candidates_f32 launched by name with its own geometry
and buffers (HipSequence.scala:15-100).
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from drift_b200 import _lib
from drift_b200.ops import CudaOps

pytestmark = pytest.mark.gpu

VOCAB = 151936


@pytest.fixture(scope="module")
def ops():
    return CudaOps()


def logits(rng, rows, width):
    values = rng.standard_normal((rows, width)).astype(np.float32)
    if width > 100:
        # ties at the top: a row's largest twice (the lower index wins), -0
        # and 0, a NaN that never wins, infinities
        values[0, 5] = values[0, width - 3] = 50.0
        values[min(1, rows - 1), 17] = np.nan
        values[min(1, rows - 1), 18] = -0.0
        values[min(1, rows - 1), 19] = 0.0
        values[rows - 1, 90] = -np.inf
        values[rows - 1, 91] = np.inf
    return values


def run_argmax(ops, values, id_offset=0):
    rows = values.shape[0]
    v = torch.from_numpy(values).cuda()
    ids = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    out = torch.empty(rows, device="cuda")
    ops.argmax(v, ids, out, id_offset)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), out.cpu().numpy()


@pytest.mark.parametrize("rows,width", [(1, VOCAB), (16, VOCAB), (3, 8193), (2, 7), (4, 1)])
def test_argmax_is_the_cpu_argmax(ops, rows, width):
    rng = np.random.default_rng(rows * 7 + width)
    values = logits(rng, rows, width)
    ids, out = run_argmax(ops, values)
    for r in range(rows):
        e = oracle.argmax(values[r])
        assert ids[r] == e, (r, ids[r], e)
        assert out[r].tobytes() == values[r, e].tobytes()


def test_argmax_nan_rules(ops):
    """CpuSequence.argmax compares with `>` from index 0: a NaN at index 0 is
    never replaced; a NaN elsewhere never wins; all -inf gives 0."""
    values = np.zeros((3, 5000), np.float32)
    values[0, 0] = np.nan
    values[0, 100] = 7.0
    values[1, 1:] = np.nan
    values[1, 0] = -1.0
    values[2, :] = -np.inf
    ids, _ = run_argmax(ops, values)
    assert list(ids) == [oracle.argmax(values[r]) for r in range(3)] == [0, 0, 0]


def run_candidates(ops, values, count, id_offset=0):
    rows, width = values.shape
    v = torch.from_numpy(values).cuda()
    ids = torch.full((rows, count), -1, dtype=torch.int32, device="cuda")
    out = torch.full((rows, count), 777.0, device="cuda")
    ops.candidates(v, count, ids, out, id_offset)
    torch.cuda.synchronize()
    kept = min(count, width)
    return ids.cpu().numpy()[:, :kept], out.cpu().numpy()[:, :kept]


@pytest.mark.parametrize("rows,width,count",
                         [(1, VOCAB, 1), (4, VOCAB, 40), (16, VOCAB, 64), (2, VOCAB, 1024),
                          (3, 5000, 300), (2, 7, 10), (5, 4096, 4096 // 4)])
def test_candidates_are_the_cpu_candidates(ops, rows, width, count):
    rng = np.random.default_rng(rows + width + count)
    values = logits(rng, rows, width)
    ids, out = run_candidates(ops, values, count)
    e_ids, e_out = oracle.candidates(values, count)
    assert np.array_equal(ids, e_ids)
    assert out.tobytes() == e_out.tobytes()


def test_candidates_with_many_equal_values(ops):
    """Ties across the whole row: the lower indices first, in index order."""
    values = np.zeros((2, VOCAB), np.float32)
    values[1, ::7] = 1.0
    ids, _ = run_candidates(ops, values, 100)
    e_ids, _ = oracle.candidates(values, 100)
    assert np.array_equal(ids, e_ids)
    assert list(ids[0][:5]) == [0, 1, 2, 3, 4]


@pytest.mark.parametrize("shards", [2, 3, 8])
def test_shards_merge_to_the_whole_rows(ops, shards):
    """Tensor parallelism's vocabulary split: each shard's argmax and
    candidates with its id offset, the (value, id) pairs gathered shard after
    shard, one merge: the whole rows' ids and values, bit for bit."""
    rng = np.random.default_rng(shards)
    rows, count = 4, 50
    values = logits(rng, rows, VOCAB)
    values[2, 3] = np.nan  # a NaN at id 3 on shard 0
    bounds = [VOCAB * s // shards for s in range(shards + 1)]
    a_vals, a_ids, c_vals, c_ids = [], [], [], []
    for s in range(shards):
        part = np.ascontiguousarray(values[:, bounds[s]:bounds[s + 1]])
        ids, out = run_argmax(ops, part, bounds[s])
        a_ids.append(ids[:, None])
        a_vals.append(out[:, None])
        ids, out = run_candidates(ops, part, count, bounds[s])
        c_ids.append(ids)
        c_vals.append(out)
    gathered = lambda parts: torch.from_numpy(np.ascontiguousarray(np.concatenate(parts, 1))).cuda()
    merged = torch.empty(rows, dtype=torch.int32, device="cuda")
    merged_values = torch.empty(rows, device="cuda")
    ops.argmax_merge(gathered(a_vals), gathered(a_ids), merged, merged_values)
    top = torch.empty(rows, count, dtype=torch.int32, device="cuda")
    top_values = torch.empty(rows, count, device="cuda")
    ops.candidates_merge(gathered(c_vals), gathered(c_ids), count, top, top_values)
    torch.cuda.synchronize()
    assert list(merged.cpu().numpy()) == [oracle.argmax(values[r]) for r in range(rows)]
    e_ids, e_out = oracle.candidates(values, count)
    assert np.array_equal(top.cpu().numpy(), e_ids)
    assert top_values.cpu().numpy().tobytes() == e_out.tobytes()


def test_refusals(ops):
    v = torch.zeros(2, 100, device="cuda")
    ids = torch.empty(2, 1025, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="1025 candidates, 1 to 1024"):
        ops.candidates(v, 1025, ids)


def launch(lib, name, grid, block, *args):
    function = ctypes.c_void_p()
    _lib.check("drift_module_get_function",
               lib.drift_module_get_function(ctypes.byref(function), None, name.encode()))
    slots = (ctypes.c_void_p * len(args))(*[ctypes.cast(ctypes.pointer(a), ctypes.c_void_p)
                                            for a in args])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(name, lib.drift_module_launch_kernel(function, grid, 1, 1, block, 1, 1, 0, stream,
                                                    slots, None))
    torch.cuda.synchronize()


def test_runner_kernels_by_name(ops):
    """argmax_f32(values, index, count) on one block of 1024 and
    candidates_f32(values, out, width, count, kept, finished) on rows x
    chunks blocks of 1024, with the runner's kept / finished buffers and its
    (value bits, index) output pairs (HipSequence.scala:15-100)."""
    lib = ops.lib
    rng = np.random.default_rng(5)
    rows, count = 3, 20
    values = logits(rng, rows, VOCAB)
    v = torch.from_numpy(values).cuda()
    index = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    launch(lib, "argmax_f32", 1, 1024, p(v), p(index), ctypes.c_int32(VOCAB))
    assert int(index.item()) == oracle.argmax(values[0])
    chunks = (VOCAB + 4095) // 4096
    out = torch.zeros(rows, count, 2, dtype=torch.int32, device="cuda")
    kept = torch.zeros(rows * chunks * count * 2, dtype=torch.int32, device="cuda")
    finished = torch.zeros(65536, dtype=torch.int32, device="cuda")
    for _ in range(2):  # finished counters are left at 0: a second call works the same
        launch(lib, "candidates_f32", rows * chunks, 1024, p(v), p(out), ctypes.c_int32(VOCAB),
               ctypes.c_int32(count), p(kept), p(finished))
        e_ids, e_out = oracle.candidates(values, count)
        got = out.cpu().numpy()
        assert np.array_equal(got[:, :, 1], e_ids)
        assert got[:, :, 0].tobytes() == e_out.view(np.int32).tobytes()
        assert int(finished.abs().sum().item()) == 0
