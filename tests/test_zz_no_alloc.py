"""drift_linear_static: the quantized product for hosts that cannot allocate
device memory on the call path (memory reserved up front, an FFM host's own
allocator, a loop that must not let cudaMalloc synchronize the device).

Its scratch is a fixed array inside the library, so these tests call it
through the C ABI directly and hold it to two things, on two calls in a row
with fresh x each time (the second must not see the first's leftovers):
- drift_linear, the entry point that allocates its scratch as it grows: the
  two run the same preparation and product kernels, so their outputs are
  equal bit for bit (a scratch-reuse fault that only moves low bits would show);
- the CPU oracle, at the tolerance the product tests use (the benchmark's
  1e-4 absolute + 1e-3 relative).
This file runs last, alone or after the others.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from drift_b200 import _lib, synthetic
from tests.conftest import within

pytestmark = pytest.mark.gpu

F32, Q4_0, Q4_1, Q8_0 = 0, 2, 3, 8


def call(name, x, weight_dtype, weight, out, m, n, k):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    x_dtype = 30 if x.dtype == torch.bfloat16 else 0
    status = getattr(lib, name)(x_dtype, ctypes.c_void_p(x.data_ptr()), weight_dtype,
                                ctypes.c_void_p(weight.data_ptr()),
                                ctypes.c_void_p(out.data_ptr()), m, n, k, stream)
    _lib.check(name, status)


def x_values(rng, m, k, bf16):
    """(device tensor, the F32 values the oracle sees)."""
    values = synthetic.gaussian(rng, m, k)
    if bf16:
        bits = synthetic.bf16_bits(values)
        return (torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16),
                synthetic.bf16_values(bits))
    return torch.from_numpy(values).cuda(), values


def weight_bytes(rng, dtype, n, k):
    if dtype == F32:
        return (0.02 * rng.standard_normal(n * k)).astype(np.float32)
    return synthetic.quantized(rng, dtype, n, k)


# (type, m, n, k, bf16 x): aligned rows (the staged kernel), a row that is not
# a whole number of 16 bytes (the direct kernel), passes of 8 rows, F32 weights
CASES = [(Q4_1, 1, 4096, 4096, True), (Q8_0, 8, 1000, 2048, False), (Q4_0, 3, 333, 1024, True),
         (Q4_1, 2, 65, 96, False), (Q4_1, 20, 512, 4096, True), (Q8_0, 31, 77, 9344, False),
         (F32, 5, 96, 2048, False), (F32, 2, 40, 512, True)]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_matches_the_allocating_entry_point_twice(case):
    dtype, m, n, k, bf16 = case
    rng = np.random.default_rng(sum(case[:4]))
    w = weight_bytes(rng, dtype, n, k)
    weight = torch.from_numpy(w).cuda()
    for call_number in range(2):
        x, x_eff = x_values(rng, m, k, bf16)
        expected = torch.full((m, n), float("nan"), device="cuda")
        actual = torch.full((m, n), float("nan"), device="cuda")
        call("drift_linear", x, dtype, weight, expected, m, n, k)
        call("drift_linear_static", x, dtype, weight, actual, m, n, k)
        torch.cuda.synchronize()
        assert torch.equal(actual, expected), \
            f"call {call_number}: differs from drift_linear in " \
            f"{int((actual != expected).sum())} of {m * n} outputs"
        reference = oracle.linear(dtype, x_eff, w.view(np.uint8), n, k)
        ok, _, _, summary = within(actual.cpu().numpy(), reference, 1e-4, 1e-3)
        assert ok, f"call {call_number} against the oracle: {summary}"


def test_refuses_what_its_scratch_cannot_hold():
    rng = np.random.default_rng(1)
    weight = torch.from_numpy(synthetic.quantized(rng, Q4_1, 16, 4096)).cuda()
    x, _ = x_values(rng, 32, 4096, False)
    out = torch.empty(32, 16, device="cuda")
    with pytest.raises(ValueError, match="takes 1 to 31 rows of x"):
        call("drift_linear_static", x, Q4_1, weight, out, 32, 16, 4096)
    # 8 rows of 40,960 columns: 1,280 blocks of 896 bytes, past 1 MiB
    big = torch.zeros(8, 40960, device="cuda")
    wide = torch.zeros(16 * 1280 * 20, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError, match="bytes of scratch"):
        call("drift_linear_static", big, Q4_1, wide, torch.empty(8, 16, device="cuda"), 8, 16,
             40960)
