"""drift_linear_static: the quantized product for hosts that cannot allocate
device memory on the call path (memory reserved up front, an FFM host's own
allocator, a loop that must not let cudaMalloc synchronize the device).

Its scratch is a fixed array inside the library, so these tests call it
through the C ABI directly and hold it to drift_linear, the entry point that
allocates its scratch as it grows: same inputs, two calls in a row (the
second must not see the first's leftovers), the tolerance the product tests
use (the benchmark's 1e-4 absolute + 1e-3 relative). This file runs last, alone
or after the others.
"""

import ctypes

import numpy as np
import pytest
import torch

from drift_b200 import _lib, synthetic
from tests.conftest import within

pytestmark = pytest.mark.gpu

Q4_0, Q4_1, Q8_0 = 2, 3, 8


def call(name, x, weight_dtype, weight, out, m, n, k):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    x_dtype = 30 if x.dtype == torch.bfloat16 else 0
    status = getattr(lib, name)(x_dtype, ctypes.c_void_p(x.data_ptr()), weight_dtype,
                                ctypes.c_void_p(weight.data_ptr()),
                                ctypes.c_void_p(out.data_ptr()), m, n, k, stream)
    _lib.check(name, status)


def x_tensor(rng, m, k, bf16):
    values = synthetic.gaussian(rng, m, k)
    if bf16:
        bits = synthetic.bf16_bits(values)
        return torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    return torch.from_numpy(values).cuda()


# (type, m, n, k, bf16 x): aligned rows (the staged kernel), a row that is not
# a whole number of 16 bytes (the direct kernel), passes of 8 rows
CASES = [(Q4_1, 1, 4096, 4096, True), (Q8_0, 8, 1000, 2048, False), (Q4_0, 3, 333, 1024, True),
         (Q4_1, 2, 65, 96, False), (Q4_1, 20, 512, 4096, True), (Q8_0, 31, 77, 9344, False)]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_matches_the_allocating_entry_point_twice(case):
    dtype, m, n, k, bf16 = case
    rng = np.random.default_rng(sum(case[:4]))
    weight = torch.from_numpy(synthetic.quantized(rng, dtype, n, k)).cuda()
    for _ in range(2):
        x = x_tensor(rng, m, k, bf16)
        expected = torch.full((m, n), float("nan"), device="cuda")
        actual = torch.full((m, n), float("nan"), device="cuda")
        call("drift_linear", x, dtype, weight, expected, m, n, k)
        call("drift_linear_static", x, dtype, weight, actual, m, n, k)
        torch.cuda.synchronize()
        ok, _, _, summary = within(actual.cpu().numpy(), expected.cpu().numpy(), 1e-4, 1e-3)
        assert ok, summary
        assert torch.isfinite(actual).all()


def test_refuses_what_its_scratch_cannot_hold():
    rng = np.random.default_rng(1)
    weight = torch.from_numpy(synthetic.quantized(rng, Q4_1, 16, 4096)).cuda()
    x = x_tensor(rng, 32, 4096, False)
    out = torch.empty(32, 16, device="cuda")
    with pytest.raises(ValueError, match="takes 1 to 31 rows of x"):
        call("drift_linear_static", x, Q4_1, weight, out, 32, 16, 4096)
    # 8 rows of 40,960 columns: 1,280 blocks of 896 bytes, past 1 MiB
    big = torch.zeros(8, 40960, device="cuda")
    wide = torch.zeros(16 * 1280 * 20, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError, match="bytes of scratch"):
        call("drift_linear_static", big, Q4_1, wide, torch.empty(8, 16, device="cuda"), 8, 16,
             40960)
