"""The C ABI without a GPU: the library loads, exports every function the
headers declare, lists its kernels by name, and refuses what the reference's
`require`s refuse -- before any CUDA call, so these run on a CPU host."""

import ctypes
import os
import re

import pytest

from drift_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]


def declared_functions():
    names = []
    for header in HEADERS:
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?\w+[\s\*]+(drift_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_headers_declare_functions():
    names = declared_functions()
    assert "drift_linear" in names and "drift_module_launch_kernel" in names
    assert len(names) >= 40


@pytest.mark.parametrize("name", declared_functions())
def test_every_declared_function_is_exported(lib, name):
    assert hasattr(lib, name), f"{name} is declared in include/ but not exported"
    assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in drift_b200/_lib.py"


def test_kernels_are_listed_by_name(lib):
    names = [lib.drift_kernel_name(i).decode() for i in range(lib.drift_kernel_count())]
    for expected in ["matvec_ring_q4_1_dp4a1", "matvec_split_q8_0_mma", "quantize_x22_mma_bf16",
                     "experts_gated_x22_q4_1_ks2", "linear_tc_q4_1",
                     # the runner's own names (runner/kernels/*.hip), with its argument lists
                     "gather_q8_0", "gather_q4_0", "gather_rows_f32", "rms_norm_f32", "gated_f32",
                     "rope_f32", "route_topk", "moe_combine", "moe_combine_norm",
                     "causal_conv_silu", "gated_rms_norm_f32", "add_f32", "matvec_rows_f32",
                     "matvec_float_x_q8_0", "matvec_float_x_narrow_q4_0",
                     "matvec_float_x_multi_q8_0", "matvec_float_x_multi_narrow_q4_0",
                     "matvec_split_q4_0",
                     # new names in the same pattern for Q4_1
                     "gather_q4_1", "matvec_float_x_q4_1", "matvec_split_q4_1"]:
        assert expected in names
    assert len(names) == len(set(names)), "a kernel name is registered twice"
    assert lib.drift_kernel_name(len(names)) is None


def test_unknown_kernel_is_refused(lib):
    f = ctypes.c_void_p()
    status = lib.drift_module_get_function(ctypes.byref(f), None, b"no_such_kernel")
    assert status == _lib.DRIFT_ERROR_INVALID_ARGUMENT
    assert b"no kernel no_such_kernel" in lib.drift_last_error_message()


def refused(status, fragment: str):
    assert status == _lib.DRIFT_ERROR_INVALID_ARGUMENT
    message = _lib.load().drift_last_error_message().decode()
    assert fragment in message, message


def test_linear_refusals(lib):
    # HipLinear.scala:112-117: no kernels for a type
    refused(lib.drift_linear(0, 8, 7, 8, 8, 1, 1, 64, None), "no kernels for")
    # DType.byteSize (DType.scala:24-30): whole blocks only
    refused(lib.drift_linear(0, 8, 3, 8, 8, 1, 1, 40, None), "not whole Q4_1 blocks of 32")
    # HipLinear.scala:126-131: rows of whole words (Q8_0, one block = 34 bytes)
    refused(lib.drift_linear(0, 8, 8, 8, 8, 1, 1, 32, None), "are not whole words")
    # x must be F32 (or BF16)
    refused(lib.drift_linear(8, 8, 3, 8, 8, 1, 1, 64, None), "takes F32 (or BF16) x")


def test_route_refusals(lib):
    refused(lib.drift_route(8, 8, 8, 1, 512, 17, None), "route: top-17 of 512")
    refused(lib.drift_route(8, 8, 8, 1, 513, 10, None), "route: top-10 of 513")


def test_rope_refusals(lib):
    refused(lib.drift_rope(8, 8, 8, 1, 1, 128, 1e6, 127, 0, None), "rotary values")
    refused(lib.drift_rope(8, 8, 8, 1, 1, 128, 1e6, 128, 2, None), "layout")


def test_experts_refusals(lib):
    refused(lib.drift_experts_linear(0, 8, 3, 3, 8, 4, 8, 64, 8, 10, 8, None),
            "for 10 slots")
    refused(lib.drift_experts_linear(0, 8, 1, 7, 8, 4, 8, 64, 8, 10, 8, None),
            "no kernels for")


def test_embedding_refusals(lib):
    refused(lib.drift_embedding(8, 8, 10, 40, 8, 1, 8, None), "not whole Q8_0 blocks")


def test_empty_products_need_no_gpu(lib):
    # zero tokens: nothing to launch
    assert lib.drift_route(None, None, None, 0, 512, 10, None) == 0
    assert lib.drift_rms_norm(None, None, 1e-6, 0.0, None, 0, 4096, None) == 0
