"""Shared pytest setup: the `gpu` marker, the repo root on sys.path, and helpers.

Tests marked `gpu` need a B200 and call the CUDA path through the C ABI; the
rest run on any CPU (oracle against golden vectors, host logic, C-ABI exports).
"""

import json
import os
import struct
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def read_safetensors(path: str) -> dict:
    """A minimal safetensors reader (8-byte header length, JSON header, data)."""
    dtypes = {"U8": np.uint8, "F32": np.float32, "F16": np.float16, "I32": np.int32}
    with open(path, "rb") as f:
        data = f.read()
    (length,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8:8 + length])
    out = {}
    base = 8 + length
    for name, info in header.items():
        if name == "__metadata__":
            continue
        start, end = info["data_offsets"]
        array = np.frombuffer(data[base + start:base + end], dtype=dtypes[info["dtype"]])
        out[name] = array.reshape(info["shape"])
    return out


def within(actual, expected, absolute: float, relative: float):
    """Comparison.of (runner/src/drift/runner/tensor/Comparison.scala:32-74):
    |a - e| <= absolute + relative * |e|, NaN and infinities only where the
    reference has the same. Returns (passed, mismatches, max_abs, summary)."""
    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    e = np.asarray(expected, dtype=np.float64).reshape(-1)
    assert a.shape == e.shape, f"comparing {a.size} values with {e.size}"
    nan = np.isnan(a) | np.isnan(e)
    inf = ~nan & (np.isinf(a) | np.isinf(e))
    finite = ~nan & ~inf
    bad = np.zeros(a.shape, dtype=bool)
    bad[nan] = ~(np.isnan(a[nan]) & np.isnan(e[nan]))
    bad[inf] = a[inf] != e[inf]
    diff = np.abs(a[finite] - e[finite])
    bad[finite] = diff > absolute + relative * np.abs(e[finite])
    max_abs = float(diff.max()) if diff.size else 0.0
    first = int(np.argmax(bad)) if bad.any() else None
    summary = (f"{int(bad.sum())}/{a.size} mismatches"
               + (f", first at {first} ({a[first]!r} vs {e[first]!r})" if first is not None else "")
               + f", max absolute {max_abs:.3g}")
    return (not bad.any()), int(bad.sum()), max_abs, summary


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")
