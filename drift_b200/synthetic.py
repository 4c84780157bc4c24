"""Seeded synthetic inputs with the benchmark configurations' shapes and value
laws (there is no dataset or checkpoint on this path: the reference's own
benchmarks also run on random weights, gpuTest/.../MatVecBenchmark.scala).

- Q8_0 (config C1): f16 scale d ~ U(0.002, 0.02), int8 codes uniform in
  [-127, 127].
- Q4_1 (config C2): d ~ U(0.002, 0.02) and m = -8 d (both f16), 4-bit codes
  uniform in 0..15, so values are symmetric about zero like Q8_0's.
- Q4_0: d ~ U(0.002, 0.02), codes uniform.
- `random_blocks`: the reference tests' weights (TestData.quantized,
  runner/test/src/drift/runner/TestData.scala:33-51): random bytes, so every
  code occurs, with f16 scales ~ N(0, 0.01).
- `k_quant_blocks`: Q4_K / Q6_K super-blocks as the reference's fixture
  recipe draws them (runner/fixtures/generate.py: random bytes, every f16
  field ~ N(0, 0.05)), scaled down to N(0, 0.005) so products stay in range.
x ~ N(0, 1) (bf16 or f32).
"""

from __future__ import annotations

import numpy as np

F32, Q4_0, Q4_1, Q8_0, Q4_K, Q6_K = 0, 2, 3, 8, 12, 14
BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q8_0: 34}
# the K-quants: (bytes per 256-value super-block, offsets of the f16 fields)
K_LAYOUT = {Q4_K: (144, [0, 2]), Q6_K: (210, [208])}


def _scales(rng: np.random.Generator, count: int) -> np.ndarray:
    return rng.uniform(0.002, 0.02, size=count).astype(np.float16)


def quantized(rng: np.random.Generator, dtype: int, n: int, k: int) -> np.ndarray:
    """[n, k] weights of `dtype` by the benchmark laws, as raw blocks (uint8)."""
    blocks = n * (k // 32)
    size = BLOCK_BYTES[dtype]
    out = np.empty((blocks, size), dtype=np.uint8)
    d = _scales(rng, blocks)
    out[:, 0:2] = d.view(np.uint8).reshape(blocks, 2)
    if dtype == Q8_0:
        codes = rng.integers(-127, 128, size=(blocks, 32), dtype=np.int16).astype(np.int8)
        out[:, 2:34] = codes.view(np.uint8)
    elif dtype == Q4_1:
        m = (-8.0 * d.astype(np.float32)).astype(np.float16)
        out[:, 2:4] = m.view(np.uint8).reshape(blocks, 2)
        out[:, 4:20] = rng.integers(0, 256, size=(blocks, 16), dtype=np.uint8)
    elif dtype == Q4_0:
        out[:, 2:18] = rng.integers(0, 256, size=(blocks, 16), dtype=np.uint8)
    else:
        raise ValueError(f"no synthetic law for type {dtype}")
    return out.reshape(-1)


def random_blocks(rng: np.random.Generator, dtype: int, n: int, k: int) -> np.ndarray:
    """The reference tests' weights: random bytes, f16 scales ~ N(0, 0.01)."""
    size = BLOCK_BYTES[dtype]
    blocks = n * (k // 32)
    out = rng.integers(0, 256, size=(blocks, size), dtype=np.uint8)
    fields = [0, 2] if dtype == Q4_1 else [0]
    for at in fields:
        scales = (rng.standard_normal(blocks) * 0.01).astype(np.float16)
        out[:, at:at + 2] = scales.view(np.uint8).reshape(blocks, 2)
    return out.reshape(-1)


def gaussian(rng: np.random.Generator, *shape) -> np.ndarray:
    return rng.standard_normal(shape).astype(np.float32)


def bf16_bits(values: np.ndarray) -> np.ndarray:
    """F32 rounded to BF16 (to nearest even) as uint16 bits."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_values(bits: np.ndarray) -> np.ndarray:
    """BF16 bits widened exactly to F32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def quantized_device(dtype: int, n: int, k: int, generator=None, device=None):
    """The `quantized` law drawn on the device (torch): for model-sized
    random-init weights, where drawing gigabytes on the host would dominate a
    run. Not the same bytes as `quantized` for a seed."""
    import torch

    device = device or torch.device("cuda")
    blocks = n * (k // 32)
    size = BLOCK_BYTES[dtype]
    out = torch.empty(blocks, size, dtype=torch.uint8, device=device)
    d = (torch.rand(blocks, generator=generator, device=device) * 0.018 + 0.002).half()
    out[:, 0:2] = d.view(torch.uint8).view(blocks, 2)
    if dtype == Q8_0:
        codes = torch.randint(-127, 128, (blocks, 32), generator=generator, device=device,
                              dtype=torch.int16).to(torch.int8)
        out[:, 2:34] = codes.view(torch.uint8)
    elif dtype == Q4_1:
        m = (-8.0 * d.float()).half()
        out[:, 2:4] = m.view(torch.uint8).view(blocks, 2)
        out[:, 4:20] = torch.randint(0, 256, (blocks, 16), generator=generator, device=device,
                                     dtype=torch.uint8)
    elif dtype == Q4_0:
        out[:, 2:18] = torch.randint(0, 256, (blocks, 16), generator=generator, device=device,
                                     dtype=torch.uint8)
    else:
        raise ValueError(f"no synthetic law for type {dtype}")
    return out.reshape(-1)


def k_quant_blocks(rng: np.random.Generator, dtype: int, n: int, k: int) -> np.ndarray:
    """[n, k] weights of Q4_K or Q6_K as raw super-blocks (uint8)."""
    size, fields = K_LAYOUT[dtype]
    count = n * (k // 256)
    out = rng.integers(0, 256, size=(count, size), dtype=np.uint8)
    for at in fields:
        halves = (rng.standard_normal(count) * 0.005).astype(np.float16)
        out[:, at:at + 2] = halves.view(np.uint8).reshape(count, 2)
    return out.reshape(-1)
