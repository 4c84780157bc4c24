"""Storage types on the hot path: a plug-in table as the reference's DType is
(runner/src/drift/runner/tensor/DType.scala:14-66, 151-175): the GGML id, the
block's elements and bytes."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class DType:
    name: str
    ggml_id: int
    block_elements: int
    block_bytes: int


F32 = DType("F32", 0, 1, 4)
F16 = DType("F16", 1, 1, 2)
Q4_0 = DType("Q4_0", 2, 32, 18)
Q4_1 = DType("Q4_1", 3, 32, 20)
Q8_0 = DType("Q8_0", 8, 32, 34)
Q4_K = DType("Q4_K", 12, 256, 144)  # tensor/KQuants.scala:99
Q6_K = DType("Q6_K", 14, 256, 210)  # tensor/KQuants.scala:122
I32 = DType("I32", 26, 1, 4)
BF16 = DType("BF16", 30, 1, 2)

DTYPES = {t.ggml_id: t for t in (F32, F16, Q4_0, Q4_1, Q8_0, Q4_K, Q6_K, I32, BF16)}


def byte_size(dtype: int, elements: int) -> int:
    """DType.byteSize (DType.scala:24-30): refuses elements that are not whole blocks."""
    t = DTYPES[dtype]
    if elements % t.block_elements:
        raise ValueError(f"{elements} elements are not whole {t.name} blocks of "
                         f"{t.block_elements}")
    return elements // t.block_elements * t.block_bytes
