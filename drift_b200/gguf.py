"""GGUF files (versions 2 and 3, little-endian): the reference's reader,
runner/src/drift/runner/formats/Gguf.scala:27-287, for this library's host.

Metadata, then tensor infos, then the data section, each tensor at a
multiple of `general.alignment` (32 when absent). GGUF lists dimensions
innermost first (ne[0] is the row length); `shape` here is outermost first,
reversed once, as the reference's Shape is. Tensors of a type this library
has no kernels for are listed in `unsupported` with the reason, as the
reference lists types without a DType. Every check of the reference's reader
is made, with its messages: the magic, the version (a big-endian file shows
as a version above 0xffff), plausible counts and lengths, at most 8
dimensions, rows of whole blocks, aligned offsets, tensors inside the file,
and each tensor's span (its bytes up to the alignment padding before the
next tensor). The file is memory-mapped; `upload` copies one tensor's raw
blocks to the device as a `Stored` weight.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from .dtypes import DTYPES

MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32


class FormatError(ValueError):
    """A malformed file (the reference's FormatException)."""


@dataclass(frozen=True)
class GgufTensor:
    name: str
    dtype: int           # GGML type id
    shape: tuple         # outermost first
    offset: int          # from the start of the file
    nbytes: int
    data: np.ndarray     # uint8 view of the mapped bytes


@dataclass
class GgufFile:
    source: str
    version: int
    metadata: dict
    alignment: int
    tensors: dict = field(default_factory=dict)
    unsupported: dict = field(default_factory=dict)

    def _value(self, key: str) -> Any:
        if key not in self.metadata:
            raise FormatError(f"{self.source} has no {key}")
        return self.metadata[key]

    def long(self, key: str) -> int:
        value = self._value(key)
        if isinstance(value, bool) or not isinstance(value, int) or not -2**63 <= value < 2**63:
            raise FormatError(f"{self.source}: {key} is {value!r}")
        return value

    def double(self, key: str) -> float:
        value = self._value(key)
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise FormatError(f"{self.source}: {key} is {value!r}")
        return float(value)

    def string(self, key: str) -> str:
        value = self._value(key)
        if not isinstance(value, str):
            raise FormatError(f"{self.source}: {key} is {value!r}")
        return value

    def boolean(self, key: str) -> bool:
        value = self._value(key)
        if not isinstance(value, bool):
            raise FormatError(f"{self.source}: {key} is {value!r}")
        return value

    def strings(self, key: str) -> list:
        value = self._value(key)
        if not isinstance(value, list) or not all(isinstance(v, str) for v in value):
            raise FormatError(f"{self.source}: {key} is {value!r}")
        return value

    @property
    def architecture(self) -> str:
        """general.architecture: the key prefix of the model's hyperparameters."""
        return self.string("general.architecture")

    def upload(self, name: str, device=None):
        """Tensor `name`'s raw blocks on the device, as a product's weight."""
        from .ops import Stored

        if name not in self.tensors:
            reason = self.unsupported.get(name, "no such tensor")
            raise FormatError(f"{self.source}: {name}: {reason}")
        t = self.tensors[name]
        return Stored.upload(t.dtype, t.shape, np.ascontiguousarray(t.data), device)


class _Reader:
    # value types 0..12 (gguf's GGUFValueType): struct formats of the scalars
    SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 10: "<Q",
               11: "<q", 12: "<d"}

    def __init__(self, data: np.ndarray, source: str):
        self.data, self.source, self.position = data, source, 0
        self.size = int(data.size)

    def fail(self, message: str):
        raise FormatError(f"{self.source}: {message}")

    def need(self, count: int) -> None:
        if count < 0 or self.position + count > self.size:
            self.fail(f"truncated at byte {self.position} (needs {count} more)")

    def scalar(self, fmt: str):
        width = struct.calcsize(fmt)
        self.need(width)
        value = struct.unpack_from(fmt, self.data, self.position)[0]
        self.position += width
        return value

    def count(self, what: str) -> int:
        value = self.scalar("<q")
        if value < 0 or value > self.size:
            self.fail(f"{what} of {value} is not plausible")
        return value

    def text(self) -> str:
        length = self.count("string length")
        self.need(length)
        raw = bytes(self.data[self.position:self.position + length])
        self.position += length
        return raw.decode("utf-8")

    def value(self, kind: int):
        if kind in self.SCALARS:
            return self.scalar(self.SCALARS[kind])
        if kind == 7:
            return self.scalar("<B") != 0
        if kind == 8:
            return self.text()
        if kind == 9:
            element = self.scalar("<I")
            length = self.count("array length")
            return [self.value(element) for _ in range(length)]
        self.fail(f"unknown metadata value type {kind}")

    def read(self) -> GgufFile:
        self.need(8)
        if bytes(self.data[:4]) != MAGIC:
            self.fail("not a GGUF file")
        self.position = 4
        version = self.scalar("<I")
        if version not in (2, 3):
            self.fail("big-endian GGUF is not supported" if version > 0xFFFF
                      else f"GGUF version {version} is not supported")
        tensor_count = self.count("tensor count")
        metadata_count = self.count("metadata count")
        metadata = {}
        for _ in range(metadata_count):
            key = self.text()
            metadata[key] = self.value(self.scalar("<I"))
        alignment = metadata.get("general.alignment", DEFAULT_ALIGNMENT)
        if (isinstance(alignment, bool) or not isinstance(alignment, int) or alignment <= 0
                or alignment & (alignment - 1)):
            self.fail(f"general.alignment is {alignment!r}")
        infos = []
        for _ in range(tensor_count):
            name = self.text()
            rank = self.scalar("<I")
            if rank > 8:
                self.fail(f"{name} has {rank} dimensions")
            dims = [self.count(f"{name} dimension") for _ in range(rank)]
            infos.append((name, dims, self.scalar("<I"), self.scalar("<q")))
        data_start = (self.position + alignment - 1) // alignment * alignment
        data_bytes = self.size - data_start
        if data_bytes < 0:
            self.fail("truncated before the data section")
        result = GgufFile(self.source, version, metadata, alignment)
        described = {}
        for name, dims, type_id, offset in infos:
            dtype = DTYPES.get(type_id)
            if dtype is None:
                result.unsupported[name] = f"GGML type {type_id} has no kernels here"
                described[name] = None
                continue
            if dims and dims[0] % dtype.block_elements:
                self.fail(f"{name}: rows of {dims[0]} are not whole {dtype.name} blocks")
            if offset % alignment:
                self.fail(f"{name} is not aligned to {alignment}")
            elements = 1
            for d in dims:
                elements *= d
            nbytes = elements // dtype.block_elements * dtype.block_bytes
            if offset + nbytes > data_bytes:
                self.fail(f"{name} runs past the end of the file")
            start = data_start + offset
            described[name] = GgufTensor(name, type_id, tuple(reversed(dims)), start, nbytes,
                                         self.data[start:start + nbytes])
        # each tensor's bytes fit the room the file gives it, up to the padding
        ordered = sorted(infos, key=lambda info: info[3])
        for index, (name, _, _, offset) in enumerate(ordered):
            tensor = described[name]
            if tensor is None:
                continue
            end = ordered[index + 1][3] if index + 1 < len(ordered) else data_bytes
            room = end - offset
            if room < tensor.nbytes or room - tensor.nbytes >= alignment:
                self.fail(f"{name} is {DTYPES[tensor.dtype].name} {list(tensor.shape)}, "
                          f"{tensor.nbytes} bytes, but the file gives it {room}")
        result.tensors = {n: t for n, t in described.items() if t is not None}
        return result


def read(data, source: str = "<bytes>") -> GgufFile:
    """Reads a whole GGUF file's bytes (a numpy uint8 array or bytes)."""
    array = np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray)) else data
    return _Reader(array, source).read()


def open_file(path: str) -> GgufFile:
    """Maps and reads a GGUF file; its tensors are views of the mapping."""
    return read(np.memmap(path, dtype=np.uint8, mode="r"), path)
