"""Tensor-parallel products across the GPUs of one box, one process per GPU.

The split of the runner's dense layers that the benchmark's decode configs name
(column-split QKV / gate / up, row-split o / down with one all-reduce; the
reference runs one device, runner/src/drift/runner/native/HipRuntime.scala:
40-43, so this is the B200 build's own layout):

- `ColumnParallelLinear`: a rank holds output rows [lo, hi) of W [N, K] -- a
  contiguous byte range of the GGML rows -- and computes y[:, lo:hi]. No
  exchange: the next product (row-split) consumes the shard as it is.
- `RowParallelLinear`: a rank holds the columns [k0, k1) of every row, in
  whole 32-value blocks (a strided copy of the raw blocks made once at load),
  multiplies its slice of x and adds the partial sums of all ranks with one
  all-reduce (NCCL over NVLink on the GPUs; gloo in the CPU tests).

Shards are even to a block: rank r of W gets blocks [B r / W, B (r+1) / W) of
the B = K / 32 blocks (or rows [N r / W, N (r+1) / W)), so every rank's rows
stay whole blocks and, where K / 32 / W is a whole number of 16-byte units,
the products keep their tensor-copy paths.

The products themselves are whatever `ops.linear` the caller passes (the
library's CudaOps on a GPU); this module owns only the partitioning and the
exchange.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Optional

import numpy as np

from .dtypes import DTYPES, byte_size

BLOCK = 32


def row_range(rows: int, rank: int, world: int) -> tuple[int, int]:
    """Output rows [lo, hi) of rank `rank` of `world` (column-split)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return rows * rank // world, rows * (rank + 1) // world


def column_range(cols: int, rank: int, world: int) -> tuple[int, int]:
    """Columns [k0, k1) of rank `rank` (row-split), in whole 32-value blocks."""
    if cols % BLOCK:
        raise ValueError(f"{cols} columns are not whole blocks of {BLOCK}")
    blocks = cols // BLOCK
    if blocks < world:
        raise ValueError(f"{blocks} blocks cannot be split {world} ways")
    lo, hi = row_range(blocks, rank, world)
    return lo * BLOCK, hi * BLOCK


def shard_rows(blocks: np.ndarray, dtype: int, rows: int, cols: int, rank: int,
               world: int) -> tuple[np.ndarray, int]:
    """The raw bytes of rank `rank`'s output rows, and their count."""
    row_bytes = byte_size(dtype, cols)
    flat = np.asarray(blocks, dtype=np.uint8).reshape(-1)
    if flat.size < rows * row_bytes:
        raise ValueError(f"{flat.size} bytes hold fewer than {rows} rows of {row_bytes}")
    lo, hi = row_range(rows, rank, world)
    return flat[lo * row_bytes:hi * row_bytes].copy(), hi - lo


def shard_columns(blocks: np.ndarray, dtype: int, rows: int, cols: int, rank: int,
                  world: int) -> tuple[np.ndarray, int, int]:
    """The raw bytes of rank `rank`'s column slice of every row ([rows,
    (k1 - k0) / 32] blocks, row-major), and (k0, k1)."""
    row_bytes = byte_size(dtype, cols)
    block_bytes = DTYPES[dtype].block_bytes
    matrix = np.asarray(blocks, dtype=np.uint8).reshape(-1)[:rows * row_bytes]
    matrix = matrix.reshape(rows, row_bytes)
    k0, k1 = column_range(cols, rank, world)
    part = matrix[:, (k0 // BLOCK) * block_bytes:(k1 // BLOCK) * block_bytes]
    return np.ascontiguousarray(part).reshape(-1), k0, k1


@dataclass
class ColumnParallelLinear:
    """This rank's output rows of a product: out [m, hi - lo] = x [m, K] .
    W[lo:hi, :]^T. `weight` is the shard as `ops.linear` takes it."""
    weight: Any
    rows: int  # the full N
    cols: int
    lo: int
    hi: int

    @staticmethod
    def from_blocks(blocks: np.ndarray, dtype: int, rows: int, cols: int, rank: int,
                    world: int, upload: Callable[[int, tuple, np.ndarray], Any]):
        part, count = shard_rows(blocks, dtype, rows, cols, rank, world)
        lo, hi = row_range(rows, rank, world)
        return ColumnParallelLinear(upload(dtype, (count, cols), part), rows, cols, lo, hi)

    def __call__(self, ops, x, out) -> None:
        ops.linear(x, self.weight, out)


@dataclass
class RowParallelLinear:
    """This rank's column slice of a product; `__call__` leaves the full
    out [m, N] = x . W^T on every rank after one all-reduce."""
    weight: Any
    rows: int
    cols: int  # the full K
    k0: int
    k1: int

    @staticmethod
    def from_blocks(blocks: np.ndarray, dtype: int, rows: int, cols: int, rank: int,
                    world: int, upload: Callable[[int, tuple, np.ndarray], Any]):
        part, k0, k1 = shard_columns(blocks, dtype, rows, cols, rank, world)
        return RowParallelLinear(upload(dtype, (rows, k1 - k0), part), rows, cols, k0, k1)

    def __call__(self, ops, x_part, out, group: Optional[Any] = None) -> None:
        """`x_part`: this rank's columns [k0, k1) of x ([m, k1 - k0]) -- the
        output of the column-split product before it, as it is."""
        import torch.distributed as dist

        ops.linear(x_part, self.weight, out)
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)


def max_over_ranks(value: float, device=None, group: Optional[Any] = None) -> float:
    """The largest of every rank's `value` (a multi-GPU time is the slowest
    rank's)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class VocabSampler:
    """The greedy choice of the next token with the lm-head split by
    vocabulary rows: each rank's argmax over its rows [offset, offset +
    rows) as (value, id) pairs -- the id global, so the reference's rule for
    a NaN at id 0 holds across shards -- one all-gather of the pairs (ids and
    value bits in one int32 tensor), then every rank merges the same pairs
    and picks the same ids (SequenceOps.argmax, CpuSequence.scala:12-22, over
    the whole vocabulary). On one rank: the argmax itself.

    `ops` supplies argmax(values, ids, out_values, id_offset) and
    argmax_merge(values, ids_in, ids, out_values) (CudaOps on a GPU); the
    gathers are torch.distributed's (NCCL, capturable in a CUDA graph)."""

    def __init__(self, ops: Any, batch: int, offset: int, group: Optional[Any] = None,
                 device=None):
        import torch
        import torch.distributed as dist

        self.ops, self.batch, self.offset, self.group = ops, batch, offset, group
        self.world = dist.get_world_size(group) if group is not None else 1
        if self.world > 1:
            # [2, batch]: row 0 the ids, row 1 the values' bits
            self.local = torch.zeros(2, batch, dtype=torch.int32, device=device)
            # the ranks' pairs one after the other: [world * 2, batch]
            self.gathered = torch.zeros(self.world * 2, batch, dtype=torch.int32, device=device)

    def __call__(self, logits, out_ids) -> None:
        """out_ids [batch] (int32) <- each row's argmax over the whole vocabulary."""
        import torch.distributed as dist

        if self.world == 1:
            self.ops.argmax(logits, out_ids, None, self.offset)
            return
        import torch

        values = self.local[1].view(torch.float32)
        self.ops.argmax(logits, self.local[0], values, self.offset)
        dist.all_gather_into_tensor(self.gathered, self.local, group=self.group)
        pairs = self.gathered.view(self.world, 2, self.batch).permute(1, 2, 0).contiguous()
        # pairs: [2, batch, world]
        self.ops.argmax_merge(pairs[1].view(torch.float32), pairs[0], out_ids, None)


class _DeviceArray:
    """A CUDA array interface over memory this library allocated, so torch
    can view it without a copy."""

    def __init__(self, pointer: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (pointer, False), "version": 3}


class PeerExchange:
    """The decode step's exchange over NVLink peer memory (the library's
    drift_comm_*): two slots of `rows` x `cols` F32 partial rows per rank,
    readable by every rank of `group`; `add_rms_norm` sums the ranks'
    partials of a slot in rank order into x and normalises, in one launch.
    Consecutive exchanges alternate slots (o, then down). A row waits for
    its peers at most `wait_limit_ns` (0: one second); a wait that runs out
    sets device error 3 and leaves the row as it was, and the exchange must
    then be closed on every rank."""

    def __init__(self, ops, group, rows: int, cols: int, wait_limit_ns: int = 0):
        import ctypes

        import torch
        import torch.distributed as dist

        from ._lib import check

        self.ops, self.lib = ops, ops.lib
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        comm = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(self.lib.drift_comm_handle_bytes())
        check("drift_comm_create", self.lib.drift_comm_create(rank, world, rows * cols * 4,
                                                              wait_limit_ns, ctypes.byref(comm),
                                                              handle))
        self.comm = comm
        handles: list = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        joined = ctypes.create_string_buffer(b"".join(handles), len(handle.raw) * world)
        check("drift_comm_open", self.lib.drift_comm_open(comm, joined))
        self.slots = []
        for slot in range(2):
            pointer = ctypes.c_void_p()
            check("drift_comm_slot", self.lib.drift_comm_slot(comm, slot, ctypes.byref(pointer)))
            self.slots.append(torch.as_tensor(_DeviceArray(pointer.value, (rows, cols)),
                                              device="cuda"))
        dist.barrier(group=group)

    def add_rms_norm(self, slot: int, x, norm, prepared=None) -> None:
        """x += the sum over ranks of slot `slot` (rank order); norm.out =
        rmsNorm(x) (and its records into `prepared`)."""
        from ._lib import check

        rows, cols = x.shape
        status = self.lib.drift_add_rms_norm_allreduce(
            self.comm, slot, x.data_ptr(), norm.weight.data_ptr(), norm.epsilon,
            norm.weight_offset, norm.out.data_ptr(), rows, cols,
            None if prepared is None else prepared.data_ptr(), self.ops._stream())
        check("drift_add_rms_norm_allreduce", status)

    def close(self) -> None:
        if self.comm:
            self.slots = []
            self.lib.drift_comm_destroy(self.comm)
            self.comm = None

