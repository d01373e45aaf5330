"""Distributed contracts for the hot path: the titan.rs `Collective` trait and
its in-process transport (projects/titan-distributed/src/lib.rs:4-135), plus the
B200 implementation that runs the trait's all_gather over NCCL/NVLink on device
buffers and the N-sharded GEMM built on it.

Sharding of the north-star configurations (one process per GPU):
  GEMM    rank r owns output columns [r*N/p, (r+1)*N/p); B (column-major, stored
          [N, K]) is sharded by rows, A is replicated; C is re-assembled with an
          all-gather of the [M, N/p] blocks.
  SDPA    batch*heads split evenly, no communication.
  conv2d  batch split evenly, weights replicated, no communication.
"""
from __future__ import annotations

import ctypes
import datetime
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _native as N
from .hal import Buffer, HalError, Session, Stream, _check


# ----------------------------------------------------------------------------- reference mirror
class CollectiveError(RuntimeError):
    """CollectiveError (projects/titan-distributed/src/lib.rs:4-16); `kind` is the variant name."""

    def __init__(self, kind: str, detail: str = ""):
        super().__init__(f"collective failed: {kind}" + (f" ({detail})" if detail else ""))
        self.kind = kind


def checksum(data: bytes) -> str:
    """FNV-1a 64 rendered as 16 hex digits (projects/titan-distributed/src/lib.rs:24-32)."""
    h = 0xCBF29CE484222325
    for b in data:
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return f"{h:016x}"


@dataclass
class LocalFrame:
    run_id: str
    epoch: int
    sequence: int
    payload: bytes
    checksum: str


class LocalTransport:
    """Run/epoch/sequence/checksum/timeout framing (projects/titan-distributed/src/lib.rs:44-93)."""

    def __init__(self, run_id: str, epoch: int, timeout: datetime.timedelta):
        self.run_id, self.epoch, self.next_sequence, self.timeout = run_id, epoch, 0, timeout

    def send(self, payload: bytes, timeout: datetime.timedelta) -> LocalFrame:
        if timeout.total_seconds() <= 0 or self.timeout.total_seconds() <= 0:
            raise CollectiveError("Timeout")
        frame = LocalFrame(self.run_id, self.epoch, self.next_sequence, bytes(payload), checksum(bytes(payload)))
        self.next_sequence += 1
        return frame

    def receive(self, frame: LocalFrame, timeout: datetime.timedelta) -> bytes:
        if timeout.total_seconds() <= 0 or self.timeout.total_seconds() <= 0:
            raise CollectiveError("Timeout")
        if frame.run_id != self.run_id:
            raise CollectiveError("RunMismatch")
        if frame.epoch != self.epoch:
            raise CollectiveError("EpochMismatch")
        if frame.sequence != self.next_sequence:
            raise CollectiveError("SequenceMismatch")
        if checksum(frame.payload) != frame.checksum:
            raise CollectiveError("ChecksumMismatch")
        self.next_sequence += 1
        return frame.payload


class Collective:
    """The `Collective` trait (projects/titan-distributed/src/lib.rs:95-99) over host shards."""

    def all_reduce_sum(self, shards: Sequence[Sequence[float]]) -> list:
        raise NotImplementedError

    def reduce_scatter_sum(self, shards: Sequence[Sequence[float]]) -> list:
        raise NotImplementedError

    def all_gather(self, shards: Sequence[Sequence[float]]) -> list:
        raise NotImplementedError


class LocalRing(Collective):
    """In-process reference implementation (projects/titan-distributed/src/lib.rs:101-135)."""

    def all_reduce_sum(self, shards):
        if not shards:
            raise CollectiveError("EmptyWorld")
        n = len(shards[0])
        if any(len(s) != n for s in shards):
            raise CollectiveError("InconsistentLengths")
        total = np.zeros(n, dtype=np.float32)
        for s in shards:
            total += np.asarray(s, dtype=np.float32)
        return total.tolist()

    def reduce_scatter_sum(self, shards):
        total = self.all_reduce_sum(shards)
        if len(total) % len(shards):
            raise CollectiveError("InconsistentLengths")
        w = len(total) // len(shards)
        return [total[i:i + w] for i in range(0, len(total), w)]

    def all_gather(self, shards):
        if not shards:
            raise CollectiveError("EmptyWorld")
        return [float(x) for s in shards for x in s]


# ----------------------------------------------------------------------------- sharding
def even_shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's even share of `total` units; total must divide by world."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if total % world:
        raise ValueError(f"{total} units do not split evenly over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def reassemble_column_blocks(gathered: np.ndarray, parts: int) -> np.ndarray:
    """Host restatement of the device re-layout after the sharded GEMM's all-gather:
    [p, M, N/p] column blocks -> row-major [M, N]."""
    p, m, np_ = gathered.shape
    assert p == parts
    return np.ascontiguousarray(gathered.transpose(1, 0, 2).reshape(m, p * np_))


class ProcessGroupCollective(Collective):
    """The trait across processes: each rank passes only ITS shard and receives the
    rank-ordered result (torch.distributed, gloo on CPU). Collective calls fail with
    an error after the process group's timeout if a peer is gone."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group

    def all_gather(self, shards):
        if len(shards) != 1:
            raise CollectiveError("InconsistentLengths", "pass exactly this rank's shard")
        import torch
        local = torch.tensor(np.asarray(shards[0], dtype=np.float32))
        world = self.dist.get_world_size(self.group)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        self.dist.all_gather(sizes, torch.tensor([local.numel()]), group=self.group)
        if any(int(s) != local.numel() for s in sizes):
            raise CollectiveError("InconsistentLengths")
        out = [torch.empty_like(local) for _ in range(world)]
        self.dist.all_gather(out, local, group=self.group)
        return torch.cat(out).tolist()

    def all_reduce_sum(self, shards):
        import torch
        if len(shards) != 1:
            raise CollectiveError("InconsistentLengths", "pass exactly this rank's shard")
        t = torch.tensor(np.asarray(shards[0], dtype=np.float32))
        self.dist.all_reduce(t, group=self.group)
        return t.tolist()

    def reduce_scatter_sum(self, shards):
        total = self.all_reduce_sum(shards)
        world = self.dist.get_world_size(self.group)
        if len(total) % world:
            raise CollectiveError("InconsistentLengths")
        w = len(total) // world
        r = self.dist.get_rank(self.group)
        return [total[r * w:(r + 1) * w]]


# ----------------------------------------------------------------------------- device (NCCL)
def new_comm_id() -> bytes:
    buf = (ctypes.c_uint8 * N.TB_COMM_ID_BYTES)()
    _check(N.lib().tb_comm_unique_id(buf))
    return bytes(buf)


def broadcast_comm_id(rank: int) -> bytes:
    """Rank 0 creates the NCCL id; torch.distributed (any backend) carries it to every rank."""
    import torch.distributed as dist
    obj = [new_comm_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


class NcclCollective:
    """`Collective::all_gather` on device buffers over NCCL (tb_comm_*)."""

    def __init__(self, session: Session, comm_id: bytes, world: int, rank: int, timeout_ms: int = 60000):
        self.session = session
        self.world, self.rank = world, rank
        cid = (ctypes.c_uint8 * N.TB_COMM_ID_BYTES).from_buffer_copy(comm_id)
        h = ctypes.c_void_p(0)
        _check(N.lib().tb_comm_init(session.ptr, cid, world, rank, timeout_ms, ctypes.byref(h)))
        self.ptr = h.value

    def all_gather(self, stream: Stream, send: Buffer, recv: Buffer, bytes_per_rank: int) -> None:
        _check(N.lib().tb_comm_all_gather(self.ptr, stream.ptr, send.ptr, recv.ptr, bytes_per_rank, None))

    def barrier(self, stream: Stream) -> None:
        _check(N.lib().tb_comm_barrier(self.ptr, stream.ptr))

    def register_buffer(self, stream: Stream, buffer: Buffer) -> None:
        """Collective: map every rank's `buffer` into every other rank (CUDA IPC over NVLink)."""
        _check(N.lib().tb_comm_register_buffer(self.ptr, stream.ptr, buffer.ptr))

    def deregister_buffer(self, buffer: Buffer) -> None:
        _check(N.lib().tb_comm_deregister_buffer(self.ptr, buffer.ptr))

    def sharded_gemm(self, stream: Stream, a, b_shard, c, workspace: Buffer | None) -> None:
        """C = A B^T with B's rows (output columns) sharded over the ranks; C complete on every rank.

        With C's buffer registered on every rank (`register_buffer`) one fused kernel
        stores this rank's columns into all ranks' C over NVLink and `workspace` may be
        None; otherwise the GEMM fills a workspace slot that NCCL all-gathers."""
        ta, tb_, tc = a.c_tensor(), b_shard.c_tensor(), c.c_tensor()
        _check(N.lib().tb_op_gemm_sharded(self.ptr, stream.ptr, ctypes.byref(ta), ctypes.byref(tb_),
                                          ctypes.byref(tc), workspace.ptr if workspace is not None else None, None))

    def close(self) -> None:
        if self.ptr:
            N.lib().tb_comm_release(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["CollectiveError", "checksum", "LocalFrame", "LocalTransport", "Collective", "LocalRing",
           "ProcessGroupCollective", "even_shard", "reassemble_column_blocks", "new_comm_id", "broadcast_comm_id",
           "NcclCollective", "HalError"]
