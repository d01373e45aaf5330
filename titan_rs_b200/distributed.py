"""Distributed contracts for the hot path: the titan.rs `Collective` trait
(projects/titan-distributed/src/lib.rs:95-99) and the B200 implementation that runs
its all_gather over NCCL/NVLink on device buffers, in place of the reference's
in-process transport, plus the N-sharded GEMM built on it.

Sharding of the north-star configurations (one process per GPU):
  GEMM    rank r owns output columns [r*N/p, (r+1)*N/p); B (column-major, stored
          [N, K]) is sharded by rows, A is replicated; C is re-assembled with an
          all-gather of the [M, N/p] blocks.
  SDPA    batch*heads split evenly, no communication.
  conv2d  batch split evenly, weights replicated, no communication.
"""
from __future__ import annotations

import ctypes
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


class Collective:
    """The `Collective` trait (projects/titan-distributed/src/lib.rs:95-99) over host shards."""

    def all_reduce_sum(self, shards: Sequence[Sequence[float]]) -> list:
        raise NotImplementedError

    def reduce_scatter_sum(self, shards: Sequence[Sequence[float]]) -> list:
        raise NotImplementedError

    def all_gather(self, shards: Sequence[Sequence[float]]) -> list:
        raise NotImplementedError


# ----------------------------------------------------------------------------- sharding
def even_shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's even share of `total` units; total must divide by world."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if total % world:
        raise ValueError(f"{total} units do not split evenly over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def shard_units(units: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's share of `units` independent units; the first
    units % world ranks take one unit more, so any count splits."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(int(units), world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _view(session, handle, first: int, count: int, unit_elems: int, shape):
    from .runtime import TensorHandle, _SIZE, contiguous_strides
    esize = _SIZE[handle.dtype]
    if tuple(handle.strides) != contiguous_strides(handle.shape):
        raise ValueError("sharded operands must be contiguous")
    nbytes = max(count * unit_elems * esize, esize)
    buf = session.wrap(handle.buffer.device_ptr + first * unit_elems * esize, nbytes)
    return TensorHandle(session, buf, handle.dtype, tuple(shape), contiguous_strides(shape))


def local_request(request, world: int, rank: int):
    """Rank r's part of an operator request that shards without communication.

    scaled_dot_product_attention shards over batch x heads: Q [B,H,Tq,D] and K, V
    [B,H,Tk,D] become views [1, n, T, D] of the rank's n = hi - lo (b, h) pairs, and
    the output spec is [1, n, Tq, D]. conv2d shards over the batch: x (NHWC or NCHW)
    becomes the rank's images, the weights and bias stay whole, and the output spec
    covers those images. The views alias the caller's buffers (no copy), so the
    inputs may be whole on every rank or hold just this rank's units at the same
    offsets. Returns (request, (lo, hi)); a rank with no units gets hi == lo and
    should skip the launch."""
    from .runtime import OpRequest, TensorSpec
    op = request.operator
    spec = request.outputs[0]
    if op == "scaled_dot_product_attention":
        q, k, v = request.inputs[:3]
        b, h, tq, d = q.shape
        tk = k.shape[2]
        lo, hi = shard_units(b * h, world, rank)
        n = hi - lo
        s = q.session
        ins = [_view(s, q, lo, n, tq * d, (1, n, tq, d)), _view(s, k, lo, n, tk * d, (1, n, tk, d)),
               _view(s, v, lo, n, tk * d, (1, n, tk, v.shape[3]))]
        out = TensorSpec(spec.dtype, (1, n, tq, spec.shape[3]))
    elif op == "conv2d":
        x = request.inputs[0]
        lo, hi = shard_units(x.shape[0], world, rank)
        n = hi - lo
        per = int(np.prod(x.shape[1:], dtype=np.int64))
        ins = [_view(x.session, x, lo, n, per, (n,) + tuple(x.shape[1:]))] + list(request.inputs[1:])
        out = TensorSpec(spec.dtype, (n,) + tuple(spec.shape[1:]))
    else:
        raise ValueError(f"{op} does not shard without communication (gemm shards through the collective)")
    return OpRequest(op, ins, [out], dict(request.attrs)), (lo, hi)


def execute_local(runtime, request, world: int, rank: int):
    """Runs rank r's units of `request` (see local_request) on this rank's Runtime.
    Returns (ExecutionHandle or None when the rank has no units, (lo, hi))."""
    local, bounds = local_request(request, world, rank)
    if bounds[1] == bounds[0]:
        return None, bounds
    return runtime.execute(local), bounds


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


__all__ = ["CollectiveError", "Collective", "ProcessGroupCollective", "even_shard", "shard_units", "local_request",
           "execute_local", "reassemble_column_blocks", "new_comm_id", "broadcast_comm_id", "NcclCollective",
           "HalError"]
