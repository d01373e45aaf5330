"""Operators on host-resident operands, streamed through the GPU.

The reference runs `gemm` on CPU tensors with its scalar loop (titan-runtime/src/lib.rs:
955-989), and its CUDA path uploads every input, runs the kernel and downloads the
result one after the other (Tensor::from_slice / to_vec, titan-tensor/src/lib.rs:
215-260). For operands that live in host memory this module overlaps the three: B is
uploaded first (every row block of C needs all of it), then A in row blocks, each
block's GEMM starting as soon as its rows have landed and each block of C going back
to the host while later blocks compute. One call is one `C = A · Bᵀ` (bf16, B stored
[N, K], fp32 accumulation, the `transpose_rhs` GEMM of `tb_op_gemm`); consecutive
calls pipeline as well: the next call's uploads start while this call's last blocks
compute and download (B alternates between two device buffers).

Each row block runs the same operator (`tb_op_gemm`) on views of one device A and one
device C, so a block's rows are computed exactly as the whole GEMM computes them when
the operator picks the same kernel for the block. Host buffers must be page-locked
(`Session.host_alloc`): the copies are asynchronous and the caller keeps them alive
until the call's work on `stream` is done. An instance keeps the events of its previous
call to order the next one, so one host thread drives it at a time.

`StreamedBatchOp` does the same for an operator whose output rows are independent over
a leading batch dimension (attention over [B, H, T, D], conv2d over NHWC images): the
batched inputs go up in batch blocks, each block runs through the native router
(`tb_execute`, the Runtime::execute of titan-runtime/src/lib.rs:1171-1256) on views of
the device tensors, and each block of the output comes back while later blocks run;
inputs without a batch dimension (the conv weights) go up once per call.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import numpy as np

from . import _native as native
from .hal import Event, PinnedHost, Session, Stream, _check
from .kernel_abi import DType, scalar_width
from .runtime import _attrs, c_tensor, contiguous_strides


def split_rows(rows: int, blocks: int, unit: int = 256):
    """Splits `rows` into at most `blocks` consecutive (first row, rows) blocks, each a
    multiple of `unit` rows (but the last) when rows >= unit * blocks."""
    if rows <= 0 or blocks <= 0:
        raise ValueError("split_rows needs positive rows and blocks")
    u = unit if rows >= unit * blocks else 1
    base = -(-rows // blocks)
    step = -(-base // u) * u
    return [(r0, min(step, rows - r0)) for r0 in range(0, rows, step)]


class StreamedGemm:
    """C[M, N] = A[M, K] · B[N, K]ᵀ from and to page-locked host buffers.

    `row_blocks` splits M into at most that many blocks (multiples of 256 rows where M
    allows, so each block still fills the GPU with 256-row CTA-pair tiles)."""

    def __init__(self, session: Session, M: int, N: int, K: int, row_blocks: int = 4):
        if min(M, N, K) <= 0:
            raise ValueError("StreamedGemm needs positive M, N and K")
        self.s, self.M, self.N, self.K = session, M, N, K
        self.blocks = split_rows(M, row_blocks)
        self.da = session.allocate(M * K * 2)
        self.db = [session.allocate(N * K * 2), session.allocate(N * K * 2)]
        self.dc = session.allocate(M * N * 2)
        self._views = []  # the wrapped buffers must outlive their tensors
        self.ta, self.tc = [], []
        for r0, n in self.blocks:
            va = session.wrap(self.da.device_ptr + r0 * K * 2, n * K * 2)
            vc = session.wrap(self.dc.device_ptr + r0 * N * 2, n * N * 2)
            self._views += [va, vc]
            self.ta.append(c_tensor(va, DType.BF16, (n, K), contiguous_strides((n, K))))
            self.tc.append(c_tensor(vc, DType.BF16, (n, N), contiguous_strides((n, N))))
        self.tb = [c_tensor(b, DType.BF16, (N, K), contiguous_strides((N, K))) for b in self.db]
        self.up = session.create_stream()    # host -> device copies, in the order they are needed
        self.down = session.create_stream()  # device -> host copies of finished row blocks
        self._key = b"transpose_rhs"
        self.attrs = (native.Attr * 1)()
        self.attrs[0].key = self._key
        self.attrs[0].value = 1
        nb = len(self.blocks)
        self._gemm_done: List[Optional[Event]] = [None] * nb  # block i's A and C views are in use until then
        self._down_done: List[Optional[Event]] = [None] * nb
        self._b_free: List[Optional[Event]] = [None, None]
        self.calls = 0

    def run(self, stream: Stream, a: PinnedHost, b: PinnedHost, c: PinnedHost, after: Optional[Event] = None) -> None:
        """Enqueues one call on `stream`: when `stream` reaches the end of it, C is in `c`.
        `after`: an event the uploads wait for (e.g. the start of a timed region)."""
        s, M, Nn, K = self.s, self.M, self.N, self.K
        if a.nbytes < M * K * 2 or b.nbytes < Nn * K * 2 or c.nbytes < M * Nn * 2:
            raise ValueError("host buffers smaller than the GEMM's operands")
        slot = self.calls & 1
        if after is not None:
            s.wait_event(self.up, after)
        if self._b_free[slot] is not None:
            s.wait_event(self.up, self._b_free[slot])  # the GEMMs of two calls ago read this B
        s.upload_pinned(self.up, self.db[slot], b, nbytes=Nn * K * 2)
        s.wait_event(stream, s.record(self.up))
        lib = native.lib()
        for i, (r0, n) in enumerate(self.blocks):
            if self._gemm_done[i] is not None:
                s.wait_event(self.up, self._gemm_done[i])  # the previous call's block i has read its A rows
            s.upload_pinned(self.up, self.da, a, nbytes=n * K * 2, dst_offset=r0 * K * 2, src_offset=r0 * K * 2)
            s.wait_event(stream, s.record(self.up))
            if self._down_done[i] is not None:
                s.wait_event(stream, self._down_done[i])  # the previous call's block i of C is on the host
            _check(lib.tb_op_gemm(s.ptr, stream.ptr, ctypes.byref(self.ta[i]), ctypes.byref(self.tb[slot]),
                                  ctypes.byref(self.tc[i]), self.attrs, 1, None))
            done = s.record(stream)
            self._gemm_done[i] = done
            s.wait_event(self.down, done)
            s.download_pinned(self.down, self.dc, c, nbytes=n * Nn * 2, src_offset=r0 * Nn * 2,
                              dst_offset=r0 * Nn * 2)
            self._down_done[i] = s.record(self.down)
        self._b_free[slot] = s.record(stream)
        s.wait_event(stream, self._down_done[-1])  # the call ends on `stream` once C is back on the host
        self.calls += 1

    def h2d_bytes(self) -> int:
        return (self.M + self.N) * self.K * 2

    def d2h_bytes(self) -> int:
        return self.M * self.N * 2


class StreamedBatchOp:
    """One operator over a leading batch dimension, inputs and output in page-locked host
    memory. `inputs`: (dtype, shape, batched) per operator input, in the operator's order;
    `output`: (dtype, shape), batch leading. The batch splits into at most `blocks` blocks."""

    def __init__(self, session: Session, operator: str, inputs, output, attrs: Optional[dict] = None,
                 blocks: int = 4):
        self.s, self.op = session, operator
        out_dtype, out_shape = output
        batch = int(out_shape[0])
        if batch <= 0:
            raise ValueError("StreamedBatchOp needs a positive batch")
        self.blocks = split_rows(batch, blocks, unit=1)
        self._keep = []  # wrapped views must outlive their tensors
        self.inputs = []  # per input: (batched, item_bytes or total bytes, device buffers, per-block tensors)
        for dtype, shape, batched in inputs:
            shape = tuple(int(x) for x in shape)
            nbytes = int(np.prod(shape)) * scalar_width(dtype)
            if batched:
                if shape[0] != batch:
                    raise ValueError("a batched input's leading dimension must equal the output's")
                item = nbytes // batch
                dev = session.allocate(nbytes)
                per_block = [self._view(dev, b0 * item, n * item, dtype, (n,) + shape[1:]) for b0, n in self.blocks]
                self.inputs.append((True, item, [dev], per_block))
            else:
                devs = [session.allocate(nbytes), session.allocate(nbytes)]  # alternate between calls
                whole = [c_tensor(d, dtype, shape, contiguous_strides(shape)) for d in devs]
                self.inputs.append((False, nbytes, devs, whole))
        out_shape = tuple(int(x) for x in out_shape)
        self.out_item = int(np.prod(out_shape)) * scalar_width(out_dtype) // batch
        self.dout = session.allocate(self.out_item * batch)
        self.outs = [self._view(self.dout, b0 * self.out_item, n * self.out_item, out_dtype, (n,) + out_shape[1:])
                     for b0, n in self.blocks]
        self.attrs, self.n_attrs, self._attr_keep = _attrs(dict(attrs or {}))
        self.up = session.create_stream()
        self.down = session.create_stream()
        nb = len(self.blocks)
        self._op_done: List[Optional[Event]] = [None] * nb
        self._down_done: List[Optional[Event]] = [None] * nb
        self._shared_free: List[Optional[Event]] = [None, None]
        self.calls = 0

    def _view(self, dev, offset, nbytes, dtype, shape):
        v = self.s.wrap(dev.device_ptr + offset, nbytes)
        self._keep.append(v)
        return c_tensor(v, dtype, shape, contiguous_strides(shape))

    def run(self, stream: Stream, hosts, out: PinnedHost, after: Optional[Event] = None) -> None:
        """Enqueues one call on `stream` (inputs: one PinnedHost per operator input, in
        order); when `stream` reaches its end, the output is in `out`."""
        s = self.s
        if len(hosts) != len(self.inputs):
            raise ValueError("one host buffer per operator input")
        for (batched, size, _, _), h in zip(self.inputs, hosts):
            if h.nbytes < (size * self.blocks[-1][0] + size * self.blocks[-1][1] if batched else size):
                raise ValueError("host buffer smaller than its operand")
        if out.nbytes < self.out_item * (self.blocks[-1][0] + self.blocks[-1][1]):
            raise ValueError("host output buffer smaller than the output")
        slot = self.calls & 1
        if after is not None:
            s.wait_event(self.up, after)
        if self._shared_free[slot] is not None:
            s.wait_event(self.up, self._shared_free[slot])  # the operators of two calls ago read these
        for (batched, size, devs, _), h in zip(self.inputs, hosts):
            if not batched:
                s.upload_pinned(self.up, devs[slot], h, nbytes=size)
        s.wait_event(stream, s.record(self.up))
        lib = native.lib()
        for i, (b0, n) in enumerate(self.blocks):
            if self._op_done[i] is not None:
                s.wait_event(self.up, self._op_done[i])  # the previous call's block i has read its inputs
            for (batched, item, devs, _), h in zip(self.inputs, hosts):
                if batched:
                    s.upload_pinned(self.up, devs[0], h, nbytes=n * item, dst_offset=b0 * item, src_offset=b0 * item)
            s.wait_event(stream, s.record(self.up))
            if self._down_done[i] is not None:
                s.wait_event(stream, self._down_done[i])  # the previous call's output block is on the host
            ins = (native.Tensor * len(self.inputs))(*[t[i] if batched else t[slot]
                                                       for batched, _, _, t in self.inputs])
            ev = ctypes.c_void_p(0)
            _check(lib.tb_execute(s.ptr, stream.ptr, self.op.encode(), ins, len(self.inputs),
                                  ctypes.byref(self.outs[i]), self.attrs, self.n_attrs, ctypes.byref(ev)))
            if ev.value:
                Event(s, ev.value)  # released when this wrapper goes away
            done = s.record(stream)
            self._op_done[i] = done
            s.wait_event(self.down, done)
            s.download_pinned(self.down, self.dout, out, nbytes=n * self.out_item, src_offset=b0 * self.out_item,
                              dst_offset=b0 * self.out_item)
            self._down_done[i] = s.record(self.down)
        self._shared_free[slot] = s.record(stream)
        s.wait_event(stream, self._down_done[-1])
        self.calls += 1

    def h2d_bytes(self) -> int:
        batch = self.blocks[-1][0] + self.blocks[-1][1]
        return sum(size * batch if batched else size for batched, size, _, _ in self.inputs)

    def d2h_bytes(self) -> int:
        return self.out_item * (self.blocks[-1][0] + self.blocks[-1][1])
