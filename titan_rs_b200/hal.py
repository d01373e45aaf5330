"""HAL session over libtitan_b200: the titan.rs `BackendDriver` / `DeviceSession`
contract (projects/titan-hal/src/lib.rs:200-237) for a B200.

Every method maps one-to-one onto a C entry point in include/titan_b200.h and
raises HalError(operation, detail) with the reference's vocabulary when the
native call fails.
"""
from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _native as N
from .kernel_abi import EncodedLaunchArgs


class HalError(RuntimeError):
    """HalError{operation, detail} (projects/titan-hal/src/lib.rs:9-14) plus the C status code."""

    def __init__(self, status: int, operation: str, detail: str):
        super().__init__(f"{operation}: {detail}")
        self.status = status
        self.operation = operation
        self.detail = detail


def _check(status: int) -> None:
    if status != N.TB_OK:
        op, detail = N.last_error()
        raise HalError(status, op, detail)


def last_candidate() -> str:
    """Name of the kernel the calling thread's most recent operator launched."""
    return (N.lib().tb_last_candidate() or b"").decode()


def launch_count() -> int:
    """Kernels this library has launched in the process so far (tb_launch_count)."""
    return int(N.lib().tb_launch_count())


def driver_available() -> bool:
    """True when libcuda loads and reports devices (the reference's no_cuda_environment inverse)."""
    try:
        return N.lib().tb_driver_open() == N.TB_OK
    except N.NativeLibraryMissing:
        return False


def enumerate_devices() -> list[dict]:
    L = N.lib()
    _check(L.tb_driver_open())
    count = ctypes.c_uint32(0)
    _check(L.tb_driver_enumerate(None, 0, ctypes.byref(count)))
    arr = (N.Fingerprint * max(count.value, 1))()
    _check(L.tb_driver_enumerate(arr, count.value, ctypes.byref(count)))
    return [_fp_dict(arr[i]) for i in range(count.value)]


def _fp_dict(fp: N.Fingerprint) -> dict:
    return {"ordinal": fp.ordinal, "model": fp.model.decode(), "driver": fp.driver.decode(),
            "capability_revision": fp.capability_revision.decode(), "sm_count": fp.sm_count,
            "total_memory": fp.total_memory}


_RELEASE_LOCK = threading.Lock()


class _Handle:
    _release = None

    def __init__(self, session: "Session", ptr: int):
        self.session = session
        self.ptr = ptr

    def release(self) -> None:
        # Handles may be dropped from any thread (the session is Send + Sync): take the
        # pointer under a lock so two threads never release the same handle.
        with _RELEASE_LOCK:
            ptr, self.ptr = self.ptr, 0
        if ptr:
            getattr(N.lib(), self._release)(ptr)

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    @property
    def _as_parameter_(self):
        return ctypes.c_void_p(self.ptr)


class Buffer(_Handle):
    _release = "tb_buffer_release"

    @property
    def byte_len(self) -> int:
        return int(N.lib().tb_buffer_byte_len(self.ptr))

    @property
    def identity(self) -> int:
        return int(N.lib().tb_buffer_identity(self.ptr))

    @property
    def device_ptr(self) -> int:
        return int(N.lib().tb_buffer_device_ptr(self.ptr))


class Stream(_Handle):
    _release = "tb_stream_release"

    @property
    def handle(self) -> int:
        return int(N.lib().tb_stream_handle(self.ptr))


class Event(_Handle):
    _release = "tb_event_release"


class GraphExec(_Handle):
    """A captured CUDA graph of a session's device work (tb_capture_begin / tb_capture_end);
    launch() replays it on a stream with one launch."""
    _release = "tb_graph_exec_release"

    def launch(self, stream: "Stream") -> None:
        _check(N.lib().tb_graph_exec_launch(self.session.ptr, self.ptr, stream.ptr))


class LoadedKernel(_Handle):
    _release = "tb_kernel_release"

    def __init__(self, session, ptr, abi_hash: str, entry: str):
        super().__init__(session, ptr)
        self.abi_hash = abi_hash
        self.entry = entry


@dataclass
class LaunchGeometry:
    """LaunchGeometry (projects/titan-hal/src/lib.rs:193-197)."""
    grid: tuple
    block: tuple
    shared_bytes: int = 0


def _out() -> ctypes.c_void_p:
    return ctypes.c_void_p(0)


class Session:
    """DeviceSession on one GPU's primary context."""

    def __init__(self, ordinal: int = 0):
        L = N.lib()
        _check(L.tb_driver_open())
        h = _out()
        _check(L.tb_session_open(ordinal, ctypes.byref(h)))
        self.ptr = h.value
        self.ordinal = ordinal

    def close(self) -> None:
        if self.ptr:
            N.lib().tb_session_release(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def _as_parameter_(self):
        return ctypes.c_void_p(self.ptr)

    def fingerprint(self) -> dict:
        fp = N.Fingerprint()
        _check(N.lib().tb_session_fingerprint(self.ptr, ctypes.byref(fp)))
        return _fp_dict(fp)

    # ---- DeviceSession ----
    def allocate(self, nbytes: int, alignment: int = 256) -> Buffer:
        h = _out()
        _check(N.lib().tb_allocate(self.ptr, nbytes, alignment, ctypes.byref(h)))
        return Buffer(self, h.value)

    def wrap(self, device_ptr: int, nbytes: int) -> Buffer:
        h = _out()
        _check(N.lib().tb_buffer_wrap(self.ptr, device_ptr, nbytes, ctypes.byref(h)))
        return Buffer(self, h.value)

    def create_stream(self) -> Stream:
        h = _out()
        _check(N.lib().tb_create_stream(self.ptr, ctypes.byref(h)))
        return Stream(self, h.value)

    def create_event(self) -> Event:
        h = _out()
        _check(N.lib().tb_create_event(self.ptr, ctypes.byref(h)))
        return Event(self, h.value)

    def upload(self, stream: Stream, dst: Buffer, src) -> Event:
        data = memoryview(np.ascontiguousarray(src)).cast("B")
        c = (ctypes.c_uint8 * len(data)).from_buffer_copy(data) if len(data) else None
        h = _out()
        _check(N.lib().tb_upload(self.ptr, stream.ptr, dst.ptr, c, len(data), ctypes.byref(h)))
        return Event(self, h.value)

    def download(self, stream: Stream, src: Buffer, dst: np.ndarray) -> Event:
        if not dst.flags["C_CONTIGUOUS"]:
            raise ValueError("download destination must be contiguous")
        h = _out()
        _check(N.lib().tb_download(self.ptr, stream.ptr, src.ptr, dst.ctypes.data_as(ctypes.c_void_p), dst.nbytes,
                                   ctypes.byref(h)))
        return Event(self, h.value)

    def copy(self, stream: Stream, dst: Buffer, src: Buffer, nbytes: int) -> Event:
        h = _out()
        _check(N.lib().tb_copy(self.ptr, stream.ptr, dst.ptr, src.ptr, nbytes, ctypes.byref(h)))
        return Event(self, h.value)

    def load(self, artifact: bytes, abi_hash: str, metadata: dict) -> LoadedKernel:
        kinds = {"buffer": N.TB_ARG_BUFFER, "scalar": N.TB_ARG_SCALAR, "shape": N.TB_ARG_SHAPE}
        args = (N.LaunchArg * max(len(metadata["arguments"]), 1))()
        for i, (kind, width) in enumerate(metadata["arguments"]):
            args[i].kind = kinds[kind]
            args[i].width = width
        md = N.LaunchMetadata()
        md.version = metadata.get("version", 1)
        md.entry = metadata["entry"].encode()
        md.arguments = args
        md.num_arguments = len(metadata["arguments"])
        for i, v in enumerate(metadata.get("block", (1, 1, 1))):
            md.block[i] = v
        md.shared_bytes = metadata.get("shared_bytes", 0)
        blob = (ctypes.c_uint8 * len(artifact)).from_buffer_copy(artifact)
        h = _out()
        _check(N.lib().tb_load(self.ptr, blob, len(artifact), abi_hash.encode(), ctypes.byref(md), ctypes.byref(h)))
        return LoadedKernel(self, h.value, abi_hash, metadata["entry"])

    def launch(self, stream: Stream, kernel: LoadedKernel, args: EncodedLaunchArgs,
               geometry: LaunchGeometry) -> Event:
        payload = (ctypes.c_uint8 * max(len(args.payload), 1)).from_buffer_copy(args.payload or b"\0")
        canon = (ctypes.c_uint8 * max(len(args.canonical_abi), 1)).from_buffer_copy(args.canonical_abi or b"\0")
        binds = (N.Binding * max(len(args.bindings), 1))()
        for i, (slot, (buf, owner)) in enumerate(sorted(args.bindings.items())):
            binds[i].slot = slot
            binds[i].buffer = buf.ptr
            binds[i].owner = owner.ptr if owner is not None else None
        enc = N.EncodedArgs(payload, len(args.payload), binds, len(args.bindings), canon, len(args.canonical_abi))
        geo = N.LaunchGeometry()
        for i in range(3):
            geo.grid[i] = geometry.grid[i] if i < len(geometry.grid) else 1
            geo.block[i] = geometry.block[i] if i < len(geometry.block) else 1
        geo.shared_bytes = geometry.shared_bytes
        h = _out()
        _check(N.lib().tb_launch(self.ptr, stream.ptr, kernel.ptr, ctypes.byref(enc), ctypes.byref(geo),
                                 ctypes.byref(h)))
        return Event(self, h.value)

    def poll(self, event: Event) -> bool:
        ready = ctypes.c_int(0)
        _check(N.lib().tb_poll(self.ptr, event.ptr, ctypes.byref(ready)))
        return bool(ready.value)

    def wait(self, event: Event) -> None:
        _check(N.lib().tb_wait(self.ptr, event.ptr))

    def wait_event(self, stream: Stream, event: Event) -> None:
        _check(N.lib().tb_wait_event(self.ptr, stream.ptr, event.ptr))

    # ---- extensions ----
    def record(self, stream: Stream) -> Event:
        h = _out()
        _check(N.lib().tb_record(self.ptr, stream.ptr, ctypes.byref(h)))
        return Event(self, h.value)

    def elapsed_ms(self, start: Event, end: Event) -> float:
        ms = ctypes.c_float(0)
        _check(N.lib().tb_event_elapsed_ms(self.ptr, start.ptr, end.ptr, ctypes.byref(ms)))
        return float(ms.value)

    def synchronize(self, stream: Stream) -> None:
        _check(N.lib().tb_stream_synchronize(self.ptr, stream.ptr))

    def capture_begin(self, stream: Stream) -> None:
        """Starts capturing this thread's device work on `stream` into a CUDA graph."""
        _check(N.lib().tb_capture_begin(self.ptr, stream.ptr))

    def capture_end(self, stream: Stream) -> GraphExec:
        """Ends the capture; the graph replays the captured work on the same buffers."""
        h = _out()
        _check(N.lib().tb_capture_end(self.ptr, stream.ptr, ctypes.byref(h)))
        return GraphExec(self, h.value)

    def host_alloc(self, nbytes: int) -> "PinnedHost":
        p = _out()
        _check(N.lib().tb_host_alloc(self.ptr, nbytes, ctypes.byref(p)))
        return PinnedHost(self, p.value, nbytes)

    def upload_pinned(self, stream: Stream, dst: Buffer, src: "PinnedHost", nbytes: Optional[int] = None,
                      dst_offset: int = 0, src_offset: int = 0) -> None:
        n = src.nbytes if nbytes is None else nbytes
        _check(N.lib().tb_upload_pinned(self.ptr, stream.ptr, dst.ptr, dst_offset, src.ptr + src_offset, n, None))

    def download_pinned(self, stream: Stream, src: Buffer, dst: "PinnedHost", nbytes: Optional[int] = None,
                        src_offset: int = 0, dst_offset: int = 0) -> None:
        n = dst.nbytes if nbytes is None else nbytes
        _check(N.lib().tb_download_pinned(self.ptr, stream.ptr, src.ptr, src_offset, dst.ptr + dst_offset, n, None))


class PinnedHost:
    """Page-locked host memory owned by a session, viewable as a numpy array."""

    def __init__(self, session: Session, ptr: int, nbytes: int):
        self.session = session
        self.ptr = ptr
        self.nbytes = nbytes

    def array(self, dtype, shape) -> np.ndarray:
        n = int(np.prod(shape)) * np.dtype(dtype).itemsize
        if n > self.nbytes:
            raise ValueError("view exceeds pinned allocation")
        buf = (ctypes.c_uint8 * n).from_address(self.ptr)
        return np.frombuffer(buf, dtype=dtype).reshape(shape)

    def free(self) -> None:
        if self.ptr:
            _check(N.lib().tb_host_free(self.session.ptr, self.ptr))
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
