"""Operator entry: the titan.rs `Runtime::execute(OpRequest)` path for the four
hot-path operators, dispatched to libtitan_b200's tb_op_* entry points.

Mirrors projects/titan-runtime/src/lib.rs:1171-1256 (dispatch by operator name
when the first input lives on the CUDA backend), TensorHandle/TensorSpec
(projects/titan-tensor/src/lib.rs:17-123, projects/titan-graph/src/graph.rs) and
ExecutionError{operator, phase, message} (projects/titan-runtime/src/lib.rs:279-285).
The contract checks themselves live in the native library, so a Rust caller
binding the C ABI gets the same messages.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _native as N
from .hal import Buffer, Event, HalError, Session, Stream
from .kernel_abi import DType

_NP = {DType.F32: np.float32, DType.BF16: np.uint16, DType.F16: np.float16, DType.I32: np.int32,
       DType.I64: np.int64}
_SIZE = {DType.F32: 4, DType.BF16: 2, DType.F16: 2, DType.I32: 4, DType.I64: 8}


def contiguous_strides(shape: Sequence[int]) -> tuple:
    """contiguous_strides (projects/titan-runtime/src/lib.rs:485-493)."""
    out, step = [0] * len(shape), 1
    for a in range(len(shape) - 1, -1, -1):
        out[a] = step
        step *= int(shape[a])
    return tuple(out)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit pattern."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    nan = ((b & 0x7F800000) == 0x7F800000) & ((b & 0x007FFFFF) != 0)
    if nan.any():
        r[nan] = ((b[nan] >> 16) | 0x0040).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class TensorHandle:
    """A device tensor: buffer + dtype + shape + element strides (TensorHandle, titan-tensor/src/lib.rs:17-123)."""
    session: Session
    buffer: Buffer
    dtype: DType
    shape: tuple
    strides: tuple

    @classmethod
    def allocate(cls, session: Session, dtype: DType, shape: Sequence[int]) -> "TensorHandle":
        shape = tuple(int(s) for s in shape)
        nbytes = int(np.prod(shape, dtype=np.int64)) * _SIZE[dtype] if shape else _SIZE[dtype]
        return cls(session, session.allocate(nbytes), dtype, shape, contiguous_strides(shape))

    @classmethod
    def from_numpy(cls, session: Session, array: np.ndarray, dtype: Optional[DType] = None,
                   stream: Optional[Stream] = None) -> "TensorHandle":
        """Uploads `array` (float32 for F32; uint16 bf16 bit patterns or float32 for BF16)."""
        dtype = dtype or DType.F32
        if dtype == DType.BF16 and array.dtype != np.uint16:
            array = f32_to_bf16_bits(array)
        array = np.ascontiguousarray(array, dtype=_NP[dtype])
        t = cls.allocate(session, dtype, array.shape)
        s = stream or session.create_stream()
        session.wait(session.upload(s, t.buffer, array))
        return t

    def to_numpy(self, stream: Optional[Stream] = None) -> np.ndarray:
        """Downloads the tensor (the reference's to_vec_f32 waits and reads back, titan-tensor/src/lib.rs:79-95)."""
        out = np.empty(self.shape, dtype=_NP[self.dtype])
        s = stream or self.session.create_stream()
        self.session.download(s, self.buffer, out)
        return out

    def to_f32(self, stream: Optional[Stream] = None) -> np.ndarray:
        a = self.to_numpy(stream)
        return bf16_bits_to_f32(a).reshape(self.shape) if self.dtype == DType.BF16 else a.astype(np.float32)

    def c_tensor(self) -> N.Tensor:
        return c_tensor(self.buffer, self.dtype, self.shape, self.strides)


def c_tensor(buffer: Optional[Buffer], dtype: DType, shape: Sequence[int], strides: Sequence[int]) -> N.Tensor:
    t = N.Tensor()
    t.buffer = buffer.ptr if buffer is not None else None
    t.dtype = dtype.value
    t.rank = len(shape)
    if len(shape) > N.TB_MAX_RANK:
        raise ValueError("rank exceeds TB_MAX_RANK")
    for i, (s, st) in enumerate(zip(shape, strides)):
        t.shape[i] = int(s)
        t.strides[i] = int(st)
    return t


@dataclass
class TensorSpec:
    """Output declaration of an OpRequest (TensorSpec, projects/titan-graph/src/graph.rs)."""
    dtype: DType
    shape: tuple
    strides: Optional[tuple] = None
    layout: str = "Contiguous"

    def resolved_strides(self) -> tuple:
        if self.layout != "Contiguous":
            # A Layout::Strided spec is never the contiguous output the CUDA
            # operators require; zero strides make the native check reject it.
            return tuple(0 for _ in self.shape)
        return tuple(self.strides) if self.strides is not None else contiguous_strides(self.shape)


@dataclass
class OpRequest:
    """OpRequest{operator, inputs, outputs, attrs} (projects/titan-graph/src/graph.rs:313-327)."""
    operator: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)


class ExecutionError(RuntimeError):
    """ExecutionError{operator, phase, message} (projects/titan-runtime/src/lib.rs:279-285)."""

    def __init__(self, operator: str, phase: str, message: str, status: int = N.TB_ERR_INVALID):
        super().__init__(f"{operator} [{phase}]: {message}")
        self.operator = operator
        self.phase = phase
        self.message = message
        self.status = status


@dataclass
class ExecutionHandle:
    outputs: list
    candidate: str
    kernel: str
    event: Event

    def wait(self) -> "ExecutionHandle":
        self.outputs[0].session.wait(self.event)
        return self


def _attrs(attrs: dict):
    arr = (N.Attr * max(len(attrs), 1))()
    keep = []
    for i, (k, v) in enumerate(attrs.items()):
        kb = k.encode()
        keep.append(kb)
        arr[i].key = kb
        if isinstance(v, (str, float)):
            # Floats cross the C ABI as their shortest round-tripping decimal string.
            sb = (v if isinstance(v, str) else repr(float(v))).encode()
            keep.append(sb)
            arr[i].str = sb
            arr[i].value = 0
        else:
            arr[i].value = int(v)
            arr[i].str = None
    return arr, len(attrs), keep


_OPS = {"softmax": "tb_op_softmax", "gemm": "tb_op_gemm", "scaled_dot_product_attention": "tb_op_sdpa",
        "conv2d": "tb_op_conv2d", "gemm.bias_act": "tb_op_gemm_bias_act", "attention.fused": "tb_op_sdpa"}
_ARITY = {"softmax": (1, 1), "gemm": (2, 2), "scaled_dot_product_attention": (3, 3), "conv2d": (2, 3),
          "gemm.bias_act": (2, 3), "attention.fused": (3, 3)}
_ARITY_MSG = {"softmax": "CUDA softmax requires exactly one input and one output",
              "gemm": "gemm requires exactly two rank-2 inputs",
              "scaled_dot_product_attention": "scaled dot-product attention requires exactly three rank-4 BHTD inputs",
              "conv2d": "conv2d requires rank-4 NCHW input, rank-4 OIHW weight, and optional bias",
              "gemm.bias_act": "gemm.bias_act requires two rank-2 inputs, an optional bias and one output",
              "attention.fused": "attention.fused requires Q, K and V"}


class Runtime:
    """Dispatches OpRequests for the hot-path operators to the B200 kernels.

    With an `autotuner` (autotune.Autotuner), a request without an explicit `candidate`
    attribute runs the candidate its exact TuneKey selected; the first request of a key
    tunes it (capability, correctness against the first capable candidate, event-timed
    benchmark, selection) and persists the decision. This is the runtime candidate
    dispatch the reference leaves unwired (titan-runtime/src/lib.rs:3493-3495)."""

    def __init__(self, session: Session, stream: Optional[Stream] = None, autotuner=None, budget=None):
        self.session = session
        self.stream = stream or session.create_stream()
        self.autotuner = autotuner
        self.budget = budget
        self.last_tune = None  # TuneResult of the most recent search (None on cache hits)
        self._device_key = None
        self._artifact = None

    def execute(self, request: OpRequest, output: Optional[TensorHandle] = None) -> ExecutionHandle:
        name = request.operator
        if name not in _OPS:
            raise ExecutionError(name, "contract", f"operator {name} is not on the B200 hot path (does not implement)",
                                 N.TB_ERR_UNSUPPORTED)
        lo, hi = _ARITY[name]
        if not (lo <= len(request.inputs) <= hi) or len(request.outputs) != 1:
            raise ExecutionError(name, "contract", _ARITY_MSG[name])
        for t in request.inputs:
            if t.session is not self.session:
                raise ExecutionError(name, "contract", f"CUDA {name} requires inputs from the same session")
        spec = request.outputs[0]
        if output is None:
            try:
                output = TensorHandle.allocate(self.session, spec.dtype, spec.shape)
            except HalError as e:
                raise ExecutionError(name, "allocate", str(e), e.status) from e
        attrs = dict(request.attrs)
        self.last_tune = None
        if self.autotuner is not None and "candidate" not in attrs:
            chosen = self._tuned_candidate(request, output, attrs)
            if chosen:
                attrs["candidate"] = chosen
        ev = self._launch(name, request, output, attrs)
        L = N.lib()
        return ExecutionHandle([TensorHandle(self.session, output.buffer, spec.dtype, tuple(spec.shape),
                                             contiguous_strides(spec.shape))],
                               L.tb_last_candidate().decode(), L.tb_last_candidate().decode(),
                               Event(self.session, ev))

    def _launch(self, name: str, request: OpRequest, output: TensorHandle, attrs_dict: dict) -> int:
        """One request through tb_execute, the native Runtime::execute router."""
        spec = request.outputs[0]
        out_c = c_tensor(output.buffer, spec.dtype, spec.shape, spec.resolved_strides())
        ins = (N.Tensor * len(request.inputs))(*[t.c_tensor() for t in request.inputs])
        attrs, nattrs, _keep = _attrs(attrs_dict)
        ev = ctypes.c_void_p(0)
        st = N.lib().tb_execute(self.session.ptr, self.stream.ptr, name.encode(), ins, len(request.inputs),
                                ctypes.byref(out_c), attrs, nattrs, ctypes.byref(ev))
        if st != N.TB_OK:
            op, detail = N.last_error()
            raise ExecutionError(name, op or "launch", detail, st)
        return ev.value

    # ---- candidate dispatch ----
    def tune_key(self, request: OpRequest):
        """The exact TuneKey of a request (shapes, strides, dtypes, semantic attributes, device, library)."""
        from . import autotune as A
        if self._device_key is None:
            fp = self.session.fingerprint()
            self._device_key = f"{fp['model']}/{fp['capability_revision']}/{fp['sm_count']}sm"
            self._artifact = A.library_identity()
        spec = request.outputs[0]
        shape = ",".join(str(list(t.shape)) for t in request.inputs) + "->" + str(list(spec.shape))
        dtype = ",".join(t.dtype.name for t in request.inputs) + "->" + spec.dtype.name
        sem = {k: v for k, v in sorted(request.attrs.items()) if k != "candidate"}
        layout = (";".join(str(list(t.strides)) for t in request.inputs) + "->" + str(list(spec.resolved_strides()))
                  + ";" + ",".join(f"{k}={v}" for k, v in sem.items()))
        return A.TuneKey(operator=request.operator, device=self._device_key, shape=shape, dtype=dtype,
                         layout=layout, artifact=self._artifact)

    def _tuned_candidate(self, request: OpRequest, output: TensorHandle, attrs: dict) -> Optional[str]:
        from . import autotune as A
        name = request.operator
        cands = A.CANDIDATES.get((name, request.inputs[0].dtype.name))
        if not cands:
            return None
        key = self.tune_key(request)
        hit = self.autotuner.get(key)
        if hit is not None:
            return hit.candidate
        spec = request.outputs[0]

        def run(c):
            try:
                self._launch(name, request, output, {**attrs, "candidate": c})
                self.session.synchronize(self.stream)
            except ExecutionError as e:
                if e.status == N.TB_ERR_UNSUPPORTED:
                    raise A.CandidateUnsupported(e.message) from e
                raise

        def read_output():
            return TensorHandle(self.session, output.buffer, spec.dtype, tuple(spec.shape),
                                contiguous_strides(spec.shape)).to_f32(self.stream)

        def time_ns(c, warmups, samples):
            cand_attrs = {**attrs, "candidate": c}
            for _ in range(warmups):
                self._launch(name, request, output, cand_attrs)
            marks = [self.session.record(self.stream)]
            for _ in range(samples):
                self._launch(name, request, output, cand_attrs)
                marks.append(self.session.record(self.stream))
            self.session.synchronize(self.stream)
            return [self.session.elapsed_ms(marks[i], marks[i + 1]) * 1e6 for i in range(samples)]

        tol = A.TOLERANCE.get(spec.dtype.name, 1e-2)
        result = self.autotuner.tune(key, cands[0], cands[1], run, read_output, time_ns, tol,
                                     self.budget or A.TuneBudget())
        self.autotuner.flush()
        self.last_tune = result
        return result.entry.candidate


def fill_normal(count: int, seed: int, mean: float = 0.0, std: float = 1.0, dtype: DType = DType.F32,
                threads: int = 0) -> np.ndarray:
    """Seeded counter-based N(mean, std^2) samples (tb_fill_normal); bf16 as uint16 bit patterns."""
    out = np.empty(count, dtype=_NP[dtype])
    st = N.lib().tb_fill_normal(out.ctypes.data_as(ctypes.c_void_p), dtype.value, count, seed, mean, std, threads)
    if st != N.TB_OK:
        raise HalError(st, *N.last_error())
    return out


def fill_uniform(count: int, seed: int, low: float = 0.0, high: float = 1.0, dtype: DType = DType.F32,
                 threads: int = 0) -> np.ndarray:
    """Seeded counter-based U[low, high) samples (tb_fill_uniform)."""
    out = np.empty(count, dtype=_NP[dtype])
    st = N.lib().tb_fill_uniform(out.ctypes.data_as(ctypes.c_void_p), dtype.value, count, seed, low, high, threads)
    if st != N.TB_OK:
        raise HalError(st, *N.last_error())
    return out
