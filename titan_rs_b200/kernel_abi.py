"""Kernel ABI: the titan.rs launch-argument contract, byte for byte.

Restates projects/titan-kernel/src/lib.rs:113-282 (KernelAbi, AbiArg,
KernelArg, encode/decode, canonical hash) and the four fixed f32 ABIs of the
CUDA backend (projects/titan-backend-cuda/src/lib.rs:343-355, 663-729). The
canonical bytes are the reference's `format!("v{}:{:?}:{:?}:{}")` string, so an
artifact loaded with this hash accepts payloads encoded by the Rust crate and
vice versa.
"""
from __future__ import annotations

import enum
import struct
from dataclasses import dataclass, field
from typing import Sequence, Union


class DType(enum.Enum):
    """titan_types::DType (projects/titan-types/src/lib.rs:42-49); value = C ABI code."""
    F32 = 0
    F16 = 1
    BF16 = 2
    I32 = 3
    I64 = 4


def scalar_width(dtype: DType) -> int:
    """projects/titan-kernel/src/lib.rs:258-264."""
    return {DType.F32: 4, DType.I32: 4, DType.F16: 2, DType.BF16: 2, DType.I64: 8}[dtype]


class KernelError(ValueError):
    """KernelError (projects/titan-kernel/src/lib.rs:381-395): kind + detail."""

    def __init__(self, kind: str, detail: str = ""):
        super().__init__(f"{kind}({detail!r})" if detail else kind)
        self.kind = kind
        self.detail = detail


@dataclass(frozen=True)
class BufferArg:
    dtype: DType
    writable: bool
    alignment: int

    def debug(self) -> str:
        return (f"Buffer {{ dtype: {self.dtype.name}, writable: {'true' if self.writable else 'false'}, "
                f"alignment: {self.alignment} }}")


@dataclass(frozen=True)
class ScalarArg:
    dtype: DType

    def debug(self) -> str:
        return f"Scalar {{ dtype: {self.dtype.name} }}"


@dataclass(frozen=True)
class ShapeArg:
    rank: int

    def debug(self) -> str:
        return f"Shape {{ rank: {self.rank} }}"


AbiArg = Union[BufferArg, ScalarArg, ShapeArg]


@dataclass(frozen=True)
class LaunchConfig:
    """projects/titan-kernel/src/lib.rs:101-111."""
    block_size: int = 256
    vector_width: int = 1
    pipeline_depth: int = 1

    def debug(self) -> str:
        return (f"LaunchConfig {{ block_size: {self.block_size}, vector_width: {self.vector_width}, "
                f"pipeline_depth: {self.pipeline_depth} }}")


# Encoding inputs (KernelArg, projects/titan-kernel/src/lib.rs:266-282).
@dataclass
class KBuffer:
    slot: int
    dtype: DType
    writable: bool
    alignment: int
    buffer: object  # hal.Buffer


@dataclass
class KBufferSlot:
    slot: int


@dataclass
class KScalar:
    dtype: DType
    data: bytes


@dataclass
class KShape:
    values: Sequence[int]


KernelArg = Union[KBuffer, KBufferSlot, KScalar, KShape]


def scalar_i32(v: int) -> KScalar:
    return KScalar(DType.I32, struct.pack("<i", v))


def scalar_f32(v: float) -> KScalar:
    return KScalar(DType.F32, struct.pack("<f", v))


@dataclass
class EncodedLaunchArgs:
    """EncodedLaunchArgs (projects/titan-hal/src/lib.rs:110): payload, slot -> binding, canonical ABI bytes."""
    payload: bytes
    bindings: dict  # slot -> (buffer, owner session)
    canonical_abi: bytes


@dataclass
class KernelAbi:
    version: int
    args: list
    launch: LaunchConfig = field(default_factory=LaunchConfig)
    workspace_bytes: int = 0

    def hash(self) -> str:
        """`format!("v{}:{:?}:{:?}:{}", version, args, launch, workspace_bytes)` (lib.rs:127-129)."""
        args = "[" + ", ".join(a.debug() for a in self.args) + "]"
        return f"v{self.version}:{args}:{self.launch.debug()}:{self.workspace_bytes}"

    def canonical_bytes(self) -> bytes:
        return self.hash().encode()

    def launch_metadata(self, entry: str) -> dict:
        """KernelAbi::launch_metadata (lib.rs:139-156)."""
        kinds = []
        for a in self.args:
            if isinstance(a, BufferArg):
                kinds.append(("buffer", 0))
            elif isinstance(a, ScalarArg):
                kinds.append(("scalar", scalar_width(a.dtype)))
            else:
                kinds.append(("shape", a.rank))
        return {"version": self.version, "entry": entry, "arguments": kinds, "block": (self.launch.block_size, 1, 1),
                "shared_bytes": 0}

    def encode(self, args: Sequence[KernelArg]) -> EncodedLaunchArgs:
        """KernelAbi::encode (lib.rs:158-207)."""
        if len(args) != len(self.args):
            raise KernelError("InvalidAbi", f"expected {len(self.args)} arguments, got {len(args)}")
        out = bytearray()
        bindings = {}
        session = None
        for decl, arg in zip(self.args, args):
            if isinstance(decl, BufferArg) and isinstance(arg, KBuffer) and decl.dtype == arg.dtype \
                    and decl.writable == arg.writable and arg.alignment >= decl.alignment:
                owner = arg.buffer.session
                if session is None:
                    session = owner
                elif owner is not session:
                    raise KernelError("CrossSessionBinding", "buffers from different sessions")
                if arg.slot in bindings:
                    raise KernelError("DuplicateBinding", str(arg.slot))
                bindings[arg.slot] = (arg.buffer, owner)
                out += struct.pack("<I", arg.slot)
            elif isinstance(decl, BufferArg) and isinstance(arg, KBufferSlot):
                raise KernelError("MissingBinding", str(arg.slot))
            elif isinstance(decl, ScalarArg) and isinstance(arg, KScalar) and decl.dtype == arg.dtype:
                expected = scalar_width(decl.dtype)
                if len(arg.data) != expected:
                    raise KernelError("InvalidAbi", f"scalar width: expected {expected}, got {len(arg.data)}")
                out += struct.pack("<I", len(arg.data)) + bytes(arg.data)
            elif isinstance(decl, ShapeArg) and isinstance(arg, KShape) and decl.rank == len(arg.values):
                for v in arg.values:
                    out += struct.pack("<Q", v)
            else:
                raise KernelError("InvalidAbi", "argument contract mismatch")
        return EncodedLaunchArgs(bytes(out), bindings, self.canonical_bytes())

    def decode(self, payload: bytes) -> list:
        """KernelAbi::decode (lib.rs:209-256): ('buffer', slot) / ('scalar', bytes) / ('shape', [u64])."""
        cursor = 0
        result = []
        for decl in self.args:
            if isinstance(decl, BufferArg):
                if cursor + 4 > len(payload):
                    raise KernelError("InvalidAbi", "truncated buffer slot")
                result.append(("buffer", struct.unpack_from("<I", payload, cursor)[0]))
                cursor += 4
            elif isinstance(decl, ScalarArg):
                if cursor + 4 > len(payload):
                    raise KernelError("InvalidAbi", "truncated scalar length")
                n = struct.unpack_from("<I", payload, cursor)[0]
                cursor += 4
                if cursor + n > len(payload):
                    raise KernelError("InvalidAbi", "truncated scalar")
                result.append(("scalar", bytes(payload[cursor:cursor + n])))
                cursor += n
            else:
                n = decl.rank * 8
                if cursor + n > len(payload):
                    raise KernelError("InvalidAbi", "truncated shape")
                result.append(("shape", list(struct.unpack_from(f"<{decl.rank}Q", payload, cursor))))
                cursor += n
        if cursor != len(payload):
            raise KernelError("InvalidAbi", "trailing ABI bytes")
        return result


def _buf(writable: bool) -> BufferArg:
    return BufferArg(DType.F32, writable, 4)


_REF_LAUNCH = LaunchConfig(block_size=128, vector_width=1, pipeline_depth=1)


def softmax_f32_abi() -> KernelAbi:
    """projects/titan-backend-cuda/src/lib.rs:343-355 (in, out, rows, cols)."""
    return KernelAbi(1, [_buf(False), _buf(True), ScalarArg(DType.I32), ScalarArg(DType.I32)], _REF_LAUNCH, 0)


def gemm_f32_abi() -> KernelAbi:
    """projects/titan-backend-cuda/src/lib.rs:663-677 (A, B, C, M, N, K)."""
    return KernelAbi(1, [_buf(False), _buf(False), _buf(True)] + [ScalarArg(DType.I32)] * 3, _REF_LAUNCH, 0)


def conv2d_f32_abi() -> KernelAbi:
    """projects/titan-backend-cuda/src/lib.rs:680-709 (x, w, bias, y + 17 i32 geometry scalars)."""
    return KernelAbi(1, [_buf(False), _buf(False), _buf(False), _buf(True)] + [ScalarArg(DType.I32)] * 17,
                     _REF_LAUNCH, 0)


def scaled_dot_product_attention_f32_abi() -> KernelAbi:
    """projects/titan-backend-cuda/src/lib.rs:712-729 (Q, K, V, O, B, H, Tq, Tk, D)."""
    return KernelAbi(1, [_buf(False)] * 3 + [_buf(True)] + [ScalarArg(DType.I32)] * 5, _REF_LAUNCH, 0)
