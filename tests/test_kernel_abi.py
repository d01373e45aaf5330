"""The Kernel ABI codec mirrors titan-kernel byte for byte (CPU only).

Cases follow projects/titan-kernel/tests/kernel.rs:24-52 and the encode/decode
rules of projects/titan-kernel/src/lib.rs:158-256.
"""
import struct

import pytest

from titan_rs_b200 import kernel_abi as K


class FakeSession:
    pass


class FakeBuffer:
    def __init__(self, session):
        self.session = session
        self.ptr = 1


def test_hash_is_the_rust_debug_format():
    assert K.softmax_f32_abi().hash() == (
        "v1:[Buffer { dtype: F32, writable: false, alignment: 4 }, Buffer { dtype: F32, writable: true, alignment: 4 }, "
        "Scalar { dtype: I32 }, Scalar { dtype: I32 }]:LaunchConfig { block_size: 128, vector_width: 1, "
        "pipeline_depth: 1 }:0")
    empty = K.KernelAbi(1, [], K.LaunchConfig(), 0)
    assert empty.hash() == "v1:[]:LaunchConfig { block_size: 256, vector_width: 1, pipeline_depth: 1 }:0"
    assert K.KernelAbi(2, [K.ShapeArg(3)], K.LaunchConfig(), 64).hash().startswith("v2:[Shape { rank: 3 }]")


def test_encode_returns_payload_bindings_and_canonical_bytes():
    abi = K.KernelAbi(1, [K.BufferArg(K.DType.F32, False, 4)], K.LaunchConfig(), 0)
    s = FakeSession()
    buf = FakeBuffer(s)
    enc = abi.encode([K.KBuffer(5, K.DType.F32, False, 4, buf)])
    assert enc.canonical_abi == abi.canonical_bytes()
    assert enc.bindings[5] == (buf, s)
    assert enc.payload == struct.pack("<I", 5)
    assert abi.decode(enc.payload) == [("buffer", 5)]


def test_encode_scalar_and_shape_layout():
    abi = K.KernelAbi(1, [K.ScalarArg(K.DType.I32), K.ShapeArg(2), K.ScalarArg(K.DType.BF16)], K.LaunchConfig(), 0)
    enc = abi.encode([K.scalar_i32(7), K.KShape([3, 4]), K.KScalar(K.DType.BF16, b"\x80\x3f")])
    assert enc.payload == struct.pack("<Ii", 4, 7) + struct.pack("<QQ", 3, 4) + struct.pack("<I", 2) + b"\x80\x3f"
    assert abi.decode(enc.payload) == [("scalar", struct.pack("<i", 7)), ("shape", [3, 4]), ("scalar", b"\x80\x3f")]


def test_encode_rejections():
    abi = K.gemm_f32_abi()
    s1, s2 = FakeSession(), FakeSession()
    b1, b2 = FakeBuffer(s1), FakeBuffer(s2)
    args = [K.KBuffer(0, K.DType.F32, False, 4, b1), K.KBuffer(1, K.DType.F32, False, 4, b2),
            K.KBuffer(2, K.DType.F32, True, 4, b1), K.scalar_i32(1), K.scalar_i32(1), K.scalar_i32(1)]
    with pytest.raises(K.KernelError) as e:
        abi.encode(args)
    assert e.value.kind == "CrossSessionBinding"
    args[1] = K.KBuffer(0, K.DType.F32, False, 4, b1)
    with pytest.raises(K.KernelError) as e:
        abi.encode(args)
    assert e.value.kind == "DuplicateBinding"
    args[1] = K.KBufferSlot(1)
    with pytest.raises(K.KernelError) as e:
        abi.encode(args)
    assert e.value.kind == "MissingBinding"
    with pytest.raises(K.KernelError, match="expected 6 arguments"):
        abi.encode(args[:3])
    args[1] = K.KBuffer(1, K.DType.F32, False, 4, b1)
    args[3] = K.KScalar(K.DType.I32, b"\x01\x00")
    with pytest.raises(K.KernelError, match="scalar width"):
        abi.encode(args)
    args[3] = K.scalar_f32(1.0)
    with pytest.raises(K.KernelError, match="contract mismatch"):
        abi.encode(args)


def test_decode_rejects_truncated_and_trailing_payloads():
    abi = K.softmax_f32_abi()
    good = struct.pack("<II", 0, 1) + struct.pack("<Ii", 4, 2) + struct.pack("<Ii", 4, 3)
    assert abi.decode(good) == [("buffer", 0), ("buffer", 1), ("scalar", struct.pack("<i", 2)),
                                ("scalar", struct.pack("<i", 3))]
    for cut, msg in ((2, "truncated buffer slot"), (10, "truncated scalar length"), (14, "truncated scalar")):
        with pytest.raises(K.KernelError, match=msg):
            abi.decode(good[:cut])
    with pytest.raises(K.KernelError, match="trailing ABI bytes"):
        abi.decode(good + b"\0")
    with pytest.raises(K.KernelError, match="truncated shape"):
        K.KernelAbi(1, [K.ShapeArg(2)]).decode(b"\0" * 15)


def test_reference_f32_abis_have_the_reference_arity():
    assert len(K.gemm_f32_abi().args) == 6
    assert len(K.conv2d_f32_abi().args) == 21
    assert len(K.scaled_dot_product_attention_f32_abi().args) == 9
    md = K.softmax_f32_abi().launch_metadata("softmax_f32")
    assert md["arguments"] == [("buffer", 0), ("buffer", 0), ("scalar", 4), ("scalar", 4)]
    assert md["block"] == (128, 1, 1)
