"""HAL contract on the B200: ownership, ABI validation and the copy/event
semantics of the titan.rs CUDA session (projects/titan-backend-cuda/src/lib.rs:1170-1536),
mirroring projects/titan-backend-cuda/tests/driver_integration.rs:680-895.
"""
import math
import struct

import numpy as np
import pytest

import titan_rs_b200 as tb
from titan_rs_b200 import _native as N
from titan_rs_b200 import kernel_abi as K
from titan_rs_b200.hal import HalError, LaunchGeometry
from titan_rs_b200.kernel_abi import DType

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sessions():
    a, b = tb.Session(0), tb.Session(0)
    yield a, b
    a.close()
    b.close()


def test_fingerprint_reports_sm100(sessions):
    fp = sessions[0].fingerprint()
    assert fp["capability_revision"] == "sm_100"
    assert fp["sm_count"] >= 100
    devices = tb.enumerate_devices()
    assert devices and devices[0]["capability_revision"] == "sm_100"


def test_upload_download_copy_round_trip(sessions):
    s, _ = sessions
    st = s.create_stream()
    data = np.arange(1 << 20, dtype=np.float32)
    a, b = s.allocate(data.nbytes), s.allocate(data.nbytes)
    up = s.upload(st, a, data)
    data[:] = -1  # upload staged its own copy
    s.wait(up)
    s.wait(s.copy(st, b, a, a.byte_len))
    out = np.empty(1 << 20, np.float32)
    ev = s.download(st, b, out)
    assert s.poll(ev)  # download completes before returning
    np.testing.assert_array_equal(out, np.arange(1 << 20, dtype=np.float32))


def test_wait_event_orders_two_streams(sessions):
    s, _ = sessions
    s1, s2 = s.create_stream(), s.create_stream()
    n = 1 << 24
    src = np.full(n, 7, np.uint8)
    a, b = s.allocate(n), s.allocate(n)
    ev = s.upload(s1, a, src)
    s.wait_event(s2, ev)
    s.copy(s2, b, a, n)
    out = np.empty(n, np.uint8)
    s.download(s2, b, out)
    assert np.all(out == 7)


def test_size_rejections(sessions):
    s, _ = sessions
    st = s.create_stream()
    a = s.allocate(16)
    with pytest.raises(HalError, match="source exceeds allocation"):
        s.upload(st, a, np.zeros(8, np.float32))
    with pytest.raises(HalError, match="destination exceeds allocation"):
        s.download(st, a, np.zeros(8, np.float32))


def test_foreign_buffer_stream_and_event_are_rejected(sessions):
    a, b = sessions
    st_a, st_b = a.create_stream(), b.create_stream()
    buf_b = b.allocate(64)
    with pytest.raises(HalError) as e:
        a.upload(st_a, buf_b, np.zeros(4, np.float32))
    assert e.value.operation == "buffer" and "foreign buffer" in e.value.detail
    with pytest.raises(HalError) as e:
        a.upload(st_b, a.allocate(64), np.zeros(4, np.float32))
    assert e.value.operation == "stream" and "foreign stream" in e.value.detail
    ev_b = b.create_event()
    with pytest.raises(HalError) as e:
        a.wait(ev_b)
    assert e.value.operation == "event" and "foreign event" in e.value.detail


def _softmax_setup(s, rows=4, cols=8):
    abi = K.softmax_f32_abi()
    kernel = s.load(N.builtin_cubin("softmax"), abi.hash(), abi.launch_metadata("softmax_f32"))
    bin_, bout = s.allocate(rows * cols * 4), s.allocate(rows * cols * 4)
    return abi, kernel, bin_, bout


def test_launch_validation_matches_reference(sessions):
    a, b = sessions
    st = a.create_stream()
    abi, kernel, bin_, bout = _softmax_setup(a)
    geo = LaunchGeometry((1, 1, 1), (128, 1, 1), 0)
    good = abi.encode([K.KBuffer(0, DType.F32, False, 4, bin_), K.KBuffer(1, DType.F32, True, 4, bout),
                       K.scalar_i32(4), K.scalar_i32(8)])
    a.wait(a.launch(st, kernel, good, geo))

    def variant(**kw):
        return K.EncodedLaunchArgs(kw.get("payload", good.payload), kw.get("bindings", dict(good.bindings)),
                                   kw.get("canonical", good.canonical_abi))

    expectations = [
        (variant(canonical=b"v1:other"), "launch", "encoded arguments do not match kernel ABI"),
        (variant(payload=good.payload[:2]), "launch", "truncated buffer slot"),
        (variant(payload=good.payload[:10]), "launch", "truncated scalar length"),
        (variant(payload=good.payload[:14]), "launch", "truncated scalar"),
        (variant(payload=good.payload + b"\0"), "launch", "trailing ABI bytes"),
        (variant(payload=good.payload[:8] + struct.pack("<Ih", 2, 4) + good.payload[16:]), "launch",
         "scalar width disagrees with ABI"),
        (variant(bindings={0: good.bindings[0]}), "launch", "missing buffer binding for slot 1"),
        (variant(bindings={0: good.bindings[0], 1: (bout, b)}), "validate_bindings", "cross-session buffer binding"),
        (variant(bindings={0: good.bindings[0], 1: (b.allocate(128), a)}), "buffer", "foreign buffer"),
    ]
    for enc, op, detail in expectations:
        with pytest.raises(HalError) as e:
            a.launch(st, kernel, enc, geo)
        assert e.value.operation == op, (op, e.value)
        assert detail in e.value.detail, (detail, e.value)
    # A kernel loaded by another session is rejected.
    kb = b.load(N.builtin_cubin("softmax"), abi.hash(), abi.launch_metadata("softmax_f32"))
    with pytest.raises(HalError) as e:
        a.launch(st, kb, good, geo)
    assert "another CUDA session" in e.value.detail


def test_load_rejects_non_artifacts_and_caches_modules(sessions):
    s, _ = sessions
    abi = K.softmax_f32_abi()
    with pytest.raises(HalError) as e:
        s.load(b"not a module", abi.hash(), abi.launch_metadata("softmax_f32"))
    assert e.value.operation == "load"
    with pytest.raises(HalError):
        s.load(N.builtin_cubin("softmax"), abi.hash(), abi.launch_metadata("no_such_entry"))
    k1 = s.load(N.builtin_cubin("softmax"), abi.hash(), abi.launch_metadata("softmax_f32"))
    k2 = s.load(N.builtin_cubin("softmax"), abi.hash(), abi.launch_metadata("softmax_f32_stream"))
    assert k1.ptr != k2.ptr


def test_event_timing_and_pinned_copies(sessions):
    s, _ = sessions
    st = s.create_stream()
    n = 1 << 22
    host = s.host_alloc(n * 4)
    arr = host.array(np.float32, (n,))
    arr[:] = np.arange(n, dtype=np.float32)
    dev = s.allocate(n * 4)
    e0 = s.record(st)
    s.upload_pinned(st, dev, host)
    back = s.host_alloc(n * 4)
    s.download_pinned(st, dev, back)
    e1 = s.record(st)
    s.synchronize(st)
    assert s.elapsed_ms(e0, e1) > 0
    np.testing.assert_array_equal(back.array(np.float32, (n,)), arr)
