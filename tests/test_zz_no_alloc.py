"""The allocation-free split-K GEMM (tb_gemm_bf16_splitk_noalloc) against the
library's allocating split-K path (tb_op_gemm) and the CPU oracle.

Callers such as a serving runtime that has planned all of HBM up front must
not let this library allocate device memory; this entry point keeps its fp32
partials in a fixed 32 MiB device array instead of per-stream scratch. The test
calls it through the C ABI several times in a row on different shapes (each
call runs on whatever the previous one left in the shared array) and checks
each result against the allocating entry point's and against the oracle on
sampled points, within the bf16 tolerance the other GEMM tests use. After each
call it reads the device-side status through
tb_gemm_bf16_splitk_noalloc_status, so a kernel that gave up a bounded wait
cannot pass as a result. One shape has N % 4 != 0, which runs the reduction's
one-column-per-thread branch. This file is named so pytest collects it last,
and it depends on no other test.
"""
import ctypes
import math

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
from titan_rs_b200 import _native as N
from titan_rs_b200.kernel_abi import DType

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2  # max|err| <= 1e-2 * max|ref|, as in test_gemm_gpu.py


def _max_rel_err(got, ref):
    return float(np.max(np.abs(got.astype(np.float64) - ref.astype(np.float64))) / max(np.max(np.abs(ref)), 1e-30))


def _status(lib, stream_handle):
    code = ctypes.c_uint32(0xFFFFFFFF)
    rc = lib.tb_gemm_bf16_splitk_noalloc_status(stream_handle, ctypes.byref(code))
    return rc, code.value


@pytest.mark.parametrize("shapes", [[(512, 512, 16384), (256, 390, 8192), (256, 384, 8192)]])
def test_no_alloc_split_k_gemm_matches_the_allocating_entry_point_and_the_oracle(shapes):
    s = tb.Session(0)
    rt = tb.Runtime(s)
    lib = N.lib()
    rng = np.random.default_rng(17)
    for call, (m, n, k) in enumerate(shapes):
        a = tb.fill_normal(m * k, seed=900 + call, dtype=DType.BF16).reshape(m, k)
        b = tb.fill_normal(n * k, seed=950 + call, std=1.0 / math.sqrt(k), dtype=DType.BF16).reshape(n, k)
        ta = tb.TensorHandle.from_numpy(s, a, DType.BF16, rt.stream)
        tbb = tb.TensorHandle.from_numpy(s, b, DType.BF16, rt.stream)
        ref = rt.execute(tb.OpRequest("gemm", [ta, tbb], [tb.TensorSpec(DType.BF16, (m, n))], {"transpose_rhs": True}))
        ref.wait()
        assert ref.candidate == "gemm_bf16_tn_splitk"
        expected = ref.outputs[0].to_f32()

        out = s.allocate(m * n * 2)
        rc = lib.tb_gemm_bf16_splitk_noalloc(rt.stream.handle, ta.buffer.device_ptr, tbb.buffer.device_ptr,
                                             out.device_ptr, m, n, k, 0)
        assert rc == N.TB_OK, N.last_error()
        rc, code = _status(lib, rt.stream.handle)
        assert rc == N.TB_OK and code == 0, (rc, hex(code), N.last_error())
        got_bits = np.empty((m, n), np.uint16)
        s.download(rt.stream, out, got_bits)
        got = tb.bf16_bits_to_f32(got_bits).reshape(m, n)
        assert np.isfinite(got).all()
        assert _max_rel_err(got, expected) <= BF16_TOL, (call, _max_rel_err(got, expected))
        rows = np.concatenate([rng.integers(0, m, 2048), [0, m - 1, 0, m - 1]])
        cols = np.concatenate([rng.integers(0, n, 2048), [0, 0, n - 1, n - 1]])
        points = oracle.gemm_bf16_points(a, b, True, m, n, k, rows, cols)
        assert _max_rel_err(got[rows, cols], points) <= BF16_TOL, (call, _max_rel_err(got[rows, cols], points))
    s.close()


def test_no_alloc_split_k_gemm_rejects_work_beyond_its_static_scratch():
    s = tb.Session(0)
    stream = s.create_stream()
    buf = s.allocate(1 << 20)
    ptr = buf.device_ptr
    # 32 splits of a 1024 x 1024 output need 33.5M partials, above the 8,388,608 the array holds.
    rc = N.lib().tb_gemm_bf16_splitk_noalloc(stream.handle, ptr, ptr, ptr, 1024, 1024, 65536, 32)
    assert rc == N.TB_ERR_INVALID
    op, detail = N.last_error()
    assert "static scratch" in detail
    # A rejected call launches nothing, so the device status stays clear.
    rc, code = _status(N.lib(), stream.handle)
    assert rc == N.TB_OK and code == 0
    s.close()
