"""Operators on host-resident operands streamed through the GPU (titan_rs_b200.streaming).

Each call uploads B, then A in row blocks, runs the operator on each block as its rows
land and downloads each block of C while later blocks compute; consecutive calls
overlap. The test makes several calls in a row with different operands into different
host buffers (so a call that read or wrote another call's device buffers shows up as a
wrong result) and checks every result against the CPU oracle on sampled points and
against the same GEMM run on device-resident operands, within the bf16 tolerance the
other GEMM tests use (max|err| <= 1e-2 * max|ref|). One shape has M not a multiple of
the block count. StreamedBatchOp (attention over (batch, head) blocks, conv2d over image
blocks with the weights uploaded once per call) is checked the same way: attention
bit for bit against the whole batch on the device, conv2d within the bf16 tolerance.
"""
import ctypes
import math

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
from titan_rs_b200 import _native as N
from titan_rs_b200.kernel_abi import DType
from titan_rs_b200.runtime import c_tensor, contiguous_strides
from titan_rs_b200.streaming import StreamedGemm

from gpu_util import max_rel_err

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2


def _device_gemm(s, stream, a_bits, b_bits, m, n, k):
    da, db, dc = s.allocate(m * k * 2), s.allocate(n * k * 2), s.allocate(m * n * 2)
    s.upload(stream, da, a_bits)
    s.upload(stream, db, b_bits)
    ta = c_tensor(da, DType.BF16, (m, k), contiguous_strides((m, k)))
    tbm = c_tensor(db, DType.BF16, (n, k), contiguous_strides((n, k)))
    tc = c_tensor(dc, DType.BF16, (m, n), contiguous_strides((m, n)))
    attrs = (N.Attr * 1)()
    key = b"transpose_rhs"
    attrs[0].key = key
    attrs[0].value = 1
    rc = N.lib().tb_op_gemm(s.ptr, stream.ptr, ctypes.byref(ta), ctypes.byref(tbm), ctypes.byref(tc), attrs, 1, None)
    assert rc == N.TB_OK, N.last_error()
    out = np.empty((m, n), np.uint16)
    s.download(stream, dc, out)
    return tb.bf16_bits_to_f32(out).reshape(m, n)


@pytest.mark.parametrize("m,n,k,blocks", [(2048, 1024, 512, 4), (1000, 768, 256, 3)])
def test_streamed_gemm_calls_in_a_row_match_the_oracle_and_the_device_gemm(m, n, k, blocks):
    s = tb.Session(0)
    stream = s.create_stream()
    g = StreamedGemm(s, m, n, k, row_blocks=blocks)
    assert sum(rows for _, rows in g.blocks) == m and 1 < len(g.blocks) <= blocks
    calls = []
    for call in range(3):
        a = s.host_alloc(m * k * 2)
        b = s.host_alloc(n * k * 2)
        c = s.host_alloc(m * n * 2)
        a.array(np.uint16, (m, k))[:] = tb.fill_normal(m * k, seed=700 + call, dtype=DType.BF16).reshape(m, k)
        b.array(np.uint16, (n, k))[:] = tb.fill_normal(n * k, seed=800 + call, std=1.0 / math.sqrt(k),
                                                         dtype=DType.BF16).reshape(n, k)
        c.array(np.uint16, (m, n))[:] = 0xFFFF  # NaN bits: a block never written stays visible
        g.run(stream, a, b, c)
        calls.append((a, b, c))
    s.synchronize(stream)
    rng = np.random.default_rng(5)
    for call, (a, b, c) in enumerate(calls):
        a_bits, b_bits = a.array(np.uint16, (m, k)), b.array(np.uint16, (n, k))
        got = tb.bf16_bits_to_f32(c.array(np.uint16, (m, n))).reshape(m, n)
        assert np.isfinite(got).all(), call
        ref = _device_gemm(s, stream, a_bits, b_bits, m, n, k)
        assert max_rel_err(got, ref) <= BF16_TOL, (call, max_rel_err(got, ref))
        rows = np.concatenate([rng.integers(0, m, 1024), [0, m - 1] + [r0 for r0, _ in g.blocks]])
        cols = np.concatenate([rng.integers(0, n, 1024), [n - 1, 0] + [n - 1] * len(g.blocks)])
        points = oracle.gemm_bf16_points(a_bits, b_bits, True, m, n, k, rows, cols)
        assert max_rel_err(got[rows, cols], points) <= BF16_TOL, (call, max_rel_err(got[rows, cols], points))
    s.close()


def test_streamed_gemm_rejects_short_host_buffers():
    s = tb.Session(0)
    stream = s.create_stream()
    g = StreamedGemm(s, 256, 256, 256, row_blocks=1)
    small = s.host_alloc(256 * 256)
    ok = s.host_alloc(256 * 256 * 2)
    with pytest.raises(ValueError):
        g.run(stream, small, ok, ok)
    s.close()


def _pinned(s, bits):
    h = s.host_alloc(bits.nbytes)
    h.array(bits.dtype, bits.shape)[:] = bits
    return h


def test_streamed_attention_blocks_match_the_whole_batch_bit_for_bit():
    """Attention over batch blocks: every (batch, head) is independent, so each block's
    rows equal the whole batch's (the same pair kernel), and the oracle on sampled rows."""
    from titan_rs_b200.streaming import StreamedBatchOp
    b, h, t, d = 4, 3, 512, 128
    s = tb.Session(0)
    rt = tb.Runtime(s)
    stream = s.create_stream()
    spec = (DType.BF16, (b, h, t, d), True)
    g = StreamedBatchOp(s, "scaled_dot_product_attention", [spec, spec, spec], (DType.BF16, (b, h, t, d)),
                        {"causal": 1}, blocks=4)
    assert len(g.blocks) == 4
    results = []
    for call in range(2):
        qkv = [tb.fill_normal(b * h * t * d, seed=900 + 3 * call + i, dtype=DType.BF16).reshape(b, h, t, d)
               for i in range(3)]
        hosts = [_pinned(s, x) for x in qkv]
        out = s.host_alloc(b * h * t * d * 2)
        out.array(np.uint16, (b, h, t, d))[:] = 0xFFFF
        g.run(stream, hosts, out)
        results.append((qkv, hosts, out))
    s.synchronize(stream)
    for qkv, _, out in results:
        got = out.array(np.uint16, (b, h, t, d)).copy()
        ins = [tb.TensorHandle.from_numpy(s, x, DType.BF16, rt.stream) for x in qkv]
        whole = rt.execute(tb.OpRequest("scaled_dot_product_attention", ins,
                                        [tb.TensorSpec(DType.BF16, (b, h, t, d))], {"causal": True}))
        whole.wait()
        np.testing.assert_array_equal(got, whole.outputs[0].to_numpy(rt.stream))
        ids = np.array([0, 1, 127, 128, 511, t + 5, 2 * t * h - 1, b * h * t - 1])
        ref = oracle.sdpa_bf16_rows(*qkv, b, h, t, t, d, True, ids)
        assert max_rel_err(tb.bf16_bits_to_f32(got.reshape(-1, d)[ids]).reshape(-1, d), ref) <= BF16_TOL
    s.close()


def test_streamed_conv2d_over_image_blocks_matches_the_oracle():
    """conv2d NHWC with the weights uploaded once per call and the images in blocks."""
    from titan_rs_b200.streaming import StreamedBatchOp
    n, hh, ww, cin, cout = 6, 20, 20, 64, 128
    s = tb.Session(0)
    rt = tb.Runtime(s)
    stream = s.create_stream()
    attrs = {"stride_h": 1, "stride_w": 1, "pad_h": 1, "pad_w": 1, "dilation_h": 1, "dilation_w": 1, "groups": 1,
             "layout": "NHWC"}
    g = StreamedBatchOp(s, "conv2d", [(DType.BF16, (n, hh, ww, cin), True), (DType.BF16, (cout, 3, 3, cin), False)],
                        (DType.BF16, (n, hh, ww, cout)), attrs, blocks=3)
    assert [blk for _, blk in g.blocks] == [2, 2, 2]
    results = []
    for call in range(3):
        x = tb.fill_normal(n * hh * ww * cin, seed=40 + call, dtype=DType.BF16).reshape(n, hh, ww, cin)
        w = tb.fill_normal(cout * 9 * cin, seed=50 + call, std=math.sqrt(2.0 / (9 * cin)),
                           dtype=DType.BF16).reshape(cout, 3, 3, cin)
        out = s.host_alloc(n * hh * ww * cout * 2)
        out.array(np.uint16, (n, hh, ww, cout))[:] = 0xFFFF
        g.run(stream, [_pinned(s, x), _pinned(s, w)], out)
        results.append((x, w, out))
    s.synchronize(stream)
    rng = np.random.default_rng(9)
    for x, w, out in results:
        got = tb.bf16_bits_to_f32(out.array(np.uint16, (n, hh, ww, cout))).reshape(-1)
        assert np.isfinite(got).all()
        ins = [tb.TensorHandle.from_numpy(s, x, DType.BF16, rt.stream), tb.TensorHandle.from_numpy(s, w, DType.BF16,
                                                                                                   rt.stream)]
        whole = rt.execute(tb.OpRequest("conv2d", ins, [tb.TensorSpec(DType.BF16, (n, hh, ww, cout))], attrs))
        whole.wait()
        assert max_rel_err(got, whole.outputs[0].to_f32(rt.stream).reshape(-1)) <= BF16_TOL
        idx = np.concatenate([rng.integers(0, got.size, 2048), [0, got.size - 1]])
        ref = oracle.conv2d_nhwc_bf16_points(x, w, None, n, hh, ww, cin, cout, 3, 3, (1, 1), (1, 1), (1, 1), hh, ww,
                                             idx)
        assert max_rel_err(got[idx], ref) <= BF16_TOL
    s.close()
