"""CUDA-graph capture of a session's device work (tb_capture_begin / tb_capture_end /
tb_graph_exec_launch).

Operators enqueued on a stream during capture become one graph; each replay runs them
again on the same device buffers, so new inputs uploaded between replays give new
results. The test captures a softmax and a bf16 GEMM whose shape takes the split-K path
(its per-stream scratch is allocated by an eager run before the capture), replays the
graph on three sets of inputs and checks every result against the CPU oracle. Host-staged
uploads and downloads are refused inside a capture (a replay would copy from or to
memory the call no longer owns), and the session stays usable after such a refusal.
"""
import math

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
from titan_rs_b200.hal import HalError
from titan_rs_b200.kernel_abi import DType

from gpu_util import elementwise_rel_err, max_rel_err

pytestmark = pytest.mark.gpu


def test_captured_operators_replay_on_new_inputs():
    s = tb.Session(0)
    rt = tb.Runtime(s)
    rows, cols = 512, 1024
    m, n, k = 256, 384, 4096  # few output tiles and a long K: the split-K GEMM
    x = tb.TensorHandle.allocate(s, DType.F32, (rows, cols))
    y = tb.TensorHandle.allocate(s, DType.F32, (rows, cols))
    a = tb.TensorHandle.allocate(s, DType.BF16, (m, k))
    b = tb.TensorHandle.allocate(s, DType.BF16, (n, k))
    c = tb.TensorHandle.allocate(s, DType.BF16, (m, n))

    def enqueue():
        rt.execute(tb.OpRequest("softmax", [x], [tb.TensorSpec(DType.F32, (rows, cols))]), output=y)
        h = rt.execute(tb.OpRequest("gemm", [a, b], [tb.TensorSpec(DType.BF16, (m, n))], {"transpose_rhs": True}),
                       output=c)
        return h.candidate

    def inputs(seed):
        xv = (np.random.default_rng(seed).standard_normal((rows, cols)) * 2.0).astype(np.float32)
        av = tb.fill_normal(m * k, seed=seed, dtype=DType.BF16).reshape(m, k)
        bv = tb.fill_normal(n * k, seed=seed + 1, std=1.0 / math.sqrt(k), dtype=DType.BF16).reshape(n, k)
        s.wait(s.upload(rt.stream, x.buffer, xv))
        s.wait(s.upload(rt.stream, a.buffer, av))
        s.wait(s.upload(rt.stream, b.buffer, bv))
        return xv, av, bv

    inputs(1)
    assert enqueue() == "gemm_bf16_tn_splitk"  # eager run: allocates the stream's scratch
    s.synchronize(rt.stream)
    s.capture_begin(rt.stream)
    enqueue()
    graph = s.capture_end(rt.stream)
    for seed in (10, 20, 30):
        xv, av, bv = inputs(seed)
        graph.launch(rt.stream)
        s.synchronize(rt.stream)
        assert elementwise_rel_err(y.to_numpy(rt.stream), oracle.softmax(xv)) <= 1e-5
        got = c.to_f32(rt.stream)
        rr = np.arange(0, m, 7)
        cc = np.arange(0, n, 5)
        rows_i, cols_i = np.repeat(rr, cc.size), np.tile(cc, rr.size)
        ref = oracle.gemm_bf16_points(av, bv, True, m, n, k, rows_i, cols_i)
        assert max_rel_err(got[rows_i, cols_i], ref) <= 1e-2
    graph.release()
    s.close()


def test_capture_refuses_host_staged_copies():
    s = tb.Session(0)
    st = s.create_stream()
    buf = s.allocate(4096)
    host = np.arange(1024, dtype=np.float32)
    s.capture_begin(st)
    with pytest.raises(HalError) as e:
        s.upload(st, buf, host)
    assert "graph capture" in str(e.value)
    with pytest.raises(HalError) as e:
        s.download(st, buf, np.empty(1024, np.float32))
    assert "graph capture" in str(e.value)
    g = s.capture_end(st)
    g.release()
    s.wait(s.upload(st, buf, host))  # the stream works normally after the capture
    back = np.empty(1024, np.float32)
    s.download(st, buf, back)
    np.testing.assert_array_equal(back, host)
    s.close()
