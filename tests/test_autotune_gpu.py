"""Runtime candidate dispatch through the autotuner on the B200: each operator's first
request of a shape tunes over the registered kernels, later requests (and a new process
reading the `.tune` file) dispatch the stored winner without tuning again."""
import numpy as np
import pytest

import titan_rs_b200 as tb
from titan_rs_b200 import autotune as A
from titan_rs_b200.kernel_abi import DType

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def session():
    s = tb.Session(0)
    yield s
    s.close()


def _bf16(session, arr):
    return tb.TensorHandle.from_numpy(session, arr, DType.BF16)


def _stages(result):
    return {r.candidate: r.stage for r in result.rejections}


def test_gemm_tunes_once_and_matches_the_explicit_candidate(session, tmp_path):
    m, n, k = 256, 512, 2048  # 8 output tiles: split-K is a real contender
    a = tb.fill_normal(m * k, seed=71, dtype=DType.BF16).reshape(m, k)
    b = tb.fill_normal(n * k, seed=72, std=0.02, dtype=DType.BF16).reshape(n, k)
    tuner = A.Autotuner(tmp_path / "kernels")
    rt = tb.Runtime(session, autotuner=tuner)
    req = tb.OpRequest("gemm", [_bf16(session, a), _bf16(session, b)], [tb.TensorSpec(DType.BF16, (m, n))],
                       {"transpose_rhs": True})
    h = rt.execute(req).wait()
    res = rt.last_tune
    assert res is not None and tuner.tunings == 1
    assert {x.candidate for x in res.measured} == {"gemm_bf16_tn_2sm", "gemm_bf16_tn", "gemm_bf16_tn_splitk"}
    assert _stages(res)["gemm_bf16_generic"] == "selection"
    assert h.candidate == res.entry.candidate
    got = h.outputs[0].to_numpy()
    explicit = tb.Runtime(session).execute(tb.OpRequest("gemm", req.inputs, req.outputs,
                                                        {"transpose_rhs": True, "candidate": h.candidate})).wait()
    np.testing.assert_array_equal(got, explicit.outputs[0].to_numpy())
    # Cache hit: no second search, same kernel.
    h2 = rt.execute(req).wait()
    assert rt.last_tune is None and tuner.tunings == 1 and h2.candidate == h.candidate
    # A new store reads the decision back from disk.
    tuner2 = A.Autotuner(tmp_path / "kernels")
    rt2 = tb.Runtime(session, autotuner=tuner2)
    h3 = rt2.execute(req).wait()
    assert rt2.last_tune is None and tuner2.tunings == 0 and h3.candidate == h.candidate


def test_softmax_rejects_small_register_variants_by_capability(session, tmp_path):
    x = tb.fill_normal(64 * 1000, seed=73).reshape(64, 1000).astype(np.float32)
    rt = tb.Runtime(session, autotuner=A.Autotuner(tmp_path / "k"))
    xi = tb.TensorHandle.from_numpy(session, x)
    h = rt.execute(tb.OpRequest("softmax", [xi], [tb.TensorSpec(DType.F32, (64, 1000))], {"axis": 1})).wait()
    st = _stages(rt.last_tune)
    assert all(st[c] == "capability" for c in ("softmax_f32_warp1", "softmax_f32_warp2", "softmax_f32_warp4"))
    assert {m.candidate for m in rt.last_tune.measured} == {"softmax_f32_warp8", "softmax_f32_warp16",
                                                             "softmax_f32_warp32", "softmax_f32_stream"}
    e = np.exp(x - x.max(axis=1, keepdims=True))
    np.testing.assert_allclose(h.outputs[0].to_numpy(), e / e.sum(axis=1, keepdims=True), rtol=2e-5, atol=1e-7)


def test_attention_tunes_over_the_tensor_core_candidates(session, tmp_path):
    b, hh, t, d = 1, 4, 512, 128
    q, k, v = (tb.fill_normal(b * hh * t * d, seed=74 + i, dtype=DType.BF16).reshape(b, hh, t, d) for i in range(3))
    rt = tb.Runtime(session, autotuner=A.Autotuner(tmp_path / "k"))
    h = rt.execute(tb.OpRequest("scaled_dot_product_attention", [_bf16(session, x) for x in (q, k, v)],
                                [tb.TensorSpec(DType.BF16, (b, hh, t, d))], {"causal": True})).wait()
    res = rt.last_tune
    assert {m.candidate for m in res.measured} == {"sdpa_fwd_bf16_d128_pair", "sdpa_fwd_bf16_d128_bn64",
                                                    "sdpa_fwd_bf16_d128"}
    assert _stages(res)["sdpa_bf16_generic"] == "selection"
    assert h.candidate == res.entry.candidate
    # A head dimension the tensor-core kernels do not take falls back, with records.
    q2, k2, v2 = (tb.fill_normal(1 * 2 * 64 * 64, seed=80 + i, dtype=DType.BF16).reshape(1, 2, 64, 64)
                  for i in range(3))
    h2 = rt.execute(tb.OpRequest("scaled_dot_product_attention", [_bf16(session, x) for x in (q2, k2, v2)],
                                 [tb.TensorSpec(DType.BF16, (1, 2, 64, 64))], {"causal": True})).wait()
    assert h2.candidate == "sdpa_bf16_generic"
    assert all(s == "capability" for c, s in _stages(rt.last_tune).items())


def test_conv2d_tunes_and_respects_capability(session, tmp_path):
    n, hgt, wid, c, kk = 2, 14, 14, 64, 64
    x = tb.fill_normal(n * hgt * wid * c, seed=90, dtype=DType.BF16).reshape(n, hgt, wid, c)
    w = tb.fill_normal(kk * 3 * 3 * c, seed=91, std=0.05, dtype=DType.BF16).reshape(kk, 3, 3, c)
    rt = tb.Runtime(session, autotuner=A.Autotuner(tmp_path / "k"))
    attrs = {"layout": "NHWC", "stride_h": 1, "stride_w": 1, "pad_h": 1, "pad_w": 1, "dilation_h": 1,
             "dilation_w": 1, "groups": 1}
    h = rt.execute(tb.OpRequest("conv2d", [_bf16(session, x), _bf16(session, w)],
                                [tb.TensorSpec(DType.BF16, (n, hgt, wid, kk))], attrs)).wait()
    tensor_core = ("conv2d_fprop_bf16_nhwc", "conv2d_fprop_bf16_nhwc_2sm")  # whichever measured faster
    assert h.candidate in tensor_core
    # Stride 2 runs on the tensor cores too (TMA traversal strides).
    attrs2 = {**attrs, "stride_h": 2, "stride_w": 2}
    h2 = rt.execute(tb.OpRequest("conv2d", [_bf16(session, x), _bf16(session, w)],
                                 [tb.TensorSpec(DType.BF16, (n, 7, 7, kk))], attrs2)).wait()
    assert h2.candidate in tensor_core
    # Two groups are not taken by the tensor-core kernel: the generic kernel wins, with the record.
    w2 = np.ascontiguousarray(w[..., : c // 2])
    attrs3 = {**attrs, "groups": 2}
    h3 = rt.execute(tb.OpRequest("conv2d", [_bf16(session, x), _bf16(session, w2)],
                                 [tb.TensorSpec(DType.BF16, (n, hgt, wid, kk))], attrs3)).wait()
    assert h3.candidate == "conv2d_bf16_nhwc_generic"
    assert _stages(rt.last_tune)["conv2d_fprop_bf16_nhwc"] == "capability"
    assert _stages(rt.last_tune)["conv2d_fprop_bf16_nhwc_2sm"] == "capability"


def test_explicit_candidate_bypasses_the_tuner(session, tmp_path):
    tuner = A.Autotuner(tmp_path / "k")
    rt = tb.Runtime(session, autotuner=tuner)
    x = tb.TensorHandle.from_numpy(session, np.ones((4, 256), np.float32))
    h = rt.execute(tb.OpRequest("softmax", [x], [tb.TensorSpec(DType.F32, (4, 256))],
                                {"candidate": "softmax_f32_stream"})).wait()
    assert h.candidate == "softmax_f32_stream" and tuner.tunings == 0
    with pytest.raises(tb.ExecutionError, match="unknown softmax candidate"):
        rt.execute(tb.OpRequest("softmax", [x], [tb.TensorSpec(DType.F32, (4, 256))], {"candidate": "nope"}))
