"""Attention sharded over batch x heads and conv2d sharded over the batch, with no
communication (the north star's SDPA and conv2d partitioning of one 8-GPU box).

Each rank's part (distributed.local_request / execute_local) is a view of its units,
so every rank's result can be produced on one GPU, one rank after another, and
checked: against the CPU oracle on that rank's rows/outputs, and bit for bit against
the same units of the unsharded call (every unit is computed by the same kernel
code whichever grid it sits in). Ragged splits (units % ranks != 0) included. The
2-process form over two GPUs is in test_multigpu_gpu.py."""
import math

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
from titan_rs_b200 import distributed as D
from titan_rs_b200.kernel_abi import DType

from gpu_util import max_rel_err, upload

pytestmark = pytest.mark.gpu
BF16_TOL = 1e-2


@pytest.fixture(scope="module")
def session():
    s = tb.Session(0)
    yield s
    s.close()


@pytest.fixture(scope="module")
def rt(session):
    return tb.Runtime(session)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_sdpa_bh_shards_match_the_oracle_and_the_whole_call(session, rt, world):
    b, h, t, d = 2, 3, 384, 128  # 6 (b, h) pairs: 3 and 8 ranks split them unevenly
    q, k, v = (tb.fill_normal(b * h * t * d, seed=300 + i, dtype=DType.BF16).reshape(b, h, t, d) for i in range(3))
    ins = [upload(session, rt.stream, x, DType.BF16) for x in (q, k, v)]
    req = tb.OpRequest("scaled_dot_product_attention", ins, [tb.TensorSpec(DType.BF16, q.shape)], {"causal": True})
    whole = rt.execute(req)
    whole.wait()
    full = whole.outputs[0].to_numpy().reshape(b * h, t, d)
    covered = []
    for rank in range(world):
        hdl, (lo, hi) = D.execute_local(rt, req, world, rank)
        covered.extend(range(lo, hi))
        if hdl is None:
            assert hi == lo
            continue
        hdl.wait()
        assert hdl.candidate == "sdpa_fwd_bf16_d128_pair"
        got = hdl.outputs[0].to_numpy().reshape(hi - lo, t, d)
        np.testing.assert_array_equal(got, full[lo:hi])
        rows = np.arange(lo * t, hi * t)
        ref = oracle.sdpa_bf16_rows(q, k, v, b, h, t, t, d, True, rows).reshape(hi - lo, t, d)
        assert max_rel_err(tb.bf16_bits_to_f32(got).reshape(ref.shape), ref) <= BF16_TOL
    assert covered == list(range(b * h))


@pytest.mark.parametrize("world", [2, 3])
def test_conv2d_batch_shards_match_the_oracle_and_the_whole_call(session, rt, world):
    n, hw, cin, cout = 5, 14, 64, 256
    x = tb.fill_normal(n * hw * hw * cin, seed=320, dtype=DType.BF16).reshape(n, hw, hw, cin)
    w = tb.fill_normal(cout * 9 * cin, seed=321, std=math.sqrt(2.0 / (9 * cin)), dtype=DType.BF16).reshape(
        cout, 3, 3, cin)
    attrs = {"stride_h": 1, "stride_w": 1, "pad_h": 1, "pad_w": 1, "dilation_h": 1, "dilation_w": 1, "groups": 1,
             "layout": "NHWC"}
    ins = [upload(session, rt.stream, x, DType.BF16), upload(session, rt.stream, w, DType.BF16)]
    req = tb.OpRequest("conv2d", ins, [tb.TensorSpec(DType.BF16, (n, hw, hw, cout))], attrs)
    whole = rt.execute(req)
    whole.wait()
    full = whole.outputs[0].to_numpy()
    per_image = hw * hw * cout
    covered = []
    for rank in range(world):
        hdl, (lo, hi) = D.execute_local(rt, req, world, rank)
        covered.extend(range(lo, hi))
        hdl.wait()
        got = hdl.outputs[0].to_numpy()
        assert got.shape == (hi - lo, hw, hw, cout)
        np.testing.assert_array_equal(got, full[lo:hi])
        idx = np.arange(lo * per_image, hi * per_image)
        ref = oracle.conv2d_nhwc_bf16_points(x, w, None, n, hw, hw, cin, cout, 3, 3, (1, 1), (1, 1), (1, 1), hw, hw,
                                             idx)
        assert max_rel_err(tb.bf16_bits_to_f32(got).ravel(), ref) <= BF16_TOL
    assert covered == list(range(n))


def test_gemm_is_not_a_communication_free_shard(session, rt):
    a = upload(session, rt.stream, np.zeros((8, 8), np.float32))
    with pytest.raises(ValueError, match="collective"):
        D.local_request(tb.OpRequest("gemm", [a, a], [tb.TensorSpec(DType.F32, (8, 8))]), 2, 0)
