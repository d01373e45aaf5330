"""Pins the CPU oracle against titan.rs's own known-answer vectors (CPU only).

Every case in tests/golden/reference_kats.json is transcribed from a reference
test file (cited in the fixture). The oracle must reproduce each within the
tolerance that reference test uses, and must reject the same invalid contracts.
"""
import json
import math
import pathlib

import numpy as np
import pytest

import oracle

KATS = json.loads((pathlib.Path(__file__).parent / "golden" / "reference_kats.json").read_text())


def _cases(op):
    return [c for c in KATS["cases"] if c["op"] == op]


@pytest.mark.parametrize("case", _cases("gemm_f32"), ids=lambda c: c["name"])
def test_gemm_kats(case):
    lhs = np.array(case["lhs"], dtype=np.float32).reshape(case["lhs_shape"])
    rhs = np.array(case["rhs"], dtype=np.float32).reshape(case["rhs_shape"])
    out = oracle.gemm(lhs, rhs, case["transpose_lhs"], case["transpose_rhs"])
    np.testing.assert_array_equal(out.ravel(), np.array(case["expected"], dtype=np.float32))


@pytest.mark.parametrize("case", _cases("softmax_f32"), ids=lambda c: c["name"])
def test_softmax_kats(case):
    x = np.array(case["input"], dtype=np.float32).reshape(case["shape"])
    y = oracle.softmax(x, axis=-1).ravel()
    assert np.max(np.abs(y - np.array(case["expected"]))) <= case["tolerance"]
    for i, e in zip(case.get("check_indices", []), case.get("expected_at_indices", [])):
        assert abs(y[i] - e) < 1e-6
    rows = y.reshape(case["shape"]).sum(axis=-1)
    assert np.all(np.abs(rows - 1.0) <= 2e-6)


@pytest.mark.parametrize("case", _cases("sdpa_f32"), ids=lambda c: c["name"])
def test_sdpa_kats(case):
    q = np.array(case["q"], dtype=np.float32).reshape(case["q_shape"])
    k = np.array(case["k"], dtype=np.float32).reshape(case["kv_shape"])
    v = np.array(case["v"], dtype=np.float32).reshape(case["kv_shape"])
    out = oracle.sdpa(q, k, v, causal=case["causal"]).ravel()
    assert np.max(np.abs(out - np.array(case["expected"]))) < case["tolerance"]


@pytest.mark.parametrize("case", _cases("conv2d_f32"), ids=lambda c: c["name"])
def test_conv2d_kats(case):
    x = np.array(case["x"], dtype=np.float32).reshape(case["x_shape"])
    w = np.array(case["w"], dtype=np.float32).reshape(case["w_shape"])
    b = None if case["bias"] is None else np.array(case["bias"], dtype=np.float32)
    out = oracle.conv2d_nchw(x, w, b, case["stride"], case["pad"], case["dilation"], case["groups"])
    assert list(out.shape) == case["out_shape"]
    assert np.max(np.abs(out.ravel() - np.array(case["expected"]))) <= max(case["tolerance"], 0.0)


def test_gemm_rejections():
    lhs = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    with pytest.raises(oracle.OracleError, match="inner dimensions"):
        oracle.gemm(lhs, np.ones((2, 2), np.float32))
    with pytest.raises(oracle.OracleError, match="rank-2"):
        oracle.gemm(np.ones(3, np.float32), np.ones((2, 2), np.float32))
    with pytest.raises(oracle.OracleError, match="output shape"):
        oracle.gemm(lhs, np.ones((3, 2), np.float32), out_shape=(3, 2))


def test_conv2d_rejections():
    x = np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3)
    w = np.array([1, 0, 0, -1], dtype=np.float32).reshape(1, 1, 2, 2)
    with pytest.raises(oracle.OracleError, match="rank-4"):
        oracle.conv2d_nchw(x[0], w, None, (1, 1), (0, 0), (1, 1), 1)
    with pytest.raises(oracle.OracleError, match="non-zero"):
        oracle.conv2d_nchw(x, w, None, (1, 1), (0, 0), (1, 1), 0, out_shape=(1, 1, 2, 2))
    with pytest.raises(oracle.OracleError, match="output shape"):
        oracle.conv2d_nchw(x, w, None, (1, 1), (0, 0), (1, 1), 1, out_shape=(1, 1, 1, 2))
    with pytest.raises(oracle.OracleError, match="channels"):
        oracle.conv2d_nchw(x, np.ones((1, 2, 2, 2), np.float32), None, (1, 1), (0, 0), (1, 1), 1)
    with pytest.raises(oracle.OracleError, match="bias"):
        oracle.conv2d_nchw(x, w, np.ones(2, np.float32), (1, 1), (0, 0), (1, 1), 1)


def test_bf16_rounding_is_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf, -np.inf], dtype=np.float32)
    bits = oracle.f32_to_bf16_bits(vals)
    back = oracle.bf16_bits_to_f32(bits)
    # 1 + 2^-8 is exactly halfway between bf16 neighbours 1 and 1+2^-7: ties to even -> 1.
    assert back[1] == 1.0
    # 1 + 3*2^-8 is halfway between 1+2^-7 and 1+2^-6: ties to even -> 1+2^-6.
    assert back[2] == 1.015625
    assert back[3] == -2.5 and np.isinf(back[5]) and np.isinf(back[6])
    lib = oracle.lib()
    for v in vals:
        assert lib.oracle_f32_to_bf16(float(v)) == int(oracle.f32_to_bf16_bits(np.array([v], np.float32))[0])


def test_gemm_bf16_points_match_full_f32_loops():
    rng = np.random.default_rng(7)
    m, n, k = 33, 47, 70
    a = oracle.f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
    bt = oracle.f32_to_bf16_bits(rng.standard_normal((n, k)).astype(np.float32))  # column-major B == [N,K]
    full = oracle.gemm(oracle.bf16_bits_to_f32(a).reshape(m, k), oracle.bf16_bits_to_f32(bt).reshape(n, k),
                       transpose_rhs=True)
    rows = np.repeat(np.arange(m), n)
    cols = np.tile(np.arange(n), m)
    pts = oracle.gemm_bf16_points(a, bt, True, m, n, k, rows, cols)
    np.testing.assert_array_equal(pts.reshape(m, n), full)
    # Row-major B gives the same numbers for the transposed storage.
    b_rm = np.ascontiguousarray(bt.reshape(n, k).T)
    pts2 = oracle.gemm_bf16_points(a, b_rm, False, m, n, k, rows, cols)
    np.testing.assert_array_equal(pts2, pts)


def test_sdpa_bf16_rows_match_full_and_causal_mask():
    rng = np.random.default_rng(3)
    b, h, t, d = 2, 3, 9, 16
    q, k, v = (oracle.f32_to_bf16_bits(rng.standard_normal((b, h, t, d)).astype(np.float32)) for _ in range(3))
    qf, kf, vf = (oracle.bf16_bits_to_f32(z).reshape(b, h, t, d) for z in (q, k, v))
    for causal in (False, True):
        full = oracle.sdpa(qf, kf, vf, causal=causal)
        ids = np.arange(b * h * t)
        rows = oracle.sdpa_bf16_rows(q, k, v, b, h, t, t, d, causal, ids)
        np.testing.assert_array_equal(rows, full.reshape(-1, d))
    # Causal row 0 attends only to key 0: output equals v[...,0,:].
    full = oracle.sdpa(qf, kf, vf, causal=True)
    np.testing.assert_array_equal(full[:, :, 0, :], vf[:, :, 0, :])
    # Against float64 numpy.
    s = np.einsum("bhid,bhjd->bhij", qf.astype(np.float64), kf.astype(np.float64)) / math.sqrt(d)
    s = np.where(np.tril(np.ones((t, t), bool)), s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ref = p @ vf.astype(np.float64)
    assert np.max(np.abs(full - ref)) < 1e-5


def test_conv2d_nhwc_points_match_nchw_reference():
    rng = np.random.default_rng(4)
    n, h, w, cin, cout, r, s = 2, 7, 6, 5, 4, 3, 3
    stride, pad, dil = (2, 1), (1, 2), (1, 2)
    x = oracle.f32_to_bf16_bits(rng.standard_normal((n, h, w, cin)).astype(np.float32))
    wt = oracle.f32_to_bf16_bits(rng.standard_normal((cout, r, s, cin)).astype(np.float32))
    bias = rng.standard_normal(cout).astype(np.float32)
    xf = oracle.bf16_bits_to_f32(x).reshape(n, h, w, cin)
    wf = oracle.bf16_bits_to_f32(wt).reshape(cout, r, s, cin)
    ref = oracle.conv2d_nchw(xf.transpose(0, 3, 1, 2), wf.transpose(0, 3, 1, 2), bias, stride, pad, dil, 1)
    ho, wo = ref.shape[2:]
    idx = np.arange(n * ho * wo * cout)
    pts = oracle.conv2d_nhwc_bf16_points(x, wt, bias, n, h, w, cin, cout, r, s, stride, pad, dil, ho, wo, idx)
    np.testing.assert_array_equal(pts.reshape(n, ho, wo, cout), ref.transpose(0, 2, 3, 1))


def test_softmax_mt_matches_single_thread():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 257)) * 2).astype(np.float32)
    np.testing.assert_array_equal(oracle.softmax_rows_mt(x), oracle.softmax(x))


def test_gelu_and_silu_match_the_reference_known_answers():
    """projects/titan-runtime/tests/cpu_reference_ops.rs:438-442."""
    x = np.array([-1.0, 0.0, 1.0], np.float32)
    s = oracle.silu(x)
    assert abs(s[0] + 0.26894143) < 1e-6 and s[1] == 0.0 and abs(s[2] - 0.7310586) < 1e-6
    g = oracle.gelu(x)
    assert abs(g[0] + 0.15865526) < 2e-6 and g[1] == 0.0 and abs(g[2] - 0.8413447) < 2e-6
    # The erf polynomial (|error| <= 1.5e-7) against the exact GELU over a range.
    from math import erf
    xs = np.linspace(-8, 8, 4001, dtype=np.float32)
    exact = np.array([0.5 * v * (1 + erf(v / 2 ** 0.5)) for v in xs.astype(np.float64)])
    assert np.max(np.abs(oracle.gelu(xs) - exact)) < 2e-6


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("seed,count", [(0, 1), (1, 4097), (33, 1 << 17), (48, 3 * (1 << 16) + 5)])
def test_oracle_generator_is_bit_identical_to_the_library(seed, count, bf16):
    """The reference arm of bench.py makes its inputs with the oracle's generator so it never
    loads the product library; both must produce the same bits for every seed and slice."""
    import titan_rs_b200 as tb
    from titan_rs_b200.kernel_abi import DType
    dt = DType.BF16 if bf16 else DType.F32
    for mean, std in [(0.0, 1.0), (0.0, 2.0), (0.5, 1.0 / 90.5)]:
        want = tb.fill_normal(count, seed=seed, mean=mean, std=std, dtype=dt)
        got = oracle.fill_normal(count, seed, mean, std, bf16=bf16, threads=3)
        assert want.dtype == got.dtype and want.tobytes() == got.tobytes()
    want = tb.fill_uniform(count, seed=seed, low=-1.0, high=1.0, dtype=dt)
    assert want.tobytes() == oracle.fill_uniform(count, seed, -1.0, 1.0, bf16=bf16).tobytes()
    # A slice made on its own equals the same slice of the whole fill (odd start included).
    lo = count // 3 | 1 if count > 2 else 0
    part = oracle.fill_normal(count - lo, seed, 0.0, 1.0, bf16=bf16, first=lo)
    assert part.tobytes() == tb.fill_normal(count, seed=seed, dtype=dt)[lo:].tobytes()
