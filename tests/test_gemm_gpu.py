"""GEMM on the B200 against the CPU oracle (restated projects/titan-runtime/src/lib.rs:955-989).

Tolerances: f32 (reference ABI) is bit-exact with the oracle, because the
kernel adds separately rounded products in the reference's k order. bf16 uses
the north-star bound max|err| <= 1e-2 * max|ref| against the f32 oracle on the
same bf16 inputs.
"""
import json
import math
import pathlib

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
from titan_rs_b200 import _native as N
from titan_rs_b200.kernel_abi import DType

from gpu_util import max_rel_err, run_op, upload

pytestmark = pytest.mark.gpu

KATS = json.loads((pathlib.Path(__file__).parent / "golden" / "reference_kats.json").read_text())
BF16_TOL = 1e-2


@pytest.fixture(scope="module")
def session():
    s = tb.Session(0)
    yield s
    s.close()


@pytest.fixture(scope="module")
def rt(session):
    return tb.Runtime(session)


def bf16_inputs(m, n, k, seed, b_col_major=True):
    a = tb.fill_normal(m * k, seed=seed * 16, dtype=DType.BF16).reshape(m, k)
    shape_b = (n, k) if b_col_major else (k, n)
    b = tb.fill_normal(n * k, seed=seed * 16 + 1, std=1.0 / math.sqrt(k), dtype=DType.BF16).reshape(shape_b)
    return a, b


@pytest.mark.parametrize("case", [c for c in KATS["cases"] if c["op"] == "gemm_f32"], ids=lambda c: c["name"])
def test_gemm_f32_reference_kats_exact(session, rt, case):
    lhs = np.array(case["lhs"], np.float32).reshape(case["lhs_shape"])
    rhs = np.array(case["rhs"], np.float32).reshape(case["rhs_shape"])
    attrs = {"transpose_lhs": case["transpose_lhs"], "transpose_rhs": case["transpose_rhs"]}
    out_shape = (len(case["expected"]) // 2, 2) if case["lhs_shape"] != [2, 4] else (2, 3)
    h = run_op(rt, "gemm", [upload(session, rt.stream, lhs), upload(session, rt.stream, rhs)], DType.F32, out_shape,
               attrs)
    np.testing.assert_array_equal(h.outputs[0].to_numpy().ravel(), np.array(case["expected"], np.float32))


@pytest.mark.parametrize("m,n,k,tl,tr", [(33, 47, 70, False, False), (64, 64, 64, True, False), (5, 129, 300, False, True),
                                         (130, 3, 17, True, True)])
def test_gemm_f32_bit_exact_with_oracle(session, rt, m, n, k, tl, tr):
    rng = np.random.default_rng(m * n + k)
    lhs = rng.uniform(-1, 1, (k, m) if tl else (m, k)).astype(np.float32)
    rhs = rng.uniform(-1, 1, (n, k) if tr else (k, n)).astype(np.float32)
    h = run_op(rt, "gemm", [upload(session, rt.stream, lhs), upload(session, rt.stream, rhs)], DType.F32, (m, n),
               {"transpose_lhs": tl, "transpose_rhs": tr})
    np.testing.assert_array_equal(h.outputs[0].to_numpy(), oracle.gemm(lhs, rhs, tl, tr))


def test_gemm_f32_c1_config_exact(session, rt):
    """C1: 256^3 f32, U[-1,1) seed 0."""
    a = tb.fill_uniform(256 * 256, seed=0, low=-1, high=1).reshape(256, 256)
    b = tb.fill_uniform(256 * 256, seed=1, low=-1, high=1).reshape(256, 256)
    h = run_op(rt, "gemm", [upload(session, rt.stream, a), upload(session, rt.stream, b)], DType.F32, (256, 256))
    np.testing.assert_array_equal(h.outputs[0].to_numpy(), oracle.gemm(a, b))


@pytest.mark.parametrize("candidate", [None, "gemm_bf16_tn", "gemm_bf16_tn_2sm"])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (200, 300, 72), (1, 8, 8), (129, 257, 1032),
                                   (1000, 1000, 1000), (512, 256, 8192), (300, 1024, 136), (2304, 4352, 520)])
def test_gemm_bf16_tcgen05_matches_oracle(session, rt, m, n, k, candidate):
    a, b = bf16_inputs(m, n, k, seed=m + n + k)
    attrs = {"transpose_rhs": True}
    if candidate:
        attrs["candidate"] = candidate
    h = run_op(rt, "gemm", [upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)],
               DType.BF16, (m, n), attrs)
    assert h.candidate == candidate if candidate else h.candidate in ("gemm_bf16_tn_2sm", "gemm_bf16_tn",
                                                                      "gemm_bf16_tn_splitk")
    got = h.outputs[0].to_f32()
    rows = np.repeat(np.arange(m), n)
    cols = np.tile(np.arange(n), m)
    ref = oracle.gemm_bf16_points(a, b, True, m, n, k, rows, cols).reshape(m, n)
    assert max_rel_err(got, ref) <= BF16_TOL, max_rel_err(got, ref)
    assert np.isfinite(got).all()


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (200, 304, 72), (1, 8, 8), (129, 264, 1032),
                                   (1000, 1000, 1000), (2304, 4352, 520)])
def test_gemm_bf16_row_major_b_on_tensor_cores(session, rt, m, n, k):
    """B stored [K, N] (the reference's default layout): gemm_bf16_nn_2sm, B tiles N-contiguous."""
    a, b = bf16_inputs(m, n, k, seed=m + n + k + 7, b_col_major=False)
    h = run_op(rt, "gemm", [upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)],
               DType.BF16, (m, n))
    assert h.candidate == "gemm_bf16_nn_2sm"
    got = h.outputs[0].to_f32()
    rows = np.repeat(np.arange(m), n)
    cols = np.tile(np.arange(n), m)
    ref = oracle.gemm_bf16_points(a, b, False, m, n, k, rows, cols).reshape(m, n)
    assert max_rel_err(got, ref) <= BF16_TOL, max_rel_err(got, ref)
    assert np.isfinite(got).all()


@pytest.mark.parametrize("tr,kernel", [(True, "gemm_bf16_ta_2sm"), (False, "gemm_bf16_ta_nn_2sm")])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (200, 304, 72), (8, 8, 8), (1000, 1000, 1000), (2304, 4352, 520)])
def test_gemm_bf16_transposed_a_on_tensor_cores(session, rt, m, n, k, tr, kernel):
    """A stored [K, M] (transpose_lhs), B stored [N, K] or [K, N]: M-contiguous A tiles."""
    a, b = bf16_inputs(m, n, k, seed=m + n + k + 11, b_col_major=tr)
    at = np.ascontiguousarray(a.T)  # the stored [K, M] operand
    h = run_op(rt, "gemm", [upload(session, rt.stream, at, DType.BF16), upload(session, rt.stream, b, DType.BF16)],
               DType.BF16, (m, n), {"transpose_lhs": True, "transpose_rhs": tr})
    assert h.candidate == kernel
    got = h.outputs[0].to_f32()
    rows = np.repeat(np.arange(m), n)
    cols = np.tile(np.arange(n), m)
    ref = oracle.gemm_bf16_points(a, b, tr, m, n, k, rows, cols).reshape(m, n)
    assert max_rel_err(got, ref) <= BF16_TOL, max_rel_err(got, ref)


def test_gemm_bf16_row_major_b_full_size(session, rt):
    """8192^3 with B stored [K, N]: sampled points and the column-checksum identity."""
    M = N = K = 8192
    a = tb.fill_normal(M * K, seed=2 * 16 + 0, dtype=DType.BF16).reshape(M, K)
    b = tb.fill_normal(K * N, seed=2 * 16 + 5, std=1.0 / math.sqrt(K), dtype=DType.BF16).reshape(K, N)
    h = run_op(rt, "gemm", [upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)],
               DType.BF16, (M, N))
    assert h.candidate == "gemm_bf16_nn_2sm"
    got = h.outputs[0].to_f32()
    rng = np.random.default_rng(3)
    rows = np.concatenate([rng.integers(0, M, 4096), [0, M - 1, 255, 256]])
    cols = np.concatenate([rng.integers(0, N, 4096), [N - 1, 0, 127, 128]])
    ref = oracle.gemm_bf16_points(a, b, False, M, N, K, rows, cols)
    assert max_rel_err(got[rows, cols], ref) <= BF16_TOL
    af = tb.bf16_bits_to_f32(a).reshape(M, K).astype(np.float64)
    bf = tb.bf16_bits_to_f32(b).reshape(K, N).astype(np.float64)
    colsum_ref = af.sum(axis=0) @ bf
    colsum = got.astype(np.float64).sum(axis=0)
    assert np.max(np.abs(colsum - colsum_ref)) <= BF16_TOL * np.max(np.abs(colsum_ref))


def test_gemm_bf16_row_major_b_and_transposed_a(session, rt):
    m, n, k = 70, 90, 40
    a, b = bf16_inputs(m, n, k, seed=5, b_col_major=False)
    h = run_op(rt, "gemm", [upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)],
               DType.BF16, (m, n))
    ref = oracle.gemm(tb.bf16_bits_to_f32(a).reshape(m, k), tb.bf16_bits_to_f32(b).reshape(k, n))
    assert max_rel_err(h.outputs[0].to_f32(), ref) <= BF16_TOL
    at = np.ascontiguousarray(a.T)
    h = run_op(rt, "gemm", [upload(session, rt.stream, at, DType.BF16), upload(session, rt.stream, b, DType.BF16)],
               DType.BF16, (m, n), {"transpose_lhs": True})
    assert max_rel_err(h.outputs[0].to_f32(), ref) <= BF16_TOL


@pytest.mark.parametrize("tl,tr,m,n,k", [
    (False, True, 300, 500, 1001),   # K % 8 != 0: no operand row starts 16-byte aligned
    (False, False, 257, 333, 515),   # B row-major [K, N] with N % 8 != 0
    (True, True, 333, 520, 777),     # A stored [K, M] with M % 8 != 0
    (True, False, 129, 130, 1023),   # both stored transposed, all extents ragged
    (False, False, 264, 130, 1001),  # A [M, K] with K ragged and B [K, N] with N ragged
    (True, True, 1000, 1001, 999),   # A [K, M] ragged, B [N, K] ragged
    (False, True, 4096, 1001, 512),  # operands fine, output rows not 16-byte aligned: C through an aligned copy
    (False, False, 520, 1000, 777),  # A [M, K] ragged; B [K, N] and C fine
])
def test_gemm_bf16_staged_for_storage_the_tma_cannot_describe(session, rt, tl, tr, m, n, k):
    """Each operand whose rows the TMA cannot read is copied in its own storage order
    with its rows padded to a multiple of 8 elements (zeros), then the tensor-core
    kernel for that order runs; the CUDA-core kernel is the cross-check."""
    a = tb.fill_normal(m * k, seed=m + k, dtype=DType.BF16).reshape((k, m) if tl else (m, k))
    b = tb.fill_normal(n * k, seed=n + k, std=1.0 / math.sqrt(k), dtype=DType.BF16).reshape((n, k) if tr else (k, n))
    ta, tbb = upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)
    attrs = {"transpose_lhs": tl, "transpose_rhs": tr}
    h = run_op(rt, "gemm", [ta, tbb], DType.BF16, (m, n), attrs)
    assert h.candidate == "gemm_bf16_staged"
    got = h.outputs[0].to_f32()
    ref = oracle.gemm(tb.bf16_bits_to_f32(a).reshape(a.shape), tb.bf16_bits_to_f32(b).reshape(b.shape), tl, tr)
    assert max_rel_err(got, ref) <= BF16_TOL
    generic = run_op(rt, "gemm", [ta, tbb], DType.BF16, (m, n), {**attrs, "candidate": "gemm_bf16_generic"})
    assert max_rel_err(got, generic.outputs[0].to_f32()) <= BF16_TOL


@pytest.mark.parametrize("candidate", [None, "gemm_bf16_tn_2sm"])
def test_gemm_bf16_full_c3_config(session, rt, candidate):
    """C3: 8192^3, A N(0,1), B column-major N(0,1/8192), seed 2. Sampled points against the
    oracle, then two size-independent properties over every element: finiteness and the
    column-checksum identity 1^T C = (1^T A) B (fp64)."""
    M = N = K = 8192
    a = tb.fill_normal(M * K, seed=2 * 16 + 0, dtype=DType.BF16).reshape(M, K)
    b = tb.fill_normal(N * K, seed=2 * 16 + 1, std=1.0 / math.sqrt(K), dtype=DType.BF16).reshape(N, K)
    attrs = {"transpose_rhs": True}
    if candidate:
        attrs["candidate"] = candidate
    h = run_op(rt, "gemm", [upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)],
               DType.BF16, (M, N), attrs)
    if candidate:
        assert h.candidate == candidate
    got = h.outputs[0].to_f32()
    rng = np.random.default_rng(2)
    rows = rng.integers(0, M, 4096)
    cols = rng.integers(0, N, 4096)
    # Corners and tile edges too.
    rows = np.concatenate([rows, [0, 0, M - 1, M - 1, 127, 128, 255, 256]])
    cols = np.concatenate([cols, [0, N - 1, 0, N - 1, 255, 256, 511, 512]])
    ref = oracle.gemm_bf16_points(a, b, True, M, N, K, rows, cols)
    assert max_rel_err(got[rows, cols], ref) <= BF16_TOL
    assert np.isfinite(got).all()
    af = tb.bf16_bits_to_f32(a).reshape(M, K).astype(np.float64)
    bf = tb.bf16_bits_to_f32(b).reshape(N, K).astype(np.float64)
    colsum_ref = af.sum(axis=0) @ bf.T
    colsum = got.astype(np.float64).sum(axis=0)
    assert np.max(np.abs(colsum - colsum_ref)) <= BF16_TOL * np.max(np.abs(colsum_ref))


def test_gemm_bf16_is_bit_reproducible(session, rt):
    a, b = bf16_inputs(640, 768, 512, seed=11)
    ta, tbb = upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)
    r1 = run_op(rt, "gemm", [ta, tbb], DType.BF16, (640, 768), {"transpose_rhs": True}).outputs[0].to_numpy()
    r2 = run_op(rt, "gemm", [ta, tbb], DType.BF16, (640, 768), {"transpose_rhs": True}).outputs[0].to_numpy()
    np.testing.assert_array_equal(r1, r2)


def test_gemm_contract_rejections(session, rt):
    """projects/titan-runtime/tests/cpu_reference_ops.rs:82-113 keywords."""
    lhs = upload(session, rt.stream, np.arange(1, 7, dtype=np.float32).reshape(2, 3))
    rhs22 = upload(session, rt.stream, np.ones((2, 2), np.float32))
    rhs32 = upload(session, rt.stream, np.ones((3, 2), np.float32))
    vec = upload(session, rt.stream, np.ones(3, np.float32))

    def err(inputs, shape, dtype=DType.F32, layout="Contiguous", attrs=None):
        with pytest.raises(tb.ExecutionError) as e:
            rt.execute(tb.OpRequest("gemm", inputs, [tb.TensorSpec(dtype, shape, layout=layout)], attrs or {}))
        assert e.value.phase == "contract"
        return e.value.message

    assert "inner dimensions" in err([lhs, rhs22], (2, 2))
    assert "rank-2" in err([vec, rhs22], (2, 2))
    assert "output shape" in err([lhs, rhs32], (3, 2))
    assert "F32" in err([lhs, rhs32], (2, 2), dtype=DType.I32)
    assert "contiguous" in err([lhs, rhs32], (2, 2), layout="Strided")
    assert "exactly two" in err([lhs], (2, 2))
    assert "unsupported attributes" in err([lhs, rhs32], (2, 2), attrs={"alpha": 2})


@pytest.mark.parametrize("m,n,k", [(128, 256, 65536), (512, 512, 16384), (300, 700, 9000), (256, 256, 1024)])
def test_gemm_bf16_split_k_matches_oracle(session, rt, m, n, k):
    """Few output tiles and a long K: the op splits K over the SMs (fp32 partials in the
    stream's scratch memory, then a fixed-order reduction)."""
    a, b = bf16_inputs(m, n, k, seed=m + n + k + 7)
    ta, tbb = upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)
    h = run_op(rt, "gemm", [ta, tbb], DType.BF16, (m, n), {"transpose_rhs": True})
    assert h.candidate == "gemm_bf16_tn_splitk"
    got = h.outputs[0].to_f32()
    rows = np.repeat(np.arange(m), n)
    cols = np.tile(np.arange(n), m)
    ref = oracle.gemm_bf16_points(a, b, True, m, n, k, rows, cols).reshape(m, n)
    assert max_rel_err(got, ref) <= BF16_TOL, max_rel_err(got, ref)
    # Same inputs, one K slice per tile: equal within bf16 rounding, and split-K is deterministic.
    whole = run_op(rt, "gemm", [ta, tbb], DType.BF16, (m, n), {"transpose_rhs": True, "candidate": "gemm_bf16_tn"})
    assert whole.candidate == "gemm_bf16_tn"
    assert max_rel_err(got, whole.outputs[0].to_f32()) <= BF16_TOL
    again = run_op(rt, "gemm", [ta, tbb], DType.BF16, (m, n), {"transpose_rhs": True})
    np.testing.assert_array_equal(again.outputs[0].to_numpy(), h.outputs[0].to_numpy())


def test_gemm_candidate_attribute(session, rt):
    a, b = bf16_inputs(256, 512, 256, seed=3)
    ta, tbb = upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)
    forced = run_op(rt, "gemm", [ta, tbb], DType.BF16, (256, 512), {"transpose_rhs": True,
                                                                    "candidate": "gemm_bf16_tn_splitk"})
    assert forced.candidate == "gemm_bf16_tn_splitk"
    generic = run_op(rt, "gemm", [ta, tbb], DType.BF16, (256, 512), {"transpose_rhs": True,
                                                                     "candidate": "gemm_bf16_generic"})
    assert generic.candidate == "gemm_bf16_generic"
    assert max_rel_err(forced.outputs[0].to_f32(), generic.outputs[0].to_f32()) <= BF16_TOL
    staged = run_op(rt, "gemm", [ta, tbb], DType.BF16, (256, 512), {"transpose_rhs": True,
                                                                    "candidate": "gemm_bf16_staged"})
    assert staged.candidate == "gemm_bf16_staged"
    assert max_rel_err(forced.outputs[0].to_f32(), staged.outputs[0].to_f32()) <= BF16_TOL
    with pytest.raises(tb.ExecutionError, match="unknown GEMM candidate"):
        run_op(rt, "gemm", [ta, tbb], DType.BF16, (256, 512), {"transpose_rhs": True, "candidate": "nope"})
    x = upload(session, rt.stream, np.ones((8, 8), np.float32))
    with pytest.raises(tb.ExecutionError, match="does not take F32") as e:
        run_op(rt, "gemm", [x, x], DType.F32, (8, 8), {"candidate": "gemm_bf16_tn"})
    assert e.value.status == N.TB_ERR_UNSUPPORTED


@pytest.mark.parametrize("tl,tr,m,n,k", [(False, False, 4096, 4095, 4096), (True, True, 4095, 4096, 4096),
                                         (False, True, 4096, 4096, 4095)])
def test_gemm_bf16_staged_at_full_width(session, rt, tl, tr, m, n, k):
    """Ragged extents at 4096: the padded copies feed the 2-SM kernels (sampled oracle points,
    the last row and column included)."""
    a = tb.fill_normal(m * k, seed=7, dtype=DType.BF16).reshape((k, m) if tl else (m, k))
    b = tb.fill_normal(n * k, seed=8, std=1.0 / math.sqrt(k), dtype=DType.BF16).reshape((n, k) if tr else (k, n))
    h = run_op(rt, "gemm", [upload(session, rt.stream, a, DType.BF16), upload(session, rt.stream, b, DType.BF16)],
               DType.BF16, (m, n), {"transpose_lhs": tl, "transpose_rhs": tr})
    assert h.candidate == "gemm_bf16_staged"
    got = h.outputs[0].to_f32()
    rng = np.random.default_rng(5)
    rows = np.concatenate([rng.integers(0, m, 2048), [0, m - 1, m - 1, 0]])
    cols = np.concatenate([rng.integers(0, n, 2048), [0, n - 1, 0, n - 1]])
    a_mk = np.ascontiguousarray(a.T) if tl else a
    ref = oracle.gemm_bf16_points(a_mk, b, tr, m, n, k, rows, cols)
    assert max_rel_err(got[rows, cols], ref) <= BF16_TOL
    assert np.isfinite(got).all()

