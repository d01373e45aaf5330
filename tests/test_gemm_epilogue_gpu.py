"""gemm.bias_act (the GEMM with a fused bias + GELU/SiLU epilogue) on the B200 against
the oracle: the reference's gemm (titan-runtime/src/lib.rs:955-989) on the same bf16
inputs, plus the bias, then its gelu (:625-640) or silu (:3064) in f32. Tolerance:
the bf16 bound max|err| <= 1e-2 * max|ref|."""
import math

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
from titan_rs_b200.kernel_abi import DType

from gpu_util import max_rel_err, run_op, upload

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


def _inputs(m, n, k, seed):
    a = tb.fill_normal(m * k, seed=seed * 16, dtype=DType.BF16)
    b = tb.fill_normal(n * k, seed=seed * 16 + 1, std=1.0 / math.sqrt(k), dtype=DType.BF16)
    bias = tb.fill_normal(n, seed=seed * 16 + 2, std=0.5)
    return a, b, bias


def _reference(a, b, bias, m, n, k, act):
    rows, cols = np.divmod(np.arange(m * n), n)
    acc = oracle.gemm_bf16_points(a, b, True, m, n, k, rows, cols).reshape(m, n)
    if bias is not None:
        acc = (acc + bias[None, :]).astype(np.float32)
    return {"none": lambda x: x, "gelu": oracle.gelu, "silu": oracle.silu}[act](acc)


@pytest.mark.parametrize("candidate", [None, "gemm_bf16_tn_bias_act_2sm"])
@pytest.mark.parametrize("act", ["none", "gelu", "silu"])
@pytest.mark.parametrize("with_bias", [True, False])
@pytest.mark.parametrize("m,n,k", [(300, 520, 1024), (128, 256, 64), (517, 264, 2048)])
def test_gemm_bias_act_matches_oracle(session, rt, m, n, k, act, with_bias, candidate):
    a, b, bias = _inputs(m, n, k, seed=m + n + k)
    ins = [upload(session, rt.stream, a.reshape(m, k), DType.BF16), upload(session, rt.stream, b.reshape(n, k), DType.BF16)]
    if with_bias:
        ins.append(upload(session, rt.stream, bias))
    attrs = {"transpose_rhs": True, "activation": act}
    if candidate:
        attrs["candidate"] = candidate
    h = run_op(rt, "gemm.bias_act", ins, DType.BF16, (m, n), attrs)
    assert h.candidate == (candidate or "gemm_bf16_tn_bias_act")
    got = h.outputs[0].to_f32()
    ref = _reference(a, b, bias if with_bias else None, m, n, k, act)
    assert np.isfinite(got).all()
    assert max_rel_err(got, ref) <= BF16_TOL, max_rel_err(got, ref)


def test_bias_act_defaults_to_pairs_on_large_outputs(session, rt):
    """1024 x 4864 holds 152 tiles of 128 x 256 (>= one wave of 148 SMs): the 2-SM kernel."""
    m, n, k = 1024, 4864, 256
    a, b, bias = _inputs(m, n, k, seed=6)
    ins = [upload(session, rt.stream, a.reshape(m, k), DType.BF16), upload(session, rt.stream, b.reshape(n, k), DType.BF16),
           upload(session, rt.stream, bias)]
    h = run_op(rt, "gemm.bias_act", ins, DType.BF16, (m, n), {"transpose_rhs": True, "activation": "gelu"})
    assert h.candidate == "gemm_bf16_tn_bias_act_2sm"
    ref = _reference(a, b, bias, m, n, k, "gelu")
    assert max_rel_err(h.outputs[0].to_f32(), ref) <= BF16_TOL


@pytest.mark.parametrize("fused_cand,plain_cand", [("gemm_bf16_tn_bias_act", "gemm_bf16_tn"),
                                                   ("gemm_bf16_tn_bias_act_2sm", "gemm_bf16_tn_2sm")])
def test_no_bias_no_activation_equals_plain_gemm_bitwise(session, rt, fused_cand, plain_cand):
    m, n, k = 640, 512, 1024
    a, b, _ = _inputs(m, n, k, seed=5)
    ta, tbb = upload(session, rt.stream, a.reshape(m, k), DType.BF16), upload(session, rt.stream, b.reshape(n, k), DType.BF16)
    fused = run_op(rt, "gemm.bias_act", [ta, tbb], DType.BF16, (m, n),
                   {"transpose_rhs": True, "activation": "none", "candidate": fused_cand})
    plain = run_op(rt, "gemm", [ta, tbb], DType.BF16, (m, n), {"transpose_rhs": True, "candidate": plain_cand})
    np.testing.assert_array_equal(fused.outputs[0].to_numpy(), plain.outputs[0].to_numpy())


@pytest.mark.parametrize("tl,tr,kernel", [(False, False, "gemm_bf16_nn_2sm"), (True, True, "gemm_bf16_ta_2sm"),
                                          (True, False, "gemm_bf16_ta_nn_2sm")])
@pytest.mark.parametrize("act", ["none", "gelu", "silu"])
def test_gemm_bias_act_other_storage_orders(session, rt, tl, tr, kernel, act):
    """A stored [K, M] and/or B stored [K, N]: the layout kernels with the same epilogue."""
    m, n, k = 264, 520, 1032
    a, b, bias = _inputs(m, n, k, seed=13)
    a2, b2 = a.reshape(m, k), b.reshape(n, k)  # the logical A [M, K] and B^T [N, K]
    a_stored = np.ascontiguousarray(a2.T) if tl else a2
    b_stored = b2 if tr else np.ascontiguousarray(b2.T)
    ins = [upload(session, rt.stream, a_stored, DType.BF16), upload(session, rt.stream, b_stored, DType.BF16),
           upload(session, rt.stream, bias)]
    h = run_op(rt, "gemm.bias_act", ins, DType.BF16, (m, n),
               {"transpose_lhs": tl, "transpose_rhs": tr, "activation": act})
    assert h.candidate == kernel
    ref = _reference(a, b, bias, m, n, k, act)
    assert max_rel_err(h.outputs[0].to_f32(), ref) <= BF16_TOL


def test_gemm_bias_act_contract(session, rt):
    m, n, k = 64, 128, 64
    a, b, bias = _inputs(m, n, k, seed=9)
    ta, tbb = upload(session, rt.stream, a.reshape(m, k), DType.BF16), upload(session, rt.stream, b.reshape(n, k), DType.BF16)

    def err(inputs, attrs, shape=(m, n)):
        with pytest.raises(tb.ExecutionError) as e:
            run_op(rt, "gemm.bias_act", inputs, DType.BF16, shape, attrs)
        return e.value

    e = err([ta, tbb, upload(session, rt.stream, bias[: n // 2])], {"transpose_rhs": True})
    assert e.phase == "contract" and "F32 [N]" in e.message
    assert "activation" in err([ta, tbb], {"transpose_rhs": True, "activation": "relu"}).message
    assert "unsupported attributes" in err([ta, tbb], {"transpose_rhs": True, "axis": 1}).message
    assert "output shape" in err([ta, tbb], {"transpose_rhs": True}, shape=(m, n + 8)).message


@pytest.mark.parametrize("tl,tr,m,n,k", [(False, False, 264, 124, 1032),   # B stored [K, N], N % 8 != 0
                                         (False, True, 300, 520, 1001),    # K % 8 != 0
                                         (True, False, 261, 136, 520),     # A stored [K, M], M % 8 != 0
                                         (False, True, 300, 522, 1024),    # only C's rows misaligned
                                         (True, True, 264, 1001, 520)])    # layout kernel order, C misaligned
@pytest.mark.parametrize("act", ["gelu", "silu"])
def test_gemm_bias_act_staged_for_storage_the_tma_cannot_describe(session, rt, tl, tr, m, n, k, act):
    """Operands the TMA cannot read are copied with rows padded to 8 elements, storage order
    kept, then the bias/activation epilogue of the kernel for that order runs."""
    a, b, bias = _inputs(m, n, k, seed=m + n + k + 1)
    a2, b2 = a.reshape(m, k), b.reshape(n, k)
    a_stored = np.ascontiguousarray(a2.T) if tl else a2
    b_stored = b2 if tr else np.ascontiguousarray(b2.T)
    ins = [upload(session, rt.stream, a_stored, DType.BF16), upload(session, rt.stream, b_stored, DType.BF16),
           upload(session, rt.stream, bias)]
    h = run_op(rt, "gemm.bias_act", ins, DType.BF16, (m, n),
               {"transpose_lhs": tl, "transpose_rhs": tr, "activation": act})
    assert h.candidate == "gemm_bf16_staged"
    ref = _reference(a, b, bias, m, n, k, act)
    assert max_rel_err(h.outputs[0].to_f32(), ref) <= BF16_TOL
