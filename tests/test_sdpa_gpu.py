"""Scaled-dot-product attention on the B200 against the CPU oracle
(restated projects/titan-runtime/src/lib.rs:1090-1151, plus the causal extension).

Tolerances: f32 (reference ABI) uses the reference GPU test's 2e-4
(projects/titan-runtime/tests/cuda_attention.rs:88-91); bf16 uses the north-star
bound max|err| <= 1e-2 * max|ref| against the f32 oracle on the same bf16 inputs.
"""
import json
import pathlib

import numpy as np
import pytest

import oracle
import titan_rs_b200 as tb
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


def qkv_bf16(b, h, tq, tk, d, seed):
    q = tb.fill_normal(b * h * tq * d, seed=seed * 16, dtype=DType.BF16).reshape(b, h, tq, d)
    k = tb.fill_normal(b * h * tk * d, seed=seed * 16 + 1, dtype=DType.BF16).reshape(b, h, tk, d)
    v = tb.fill_normal(b * h * tk * d, seed=seed * 16 + 2, dtype=DType.BF16).reshape(b, h, tk, d)
    return q, k, v


TC_CANDIDATES = ["sdpa_fwd_bf16_d128_bn64", "sdpa_fwd_bf16_d128_pair", "sdpa_fwd_bf16_d128", "sdpa_fwd_bf16_d128_persist"]


def run_sdpa(session, rt, q, k, v, causal, dtype=DType.BF16, candidate=None):
    attrs = {"causal": True} if causal else {}
    if candidate:
        attrs["candidate"] = candidate
    ins = [upload(session, rt.stream, t, dtype) for t in (q, k, v)]
    return run_op(rt, "scaled_dot_product_attention", ins, dtype, q.shape, attrs)


@pytest.mark.parametrize("case", [c for c in KATS["cases"] if c["op"] == "sdpa_f32"], ids=lambda c: c["name"])
def test_sdpa_f32_reference_kats(session, rt, case):
    q = np.array(case["q"], np.float32).reshape(case["q_shape"])
    k = np.array(case["k"], np.float32).reshape(case["kv_shape"])
    v = np.array(case["v"], np.float32).reshape(case["kv_shape"])
    h = run_sdpa(session, rt, q, k, v, False, DType.F32)
    assert np.max(np.abs(h.outputs[0].to_numpy().ravel() - np.array(case["expected"]))) <= 2e-4


def test_sdpa_f32_matches_oracle(session, rt):
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 3, 17, 40)).astype(np.float32)
    k = rng.standard_normal((2, 3, 29, 40)).astype(np.float32)
    v = rng.standard_normal((2, 3, 29, 40)).astype(np.float32)
    h = run_sdpa(session, rt, q, k, v, False, DType.F32)
    assert np.max(np.abs(h.outputs[0].to_numpy() - oracle.sdpa(q, k, v))) <= 2e-4


def test_sdpa_f32_rejects_mask_and_causal_like_the_reference(session, rt):
    """projects/titan-runtime/tests/cuda_attention.rs:93-99."""
    q = upload(session, rt.stream, np.ones((1, 1, 2, 2), np.float32))
    kv = upload(session, rt.stream, np.ones((1, 1, 3, 2), np.float32))
    for attr in ("mask", "causal"):
        with pytest.raises(tb.ExecutionError) as e:
            rt.execute(tb.OpRequest("scaled_dot_product_attention", [q, kv, kv],
                                    [tb.TensorSpec(DType.F32, (1, 1, 2, 2))], {attr: True}))
        assert e.value.phase == "contract" and "does not implement" in e.value.message


@pytest.mark.parametrize("candidate", TC_CANDIDATES)
@pytest.mark.parametrize("b,h,tq,tk,causal", [(1, 1, 128, 128, False), (1, 1, 128, 128, True), (1, 2, 256, 256, True),
                                              (2, 1, 384, 384, True), (1, 1, 200, 200, True), (1, 2, 130, 130, False),
                                              (1, 1, 256, 384, False), (1, 1, 256, 384, True),
                                              (1, 1, 384, 256, True), (2, 2, 1024, 1024, True)])
def test_sdpa_bf16_tcgen05_matches_oracle(session, rt, b, h, tq, tk, causal, candidate):
    d = 128
    q, k, v = qkv_bf16(b, h, tq, tk, d, seed=b * 1000 + h * 100 + tq + tk + causal)
    res = run_sdpa(session, rt, q, k, v, causal, candidate=candidate)
    assert res.candidate == candidate
    got = res.outputs[0].to_f32()
    ids = np.arange(b * h * tq)
    ref = oracle.sdpa_bf16_rows(q, k, v, b, h, tq, tk, d, causal, ids).reshape(b, h, tq, d)
    assert np.isfinite(got).all()
    assert max_rel_err(got, ref) <= BF16_TOL, max_rel_err(got, ref)


def test_sdpa_bf16_generic_head_dim(session, rt):
    b, h, t, d = 1, 2, 100, 64
    q, k, v = qkv_bf16(b, h, t, t, d, seed=77)
    res = run_sdpa(session, rt, q, k, v, True)
    assert res.candidate == "sdpa_bf16_generic"
    ref = oracle.sdpa_bf16_rows(q, k, v, b, h, t, t, d, True, np.arange(b * h * t)).reshape(b, h, t, d)
    assert max_rel_err(res.outputs[0].to_f32(), ref) <= BF16_TOL


@pytest.mark.parametrize("candidate", TC_CANDIDATES)
def test_sdpa_bf16_full_c4_config(session, rt, candidate):
    """C4: causal B8 H32 S4096 D128, seed 3. Sampled full rows against the oracle, and
    the size-independent property that causal row 0 of every head equals V[..., 0, :]."""
    b, h, s, d = 8, 32, 4096, 128
    q, k, v = qkv_bf16(b, h, s, s, d, seed=3)
    res = run_sdpa(session, rt, q, k, v, True, candidate=candidate)
    assert res.candidate == candidate
    got = res.outputs[0].to_numpy()
    rng = np.random.default_rng(3)
    bh = rng.integers(0, b * h, 48)
    rows = rng.integers(0, s, 48)
    rows[:8] = [0, 1, 127, 128, 129, 2047, 4094, 4095]
    ids = np.sort(bh * s + rows)
    ref = oracle.sdpa_bf16_rows(q, k, v, b, h, s, s, d, True, ids)
    got_rows = tb.bf16_bits_to_f32(got.reshape(-1, d)[ids]).reshape(-1, d)
    assert max_rel_err(got_rows, ref) <= BF16_TOL, max_rel_err(got_rows, ref)
    np.testing.assert_array_equal(got[:, :, 0, :], v[:, :, 0, :])
    assert np.isfinite(tb.bf16_bits_to_f32(got)).all()


def test_sdpa_bf16_is_bit_reproducible(session, rt):
    q, k, v = qkv_bf16(1, 4, 512, 512, 128, seed=8)
    a = run_sdpa(session, rt, q, k, v, True).outputs[0].to_numpy()
    b = run_sdpa(session, rt, q, k, v, True).outputs[0].to_numpy()
    np.testing.assert_array_equal(a, b)


def test_sdpa_default_candidate_and_unknown_candidate(session, rt):
    q, k, v = qkv_bf16(1, 1, 256, 256, 128, seed=9)
    assert run_sdpa(session, rt, q, k, v, True).candidate == "sdpa_fwd_bf16_d128_pair"
    with pytest.raises(tb.ExecutionError, match="unknown attention candidate"):
        run_sdpa(session, rt, q, k, v, True, candidate="no_such_kernel")


def test_sdpa_contract_rejections(session, rt):
    """projects/titan-runtime/tests/cpu_reference_ops.rs:231-310 keywords."""
    q = upload(session, rt.stream, np.ones((1, 1, 2, 2), np.float32))
    k = upload(session, rt.stream, np.ones((1, 1, 3, 2), np.float32))
    v = upload(session, rt.stream, np.ones((1, 1, 3, 2), np.float32))
    v2 = upload(session, rt.stream, np.ones((1, 1, 2, 2), np.float32))
    r3 = upload(session, rt.stream, np.ones((1, 2, 2), np.float32))

    def err(inputs, shape, dtype=DType.F32, layout="Contiguous"):
        with pytest.raises(tb.ExecutionError) as e:
            rt.execute(tb.OpRequest("scaled_dot_product_attention", inputs,
                                    [tb.TensorSpec(dtype, shape, layout=layout)]))
        return e.value.message

    assert "exactly three" in err([q, k], (1, 1, 2, 2))
    assert "rank-4" in err([r3, k, v], (1, 1, 2, 2))
    assert "K/V sequence" in err([q, k, v2], (1, 1, 2, 2))
    assert "output shape" in err([q, k, v], (1, 1, 3, 2))
    assert "F32" in err([q, k, v], (1, 1, 2, 2), dtype=DType.I32)
    assert "contiguous" in err([q, k, v], (1, 1, 2, 2), layout="Strided")


@pytest.mark.parametrize("candidate,d", [("sdpa_fwd_bf16_d128_pair", 128), ("sdpa_fwd_bf16_d128_bn64", 128),
                                         ("sdpa_fwd_bf16_d128", 128), ("sdpa_bf16_generic", 64)])
@pytest.mark.parametrize("scale", [1.0, 0.03])
def test_sdpa_bf16_scale_attribute(session, rt, candidate, d, scale):
    """`scale` (an extension; the reference fixes 1/sqrt(D)) multiplies Q K^T in every bf16 kernel."""
    b, h, tq, tk = 1, 2, 256, 384
    q, k, v = qkv_bf16(b, h, tq, tk, d, seed=41)
    q = (tb.bf16_bits_to_f32(q) * 0.25).reshape(q.shape)  # keeps exp() of unscaled scores in range
    q = (q.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    ins = [upload(session, rt.stream, t, DType.BF16) for t in (q, k, v)]
    res = run_op(rt, "scaled_dot_product_attention", ins, DType.BF16, q.shape,
                 {"causal": True, "scale": scale, "candidate": candidate})
    assert res.candidate == candidate
    ref = oracle.sdpa_bf16_rows(q, k, v, b, h, tq, tk, d, True, np.arange(b * h * tq), scale=scale)
    assert max_rel_err(res.outputs[0].to_f32(), ref.reshape(b, h, tq, d)) <= BF16_TOL


def test_sdpa_bf16_scale_attribute_contract(session, rt):
    q, k, v = qkv_bf16(1, 1, 128, 128, 128, seed=42)
    ins = [upload(session, rt.stream, t, DType.BF16) for t in (q, k, v)]
    for bad in ("0", "-1", "nan", "inf", "abc", "1.0x", 0.0):
        with pytest.raises(tb.ExecutionError, match="scale must be a positive finite number"):
            run_op(rt, "scaled_dot_product_attention", ins, DType.BF16, q.shape, {"scale": bad})


@pytest.mark.parametrize("b,h,t,causal", [(4, 16, 2048, True), (3, 5, 1000, True), (2, 40, 512, False)])
def test_sdpa_persistent_ctas_walk_many_items_like_the_pair_kernel(session, rt, b, h, t, causal):
    """The persistent kernel (one CTA per SM walking several (head, query-tile pair) items,
    item boundaries pipelined) computes every item with the pair kernel's arithmetic: the
    outputs are bit-identical, and sampled rows match the oracle. 512, 300 and 160 items
    over 148 SMs: several items per CTA, head groups of 16 with a ragged last group, ragged Tq."""
    d = 128
    q, k, v = qkv_bf16(b, h, t, t, d, seed=b + h + t)
    pair = run_sdpa(session, rt, q, k, v, causal, candidate="sdpa_fwd_bf16_d128_pair")
    want = pair.outputs[0].to_numpy()
    got_h = run_sdpa(session, rt, q, k, v, causal, candidate="sdpa_fwd_bf16_d128_persist")
    assert got_h.candidate == "sdpa_fwd_bf16_d128_persist"
    got = got_h.outputs[0].to_numpy()
    np.testing.assert_array_equal(got, want)
    rng = np.random.default_rng(t)
    ids = np.unique(np.concatenate([rng.integers(0, b * h * t, 512), [0, b * h * t - 1]]))
    ref = oracle.sdpa_bf16_rows(q, k, v, b, h, t, t, d, causal, ids)
    got_rows = tb.bf16_bits_to_f32(got).reshape(-1, d)[ids]
    assert max_rel_err(got_rows, ref) <= BF16_TOL

