"""Conv2d on the B200 against the CPU oracle (restated projects/titan-runtime/src/lib.rs:991-1088).

Tolerances: f32 (reference ABI, NCHW/OIHW) is bit-exact with the oracle (same
loop order, separately rounded multiply and add); the reference's own GPU test
uses 1e-5 (projects/titan-runtime/tests/cuda_conv2d.rs:96-98). bf16 NHWC uses the
north-star bound max|err| <= 1e-2 * max|ref| against the f32 oracle on the same
bf16 inputs.
"""
import json
import math
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


def conv_attrs(stride=(1, 1), pad=(0, 0), dil=(1, 1), groups=1, layout=None):
    a = {"stride_h": stride[0], "stride_w": stride[1], "pad_h": pad[0], "pad_w": pad[1], "dilation_h": dil[0],
         "dilation_w": dil[1], "groups": groups}
    if layout:
        a["layout"] = layout
    return a


def out_hw(h, w, r, s, stride, pad, dil):
    return ((h + 2 * pad[0] - dil[0] * (r - 1) - 1) // stride[0] + 1,
            (w + 2 * pad[1] - dil[1] * (s - 1) - 1) // stride[1] + 1)


@pytest.mark.parametrize("case", [c for c in KATS["cases"] if c["op"] == "conv2d_f32"], ids=lambda c: c["name"])
def test_conv2d_f32_reference_kats(session, rt, case):
    x = np.array(case["x"], np.float32).reshape(case["x_shape"])
    w = np.array(case["w"], np.float32).reshape(case["w_shape"])
    ins = [upload(session, rt.stream, x), upload(session, rt.stream, w)]
    if case["bias"] is not None:
        ins.append(upload(session, rt.stream, np.array(case["bias"], np.float32)))
    h = run_op(rt, "conv2d", ins, DType.F32, case["out_shape"],
               conv_attrs(case["stride"], case["pad"], case["dilation"], case["groups"]))
    got = h.outputs[0].to_numpy().ravel()
    assert np.max(np.abs(got - np.array(case["expected"]))) <= max(case["tolerance"], 1e-5)
    ref = oracle.conv2d_nchw(x, w, None if case["bias"] is None else np.array(case["bias"], np.float32),
                             case["stride"], case["pad"], case["dilation"], case["groups"])
    np.testing.assert_array_equal(got, ref.ravel())


def test_conv2d_f32_random_bit_exact(session, rt):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 6, 11, 9)).astype(np.float32)
    w = rng.standard_normal((4, 3, 3, 2)).astype(np.float32)
    b = rng.standard_normal(4).astype(np.float32)
    stride, pad, dil = (2, 1), (1, 2), (2, 1)
    ref = oracle.conv2d_nchw(x, w, b, stride, pad, dil, 2)
    ins = [upload(session, rt.stream, t) for t in (x, w, b)]
    h = run_op(rt, "conv2d", ins, DType.F32, ref.shape, conv_attrs(stride, pad, dil, 2))
    np.testing.assert_array_equal(h.outputs[0].to_numpy(), ref)


def nhwc_inputs(n, hh, ww, cin, cout, r, s, seed, with_bias=False):
    x = tb.fill_normal(n * hh * ww * cin, seed=seed * 16, dtype=DType.BF16).reshape(n, hh, ww, cin)
    w = tb.fill_normal(cout * r * s * cin, seed=seed * 16 + 1, std=math.sqrt(2.0 / (r * s * cin)),
                       dtype=DType.BF16).reshape(cout, r, s, cin)
    b = tb.fill_normal(cout, seed=seed * 16 + 2) if with_bias else None
    return x, w, b


def check_nhwc(session, rt, n, hh, ww, cin, cout, r, s, stride, pad, dil, with_bias, expect_candidate, seed, groups=1,
               candidate=None):
    x, w, b = nhwc_inputs(n, hh, ww, cin, cout, r, s, seed, with_bias)
    if groups > 1:
        w = np.ascontiguousarray(w[..., : cin // groups])
    ho, wo = out_hw(hh, ww, r, s, stride, pad, dil)
    ins = [upload(session, rt.stream, x, DType.BF16), upload(session, rt.stream, w, DType.BF16)]
    if b is not None:
        ins.append(upload(session, rt.stream, b, DType.F32))
    attrs = conv_attrs(stride, pad, dil, groups, "NHWC")
    if candidate:
        attrs["candidate"] = candidate
    res = run_op(rt, "conv2d", ins, DType.BF16, (n, ho, wo, cout), attrs)
    assert res.candidate == expect_candidate
    got = res.outputs[0].to_f32()
    if groups == 1:
        idx = np.arange(n * ho * wo * cout)
        ref = oracle.conv2d_nhwc_bf16_points(x, w, b, n, hh, ww, cin, cout, r, s, stride, pad, dil, ho, wo, idx)
        ref = ref.reshape(n, ho, wo, cout)
    else:
        xf = tb.bf16_bits_to_f32(x).reshape(x.shape).transpose(0, 3, 1, 2)
        wf = tb.bf16_bits_to_f32(w).reshape(w.shape).transpose(0, 3, 1, 2)
        ref = oracle.conv2d_nchw(xf, wf, b, stride, pad, dil, groups).transpose(0, 2, 3, 1)
    assert np.isfinite(got).all()
    assert max_rel_err(got, ref) <= BF16_TOL, max_rel_err(got, ref)


@pytest.mark.parametrize("n,hh,ww,cin,cout,r,s,pad,dil,bias", [
    (2, 8, 8, 64, 256, 3, 3, (1, 1), (1, 1), False),
    (2, 16, 16, 128, 256, 3, 3, (1, 1), (1, 1), True),
    (3, 13, 11, 64, 256, 3, 3, (1, 1), (1, 1), False),      # odd batch, ragged H/W tiles
    (2, 10, 12, 96, 128, 3, 3, (1, 1), (1, 1), True),       # channel tails (96 % 64, Cout < 256)
    (1, 9, 9, 64, 512, 1, 1, (0, 0), (1, 1), False),        # 1x1, two N tiles
    (2, 12, 12, 64, 256, 3, 3, (2, 2), (2, 2), False),      # dilation 2
    (4, 7, 7, 32, 64, 5, 3, (2, 1), (1, 1), True),          # non-square filter, Cin 32
])
@pytest.mark.parametrize("candidate", [None, "conv2d_fprop_bf16_nhwc_2sm"])
def test_conv2d_bf16_implicit_gemm_matches_oracle(session, rt, n, hh, ww, cin, cout, r, s, pad, dil, bias, candidate):
    """Small outputs take the 1-SM kernel by default; the 2-SM kernel is forced by name
    (its odd CTA of a final pair past the last 128-pixel block must store nothing)."""
    check_nhwc(session, rt, n, hh, ww, cin, cout, r, s, (1, 1), pad, dil, bias, candidate or "conv2d_fprop_bf16_nhwc",
               seed=n + hh + cin + cout + r, candidate=candidate)


@pytest.mark.parametrize("n,hh,ww,cin,cout,r,s,stride,pad,dil,bias", [
    (2, 9, 10, 64, 32, 3, 3, (2, 2), (1, 1), (1, 1), True),     # the reference's stride-2 case, tensor cores
    (2, 56, 56, 64, 128, 3, 3, (2, 2), (1, 1), (1, 1), False),  # ResNet-style downsampling
    (3, 17, 23, 128, 256, 3, 3, (2, 1), (1, 1), (1, 1), True),  # mixed strides, ragged tiles
    (2, 20, 20, 64, 64, 1, 1, (2, 2), (0, 0), (1, 1), False),   # 1x1 projection shortcut
    (1, 31, 29, 64, 256, 5, 5, (3, 3), (2, 2), (1, 1), False),  # stride 3
    (2, 24, 24, 64, 128, 3, 3, (2, 2), (2, 2), (2, 2), True),   # stride 2 + dilation 2
])
@pytest.mark.parametrize("candidate", [None, "conv2d_fprop_bf16_nhwc_2sm"])
def test_conv2d_bf16_strided_implicit_gemm_matches_oracle(session, rt, n, hh, ww, cin, cout, r, s, stride, pad, dil,
                                                          bias, candidate):
    """Strides reach the tensor-core kernel as TMA traversal strides (input box 8*s wide)."""
    check_nhwc(session, rt, n, hh, ww, cin, cout, r, s, stride, pad, dil, bias, candidate or "conv2d_fprop_bf16_nhwc",
               seed=n + hh + cin + cout + stride[0], candidate=candidate)


@pytest.mark.parametrize("stride,groups,cin", [((1, 1), 2, 64), ((1, 1), 1, 12), ((2, 2), 1, 12)])
def test_conv2d_bf16_generic_path(session, rt, stride, groups, cin):
    check_nhwc(session, rt, 2, 9, 10, cin, 32, 3, 3, stride, (1, 1), (1, 1), True, "conv2d_bf16_nhwc_generic",
               seed=5 + groups + cin, groups=groups)


@pytest.mark.parametrize("candidate", [None, "conv2d_fprop_bf16_nhwc"])
def test_conv2d_bf16_full_c5_config(session, rt, candidate):
    """C5: x [64,56,56,256] N(0,1), w [256,3,3,256] N(0, 2/2304), seed 4, stride 1, pad 1.
    The default at this size is the 2-SM kernel; the 1-SM kernel is forced by name."""
    n, hh, ww, cin, cout = 64, 56, 56, 256, 256
    x = tb.fill_normal(n * hh * ww * cin, seed=4 * 16, dtype=DType.BF16).reshape(n, hh, ww, cin)
    w = tb.fill_normal(cout * 9 * cin, seed=4 * 16 + 1, std=math.sqrt(2.0 / 2304), dtype=DType.BF16)
    w = w.reshape(cout, 3, 3, cin)
    ins = [upload(session, rt.stream, x, DType.BF16), upload(session, rt.stream, w, DType.BF16)]
    attrs = conv_attrs((1, 1), (1, 1), (1, 1), 1, "NHWC")
    if candidate:
        attrs["candidate"] = candidate
    res = run_op(rt, "conv2d", ins, DType.BF16, (n, hh, ww, cout), attrs)
    assert res.candidate == (candidate or "conv2d_fprop_bf16_nhwc_2sm")
    got = res.outputs[0].to_f32()
    rng = np.random.default_rng(4)
    idx = rng.integers(0, n * hh * ww * cout, 4096)
    # Borders (padding) and tile edges.
    corners = [((0 * hh + 0) * ww + 0) * cout, ((0 * hh + 55) * ww + 55) * cout + 255, ((63 * hh + 0) * ww + 55) * cout,
               ((1 * hh + 7) * ww + 8) * cout + 17, ((62 * hh + 48) * ww + 47) * cout + 128]
    idx = np.concatenate([idx, corners])
    ref = oracle.conv2d_nhwc_bf16_points(x, w, None, n, hh, ww, cin, cout, 3, 3, (1, 1), (1, 1), (1, 1), hh, ww, idx)
    assert max_rel_err(got.ravel()[idx], ref) <= BF16_TOL
    assert np.isfinite(got).all()


def test_conv2d_contract_rejections(session, rt):
    """projects/titan-runtime/tests/cpu_reference_ops.rs:156-203 keywords."""
    x = upload(session, rt.stream, np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3))
    w = upload(session, rt.stream, np.array([1, 0, 0, -1], np.float32).reshape(1, 1, 2, 2))
    r3 = upload(session, rt.stream, np.ones((1, 3, 3), np.float32))
    bad_w = upload(session, rt.stream, np.ones((1, 2, 2, 2), np.float32))
    bad_b = upload(session, rt.stream, np.ones(2, np.float32))

    def err(inputs, shape, attrs=None, dtype=DType.F32, layout="Contiguous"):
        with pytest.raises(tb.ExecutionError) as e:
            rt.execute(tb.OpRequest("conv2d", inputs, [tb.TensorSpec(dtype, shape, layout=layout)],
                                    attrs if attrs is not None else conv_attrs()))
        return e.value.message

    assert "rank-4" in err([r3, w], (1, 1, 2, 2))
    assert "non-zero" in err([x, w], (1, 1, 2, 2), conv_attrs(groups=0))
    assert "output shape" in err([x, w], (1, 1, 1, 2))
    assert "channels" in err([x, bad_w], (1, 1, 2, 2))
    assert "bias" in err([x, w, bad_b], (1, 1, 2, 2))
    assert "F32" in err([x, w], (1, 1, 2, 2), dtype=DType.I32)
    assert "contiguous" in err([x, w], (1, 1, 2, 2), layout="Strided")
    assert "unsupported attributes" in err([x, w], (1, 1, 2, 2), {**conv_attrs(), "alpha": 1})
