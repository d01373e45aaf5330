"""Writes tests/golden/reference_kats.json: the titan.rs known-answer vectors for
the MatMul / softmax / SDPA / conv2d path.

The reference is a Rust workspace and no Rust toolchain exists here, so its
tests cannot run. Instead every literal below is transcribed from the reference's
own test files (cited per case, paths inside the titan.rs project). Where the
reference test compares a CUDA result against its CPU scalar reference rather
than against literal numbers, the expected values are computed here
independently in float64 with numpy (a different code path from the C oracle),
so the oracle is pinned against both the literal reference answers and an
independent evaluation.

Run:  python tests/golden/make_reference_kats.py
"""
from __future__ import annotations

import json
import math
import pathlib

import numpy as np

OUT = pathlib.Path(__file__).with_name("reference_kats.json")


def sdpa_f64(q, k, v, causal=False):
    q, k, v = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    d = q.shape[-1]
    s = q @ np.swapaxes(k, -1, -2) / math.sqrt(d)
    if causal:
        tq, tk = s.shape[-2:]
        mask = np.tril(np.ones((tq, tk), dtype=bool))
        s = np.where(mask, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return p @ v


def conv2d_nchw_f64(x, w, b, stride, pad, dil, groups):
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    n, c, h, wd = x.shape
    assert n == 1, "fixture cases use batch 1"
    co, cpg, kh, kw = w.shape
    ho = (h + 2 * pad[0] - (dil[0] * (kh - 1) + 1)) // stride[0] + 1
    wo = (wd + 2 * pad[1] - (dil[1] * (kw - 1) + 1)) // stride[1] + 1
    xp = np.zeros((n, c, h + 2 * pad[0], wd + 2 * pad[1]))
    xp[:, :, pad[0]:pad[0] + h, pad[1]:pad[1] + wd] = x
    out = np.zeros((n, co, ho, wo))
    opg = co // groups
    for oc in range(co):
        g = oc // opg
        for oh in range(ho):
            for ow in range(wo):
                acc = 0.0 if b is None else float(b[oc])
                for ci in range(cpg):
                    for r in range(kh):
                        for s in range(kw):
                            acc += xp[0, g * cpg + ci, oh * stride[0] + r * dil[0], ow * stride[1] + s * dil[1]] * w[oc, ci, r, s]
                out[0, oc, oh, ow] = acc
    return out


def softmax_f64(x):
    x = np.asarray(x, dtype=np.float64)
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def main() -> None:
    cases = []

    # --- GEMM ---------------------------------------------------------------
    cases.append({
        "name": "gemm_2x3_3x2",
        "source": "projects/titan-runtime/tests/cpu_reference_ops.rs:58-65",
        "op": "gemm_f32", "lhs_shape": [2, 3], "rhs_shape": [3, 2],
        "lhs": [1, 2, 3, 4, 5, 6], "rhs": [7, 8, 9, 10, 11, 12],
        "transpose_lhs": False, "transpose_rhs": False,
        "expected": [58, 64, 139, 154], "tolerance": 0.0,
    })
    cases.append({
        "name": "gemm_transposed_both",
        "source": "projects/titan-runtime/tests/cpu_reference_ops.rs:67-79",
        "op": "gemm_f32", "lhs_shape": [3, 2], "rhs_shape": [2, 3],
        "lhs": [1, 4, 2, 5, 3, 6], "rhs": [7, 9, 11, 8, 10, 12],
        "transpose_lhs": True, "transpose_rhs": True,
        "expected": [58, 64, 139, 154], "tolerance": 0.0,
    })
    lhs = np.arange(1, 9, dtype=np.float64).reshape(2, 4)
    rhs = np.arange(1, 13, dtype=np.float64).reshape(4, 3)
    cases.append({
        "name": "gemm_cuda_parity_2x4_4x3",
        "source": "projects/titan-runtime/tests/cuda_gemm.rs:57-78 (CUDA == CPU, exact)",
        "op": "gemm_f32", "lhs_shape": [2, 4], "rhs_shape": [4, 3],
        "lhs": lhs.ravel().tolist(), "rhs": rhs.ravel().tolist(),
        "transpose_lhs": False, "transpose_rhs": False,
        "expected": (lhs @ rhs).ravel().tolist(), "tolerance": 0.0,
    })

    # --- softmax ------------------------------------------------------------
    cases.append({
        "name": "softmax_1to6_axis1",
        "source": "projects/titan-runtime/tests/cpu_reference_ops.rs:356-362",
        "op": "softmax_f32", "shape": [2, 3], "input": [1, 2, 3, 4, 5, 6],
        "check_indices": [0, 2, 3], "expected_at_indices": [0.09003057, 0.66524094, 0.09003057],
        "expected": softmax_f64(np.array([[1, 2, 3], [4, 5, 6]])).ravel().tolist(),
        "tolerance": 1e-6,
    })
    big = [1001.0, 1000.0, 999.0, 1.0, 2.0, 3.0]
    cases.append({
        "name": "softmax_large_offset_stability",
        "source": "projects/titan-runtime/tests/cuda_softmax.rs:84-113 (CPU tol 2e-6, GPU tol 2e-4, row sums 2e-4)",
        "op": "softmax_f32", "shape": [2, 3], "input": big,
        "expected": softmax_f64(np.array(big).reshape(2, 3)).ravel().tolist(),
        "tolerance": 2e-6, "gpu_tolerance": 2e-4,
    })

    # --- SDPA ---------------------------------------------------------------
    high = math.exp(1.0 / math.sqrt(2.0))
    hw = high / (2.0 * high + 1.0)
    lw = 1.0 / (2.0 * high + 1.0)
    cases.append({
        "name": "sdpa_analytic_tq2_tk3",
        "source": "projects/titan-runtime/tests/cpu_reference_ops.rs:209-228",
        "op": "sdpa_f32", "q_shape": [1, 1, 2, 2], "kv_shape": [1, 1, 3, 2],
        "q": [1, 0, 0, 1], "k": [1, 0, 0, 1, 1, 1], "v": [10, 0, 0, 20, 10, 10],
        "causal": False,
        "expected": [20.0 * hw, 20.0 * lw + 10.0 * hw, 10.0 * (lw + hw), 30.0 * hw],
        "tolerance": 1e-6,
    })
    q = [1.0, -0.5, 0.25, 1.5]
    k = [0.5, 1.0, -1.0, 0.25, 0.75, -0.5]
    v = [2.0, -1.0, 0.5, 3.0, -2.0, 1.5]
    cases.append({
        "name": "sdpa_cuda_parity_tq2_tk3",
        "source": "projects/titan-runtime/tests/cuda_attention.rs:61-92 (CUDA vs CPU, tol 2e-4)",
        "op": "sdpa_f32", "q_shape": [1, 1, 2, 2], "kv_shape": [1, 1, 3, 2],
        "q": q, "k": k, "v": v, "causal": False,
        "expected": sdpa_f64(np.array(q).reshape(1, 1, 2, 2), np.array(k).reshape(1, 1, 3, 2),
                             np.array(v).reshape(1, 1, 3, 2)).ravel().tolist(),
        "tolerance": 1e-6, "gpu_tolerance": 2e-4,
    })

    # --- conv2d ---------------------------------------------------------------
    cases.append({
        "name": "conv2d_3x3_2x2_bias",
        "source": "projects/titan-runtime/tests/cpu_reference_ops.rs:130-140",
        "op": "conv2d_f32", "x_shape": [1, 1, 3, 3], "w_shape": [1, 1, 2, 2],
        "x": [1, 2, 3, 4, 5, 6, 7, 8, 9], "w": [1, 0, 0, -1], "bias": [1],
        "stride": [1, 1], "pad": [0, 0], "dilation": [1, 1], "groups": 1,
        "out_shape": [1, 1, 2, 2], "expected": [-3, -3, -3, -3], "tolerance": 0.0,
    })
    cases.append({
        "name": "conv2d_grouped_1x1",
        "source": "projects/titan-runtime/tests/cpu_reference_ops.rs:142-152",
        "op": "conv2d_f32", "x_shape": [1, 2, 1, 1], "w_shape": [2, 1, 1, 1],
        "x": [2, 3], "w": [10, 20], "bias": None,
        "stride": [1, 1], "pad": [0, 0], "dilation": [1, 1], "groups": 2,
        "out_shape": [1, 2, 1, 1], "expected": [20, 60], "tolerance": 0.0,
    })
    x = list(range(1, 26)) + [-i for i in range(1, 26)]
    w = [1.0, 0.5, -1.0, 2.0, -0.5, 1.5, 0.25, -1.0]
    b = [0.75, -1.25]
    exp = conv2d_nchw_f64(np.array(x, dtype=np.float64).reshape(1, 2, 5, 5), np.array(w).reshape(2, 1, 2, 2),
                          b, (2, 2), (1, 1), (2, 2), 2)
    cases.append({
        "name": "conv2d_stride2_pad1_dil2_groups2_bias",
        "source": "projects/titan-runtime/tests/cuda_conv2d.rs:12-40,67-99 (CUDA vs CPU, tol 1e-5)",
        "op": "conv2d_f32", "x_shape": [1, 2, 5, 5], "w_shape": [2, 1, 2, 2],
        "x": x, "w": w, "bias": b,
        "stride": [2, 2], "pad": [1, 1], "dilation": [2, 2], "groups": 2,
        "out_shape": [1, 2, 3, 3], "expected": exp.ravel().tolist(), "tolerance": 1e-5,
    })

    # --- contract rejections (message keywords the reference tests grep for) ---
    rejections = [
        {"op": "gemm", "case": "inner dimensions", "source": "cpu_reference_ops.rs:85-92", "keyword": "inner dimensions"},
        {"op": "gemm", "case": "rank-1 lhs", "source": "cpu_reference_ops.rs:93-99", "keyword": "rank-2"},
        {"op": "gemm", "case": "output shape", "source": "cpu_reference_ops.rs:100-106", "keyword": "output shape"},
        {"op": "gemm", "case": "one input", "source": "cpu_reference_ops.rs:113", "keyword": "exactly two"},
        {"op": "softmax", "case": "axis 0", "source": "cuda_softmax.rs:131-137", "keyword": "last axis"},
        {"op": "softmax", "case": "F16 output", "source": "cuda_softmax.rs:139-143", "keyword": "F32"},
        {"op": "softmax", "case": "strided output", "source": "cuda_softmax.rs:145-149", "keyword": "contiguous"},
        {"op": "softmax", "case": "shape mismatch", "source": "cuda_softmax.rs:151-155", "keyword": "same shape"},
        {"op": "softmax", "case": "unknown attribute", "source": "cuda_softmax.rs:157-164", "keyword": "axis"},
        {"op": "sdpa", "case": "two inputs", "source": "cpu_reference_ops.rs:236-241", "keyword": "exactly three"},
        {"op": "sdpa", "case": "rank-3 query", "source": "cpu_reference_ops.rs:242-252", "keyword": "rank-4"},
        {"op": "sdpa", "case": "K/V length mismatch", "source": "cpu_reference_ops.rs:253-263", "keyword": "K/V sequence"},
        {"op": "sdpa", "case": "output shape", "source": "cpu_reference_ops.rs:264-273", "keyword": "output shape"},
        {"op": "sdpa", "case": "f32 path with mask", "source": "cuda_attention.rs:93-99", "keyword": "does not implement"},
        {"op": "conv2d", "case": "rank-3 input", "source": "cpu_reference_ops.rs:161-166", "keyword": "rank-4"},
        {"op": "conv2d", "case": "groups 0", "source": "cpu_reference_ops.rs:167-177", "keyword": "non-zero"},
        {"op": "conv2d", "case": "output shape", "source": "cpu_reference_ops.rs:178-183", "keyword": "output shape"},
        {"op": "conv2d", "case": "weight channels", "source": "cpu_reference_ops.rs:184-190", "keyword": "channels"},
        {"op": "conv2d", "case": "bias shape", "source": "cpu_reference_ops.rs:191-199", "keyword": "bias"},
    ]

    OUT.write_text(json.dumps({"cases": cases, "rejections": rejections}, indent=1) + "\n")
    print(f"wrote {OUT} ({len(cases)} cases, {len(rejections)} rejection keywords)")


if __name__ == "__main__":
    main()
