"""Helpers shared by the GPU tests (no test functions here)."""
from __future__ import annotations

import numpy as np

import titan_rs_b200 as tb
from titan_rs_b200.kernel_abi import DType


def upload(session, stream, array: np.ndarray, dtype: DType = DType.F32) -> tb.TensorHandle:
    return tb.TensorHandle.from_numpy(session, array, dtype, stream)


def run_op(rt: tb.Runtime, name: str, inputs, out_dtype: DType, out_shape, attrs=None, output=None):
    req = tb.OpRequest(name, list(inputs), [tb.TensorSpec(out_dtype, tuple(out_shape))], dict(attrs or {}))
    h = rt.execute(req, output=output)
    h.wait()
    return h


def max_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref| (the bf16 tolerance form of the north star)."""
    return float(np.max(np.abs(got.astype(np.float64) - ref.astype(np.float64))) / max(np.max(np.abs(ref)), 1e-30))


def elementwise_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max_i |got_i - ref_i| / |ref_i| (the fp32 softmax tolerance form)."""
    ref = ref.astype(np.float64)
    return float(np.max(np.abs(got.astype(np.float64) - ref) / np.maximum(np.abs(ref), 1e-30)))
