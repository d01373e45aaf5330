"""Zero extents never reach a kernel.

The reference's CUDA context refuses zero-byte allocations
(projects/titan-backend-cuda/src/lib.rs:122-125), and each operator refuses a zero
dimension with "non-zero" in its message: softmax (projects/titan-runtime/src/lib.rs:1548),
GEMM (titan-backend-cuda/src/lib.rs:912-913), attention (:761-762, runtime :1117) and
conv2d (:815-825). Zero-extent tensors are built here as views of real buffers, the only
way they can exist once allocation refuses zero bytes."""
import numpy as np
import pytest

import titan_rs_b200 as tb
from titan_rs_b200.hal import HalError
from titan_rs_b200.kernel_abi import DType
from titan_rs_b200.runtime import contiguous_strides

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def session():
    s = tb.Session(0)
    yield s
    s.close()


@pytest.fixture(scope="module")
def rt(session):
    return tb.Runtime(session)


def test_zero_byte_allocation_is_refused(session):
    with pytest.raises(HalError, match="zero-byte CUDA allocations are unsupported") as e:
        session.allocate(0)
    assert e.value.operation == "allocate"
    with pytest.raises(HalError, match="zero-byte"):
        tb.TensorHandle.allocate(session, DType.F32, (0, 4))


def view(backing: tb.TensorHandle, dtype: DType, shape) -> tb.TensorHandle:
    return tb.TensorHandle(backing.session, backing.buffer, dtype, tuple(shape), contiguous_strides(shape))


def rejected(rt, op, inputs, out, attrs=None):
    with pytest.raises(tb.ExecutionError) as e:
        rt.execute(tb.OpRequest(op, inputs, [tb.TensorSpec(out.dtype, out.shape)], attrs or {}), output=out)
    assert e.value.phase == "contract", e.value
    return e.value.message


@pytest.mark.parametrize("dtype", [DType.F32, DType.BF16])
def test_softmax_zero_rows_or_cols(session, rt, dtype):
    backing = tb.TensorHandle.allocate(session, DType.F32, (64,))
    for shape in [(0, 4), (4, 0), (2, 0, 3)]:
        t = view(backing, dtype, shape)
        assert "non-zero" in rejected(rt, "softmax", [t], view(backing, dtype, shape))


@pytest.mark.parametrize("dtype", [DType.F32, DType.BF16])
@pytest.mark.parametrize("m,n,k", [(0, 8, 8), (8, 0, 8), (8, 8, 0)])
def test_gemm_zero_m_n_or_k(session, rt, dtype, m, n, k):
    backing = tb.TensorHandle.allocate(session, DType.F32, (256,))
    msg = rejected(rt, "gemm", [view(backing, dtype, (m, k)), view(backing, dtype, (k, n))],
                   view(backing, dtype, (m, n)))
    assert "M, N, and K must be non-zero" in msg


@pytest.mark.parametrize("dtype", [DType.F32, DType.BF16])
@pytest.mark.parametrize("zero", range(5))
def test_attention_zero_b_h_t_or_d(session, rt, dtype, zero):
    backing = tb.TensorHandle.allocate(session, DType.F32, (1024,))
    dims = [1, 2, 8, 8, 16]  # B, H, Tq, Tk, D
    dims[zero] = 0
    b, h, tq, tk, d = dims
    q, kv, o = (b, h, tq, d), (b, h, tk, d), (b, h, tq, d)
    msg = rejected(rt, "scaled_dot_product_attention",
                   [view(backing, dtype, q), view(backing, dtype, kv), view(backing, dtype, kv)],
                   view(backing, dtype, o))
    assert "non-zero" in msg


@pytest.mark.parametrize("zero", range(8))
def test_conv2d_zero_input_or_weight_extent(session, rt, zero):
    backing = tb.TensorHandle.allocate(session, DType.F32, (4096,))
    x, w = [1, 2, 6, 6], [2, 2, 3, 3]  # NCHW, OIHW
    (x if zero < 4 else w)[zero % 4] = 0
    attrs = {"stride_h": 1, "stride_w": 1, "pad_h": 1, "pad_w": 1, "dilation_h": 1, "dilation_w": 1, "groups": 1}
    out = view(backing, DType.F32, (x[0], w[0], 6, 6))
    msg = rejected(rt, "conv2d", [view(backing, DType.F32, x), view(backing, DType.F32, w)], out, attrs)
    assert "CUDA Conv2D dimensions must be non-zero" in msg
