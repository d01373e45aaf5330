"""CPU-only checks of the native boundary and host logic (no GPU calls).

- libtitan_b200.so loads and exports every function include/titan_b200.h declares.
- Without a CUDA driver the library reports "load_driver", the reference's
  no_cuda_environment case (projects/titan-runtime/tests/cuda_gemm.rs:32-35).
- The seeded generators are deterministic, thread-count invariant and have the
  requested moments.
"""
import ctypes
import pathlib
import re
import subprocess

import numpy as np
import pytest

import titan_rs_b200 as tb
from titan_rs_b200 import _native as N
from titan_rs_b200.kernel_abi import DType

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "titan_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tb_[a-z0-9_]+)\s*\(", text)))


def test_header_declarations_are_all_exported():
    lib = N.lib()
    declared = declared_functions()
    assert len(declared) >= 50
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert set(declared) <= exported
    # Nothing but the C ABI leaks out of the library.
    assert all(name.startswith("tb_") for name in exported if not name.startswith("_"))


def test_python_binding_covers_the_header():
    assert set(declared_functions()) == set(N.EXPORTED)


def test_no_driver_reports_load_driver_like_the_reference():
    try:
        lib = ctypes.CDLL("libcuda.so.1")
        del lib
        pytest.skip("a CUDA driver is present on this machine")
    except OSError:
        pass
    assert not tb.driver_available()
    op, detail = N.last_error()
    assert op == "load_driver"
    with pytest.raises(tb.HalError) as err:
        tb.Session(0)
    assert err.value.operation == "load_driver"
    assert err.value.status == N.TB_ERR_DRIVER_UNAVAILABLE


def test_fill_normal_is_deterministic_and_thread_invariant():
    a = tb.fill_normal(1 << 17, seed=3, mean=0.0, std=1.0, threads=1)
    b = tb.fill_normal(1 << 17, seed=3, mean=0.0, std=1.0, threads=7)
    np.testing.assert_array_equal(a, b)
    c = tb.fill_normal(1 << 17, seed=4)
    assert not np.array_equal(a, c)
    # A prefix is the same whatever the total count (counter-based).
    np.testing.assert_array_equal(tb.fill_normal(1001, seed=3), a[:1001])


def test_fill_moments_match_the_configs():
    x = tb.fill_normal(1 << 20, seed=1, mean=0.0, std=2.0)  # softmax config: N(0, 2^2)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 2.0) < 0.01
    u = tb.fill_uniform(1 << 20, seed=0, low=-1.0, high=1.0)  # gemm CPU config: U[-1, 1)
    assert u.min() >= -1.0 and u.max() < 1.0 and abs(u.mean()) < 0.01
    bits = tb.fill_normal(1 << 16, seed=2, std=1.0 / np.sqrt(8192), dtype=DType.BF16)
    assert bits.dtype == np.uint16
    f = tb.bf16_bits_to_f32(bits)
    assert abs(f.std() * np.sqrt(8192) - 1.0) < 0.02
    # bf16 fill == f32 fill rounded to nearest even.
    f32 = tb.fill_normal(1 << 16, seed=2, std=1.0 / np.sqrt(8192))
    np.testing.assert_array_equal(bits, tb.f32_to_bf16_bits(f32))


def test_fill_rejects_bad_dtype():
    with pytest.raises(tb.HalError):
        tb.fill_normal(4, seed=0, dtype=DType.I32)


def test_embedded_cubins_are_sm100a_elf():
    for module in ("softmax",):
        blob = N.builtin_cubin(module)
        assert blob[:4] == b"\x7fELF"
    with pytest.raises(KeyError):
        N.builtin_cubin("no_such_module")


def test_attributes_cross_the_abi_as_ints_and_strings():
    """OpRequest attributes become TbAttr: bools and ints in `value`, strings in `str`, and
    floats (the attention `scale`) as their shortest round-tripping decimal string."""
    from titan_rs_b200.runtime import _attrs
    arr, n, keep = _attrs({"transpose_rhs": True, "axis": -1, "layout": "NHWC", "scale": 0.08838834764831845})
    assert n == 4
    got = {arr[i].key.decode(): (arr[i].value, arr[i].str) for i in range(n)}
    assert got["transpose_rhs"] == (1, None) and got["axis"] == (-1, None)
    assert got["layout"] == (0, b"NHWC")
    assert got["scale"][1] == b"0.08838834764831845" and float(got["scale"][1]) == 0.08838834764831845


def test_execute_routes_by_operator_name_before_touching_a_session():
    """tb_execute mirrors Runtime::execute (projects/titan-runtime/src/lib.rs:1171-1256): an
    operator without a route and a wrong input count fail in the contract phase."""
    L = N.lib()
    t = (N.Tensor * 4)()
    out = N.Tensor()
    ev = ctypes.c_void_p(0)

    def call(op, n):
        return L.tb_execute(None, None, op, t, n, ctypes.byref(out), None, 0, ctypes.byref(ev))

    assert call(b"layer_norm", 1) == N.TB_ERR_UNSUPPORTED
    assert N.last_error() == ("contract", "operator layer_norm is not on the B200 hot path (does not implement)")
    for op, bad, keyword in [(b"softmax", 2, "exactly one input"), (b"gemm", 3, "exactly two"),
                             (b"scaled_dot_product_attention", 2, "exactly three"), (b"conv2d", 1, "optional bias"),
                             (b"conv2d", 4, "optional bias"), (b"gemm.bias_act", 4, "optional bias")]:
        assert call(op, bad) == N.TB_ERR_INVALID, op
        operation, detail = N.last_error()
        assert operation == "contract" and keyword in detail, (op, detail)


def test_execute_takes_the_fused_graph_nodes():
    """tb_execute routes the graph compiler's fused nodes; attention.fused wants contiguous
    rank-2 [T, D] tensors (viewed as [1, 1, T, D]) before any session is touched."""
    L = N.lib()

    def t2(rows, cols, strides=None):
        t = N.Tensor()
        t.dtype, t.rank = N.TB_BF16, 2
        t.shape[0], t.shape[1] = rows, cols
        t.strides[0], t.strides[1] = strides or (cols, 1)
        return t

    ev = ctypes.c_void_p(0)
    ins = (N.Tensor * 3)(t2(4, 8), t2(6, 8, (1, 6)), t2(6, 8))
    assert L.tb_execute(None, None, b"attention.fused", ins, 3, ctypes.byref(t2(4, 8)), None, 0,
                        ctypes.byref(ev)) == N.TB_ERR_INVALID
    assert N.last_error() == ("contract", "attention.fused requires contiguous rank-2 [T, D] Q, K, V and output")
    assert L.tb_execute(None, None, b"attention.fused", ins, 2, ctypes.byref(t2(4, 8)), None, 0,
                        ctypes.byref(ev)) == N.TB_ERR_INVALID
    assert N.last_error()[1] == "attention.fused requires Q, K and V"
    # Contiguous views pass the router and reach the attention operator's own checks.
    ins = (N.Tensor * 3)(t2(4, 8), t2(6, 8), t2(6, 8))
    assert L.tb_execute(None, None, b"attention.fused", ins, 3, ctypes.byref(t2(4, 8)), None, 0,
                        ctypes.byref(ev)) != N.TB_OK
    assert "attention.fused" not in N.last_error()[1]
