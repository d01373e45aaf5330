"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU parity oracle (oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this module, and only as the checker or the timed CPU
baseline. The product path (titan_rs_b200) never imports it.

The functions restate titan.rs's CPU scalar operators
(projects/titan-runtime/src/lib.rs:933-1151); see oracle.h for the contract.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

_HERE = pathlib.Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t


def build() -> pathlib.Path:
    """Compiles liboracle.so with the committed Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    L = ctypes.CDLL(str(_LIB_PATH))
    L.oracle_last_error.restype = ctypes.c_char_p
    L.oracle_num_threads.restype = ctypes.c_int
    L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
    L.oracle_f32_to_bf16.restype = ctypes.c_uint16
    L.oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
    L.oracle_bf16_to_f32.restype = ctypes.c_float
    L.oracle_softmax_f32.argtypes = [_f32p, _f32p, _sz, _sz, _sz]
    L.oracle_softmax_rows_f32_mt.argtypes = [_f32p, _f32p, _sz, _sz, ctypes.c_int]
    L.oracle_gemm_f32.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, ctypes.c_int, ctypes.c_int, _sz, _sz]
    L.oracle_gemm_f32_mt.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, ctypes.c_int]
    L.oracle_conv2d_nchw_f32.argtypes = [_f32p, _f32p, ctypes.c_void_p, _f32p] + [_sz] * 19
    L.oracle_sdpa_f32.argtypes = [_f32p, _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, ctypes.c_int]
    L.oracle_gemm_bf16_points.argtypes = [_u16p, _u16p, ctypes.c_int, _sz, _sz, _sz, _i64p, _i64p, _sz, _f32p,
                                          ctypes.c_int]
    L.oracle_sdpa_bf16_rows.argtypes = [_u16p, _u16p, _u16p, _sz, _sz, _sz, _sz, _sz, ctypes.c_int, ctypes.c_float,
                                        _i64p, _sz, _f32p, ctypes.c_int]
    L.oracle_conv2d_nhwc_bf16_points.argtypes = [_u16p, _u16p, ctypes.c_void_p] + [_sz] * 15 + [_i64p, _sz, _f32p,
                                                                                              ctypes.c_int]
    for name in ("oracle_fill_uniform", "oracle_fill_normal"):
        getattr(L, name).argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, _sz, ctypes.c_uint64,
                                     ctypes.c_double, ctypes.c_double, ctypes.c_int]
    _lib = L
    return L


class OracleError(ValueError):
    pass


def _check(status: int) -> None:
    if status != 0:
        raise OracleError(lib().oracle_last_error().decode())


def num_threads() -> int:
    return int(lib().oracle_num_threads())


# ---- bf16 helpers (bit patterns carried as uint16) ----

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit pattern (vectorised restatement of oracle_f32_to_bf16)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7F800000) == 0x7F800000
    nan &= (b & 0x007FFFFF) != 0
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x0040).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- restated reference operators ----

def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    axis = axis % x.ndim
    outer = int(np.prod(x.shape[:axis], dtype=np.int64))
    inner = int(np.prod(x.shape[axis + 1:], dtype=np.int64))
    y = np.empty_like(x)
    _check(lib().oracle_softmax_f32(x, y, outer, x.shape[axis], inner))
    return y


def softmax_rows_mt(x: np.ndarray, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    _check(lib().oracle_softmax_rows_f32_mt(x, y, x.shape[0], x.shape[1], threads))
    return y


def gemm(lhs: np.ndarray, rhs: np.ndarray, transpose_lhs=False, transpose_rhs=False, out_shape=None) -> np.ndarray:
    lhs = np.ascontiguousarray(lhs, dtype=np.float32)
    rhs = np.ascontiguousarray(rhs, dtype=np.float32)
    if lhs.ndim != 2 or rhs.ndim != 2:
        raise OracleError("gemm requires exactly two rank-2 inputs")
    m = lhs.shape[1] if transpose_lhs else lhs.shape[0]
    n = rhs.shape[0] if transpose_rhs else rhs.shape[1]
    out_shape = tuple(out_shape) if out_shape is not None else (m, n)
    out = np.empty((max(out_shape[0], 0) * max(out_shape[1], 0),), dtype=np.float32)
    if out.size < m * n:
        out = np.empty((m * n,), dtype=np.float32)
    _check(lib().oracle_gemm_f32(lhs, rhs, out, lhs.shape[0], lhs.shape[1], rhs.shape[0], rhs.shape[1],
                                 int(transpose_lhs), int(transpose_rhs), out_shape[0], out_shape[1]))
    return out[: m * n].reshape(m, n)


def gemm_mt(lhs: np.ndarray, rhs: np.ndarray, threads: int = 0) -> np.ndarray:
    lhs = np.ascontiguousarray(lhs, dtype=np.float32)
    rhs = np.ascontiguousarray(rhs, dtype=np.float32)
    out = np.empty((lhs.shape[0], rhs.shape[1]), dtype=np.float32)
    _check(lib().oracle_gemm_f32_mt(lhs, rhs, out, lhs.shape[0], rhs.shape[1], lhs.shape[1], threads))
    return out


def conv2d_nchw(x, w, bias, stride, pad, dilation, groups, out_shape=None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    if x.ndim != 4 or w.ndim != 4:
        raise OracleError("conv2d requires rank-4 NCHW input, rank-4 OIHW weight, and optional bias")
    n, c, h, wd = x.shape
    co, wc, kh, kw = w.shape
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        if bias.shape != (co,):
            raise OracleError("conv2d bias must have shape [output_channels]")
    if out_shape is None:
        eh = dilation[0] * (kh - 1) + 1
        ew = dilation[1] * (kw - 1) + 1
        out_shape = (n, co, max((h + 2 * pad[0] - eh) // max(stride[0], 1) + 1, 0),
                     max((wd + 2 * pad[1] - ew) // max(stride[1], 1) + 1, 0))
    out = np.zeros(int(np.prod(out_shape)), dtype=np.float32)
    bptr = bias.ctypes.data_as(ctypes.c_void_p) if bias is not None else None
    _check(lib().oracle_conv2d_nchw_f32(x, w, bptr, out, n, c, h, wd, co, wc, kh, kw, stride[0], stride[1],
                                        pad[0], pad[1], dilation[0], dilation[1], groups, *out_shape))
    return out.reshape(out_shape)


def sdpa(q, k, v, causal=False) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    b, h, tq, d = q.shape
    tk = k.shape[2]
    out = np.empty_like(q)
    _check(lib().oracle_sdpa_f32(q, k, v, out, b, h, tq, tk, d, int(causal)))
    return out


def gelu(x: np.ndarray) -> np.ndarray:
    """titan-runtime/src/lib.rs:625-640: 0.5 x (1 + erf(x / sqrt 2)) with erf from the
    Abramowitz & Stegun 7.1.26 polynomial evaluated in f64 and rounded to f32, as the
    reference's `erf_approximation` does; x / sqrt 2 is the f32 product (FRAC_1_SQRT_2)."""
    x = np.asarray(x, dtype=np.float32)
    z32 = (x * np.float32(0.70710678118654752)).astype(np.float32)
    sign = np.sign(z32).astype(np.float64)
    z = np.abs(z32).astype(np.float64)
    t = 1.0 / (1.0 + 0.3275911 * z)
    p = 1.061405429
    p = p * t - 1.453152027
    p = p * t + 1.421413741
    p = p * t - 0.284496736
    p = p * t + 0.254829592
    erf = (sign * (1.0 - p * t * np.exp(-z * z))).astype(np.float32)
    return (np.float32(0.5) * x * (np.float32(1.0) + erf)).astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    """titan-runtime/src/lib.rs:3064: value / (1 + exp(-value)) in f32."""
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def gemm_bf16_points(a_bits, b_bits, b_col_major, m, n, k, rows, cols, threads=0) -> np.ndarray:
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    cols = np.ascontiguousarray(cols, dtype=np.int64)
    out = np.empty(rows.shape[0], dtype=np.float32)
    _check(lib().oracle_gemm_bf16_points(np.ascontiguousarray(a_bits).ravel(), np.ascontiguousarray(b_bits).ravel(),
                                         int(b_col_major), m, n, k, rows, cols, rows.shape[0], out, threads))
    return out


def sdpa_bf16_rows(q_bits, k_bits, v_bits, b, h, tq, tk, d, causal, row_ids, scale=0.0, threads=0) -> np.ndarray:
    row_ids = np.ascontiguousarray(row_ids, dtype=np.int64)
    out = np.empty((row_ids.shape[0], d), dtype=np.float32)
    _check(lib().oracle_sdpa_bf16_rows(np.ascontiguousarray(q_bits).ravel(), np.ascontiguousarray(k_bits).ravel(),
                                       np.ascontiguousarray(v_bits).ravel(), b, h, tq, tk, d, int(causal),
                                       float(scale), row_ids, row_ids.shape[0], out, threads))
    return out


def conv2d_nhwc_bf16_points(x_bits, w_bits, bias, n, h, w, cin, cout, r, s, stride, pad, dilation, out_h, out_w,
                            idx, threads=0) -> np.ndarray:
    idx = np.ascontiguousarray(idx, dtype=np.int64)
    out = np.empty(idx.shape[0], dtype=np.float32)
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
    bptr = bias.ctypes.data_as(ctypes.c_void_p) if bias is not None else None
    _check(lib().oracle_conv2d_nhwc_bf16_points(
        np.ascontiguousarray(x_bits).ravel(), np.ascontiguousarray(w_bits).ravel(), bptr, n, h, w, cin, cout, r, s,
        stride[0], stride[1], pad[0], pad[1], dilation[0], dilation[1], out_h, out_w, idx, idx.shape[0], out,
        threads))
    return out


def cpu_count() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


# ---- seeded synthetic inputs (the benchmark's generator, without the product library) ----

def _fill(fn, count, seed, a, b, bf16, first, threads):
    out = np.empty(int(count), dtype=np.uint16 if bf16 else np.float32)
    _check(fn(out.ctypes.data_as(ctypes.c_void_p), int(bool(bf16)), int(first), int(count), int(seed), float(a),
              float(b), int(threads)))
    return out


def fill_normal(count, seed, mean=0.0, std=1.0, bf16=False, first=0, threads=0) -> np.ndarray:
    """Elements [first, first + count) of the seeded normal fill (f32, or bf16 bit patterns)."""
    return _fill(lib().oracle_fill_normal, count, seed, mean, std, bf16, first, threads)


def fill_uniform(count, seed, low=0.0, high=1.0, bf16=False, first=0, threads=0) -> np.ndarray:
    """Elements [first, first + count) of the seeded uniform fill in [low, high)."""
    return _fill(lib().oracle_fill_uniform, count, seed, low, high, bf16, first, threads)

