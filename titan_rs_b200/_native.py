"""ctypes binding of libtitan_b200.so (the C ABI in include/titan_b200.h).

The library is built in-tree by titan_rs_b200.build. Loading fails loudly when
it is missing: there is no CPU or Python fallback for any operator.
"""
from __future__ import annotations

import ctypes
import pathlib

_PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = _PKG / "libtitan_b200.so"

TB_OK = 0
TB_ERR_DRIVER_UNAVAILABLE = 1
TB_ERR_INVALID = 2
TB_ERR_FOREIGN = 3
TB_ERR_CUDA = 4
TB_ERR_UNSUPPORTED = 5
TB_ERR_TIMEOUT = 6
TB_ERR_NCCL = 7
TB_ERR_OUT_OF_MEMORY = 8
TB_ERR_IO = 9

TB_F32, TB_F16, TB_BF16, TB_I32, TB_I64 = 0, 1, 2, 3, 4
TB_ARG_BUFFER, TB_ARG_SCALAR, TB_ARG_SHAPE = 0, 1, 2
TB_MAX_RANK = 6
TB_COMM_ID_BYTES = 128


class TuneMeasurement(ctypes.Structure):
    _fields_ = [("candidate", ctypes.c_char_p), ("median_ns", ctypes.c_uint64), ("p95_ns", ctypes.c_uint64),
                ("workspace_bytes", ctypes.c_uint64)]


class Fingerprint(ctypes.Structure):
    _fields_ = [("ordinal", ctypes.c_uint32), ("model", ctypes.c_char * 128), ("driver", ctypes.c_char * 32),
                ("capability_revision", ctypes.c_char * 16), ("sm_count", ctypes.c_uint32),
                ("total_memory", ctypes.c_uint64)]


class LaunchArg(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_uint32), ("width", ctypes.c_uint32)]


class LaunchMetadata(ctypes.Structure):
    _fields_ = [("version", ctypes.c_uint32), ("entry", ctypes.c_char_p), ("arguments", ctypes.POINTER(LaunchArg)),
                ("num_arguments", ctypes.c_uint32), ("block", ctypes.c_uint32 * 3), ("shared_bytes", ctypes.c_uint32)]


class Binding(ctypes.Structure):
    _fields_ = [("slot", ctypes.c_uint32), ("buffer", ctypes.c_void_p), ("owner", ctypes.c_void_p)]


class EncodedArgs(ctypes.Structure):
    _fields_ = [("payload", ctypes.POINTER(ctypes.c_uint8)), ("payload_len", ctypes.c_size_t),
                ("bindings", ctypes.POINTER(Binding)), ("num_bindings", ctypes.c_uint32),
                ("canonical_abi", ctypes.POINTER(ctypes.c_uint8)), ("canonical_abi_len", ctypes.c_size_t)]


class LaunchGeometry(ctypes.Structure):
    _fields_ = [("grid", ctypes.c_uint32 * 3), ("block", ctypes.c_uint32 * 3), ("shared_bytes", ctypes.c_uint32)]


class Tensor(ctypes.Structure):
    _fields_ = [("buffer", ctypes.c_void_p), ("dtype", ctypes.c_uint32), ("rank", ctypes.c_uint32),
                ("shape", ctypes.c_uint64 * TB_MAX_RANK), ("strides", ctypes.c_int64 * TB_MAX_RANK)]


class Attr(ctypes.Structure):
    _fields_ = [("key", ctypes.c_char_p), ("value", ctypes.c_int64), ("str", ctypes.c_char_p)]


_P = ctypes.c_void_p
_PP = ctypes.POINTER(ctypes.c_void_p)
_S = ctypes.c_int
_SZ = ctypes.c_size_t
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64

# name -> (restype, argtypes)
_SIGNATURES = {
    "tb_last_error_operation": (ctypes.c_char_p, []),
    "tb_last_error_detail": (ctypes.c_char_p, []),
    "tb_version": (ctypes.c_char_p, []),
    "tb_last_candidate": (ctypes.c_char_p, []),
    "tb_launch_count": (_U64, []),
    "tb_driver_open": (_S, []),
    "tb_driver_enumerate": (_S, [ctypes.POINTER(Fingerprint), _U32, ctypes.POINTER(_U32)]),
    "tb_session_open": (_S, [_U32, _PP]),
    "tb_session_retain": (None, [_P]),
    "tb_session_release": (None, [_P]),
    "tb_session_fingerprint": (_S, [_P, ctypes.POINTER(Fingerprint)]),
    "tb_allocate": (_S, [_P, _SZ, _SZ, _PP]),
    "tb_buffer_wrap": (_S, [_P, _U64, _SZ, _PP]),
    "tb_buffer_retain": (None, [_P]),
    "tb_buffer_release": (None, [_P]),
    "tb_buffer_byte_len": (_SZ, [_P]),
    "tb_buffer_identity": (_U64, [_P]),
    "tb_buffer_device_ptr": (_U64, [_P]),
    "tb_create_stream": (_S, [_P, _PP]),
    "tb_stream_release": (None, [_P]),
    "tb_create_event": (_S, [_P, _PP]),
    "tb_event_release": (None, [_P]),
    "tb_upload": (_S, [_P, _P, _P, _P, _SZ, _PP]),
    "tb_download": (_S, [_P, _P, _P, _P, _SZ, _PP]),
    "tb_copy": (_S, [_P, _P, _P, _P, _SZ, _PP]),
    "tb_load": (_S, [_P, _P, _SZ, ctypes.c_char_p, ctypes.POINTER(LaunchMetadata), _PP]),
    "tb_kernel_release": (None, [_P]),
    "tb_builtin_cubin": (_S, [ctypes.c_char_p, _PP, ctypes.POINTER(_SZ)]),
    "tb_launch": (_S, [_P, _P, _P, ctypes.POINTER(EncodedArgs), ctypes.POINTER(LaunchGeometry), _PP]),
    "tb_poll": (_S, [_P, _P, ctypes.POINTER(ctypes.c_int)]),
    "tb_wait": (_S, [_P, _P]),
    "tb_wait_event": (_S, [_P, _P, _P]),
    "tb_record": (_S, [_P, _P, _PP]),
    "tb_event_elapsed_ms": (_S, [_P, _P, _P, ctypes.POINTER(ctypes.c_float)]),
    "tb_stream_synchronize": (_S, [_P, _P]),
    "tb_stream_handle": (_U64, [_P]),
    "tb_capture_begin": (_S, [_P, _P]),
    "tb_capture_end": (_S, [_P, _P, _PP]),
    "tb_graph_exec_launch": (_S, [_P, _P, _P]),
    "tb_graph_exec_release": (None, [_P]),
    "tb_host_alloc": (_S, [_P, _SZ, _PP]),
    "tb_host_free": (_S, [_P, _P]),
    "tb_upload_pinned": (_S, [_P, _P, _P, _SZ, _P, _SZ, _PP]),
    "tb_download_pinned": (_S, [_P, _P, _P, _SZ, _P, _SZ, _PP]),
    "tb_op_softmax": (_S, [_P, _P, ctypes.POINTER(Tensor), ctypes.POINTER(Tensor), ctypes.POINTER(Attr), _U32, _PP]),
    "tb_op_gemm": (_S, [_P, _P, ctypes.POINTER(Tensor), ctypes.POINTER(Tensor), ctypes.POINTER(Tensor),
                        ctypes.POINTER(Attr), _U32, _PP]),
    "tb_op_sdpa": (_S, [_P, _P, ctypes.POINTER(Tensor), ctypes.POINTER(Tensor), ctypes.POINTER(Tensor),
                        ctypes.POINTER(Tensor), ctypes.POINTER(Attr), _U32, _PP]),
    "tb_op_conv2d": (_S, [_P, _P, ctypes.POINTER(Tensor), ctypes.POINTER(Tensor), ctypes.POINTER(Tensor),
                          ctypes.POINTER(Tensor), ctypes.POINTER(Attr), _U32, _PP]),
    "tb_comm_unique_id": (_S, [ctypes.POINTER(ctypes.c_uint8)]),
    "tb_comm_init": (_S, [_P, ctypes.POINTER(ctypes.c_uint8), _S, _S, _U32, _PP]),
    "tb_comm_release": (None, [_P]),
    "tb_comm_rank": (_S, [_P]),
    "tb_comm_size": (_S, [_P]),
    "tb_comm_all_gather": (_S, [_P, _P, _P, _P, _SZ, _PP]),
    "tb_comm_barrier": (_S, [_P, _P]),
    "tb_comm_register_buffer": (_S, [_P, _P, _P]),
    "tb_comm_deregister_buffer": (_S, [_P, _P]),
    "tb_op_gemm_bias_act": (_S, [_P, _P, ctypes.POINTER(Tensor), ctypes.POINTER(Tensor), ctypes.POINTER(Tensor),
                                 ctypes.POINTER(Tensor), ctypes.POINTER(Attr), _U32, _PP]),
    "tb_op_gemm_sharded": (_S, [_P, _P, ctypes.POINTER(Tensor), ctypes.POINTER(Tensor), ctypes.POINTER(Tensor), _P,
                                _PP]),
    "tb_gemm_bf16_splitk_noalloc": (_S, [_U64, _P, _P, _P, _S, _S, _S, _S]),
    "tb_gemm_bf16_splitk_noalloc_status": (_S, [_U64, ctypes.POINTER(_U32)]),
    "tb_fill_normal": (_S, [_P, _U32, _SZ, _U64, ctypes.c_double, ctypes.c_double, _S]),
    "tb_fill_uniform": (_S, [_P, _U32, _SZ, _U64, ctypes.c_double, ctypes.c_double, _S]),
    "tb_execute": (_S, [_P, _P, ctypes.c_char_p, ctypes.POINTER(Tensor), _U32, ctypes.POINTER(Tensor),
                        ctypes.POINTER(Attr), _U32, _PP]),
    "tb_graph_compile": (_S, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _SZ, ctypes.POINTER(_SZ)]),
    "tb_tune_open": (_S, [ctypes.c_char_p, _PP]),
    "tb_tune_release": (None, [_P]),
    "tb_tune_insert": (_S, [_P, ctypes.c_char_p, ctypes.c_char_p]),
    "tb_tune_get": (_S, [_P, ctypes.c_char_p, ctypes.c_char_p, _SZ, ctypes.POINTER(_SZ)]),
    "tb_tune_flush": (_S, [_P]),
    "tb_tune_stats": (_S, [_P, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "tb_tune_record": (_S, [_P, _SZ, ctypes.c_char_p, _SZ, ctypes.POINTER(_SZ), ctypes.c_char_p, _SZ,
                            ctypes.POINTER(_SZ)]),
    "tb_tune_canonical_json": (_S, [ctypes.c_char_p, ctypes.c_char_p, _SZ, ctypes.POINTER(_SZ)]),
    "tb_tune_select": (_S, [ctypes.POINTER(TuneMeasurement), _SZ, ctypes.POINTER(_SZ)]),
    "tb_sha256_hex": (_S, [ctypes.c_char_p, _SZ, ctypes.c_char_p]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


class NativeLibraryMissing(RuntimeError):
    pass


def lib():
    """Loads libtitan_b200.so once; raises NativeLibraryMissing when it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise NativeLibraryMissing(
            f"{LIB_PATH} is not built: run `python -m titan_rs_b200.build` (there is no fallback path)")
    L = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def builtin_cubin(module: str) -> bytes:
    """Bytes of an embedded sm_100a cubin (tb_builtin_cubin)."""
    L = lib()
    data = ctypes.c_void_p(0)
    n = ctypes.c_size_t(0)
    if L.tb_builtin_cubin(module.encode(), ctypes.byref(data), ctypes.byref(n)) != TB_OK:
        raise KeyError(module)
    return ctypes.string_at(data.value, n.value)


def last_error() -> tuple[str, str]:
    L = lib()
    return L.tb_last_error_operation().decode(), L.tb_last_error_detail().decode()


def _text_out(call, *args):
    """Runs a tb_* call whose last three arguments are (out, cap, len); grows the buffer
    until the text fits. Returns the text, or None when *len is 0."""
    cap = 512
    n = ctypes.c_size_t(0)
    while True:
        buf = ctypes.create_string_buffer(cap)
        status = call(*args, buf, cap, ctypes.byref(n))
        if status == TB_OK:
            return buf.raw[:n.value].decode() if n.value else None
        if n.value < cap:
            raise ValueError(last_error()[1])
        cap = n.value + 1


def sha256_hex(data: bytes) -> str:
    out = ctypes.create_string_buffer(65)
    if lib().tb_sha256_hex(data, len(data), out) != TB_OK:
        raise ValueError(last_error()[1])
    return out.value.decode()


def canonical_json(text: str) -> str:
    return _text_out(lib().tb_tune_canonical_json, text.encode())


class TuneStore:
    """Owner of a native `.tune` version 2 store (tb_tune_*); records are canonical JSON text."""

    def __init__(self, path):
        self._lib = lib()
        h = ctypes.c_void_p(0)
        if self._lib.tb_tune_open(str(path).encode(), ctypes.byref(h)) != TB_OK:
            raise ValueError(last_error()[1])
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._lib.tb_tune_release(h)
            self._h = None

    def insert(self, key_json: str, entry_json: str) -> None:
        if self._lib.tb_tune_insert(self._h, key_json.encode(), entry_json.encode()) != TB_OK:
            raise ValueError(last_error()[1])

    def get(self, key_json: str):
        return _text_out(self._lib.tb_tune_get, self._h, key_json.encode())

    def flush(self) -> None:
        status = self._lib.tb_tune_flush(self._h)
        if status == TB_ERR_IO:
            raise OSError(last_error()[1])
        if status != TB_OK:
            raise ValueError(last_error()[1])

    def stats(self) -> tuple[int, int]:
        records, ignored = ctypes.c_size_t(0), ctypes.c_size_t(0)
        self._lib.tb_tune_stats(self._h, ctypes.byref(records), ctypes.byref(ignored))
        return records.value, ignored.value

    def records(self) -> list[tuple[str, str]]:
        out = []
        kcap = ecap = 512
        kn, en = ctypes.c_size_t(0), ctypes.c_size_t(0)
        for i in range(self.stats()[0]):
            while True:
                kb, eb = ctypes.create_string_buffer(kcap), ctypes.create_string_buffer(ecap)
                status = self._lib.tb_tune_record(self._h, i, kb, kcap, ctypes.byref(kn), eb, ecap, ctypes.byref(en))
                if status == TB_OK:
                    out.append((kb.raw[:kn.value].decode(), eb.raw[:en.value].decode()))
                    break
                if kn.value < kcap and en.value < ecap:
                    raise ValueError(last_error()[1])
                kcap, ecap = max(kcap, kn.value + 1), max(ecap, en.value + 1)
        return out
