"""ctypes binding of the C ABI declared in include/lmce.h (liblmce.so).

The library is loaded from the package directory only. There is no fallback:
if the shared object is missing or the device is not sm_100, every call
raises. Status codes are mapped to ``LmceError`` with the library's message.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblmce.so"

LMCE_OK = 0
LMCE_ERR_INVALID_ARGUMENT = 1
LMCE_ERR_UNSUPPORTED = 2
LMCE_ERR_CUDA = 3
LMCE_ERR_TIMEOUT = 4
LMCE_ERR_LABEL_RANGE = 5
LMCE_ERR_WORKSPACE = 6

LMCE_DTYPE_F16 = 0
LMCE_DTYPE_BF16 = 1

PART_BYTES = 24  # sizeof(lmce_part)


class DxExchange(ctypes.Structure):
    """struct lmce_dx_exchange (buffers of the fused cross-GPU dX sum)."""
    _fields_ = [
        ("partial", ctypes.c_void_p),
        ("partial_mc", ctypes.c_void_p),
        ("out_mc", ctypes.c_void_p),
        ("flags", ctypes.c_void_p),
        ("flags_mc", ctypes.c_void_p),
        ("epoch", ctypes.c_uint32),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
    ]

_ERR_NAMES = {
    LMCE_ERR_INVALID_ARGUMENT: "LMCE_ERR_INVALID_ARGUMENT",
    LMCE_ERR_UNSUPPORTED: "LMCE_ERR_UNSUPPORTED",
    LMCE_ERR_CUDA: "LMCE_ERR_CUDA",
    LMCE_ERR_TIMEOUT: "LMCE_ERR_TIMEOUT",
    LMCE_ERR_LABEL_RANGE: "LMCE_ERR_LABEL_RANGE",
    LMCE_ERR_WORKSPACE: "LMCE_ERR_WORKSPACE",
}


class LmceError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{_ERR_NAMES.get(code, code)}: {message}")
        self.code = code


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

# name -> (restype, argtypes); mirrors include/lmce.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "lmce_abi_version": (_int, []),
    "lmce_last_error": (ctypes.c_char_p, []),
    "lmce_device_error": (_int, [_int]),
    "lmce_fwd_num_parts": (_i64, [_i64, _i64]),
    "lmce_fwd_stats": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _i64, _vp]),
    "lmce_stats_reduce": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "lmce_stats_finish": (
        _int,
        [_vp, _i64, _i64, _i64, _vp, _i64, _vp, ctypes.c_double, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
    "lmce_bwd_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64, _i64]),
    "lmce_backward": (
        _int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _vp, _vp, _vp, _vp, _i64, _vp, ctypes.c_size_t, _vp],
    ),
    "lmce_backward_nvls": (
        _int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _vp, ctypes.POINTER(DxExchange), _vp, _i64, _vp,
         ctypes.c_size_t, _vp],
    ),
    "lmce_dx_copy_labelled": (_int, [_vp, _vp, _i64, _i64, _int, _vp, _vp]),
    "lmce_pack_tokens": (_int, [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _int, _vp, _vp]),
    "lmce_scatter_token_outputs": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp]),
    "lmce_embedding_grad_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "lmce_embedding_grad_add": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _vp, ctypes.c_size_t, _vp]),
    "lmce_embedding_lookup": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "lmce_rmsnorm_pack": (_int, [_vp, _vp, ctypes.c_float, _vp, _vp, _i64, _i64, _int, _vp, _vp, _vp]),
    "lmce_rmsnorm_backward": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _vp, _vp]),
    "lmce_dx_finalize": (_int, [_vp, _i64, _i64, _int, _vp, _vp]),
    "lmce_selftest_wait_timeout": (_int, [ctypes.c_uint64, _vp]),
    "lmce_launch_count": (ctypes.c_uint64, []),
    "lmce_set_timing_events": (_int, [_int, _vp, _vp]),
    "lmce_profile_read": (_int, [_vp, ctypes.c_size_t, _vp, ctypes.c_size_t, _int]),
    "lmce_probe_tma_rate": (_int, [_vp, _i64, _i64, _int, _int, _vp, _i64, _vp]),
    "lmce_probe_tma_pipeline": (_int, [_vp, _i64, _i64, _int, _int, _int, _int, _int, _vp, _i64, _vp]),
    "lmce_forward_noalloc": (
        _int,
        [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, ctypes.c_double, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load liblmce.so (once). Raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise LmceError(
                    LMCE_ERR_UNSUPPORTED,
                    f"{LIB_PATH} is missing: build it with `python -m rus_b200.build` (there is no CPU fallback)",
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.lmce_abi_version() != 1:
                raise LmceError(LMCE_ERR_UNSUPPORTED, "liblmce.so ABI version mismatch")
            _lib = lib
        return _lib


def check(rc: int) -> None:
    if rc != LMCE_OK:
        msg = load().lmce_last_error()
        raise LmceError(rc, msg.decode() if msg else "")


def call(name: str, *args) -> int:
    fn = getattr(load(), name)
    rc = fn(*args)
    check(rc)
    return rc


def launch_count() -> int:
    """Kernels launched by liblmce.so in this process so far."""
    return int(load().lmce_launch_count())


def device_error(reset: bool = True) -> int:
    """Synchronously read (and by default clear) the current device's error word."""
    return load().lmce_device_error(1 if reset else 0)
