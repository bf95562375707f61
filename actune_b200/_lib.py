"""ctypes binding of libactune_b200.so (the C ABI declared in include/actune_b200.h).

The library is built in-tree by ``python -m actune_b200.build`` (or
``__graft_entry__.build()``).  There is no fallback: if the library is missing
or the current device is not an sm_100 GPU, every call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libactune_b200.so")

OK = 0
ERR_INVALID_VALUE = 1
ERR_MISALIGNED = 2
ERR_DEVICE = 3
ERR_CUDA = 4
ERR_WORKSPACE = 5

DTYPE_NONE, DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2, 3
VARIANT_AUTO, VARIANT_BN32, VARIANT_BN64, VARIANT_BN128 = 0, 1, 2, 3
VARIANT_WT16, VARIANT_WT32, VARIANT_WT64, VARIANT_WT128 = 4, 5, 6, 7
VARIANT_GEMV = 8
VARIANT_BN32X2, VARIANT_BN64X2, VARIANT_BN128X2 = 9, 10, 11
VARIANT_BN64P, VARIANT_BN128P = 12, 13
VARIANT_MAX = VARIANT_BN128P

# Every symbol the header declares (checked by the CPU test suite).
EXPORTS = (
    "actune_quantize_group64",
    "actune_quantize_group64_codes",
    "actune_packed_linear",
    "actune_quantize_rows_a8",
    "actune_tokenwise_linear",
    "actune_quantize_rows_a4",
    "actune_rowwise_linear",
    "actune_packed_linear_dots",
    "actune_weight_codes",
    "actune_r4_refine",
    "actune_pack_rows",
    "actune_grouped_linear_workspace_size",
    "actune_grouped_linear",
    "actune_status_string",
    "actune_device_error",
    "actune_abi_version",
    "actune_last_cuda_error",
    "actune_grouped_linear_noalloc",
    "actune_set_wait_limit_ns",
    "actune_wait_limit_ns",
    "actune_selftest_wait_timeout",
)

_LIB = None
_LOCK = threading.Lock()


class ActuneError(RuntimeError):
    """A C-ABI call returned a non-zero actune_status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _declare(L):
    p, i32, i64, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
    L.actune_quantize_group64.argtypes = [p, i32, i64, i64, i32, p, p, p]
    L.actune_quantize_group64_codes.argtypes = [p, i32, i64, i64, i32, p, p, p]
    L.actune_packed_linear.argtypes = [p, p, p, p, p, i32, p, i32, i64, i64, i64, i32, i32, i32, p]
    L.actune_packed_linear_dots.argtypes = [p, p, p, i64, i64, i64, i32, i32, i32, p]
    L.actune_quantize_rows_a8.argtypes = [p, i32, i64, i64, p, p, p]
    L.actune_tokenwise_linear.argtypes = [p, p, p, p, p, i32, p, i32, i64, i64, i64, i32, i32, p]
    L.actune_quantize_rows_a4.argtypes = [p, i32, i64, i64, p, p, p]
    L.actune_rowwise_linear.argtypes = [p, i32, p, p, i32, p, p, i32, p, i32, i64, i64, i64, i32, i32, p]
    L.actune_weight_codes.argtypes = [p, i32, i64, i64, i32, i32, p, p, p, p]
    L.actune_r4_refine.argtypes = [p, i32, i64, i64, p, p, p, p, p]
    L.actune_pack_rows.argtypes = [p, i64, i64, i32, p, p]
    L.actune_grouped_linear_workspace_size.argtypes = [i64, i64, i32]
    L.actune_grouped_linear_workspace_size.restype = sz
    L.actune_grouped_linear.argtypes = [p, i32, i64, i64, p, p, p, i32, i64, i32, i32, p, i32, p, sz, i32, p]
    L.actune_status_string.argtypes = [i32]
    L.actune_status_string.restype = ctypes.c_char_p
    L.actune_device_error.argtypes = [ctypes.POINTER(i32), ctypes.POINTER(i32), i32]
    L.actune_abi_version.argtypes = []
    L.actune_last_cuda_error.argtypes = []
    L.actune_grouped_linear_noalloc.argtypes = [p, i32, i64, i64, p, p, p, i32, i64, i32, i32, p, i32, i32, p]
    L.actune_set_wait_limit_ns.argtypes = [ctypes.c_uint64]
    L.actune_wait_limit_ns.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
    L.actune_selftest_wait_timeout.argtypes = [i32, p]
    for name in EXPORTS:
        if name not in ("actune_status_string", "actune_grouped_linear_workspace_size"):
            getattr(L, name).restype = i32
    return L


def lib():
    """Load (once) and return the CDLL; raises if the library was not built."""
    global _LIB
    if _LIB is None:
        with _LOCK:
            if _LIB is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH.name} is not built; run `python -m actune_b200.build` "
                        "(the packed-integer path has no fallback implementation)")
                _LIB = _declare(ctypes.CDLL(str(LIB_PATH)))
    return _LIB


def status_string(status: int) -> str:
    return lib().actune_status_string(int(status)).decode()


def check(status: int, what: str = "") -> None:
    if status != OK:
        msg = f"actune_b200{(' ' + what) if what else ''}: {status_string(status)} (status {status})"
        if status == ERR_CUDA:
            msg += f" [cudaError {lib().actune_last_cuda_error()}]"
        raise ActuneError(status, msg)


def wait_limit_ns() -> int:
    """The current device's pipeline wait limit (ns)."""
    v = ctypes.c_uint64(0)
    check(lib().actune_wait_limit_ns(ctypes.byref(v)), "wait_limit_ns")
    return v.value


def set_wait_limit_ns(ns: int) -> None:
    """Set the current device's pipeline wait limit (1 ms .. 60 s)."""
    check(lib().actune_set_wait_limit_ns(int(ns)), "set_wait_limit_ns")


def device_error(reset: bool = False):
    """(code, site) of the current device's error word (synchronises the device)."""
    code, site = ctypes.c_int(0), ctypes.c_int(0)
    check(lib().actune_device_error(ctypes.byref(code), ctypes.byref(site), 1 if reset else 0), "device_error")
    return code.value, site.value
