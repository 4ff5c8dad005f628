"""ctypes binding of libnsq.so (the C ABI declared in include/nsq.h).

The library is loaded from the package directory only. There is no fallback:
if it is missing or fails to load, every operation raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libnsq.so")

# element type codes (include/nsq.h)
DTYPE_NONE = -1
DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_F32 = 2

# return codes
OK = 0
EINVAL = 1
EALIGN = 2
ENOTSUP = 3
ECUDA = 4
EWORKSPACE = 5
EDEVICE_TIMEOUT = 6

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_size_t = ctypes.c_size_t

# name -> (restype, argtypes); the complete exported surface of include/nsq.h
SIGNATURES = {
    "nsq_strerror": (ctypes.c_char_p, [c_int]),
    "nsq_version": (c_int, []),
    "nsq_device_status": (c_int, [ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "nsq_device_status_reset": (c_int, []),
    "nsq_awq_dequant": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "nsq_awq_linear": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                               c_int64, c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "nsq_fp8_linear": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                               c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "nsq_awq_linear_multi": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_int64, c_void_p, c_int, c_void_p, c_int64, c_void_p]),
    "nsq_fp8_linear_multi": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_int, c_void_p, c_int64, c_void_p]),
    "nsq_awq_gate_up_silu": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "nsq_fp8_gate_up_silu": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_void_p]),
    "nsq_fp8_dequant": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "nsq_awq_quantize": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                 c_void_p]),
    "nsq_awq_from_autoawq": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                     c_void_p, c_void_p]),
    "nsq_fp8_quantize_workspace_size": (c_size_t, [c_int64, c_int64]),
    "nsq_linear_workspace_size": (c_size_t, [c_int, c_int64, c_int64, c_int64, c_int64]),
    "nsq_fp8_quantize": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_size_t,
                                 c_void_p]),
    "nsq_fp8_quantize_noalloc": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "nsq_set_pdl": (c_int, [c_int]),
    "nsq_set_wait_limit_ns": (c_int, [ctypes.c_uint64]),
    "nsq_set_sm_reserve": (c_int, [c_int]),
    "nsq_peer_workspace_size": (c_size_t, [c_int, c_int64]),
    "nsq_peer_workspace_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p)]),
    "nsq_peer_workspace_free": (c_int, [c_void_p]),
    "nsq_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "nsq_ipc_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "nsq_ipc_close": (c_int, [c_void_p]),
    "nsq_peer_allreduce": (c_int, [c_void_p, c_int, c_int, c_int64, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "nsq_test_withhold_weight_load": (c_int, [c_int]),
}

_lib = None
_lock = threading.Lock()


class NsqError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = strerror(code) if _lib is not None else f"nsq error {code}"
        super().__init__(f"{what}: {msg} (nsq code {code})" if what else msg)


def load() -> ctypes.CDLL:
    """Load libnsq.so (once). Raises if it is absent: there is no CPU path."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libnsq.so not found at {LIB_PATH}; build it with "
                "`python -m nanosglang_b200._build` (nvcc, sm_100a). There is no CPU fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def strerror(code: int) -> str:
    return load().nsq_strerror(int(code)).decode()


def check(code: int, what: str = "") -> None:
    if code != OK:
        raise NsqError(code, what)


def set_pdl(enable: bool) -> bool:
    """Opt in to programmatic dependent launch for the linear kernels."""
    return bool(load().nsq_set_pdl(1 if enable else 0))


def device_status():
    """(code, where, block) of the device status word (synchronises)."""
    w = c_int(0)
    b = c_int(0)
    code = load().nsq_device_status(ctypes.byref(w), ctypes.byref(b))
    return code, w.value, b.value


def device_status_reset() -> None:
    """Clear the device status word (also restores the default wait limit)."""
    check(load().nsq_device_status_reset(), "nsq_device_status_reset")


def set_sm_reserve(n: int) -> int:
    """SMs the linear kernels leave free for a concurrent collective; returns the previous value."""
    return int(load().nsq_set_sm_reserve(int(n)))


def set_wait_limit_ns(ns: int) -> None:
    """Limit of every bounded device wait that reports to the status word (0 = the 2 s default)."""
    check(load().nsq_set_wait_limit_ns(int(ns)), "nsq_set_wait_limit_ns")


def withhold_weight_load_for_test(enable: bool) -> bool:
    """Failure-path test hook (see include/nsq.h); returns the previous setting."""
    return bool(load().nsq_test_withhold_weight_load(1 if enable else 0))
