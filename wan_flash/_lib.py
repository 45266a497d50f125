"""ctypes binding of ``libwanflash.so`` (the C ABI in include/wan_flash.h).

There is no CPU fallback: if the library is missing or fails to load, every
entry point raises.  ``lib()`` loads it once per process.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

_LIB_PATH = pathlib.Path(__file__).resolve().parent / "libwanflash.so"
_lock = threading.Lock()
_lib = None

# wf_status codes (include/wan_flash.h)
WF_OK = 0
STATUS_NAMES = {
    0: "WF_OK",
    -1: "WF_ERR_INVALID_ARG",
    -2: "WF_ERR_UNSUPPORTED",
    -3: "WF_ERR_MISALIGNED",
    -4: "WF_ERR_CUDA",
    -5: "WF_ERR_NO_DEVICE",
    -6: "WF_ERR_WAIT_TIMEOUT",
    -7: "WF_ERR_SMEM_ALIGN",
}

EXPORTS = (
    "wf_fwd", "wf_fwd_dual", "wf_bwd_pre", "wf_bwd_main", "wf_bwd_convert", "wf_bwd_noalloc", "wf_last_error",
    "wf_device_status", "wf_set_wait_limit_ns", "wf_selftest_wait_timeout", "wf_num_sms", "wf_version",
)


class FwdCfg(ctypes.Structure):
    _fields_ = [("rescale_threshold", ctypes.c_float), ("scheduler", ctypes.c_int), ("num_sms", ctypes.c_int),
                ("cluster_m", ctypes.c_int)]


class BwdCfg(ctypes.Structure):
    _fields_ = [("nsplit", ctypes.c_int), ("cluster_n", ctypes.c_int), ("deterministic", ctypes.c_int),
                ("pdl_off", ctypes.c_int), ("sem", ctypes.c_void_p)]


class WanFlashError(RuntimeError):
    def __init__(self, code: int, message: str):
        self.code = code
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {message}")


def _declare(lib):
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fp = ctypes.POINTER(ctypes.c_float)
    lib.wf_fwd.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, ctypes.POINTER(FwdCfg), vp]
    lib.wf_fwd_dual.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, i, ctypes.POINTER(FwdCfg), vp]
    lib.wf_bwd_pre.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, i, vp]
    lib.wf_bwd_main.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, ctypes.POINTER(BwdCfg), vp]
    lib.wf_bwd_convert.argtypes = [vp, vp, f, i, i, i, vp]
    lib.wf_bwd_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, vp]
    lib.wf_last_error.argtypes = [ctypes.c_char_p, i]
    lib.wf_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    lib.wf_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
    lib.wf_selftest_wait_timeout.argtypes = [ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_uint)]
    for name in EXPORTS:
        getattr(lib, name).restype = ctypes.c_int
    del fp


def lib_path() -> pathlib.Path:
    return _LIB_PATH


def lib():
    """Load (once) and return the CUDA library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"{_LIB_PATH} is missing: build the sm_100a library first "
                    "(python -m wan_flash.build); there is no CPU fallback"
                )
            handle = ctypes.CDLL(str(_LIB_PATH))
            _declare(handle)
            _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().wf_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(code: int):
    if code != WF_OK:
        raise WanFlashError(code, last_error())


def device_status() -> tuple[int, list[int]]:
    """Synchronise and read (and clear) the device error word."""
    info = (ctypes.c_uint * 4)()
    code = lib().wf_device_status(info)
    return code, list(info)


def check_device():
    code, _ = device_status()
    check(code)
