"""ctypes binding of libzipfft_b200.so (C ABI in include/zipfft_b200.h).

The library is loaded from the package directory, where
`python -m zipfft_b200.build` puts it.  There is no fallback: if the library
is missing or fails to load, every call raises RuntimeError.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "libzipfft_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

ZFFT_SUCCESS = 0
ZFFT_ERROR_INVALID_VALUE = 1
ZFFT_ERROR_UNSUPPORTED = 2
ZFFT_ERROR_CUDA = 3
ZFFT_ERROR_TIMEOUT = 4

# Every symbol include/zipfft_b200.h declares: name -> (restype, argtypes).
_c_int, _c_size, _vp = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p
_CONV_ARGS = [_vp, _c_int, _c_int, _c_int, _vp, _c_size, _vp, _vp, _c_int, _c_int, _c_int,
              _c_int, _c_int, _vp]
SIGNATURES = {
    "zfft_padded_real_corr_2d": (_c_int, _CONV_ARGS),
    "zfft_padded_real_conv_2d": (_c_int, _CONV_ARGS),
    "zfft_padded_real_corr_2d_noalloc": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _c_int,
                                                  _c_int, _c_int, _c_int, _c_int, _vp]),
    "zfft_padded_real_corr_2d_max": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _c_size, _vp, _vp,
                                              _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                              _c_int, _vp]),
    "zfft_padded_real_corr_2d_peaks": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _c_size, _vp,
                                                _vp, _c_int, _c_int, _c_int, _c_int, _vp, _c_int,
                                                _vp]),
    "zfft_padded_real_corr_2d_max_stats": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _c_size,
                                                    _vp, _vp, _vp, _vp, _vp, _c_int, _c_int,
                                                    _c_int, _c_int, _c_int, _c_int, _c_int, _vp]),
    "zfft_pack_max_arg": (_c_int, [_vp, _vp, _vp, _c_size, _c_int, _vp]),
    "zfft_unpack_max_arg": (_c_int, [_vp, _vp, _vp, _c_size, _c_int, _vp]),
    "zfft_image_spectrum": (_c_int, [_vp, _c_int, _c_int, _vp, _c_size, _c_int, _vp]),
    "zfft_workspace_bytes": (_c_size, [_c_int, _c_int]),
    "zfft_is_fft_size_supported": (_c_int, [_c_int]),
    "zfft_get_supported_conv_configs": (_c_int, [ctypes.POINTER(ctypes.c_int), _c_int]),
    "zfft_get_last_error": (ctypes.c_char_p, []),
    "zfft_get_version": (_c_int, []),
    "zfft_check_device_status": (_c_int, [_c_int, _vp, ctypes.POINTER(ctypes.c_int)]),
    "zfft_selftest_wait_timeout": (_c_int, [_c_int, _vp]),
    "zfft_stage_timing_enable": (_c_int, [_c_int]),
    "zfft_stage_timing_read": (_c_int, [ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_int), _c_int]),
}

STAGE_NAMES = ("k_row_r2c", "k_col_fused", "k_row_c2r")


def stage_timing(enable: bool) -> None:
    """Turn per-stage event timing on or off for the calling thread."""
    check(load().zfft_stage_timing_enable(1 if enable else 0))


def stage_timing_read() -> dict:
    """{stage name: (total ms, launches)} since the last read (synchronises)."""
    ms = (ctypes.c_double * 3)()
    n = (ctypes.c_int * 3)()
    check(load().zfft_stage_timing_read(ms, n, 3))
    return {STAGE_NAMES[i]: (ms[i], n[i]) for i in range(3)}

_lock = threading.Lock()
_lib = None
_load_error: str | None = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the library once and declare every exported signature."""
    global _lib, _load_error
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            _load_error = (f"{LIB_NAME} not found at {p}; build it with "
                           "`python -m zipfft_b200.build` (nvcc, sm_100a)")
            raise RuntimeError(_load_error)
        try:
            lib = ctypes.CDLL(p)
        except OSError as exc:  # pragma: no cover - depends on the host
            _load_error = f"failed to load {p}: {exc}"
            raise RuntimeError(_load_error) from exc
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def last_error() -> str:
    msg = load().zfft_get_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    """Raise RuntimeError carrying the library's message for a non-zero status."""
    if status != ZFFT_SUCCESS:
        raise RuntimeError(last_error() or f"zipfft_b200 call failed with status {status}")


def check_device_status(device: int, stream=None) -> int:
    """Synchronize `stream` on `device` and return (and clear) the device
    status word: 0, or ZFFT_ERROR_TIMEOUT if a kernel gave up on a wait."""
    st = ctypes.c_int(0)
    check(load().zfft_check_device_status(int(device), stream, ctypes.byref(st)))
    return st.value
