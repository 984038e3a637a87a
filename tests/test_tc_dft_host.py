"""The tensor-core column-FFT A/B library builds for sm_100a and exports its
C ABI (no GPU needed)."""
import ctypes

from zipfft_b200 import tc_dft as T


def test_tc_dft_library_builds_and_exports():
    path = T.build()
    lib = ctypes.CDLL(path)
    for name in T.EXPORTS:
        assert hasattr(lib, name), name


def test_tc_dft_rejects_bad_arguments_without_a_launch():
    lib = T.load()
    # misaligned pointer and negative column count fail before any CUDA call
    assert lib.zftc_col_fft4096(ctypes.c_void_p(8), -1, 1, 1, 0, 0, None) == 1
    assert b"invalid" in lib.zftc_last_error()
    assert lib.zftc_col_fft4096(ctypes.c_void_p(16), 4, 0, 1, 0, 0, None) == 1  # passes < 1
    assert lib.zftc_col_fft4096(ctypes.c_void_p(16), 4, 1, 1, 9, 0, None) == 1  # blocks/SM > 8
    assert lib.zftc_col_fft4096(ctypes.c_void_p(8), 1, 1, 1, 0, 99, None) == 1
