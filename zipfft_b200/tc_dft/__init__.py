"""Radix-16 FFT stages on the tensor cores (tcgen05.mma kind::tf32, 3-pass
split) against the same stages on the CUDA cores: the measured A/B behind the
choice of CUDA-core butterflies for the column FFTs.  Not on the product path.

    python -m zipfft_b200.tc_dft [--columns N] [--windows W] [--reps R]

runs both kernels of `col_fft_tc.cu` -- the same in-place 4096-point forward
FFT over N contiguous columns (default 4098: two templates' worth of the
4096^2 column pass, 134 MB, more than the L2), the 16-point DFTs on the CUDA
cores or as a GEMM on the tensor cores -- checks both against numpy's
float64 FFT, times them in interleaved windows with CUDA events and prints
one JSON line.  The kernels stand for the column FFTs of the cuFFTDx-based
passes at src/cuda/real_conv_2d.cuh:84,114.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "col_fft_tc.cu")
LIB = os.path.join(HERE, "libzftc.so")
STAMP = LIB + ".stamp"
_DEPS = [SRC, os.path.join(HERE, "..", "csrc", "fft_core.cuh"),
         os.path.join(HERE, "..", "csrc", "async_copy.cuh")]
EXPORTS = ("zftc_col_fft4096", "zftc_kernel_info", "zftc_occupancy", "zftc_status",
           "zftc_last_error")
N = 4096


def _hash() -> str:
    from zipfft_b200.build import NVCC_FLAGS

    h = hashlib.sha256()
    for f in _DEPS:
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False) -> str:
    """Compile col_fft_tc.cu into libzftc.so (sm_100a) if the sources changed."""
    from zipfft_b200.build import NVCC_FLAGS, nvcc

    want = _hash()
    if not force and os.path.exists(LIB) and os.path.exists(STAMP):
        with open(STAMP) as fh:
            if fh.read().strip() == want:
                return LIB
    tmp = LIB + ".tmp"
    res = subprocess.run([nvcc(), *NVCC_FLAGS, "-shared", "-cudart", "static", "-o", tmp, SRC],
                         capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {SRC}:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    with open(STAMP, "w") as fh:
        fh.write(want + "\n")
    return LIB


_lib = None


def load() -> ctypes.CDLL:
    """The built library (raises if it is missing or stale: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise RuntimeError(f"{LIB} is not built: python -c 'import zipfft_b200.tc_dft as t; t.build()'")
        lib = ctypes.CDLL(LIB)
        lib.zftc_col_fft4096.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        lib.zftc_occupancy.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_int)]
        lib.zftc_kernel_info.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                         ctypes.POINTER(ctypes.c_int)]
        lib.zftc_status.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        lib.zftc_last_error.restype = ctypes.c_char_p
        _lib = lib
    return _lib


def col_fft4096(x, tensor_cores: bool, passes: int = 1, blocks_per_sm: int = 0) -> None:
    """In-place forward FFT of each row of x: (columns, 4096) complex64,
    contiguous, on a CUDA device, applied `passes` times; launched on the
    current stream.  blocks_per_sm > 0 overrides the occupancy calculator's
    blocks per SM for the persistent grid."""
    import torch

    if x.dtype != torch.complex64 or x.dim() != 2 or x.shape[1] != N or not x.is_contiguous() \
            or x.device.type != "cuda":
        raise RuntimeError("expected a contiguous (columns, 4096) complex64 CUDA tensor")
    lib = load()
    dev = x.device.index
    st = lib.zftc_col_fft4096(x.data_ptr(), x.shape[0], int(passes), 1 if tensor_cores else 0,
                              int(blocks_per_sm), dev,
                              torch.cuda.current_stream(dev).cuda_stream)
    if st:
        raise RuntimeError(lib.zftc_last_error().decode())


def kernel_info(tensor_cores: bool, device: int = 0) -> tuple[int, int]:
    """(registers per thread, resident blocks per SM) of one kernel."""
    lib = load()
    regs, occ = ctypes.c_int(), ctypes.c_int()
    if lib.zftc_kernel_info(1 if tensor_cores else 0, device, ctypes.byref(regs), ctypes.byref(occ)):
        raise RuntimeError(lib.zftc_last_error().decode())
    return regs.value, occ.value


def occupancy(tensor_cores: bool, smem: int, device: int = 0) -> int:
    """Resident blocks per SM of one kernel with `smem` bytes of dynamic
    shared memory (the occupancy calculator's answer)."""
    lib = load()
    occ = ctypes.c_int()
    if lib.zftc_occupancy(1 if tensor_cores else 0, device, int(smem), ctypes.byref(occ)):
        raise RuntimeError(lib.zftc_last_error().decode())
    return occ.value


def status(device: int = 0) -> int:
    """The device status word (4 = a bounded wait gave up), then cleared."""
    lib = load()
    out = ctypes.c_int()
    if lib.zftc_status(device, ctypes.byref(out)):
        raise RuntimeError(lib.zftc_last_error().decode())
    return out.value
