"""zipfft_b200: B200-native (sm_100a) implicitly zero-padded real 2D FFT
convolution / cross-correlation with zipFFT's Python operator API.

    import torch, zipfft            # or: import zipfft_b200 as zipfft
    zipfft.padded_rconv2d.corr(kernel, workspace, image_fft_T, output, H, W)

Package-level helpers mirror the reference's src/zipfft/__init__.py:25-45.
"""
from __future__ import annotations

from typing import List

from . import _lib
from . import padded_rconv2d

__version__ = "0.3.0"

CUDA_ARCHITECTURES = ["10.0a"]


def is_extension_available(extension_name: str) -> bool:
    """True if `extension_name` is built and loads (src/zipfft/__init__.py:25-27)."""
    return extension_name == "padded_rconv2d" and _lib.available()


def get_available_extensions() -> List[str]:
    """Extensions that load (src/zipfft/__init__.py:30-32)."""
    return ["padded_rconv2d"] if _lib.available() else []


def get_cuda_architectures() -> List[str]:
    """CUDA architectures the library is compiled for (src/zipfft/__init__.py:35-37)."""
    return list(CUDA_ARCHITECTURES)


__all__ = [
    "is_extension_available",
    "get_available_extensions",
    "get_cuda_architectures",
    "padded_rconv2d",
]
