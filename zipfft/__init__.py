"""`import zipfft` alias of zipfft_b200, so code written against the
reference package (mgiammar/zipFFT src/zipfft/__init__.py) runs unchanged."""
from zipfft_b200 import (  # noqa: F401
    __version__,
    CUDA_ARCHITECTURES,
    get_available_extensions,
    get_cuda_architectures,
    is_extension_available,
    padded_rconv2d,
)

__all__ = [
    "is_extension_available",
    "get_available_extensions",
    "get_cuda_architectures",
    "padded_rconv2d",
]
