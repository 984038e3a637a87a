"""CPU oracle for the implicitly zero-padded real 2D FFT cross-correlation.

TEST INFRASTRUCTURE ONLY (tests/, __graft_entry__.smoke(), bench.py's CPU
baseline and reference arm).  The library never imports this module.

Restates mgiammar/zipFFT's own correctness oracle, the torch.fft path of
tests/test_real_conv_2d.py:110-123:

    filter_fft = rfftn(filter, s=(H, W))                    (test:111)
    result_fft = image_fft * conj(filter_fft)   # corr      (test:113-115)
               = image_fft * filter_fft         # conv      (test:116-118)
    result     = irfftn(result_fft, norm="backward")        (test:120-122)
    result     = result[..., :H-h+1, :W-w+1]                (test:123)

with the image spectrum passed transposed, (W/2+1, H) (test:125-127,
real_conv_2d_binding.cu:248-255).  The reference's CUDA path cannot run here
(it needs cuFFTDx, absent from this environment, and has no sm_100 case:
real_conv_2d.cuh:306-331), so the oracle is pinned instead by
  * direct_corr2d (oracle/direct_corr.c): the correlation's definition as a
    brute-force double-precision sum, and
  * the committed golden fixtures in tests/golden/ (made by
    tests/golden/make_golden.py from this torch path and the direct sum).
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))


def image_spectrum_T(image, dtype=np.complex64) -> np.ndarray:
    """rfft2 of a real (H, W) image, transposed to (W/2+1, H).

    The layout zipFFT's operator expects for `conv_data`, which the reference's
    callers compute as `torch.fft.rfftn(image).transpose(-2, -1)` (README.md:
    224-228, test:89-90 and :125-127).  Computed in float64 and rounded once to
    `dtype` (complex64 by default; complex128 keeps the float64 values)."""
    img = np.asarray(image, dtype=np.float64)
    return np.ascontiguousarray(np.fft.rfft2(img).T).astype(dtype)


def out_shape(h: int, w: int, H: int, W: int, full: bool) -> Tuple[int, int]:
    """Valid crop (H-h+1, W-w+1) as in the reference (binding.cu:230-231,
    :257-263), or the full circular map (H, W)."""
    return (H, W) if full else (H - h + 1, W - w + 1)


def padded_corr2d_f64(templates, spec_T, H: int, W: int, cross_correlate: bool = True,
                      full: bool = False) -> np.ndarray:
    """Float64 restatement of test:110-123 given the transposed image spectrum.

    templates: (B, h, w) or (h, w) real; spec_T: (W/2+1, H) complex (the same
    values the kernel receives).  Returns float64 of shape (B, oy, ox) or
    (oy, ox)."""
    t = np.asarray(templates, dtype=np.float64)
    squeeze = t.ndim == 2
    if squeeze:
        t = t[None]
    B, h, w = t.shape
    S = np.asarray(spec_T).astype(np.complex128).T  # (H, W/2+1)
    assert S.shape == (H, W // 2 + 1), (S.shape, H, W)
    F = np.fft.rfft2(t, s=(H, W), axes=(-2, -1))
    prod = S[None] * (np.conj(F) if cross_correlate else F)
    res = np.fft.irfft2(prod, s=(H, W), axes=(-2, -1))
    oy, ox = out_shape(h, w, H, W, full)
    res = res[:, :oy, :ox]
    return res[0] if squeeze else res


def reference_torch_path(templates, image_fft, H: int, W: int, cross_correlate: bool = True,
                         full: bool = False):
    """The reference test's torch.fft computation (test:110-123), on whatever
    device the tensors live on (CPU for the baseline).  image_fft is the
    untransposed rfftn of the image, (H, W/2+1) complex64."""
    import torch

    filt = templates
    filter_fft = torch.fft.rfftn(filt, s=(H, W), dim=(-2, -1))
    if cross_correlate:
        res_fft = image_fft[None, ...] * torch.conj(filter_fft)
    else:
        res_fft = image_fft[None, ...] * filter_fft
    res = torch.fft.irfftn(res_fft, dim=(-2, -1), norm="backward")
    h, w = filt.shape[-2], filt.shape[-1]
    oy, ox = out_shape(h, w, H, W, full)
    return res[..., :oy, :ox]


# ---------------------------------------------------------------------------
# Brute-force definition (C): out[u,v] = sum_{y<h,x<w} T[y,x] I[(y+u)%H, (x+v)%W]
# for correlation, I[(u-y)%H, (v-x)%W] for convolution.
# ---------------------------------------------------------------------------
_direct_lib: Optional[ctypes.CDLL] = None


def direct_lib_path() -> str:
    return os.path.join(_HERE, "_build", "liboracle_direct.so")


def build_direct(force: bool = False) -> str:
    """Compile oracle/direct_corr.c (gcc) into oracle/_build/."""
    import subprocess

    src = os.path.join(_HERE, "direct_corr.c")
    out = direct_lib_path()
    if force or not os.path.exists(out) or os.path.getmtime(out) < os.path.getmtime(src):
        os.makedirs(os.path.dirname(out), exist_ok=True)
        subprocess.check_call(["gcc", "-O2", "-shared", "-fPIC", "-o", out, src])
    return out


def _direct() -> ctypes.CDLL:
    global _direct_lib
    if _direct_lib is None:
        path = direct_lib_path()
        if not os.path.exists(path):
            path = build_direct()
        lib = ctypes.CDLL(path)
        dp = ctypes.POINTER(ctypes.c_double)
        lib.direct_corr2d.argtypes = [dp, ctypes.c_int, ctypes.c_int, dp, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, dp, ctypes.c_int, ctypes.c_int]
        lib.direct_corr2d.restype = None
        _direct_lib = lib
    return _direct_lib


def direct_corr2d(template, image, cross_correlate: bool = True, full: bool = False) -> np.ndarray:
    """Definition of the circular correlation / convolution by direct summation
    in double precision (independent of any FFT).  template (h, w), image (H, W)."""
    t = np.ascontiguousarray(template, dtype=np.float64)
    im = np.ascontiguousarray(image, dtype=np.float64)
    h, w = t.shape
    H, W = im.shape
    oy, ox = out_shape(h, w, H, W, full)
    out = np.zeros((oy, ox), dtype=np.float64)
    dp = ctypes.POINTER(ctypes.c_double)
    _direct().direct_corr2d(t.ctypes.data_as(dp), h, w, im.ctypes.data_as(dp), H, W,
                            1 if cross_correlate else 0, out.ctypes.data_as(dp), oy, ox)
    return out


# ---------------------------------------------------------------------------
# Error metrics (tolerances of BASELINE north star and the reference test)
# ---------------------------------------------------------------------------
def rel_l2(ref, out) -> float:
    """||ref - out|| / ||ref|| (test:173); complex inputs keep both parts."""
    cplx = np.iscomplexobj(ref) or np.iscomplexobj(out)
    dt = np.complex128 if cplx else np.float64
    ref = np.asarray(ref, dtype=dt)
    out = np.asarray(out, dtype=dt)
    return float(np.linalg.norm(ref - out) / max(np.linalg.norm(ref), 1e-300))


def max_abs_over_peak(ref, out) -> float:
    ref = np.asarray(ref, dtype=np.float64)
    out = np.asarray(out, dtype=np.float64)
    return float(np.max(np.abs(ref - out)) / max(np.max(np.abs(ref)), 1e-300))
