"""zipfft.padded_rconv2d: padded real 2D convolution / cross-correlation.

Drop-in for the reference's pybind11 module of the same name
(mgiammar/zipFFT src/cuda/real_conv_2d_binding.cu:301-308): same functions,
argument order and meaning, the same validation messages (binding.cu:196-263)
raised as RuntimeError, and the same stream/device behaviour (launch on
torch.cuda.current_stream of the input's device, no host synchronisation,
binding.cu:192-194 and :266).

Differences, all supersets of the reference:
  * shapes are run-time values: any signal size up to the FFT size and any
    batch, for the FFT sizes in `supported_fft_sizes()` (the reference only
    accepts the 45 compiled shapes of binding.cu:51-106);
  * `output` may also be the full circular map (..., H, W) instead of the
    valid crop (..., H-h+1, W-w+1);
  * tensors must be contiguous (the reference silently assumed it);
  * CUDA failures raise instead of terminating the process.
The computation runs only in libzipfft_b200.so (CUDA, sm_100a); there is no
CPU path.
"""
from __future__ import annotations

from typing import List, Tuple

import torch

from . import _lib

__all__ = ["corr", "conv", "corr_max", "image_spectrum", "get_supported_conv_configs",
           "supported_fft_sizes", "workspace_bytes"]


# The current stream's handle without building a torch.cuda.Stream object
# (the public call below is the fallback).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _current_stream(device: int) -> int:
    """Handle of torch's current CUDA stream on `device`."""
    if _raw_stream is not None:
        return _raw_stream(device)
    return torch.cuda.current_stream(device).cuda_stream


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _validate(input: torch.Tensor, fft_workspace: torch.Tensor, conv_data: torch.Tensor,
              output: torch.Tensor, fft_size_y: int, fft_size_x: int, *,
              output_is_shape_stand_in: bool = False):
    """Checks of real_conv_2d_binding.cu:196-263, same order and messages.

    output_is_shape_stand_in: `output` is an expanded view that only carries
    the per-template map shape (corr_max, whose kernels write the running maps
    instead); its contiguity is not checked.  Every caller whose `output`
    receives the maps leaves this False, so an expanded or overlapping output
    (stride 0 over the batch) is rejected before anything launches."""
    # Each tensor's attributes are read once (a torch attribute read costs
    # a few hundred ns of host time; the small-image calls take ~25 us).
    idev, wdev, cdev, odev = input.device, fft_workspace.device, conv_data.device, output.device
    _check(idev.type == "cuda", "Input tensor must be on CUDA device")
    _check(wdev.type == "cuda", "FFT workspace tensor must be on CUDA device")
    _check(cdev.type == "cuda", "Convolution data tensor must be on CUDA device")
    _check(odev.type == "cuda", "Output tensor must be on CUDA device")
    _check(wdev == idev, "FFT workspace tensor must be on the same device as the input tensor")
    _check(cdev == idev, "Convolution data tensor must be on the same device as the input tensor")
    _check(odev == idev, "Output tensor must be on the same device as the input tensor")
    _check(input.dtype == torch.float32, "Input tensor must be of type torch.float32")
    _check(fft_workspace.dtype == torch.complex64,
           "FFT workspace tensor must be of type torch.complex64 (float2)")
    _check(conv_data.dtype == torch.complex64,
           "Convolution data tensor must be of type torch.complex64 (float2)")
    _check(output.dtype == torch.float32, "Output tensor must be of type torch.float32")

    ishape, wshape, cshape, oshape = input.shape, fft_workspace.shape, conv_data.shape, output.shape
    ndim = len(ishape)
    if ndim == 2:
        batch, sy, sx = 1, ishape[0], ishape[1]
    elif ndim == 3:
        batch, sy, sx = ishape
    else:
        raise RuntimeError(f"Input tensor must be 2D or 3D. Got {ndim}D.")

    stride = fft_size_x // 2 + 1
    _check(len(wshape) == ndim,
           "FFT workspace tensor must have the same number of dimensions as the input tensor")
    _check(wshape[-1] == stride, "FFT workspace tensor last dimension must be fft_size_x/2 + 1")
    _check(wshape[-2] == fft_size_y,
           "FFT workspace tensor second-to-last dimension must be fft_size_y")
    if batch > 1:
        _check(wshape[0] == batch,
               "FFT workspace tensor first dimension (batch) must match input batch size")

    # The two messages below are the reference's text verbatim (binding.cu:252-255).
    _check(len(cshape) == 2, f"Convolution data tensor must be 2D. Got {len(cshape)}D.")
    _check(cshape[0] == stride, "Convolution data tensor first dimension must match fft_size_y")
    _check(cshape[1] == fft_size_y,
           "Convolution data tensor second dimension must be fft_size_x/2 + 1")

    vx, vy = fft_size_x - sx + 1, fft_size_y - sy + 1
    _check(len(oshape) == ndim,
           "Output tensor must have the same number of dimensions as the input tensor")
    oy, ox = oshape[-2], oshape[-1]
    full = ox == fft_size_x and oy == fft_size_y
    if not full:
        _check(ox == vx, "Output tensor last dimension must be fft_size_x - signal_length_x + 1")
        _check(oy == vy,
               "Output tensor second-to-last dimension must be fft_size_y - signal_length_y + 1")
    if len(oshape) == 3:
        _check(oshape[0] == batch, "Output tensor first dimension (batch) must match input "
                                   "batch size")
    _check(input.is_contiguous(), "Input tensor must be contiguous")
    _check(fft_workspace.is_contiguous(), "FFT workspace tensor must be contiguous")
    _check(conv_data.is_contiguous(), "Convolution data tensor must be contiguous")
    _check(output_is_shape_stand_in or output.is_contiguous(), "Output tensor must be contiguous")
    return batch, sy, sx, oy, ox


def _run(fn_name: str, input, fft_workspace, conv_data, output, fft_size_y: int,
         fft_size_x: int) -> None:
    batch, sy, sx, oy, ox = _validate(input, fft_workspace, conv_data, output, int(fft_size_y),
                                      int(fft_size_x))
    lib = _lib.load()
    device = input.device.index if input.device.index is not None else torch.cuda.current_device()
    stream = _current_stream(device)
    ws_bytes = fft_workspace.numel() * fft_workspace.element_size()
    status = getattr(lib, fn_name)(input.data_ptr(), batch, sy, sx, fft_workspace.data_ptr(),
                                   ws_bytes, conv_data.data_ptr(), output.data_ptr(), oy, ox,
                                   int(fft_size_y), int(fft_size_x), device, stream)
    _lib.check(status)


def corr(input: torch.Tensor, fft_workspace: torch.Tensor, conv_data: torch.Tensor,
         output: torch.Tensor, fft_size_y: int, fft_size_x: int, *,
         peaks: torch.Tensor = None) -> None:
    """2D padded real cross-correlation (binding.cu:295-299, :304).

    input (h, w) or (B, h, w) float32; fft_workspace complex64 (H, W/2+1) or
    (B, H, W/2+1), clobbered; conv_data complex64 (W/2+1, H) = rfftn(image).T;
    output float32 (..., H-h+1, W-w+1) or (..., H, W), written in place.

    peaks (keyword only, not in the reference): a float32 tensor of B values
    (one per template; 1 value for a 2D input) that receives each output
    map's largest value, computed by the kernel that writes the map."""
    if peaks is None:
        _run("zfft_padded_real_corr_2d", input, fft_workspace, conv_data, output, fft_size_y,
             fft_size_x)
        return
    batch, sy, sx, oy, ox = _validate(input, fft_workspace, conv_data, output, int(fft_size_y),
                                      int(fft_size_x))
    _check(peaks.dtype == torch.float32, "Peaks tensor must be of type torch.float32")
    _check(peaks.device == input.device, "Peaks tensor must be on the same device as the input")
    _check(peaks.numel() == batch and peaks.is_contiguous(),
           f"Peaks tensor must be contiguous with {batch} elements (one per template)")
    lib = _lib.load()
    device = input.device.index if input.device.index is not None else torch.cuda.current_device()
    stream = _current_stream(device)
    ws_bytes = fft_workspace.numel() * fft_workspace.element_size()
    status = lib.zfft_padded_real_corr_2d_peaks(input.data_ptr(), batch, sy, sx,
                                                fft_workspace.data_ptr(), ws_bytes,
                                                conv_data.data_ptr(), output.data_ptr(), oy, ox,
                                                int(fft_size_y), int(fft_size_x),
                                                peaks.data_ptr(), device, stream)
    _lib.check(status)


def conv(input: torch.Tensor, fft_workspace: torch.Tensor, conv_data: torch.Tensor,
         output: torch.Tensor, fft_size_y: int, fft_size_x: int) -> None:
    """2D padded real convolution (binding.cu:288-292, :303); arguments as corr."""
    _run("zfft_padded_real_conv_2d", input, fft_workspace, conv_data, output, fft_size_y,
         fft_size_x)


def corr_max(input: torch.Tensor, fft_workspace: torch.Tensor, conv_data: torch.Tensor,
             max_map: torch.Tensor, arg_map: torch.Tensor, fft_size_y: int, fft_size_x: int,
             template_index_base: int = 0, reset: bool = False,
             sum_map: torch.Tensor = None, sumsq_map: torch.Tensor = None) -> None:
    """Cross-correlate every template like `corr`, folding the results into
    running per-pixel maps instead of writing one map per template.

    max_map (float32) keeps the largest correlation per pixel, arg_map (int32)
    the index of the template that produced it; template t of `input` has
    index template_index_base + t and ties keep the lower index.  Both maps
    are (H-h+1, W-w+1) or (H, W).  reset=True: this call's first template
    overwrites the maps (no initialisation needed).  With sum_map and
    sumsq_map (float32, same shape) every correlation and its square are also
    added to them per pixel (reset overwrites them too): the statistics 2D
    template matching normalises its scores with.  No counterpart in the
    reference; the 2D template-matching search its README motivates."""
    _check(max_map.dtype == torch.float32, "Max map tensor must be of type torch.float32")
    _check(arg_map.dtype == torch.int32, "Argmax map tensor must be of type torch.int32")
    _check(max_map.dim() == 2 and arg_map.shape == max_map.shape,
           "Max and argmax maps must be 2D tensors of the same shape")
    _check(max_map.device == input.device and arg_map.device == input.device,
           "Max and argmax maps must be on the same device as the input tensor")
    _check(max_map.is_contiguous() and arg_map.is_contiguous(), "Maps must be contiguous")
    stats = sum_map is not None or sumsq_map is not None
    if stats:
        _check(sum_map is not None and sumsq_map is not None,
               "Sum and sum-of-squares maps must be given together")
        for name, m in (("Sum", sum_map), ("Sum-of-squares", sumsq_map)):
            _check(m.dtype == torch.float32, f"{name} map tensor must be of type torch.float32")
            _check(m.shape == max_map.shape, f"{name} map must have the max map's shape")
            _check(m.device == input.device,
                   f"{name} map must be on the same device as the input tensor")
            _check(m.is_contiguous(), "Maps must be contiguous")
    lead = (input.size(0),) if input.dim() == 3 else ()
    # Validate everything else exactly as corr does, with a shape stand-in for
    # the per-template output.
    batch, sy, sx, oy, ox = _validate(input, fft_workspace, conv_data,
                                      max_map.expand(*lead, *max_map.shape), int(fft_size_y),
                                      int(fft_size_x), output_is_shape_stand_in=True)
    lib = _lib.load()
    device = input.device.index if input.device.index is not None else torch.cuda.current_device()
    stream = _current_stream(device)
    ws_bytes = fft_workspace.numel() * fft_workspace.element_size()
    if stats:
        status = lib.zfft_padded_real_corr_2d_max_stats(
            input.data_ptr(), batch, sy, sx, fft_workspace.data_ptr(), ws_bytes,
            conv_data.data_ptr(), max_map.data_ptr(), arg_map.data_ptr(), sum_map.data_ptr(),
            sumsq_map.data_ptr(), oy, ox, int(fft_size_y), int(fft_size_x),
            int(template_index_base), 1 if reset else 0, device, stream)
    else:
        status = lib.zfft_padded_real_corr_2d_max(input.data_ptr(), batch, sy, sx,
                                                  fft_workspace.data_ptr(), ws_bytes,
                                                  conv_data.data_ptr(), max_map.data_ptr(),
                                                  arg_map.data_ptr(), oy, ox, int(fft_size_y),
                                                  int(fft_size_x), int(template_index_base),
                                                  1 if reset else 0, device, stream)
    _lib.check(status)


def image_spectrum(image: torch.Tensor, conv_data: torch.Tensor = None) -> torch.Tensor:
    """The image spectrum that corr / conv take as conv_data:
    rfftn(image).transpose(-2, -1), complex64 (W/2+1, H), computed on the GPU
    by the library's own row and column kernels.  The reference leaves this to
    the caller (README.md:224-228, tests/test_real_conv_2d.py:89-90).

    image: float32 (H, W) contiguous CUDA tensor, H and W supported FFT sizes.
    conv_data: optional complex64 (W/2+1, H) contiguous output on the same
    device; allocated when omitted.  Returns conv_data."""
    _check(image.is_cuda, "Image tensor must be on a CUDA device")
    _check(image.dtype == torch.float32, "Image tensor must be of type torch.float32")
    _check(image.dim() == 2, "Image tensor must be 2D (H, W)")
    _check(image.is_contiguous(), "Image tensor must be contiguous")
    H, W = image.shape
    if conv_data is None:
        conv_data = torch.empty(W // 2 + 1, H, dtype=torch.complex64, device=image.device)
    _check(conv_data.dtype == torch.complex64,
           "Convolution data tensor must be of type torch.complex64")
    _check(conv_data.device == image.device,
           "Convolution data tensor must be on the same device as the image tensor")
    _check(tuple(conv_data.shape) == (W // 2 + 1, H),
           f"Convolution data tensor must have shape ({W // 2 + 1}, {H}). "
           f"Got {tuple(conv_data.shape)}.")
    _check(conv_data.is_contiguous(), "Convolution data tensor must be contiguous")
    lib = _lib.load()
    device = image.device.index if image.device.index is not None else torch.cuda.current_device()
    stream = _current_stream(device)
    status = lib.zfft_image_spectrum(image.data_ptr(), H, W, conv_data.data_ptr(),
                                     conv_data.numel() * conv_data.element_size(), device, stream)
    _lib.check(status)
    return conv_data


def get_supported_conv_configs() -> List[Tuple[int, int, int, int, int, bool]]:
    """(signal_y, signal_x, fft_y, fft_x, batch, cross_correlate) tuples
    (binding.cu:160-170): the reference's 45 shapes plus the 2DTM workloads.
    Any other shape with supported FFT sizes runs as well."""
    import ctypes

    lib = _lib.load()
    n = lib.zfft_get_supported_conv_configs(None, 0)
    buf = (ctypes.c_int * (6 * n))()
    lib.zfft_get_supported_conv_configs(buf, n)
    return [(buf[6 * i], buf[6 * i + 1], buf[6 * i + 2], buf[6 * i + 3], buf[6 * i + 4],
             bool(buf[6 * i + 5])) for i in range(n)]


def supported_fft_sizes() -> List[int]:
    """FFT sizes (for both H and W) compiled into the library."""
    lib = _lib.load()
    return [n for n in range(16, 8193) if lib.zfft_is_fft_size_supported(n)]


def workspace_bytes(fft_size_y: int, fft_size_x: int) -> int:
    """Workspace bytes the kernels use (one H x W/2 complex64 slice)."""
    return int(_lib.load().zfft_workspace_bytes(int(fft_size_y), int(fft_size_x)))
