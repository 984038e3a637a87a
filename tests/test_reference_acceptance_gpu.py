"""The reference's own test, run against this library through the same API.

Mirrors mgiammar/zipFFT tests/test_real_conv_2d.py: every configuration of
get_supported_conv_configs() (the reference's 45 plus the 2DTM shapes),
random inputs, the torch.fft path on the same GPU as the expected value, the
reference's tolerances (test:39-40, :168-174), the non-default stream test
(test:253-279) and the non-zero device test (test:282-309).
"""
import pytest
import torch

import zipfft

pytestmark = pytest.mark.gpu

TYPE_MAP = {"float32": torch.float32, "complex64": torch.complex64}
FFT_NORMALIZATION_DIRECTION = "backward"

if torch.cuda.is_available() and zipfft.is_extension_available("padded_rconv2d"):
    ALL_CONFIGS = zipfft.padded_rconv2d.get_supported_conv_configs()
else:
    ALL_CONFIGS = []
CONV_CONFIGS = [c[:5] for c in ALL_CONFIGS if c[5] is False]
CROSS_CORR_CONFIGS = [c[:5] for c in ALL_CONFIGS if c[5] is True]

RTOL = 3e1
ATOL = 5e-6


def repeats(fy, fx, batch):
    # The reference repeats each case 10 times (test:38); the large 2DTM
    # shapes run fewer repeats to keep the suite within minutes.
    work = batch * fy * fx
    return 10 if work <= (1 << 26) else (2 if work <= (1 << 30) else 1)


def run_conv_or_corr_2d_test(signal_length_y, signal_length_x, fft_size_y, fft_size_x,
                             batch_size, cross_correlate, dtype=torch.float32, rtol=RTOL,
                             atol=ATOL, device="cuda:0", seed=0):
    # Inputs are seeded here; the reference draws them unseeded.  Its small-size
    # check (allclose with rtol applied to |output|) fails whenever an output
    # lands within ~1e-6 of zero while two fp32 FFTs differ there by their
    # normal ~1e-7 relative rounding, so an unseeded run flakes at random.
    torch.manual_seed(seed)
    filter_shape = (signal_length_y, signal_length_x)
    image_shape = (fft_size_y, fft_size_x)
    output_shape = (fft_size_y - signal_length_y + 1, fft_size_x - signal_length_x + 1)
    if batch_size > 1:
        filter_shape = (batch_size,) + filter_shape
        output_shape = (batch_size,) + output_shape
    stride_y = fft_size_x // 2 + 1
    input_image = torch.randn(image_shape, dtype=dtype, device=device)
    input_image_fft = torch.fft.rfftn(input_image).contiguous()
    input_filter = torch.randn(filter_shape, dtype=dtype, device=device)
    if batch_size > 1:
        workspace_shape = (batch_size, fft_size_y, stride_y)
    else:
        workspace_shape = (fft_size_y, stride_y)
    fft_workspace = torch.empty(workspace_shape, dtype=torch.complex64, device=device)
    output = torch.empty(output_shape, dtype=dtype, device=device)

    filter_fft = torch.fft.rfftn(input_filter, s=(fft_size_y, fft_size_x), dim=(-2, -1))
    if cross_correlate:
        torch_result_fft = input_image_fft[None, ...] * torch.conj(filter_fft)
    else:
        torch_result_fft = input_image_fft[None, ...] * filter_fft
    torch_result = torch.fft.irfftn(torch_result_fft, dim=(-2, -1),
                                    norm=FFT_NORMALIZATION_DIRECTION)
    torch_result = torch_result[..., : output_shape[-2], : output_shape[-1]]
    del torch_result_fft, filter_fft
    input_image_fft = input_image_fft.transpose(-2, -1).contiguous()

    if cross_correlate:
        zipfft.padded_rconv2d.corr(input_filter, fft_workspace, input_image_fft, output,
                                   fft_size_y, fft_size_x)
    else:
        zipfft.padded_rconv2d.conv(input_filter, fft_workspace, input_image_fft, output,
                                   fft_size_y, fft_size_x)
    torch.cuda.synchronize()

    max_abs_diff = torch.max(torch.abs(torch_result - output))
    op_name = "cross-correlation" if cross_correlate else "convolution"
    error_msg = (f"Real 2D {op_name} results do not match ground truth. "
                 f"Max abs diff: {max_abs_diff}.")
    if max(fft_size_y, fft_size_x) < 512:
        assert torch.allclose(torch_result, output, rtol=rtol, atol=atol), error_msg
    else:
        l2_norm = torch.norm(torch_result - output) / torch.norm(torch_result)
        assert l2_norm < atol, error_msg + f" L2 norm: {l2_norm}"


@pytest.mark.parametrize("signal_length_y,signal_length_x,fft_size_y,fft_size_x,batch_size",
                         CONV_CONFIGS)
def test_convolution_2d(signal_length_y, signal_length_x, fft_size_y, fft_size_x, batch_size):
    for rep in range(repeats(fft_size_y, fft_size_x, batch_size)):
        run_conv_or_corr_2d_test(signal_length_y, signal_length_x, fft_size_y, fft_size_x,
                                 batch_size, cross_correlate=False, seed=rep)


@pytest.mark.parametrize("signal_length_y,signal_length_x,fft_size_y,fft_size_x,batch_size",
                         CROSS_CORR_CONFIGS)
def test_cross_correlation_2d(signal_length_y, signal_length_x, fft_size_y, fft_size_x,
                              batch_size):
    for rep in range(repeats(fft_size_y, fft_size_x, batch_size)):
        run_conv_or_corr_2d_test(signal_length_y, signal_length_x, fft_size_y, fft_size_x,
                                 batch_size, cross_correlate=True, seed=rep)


def test_non_standard_stream():
    stream = torch.cuda.Stream()
    sy, sx, fy, fx, b = CONV_CONFIGS[0]
    for rep in range(10):
        with torch.cuda.stream(stream):
            run_conv_or_corr_2d_test(sy, sx, fy, fx, b, cross_correlate=False, seed=rep)
    stream.synchronize()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="Less than 2 CUDA devices available")
def test_non_standard_device():
    sy, sx, fy, fx, b = CROSS_CORR_CONFIGS[0]
    for rep in range(10):
        run_conv_or_corr_2d_test(sy, sx, fy, fx, b, cross_correlate=True, device="cuda:1",
                                 seed=rep)
