"""The image-spectrum path (zfft_image_spectrum / padded_rconv2d.image_spectrum):
the conv_data the operator takes, rfftn(image).transpose(-2, -1), computed by
the library's row and in-place column kernels.  The reference leaves this step
to its callers (README.md:224-228, tests/test_real_conv_2d.py:89-90), so the
oracle is the float64 rfft2 of the same float32 image; tolerances are the
reference test's rel L2 < 5e-6 and max |err| < 1e-5 x peak."""
import numpy as np
import pytest
import torch

from oracle import xcorr_oracle as O
from tests.gpu_helpers import assert_parity, capi_corr
from zipfft_b200 import _lib
from zipfft_b200 import padded_rconv2d as P

pytestmark = pytest.mark.gpu

SIZES = [(64, 64), (128, 256), (256, 128), (512, 512), (1024, 1024), (2048, 4096),
         (4096, 4096), (120, 240), (1920, 960), (3840, 3840)]


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    assert _lib.check_device_status(0) == 0


def _image(H, W, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((H, W), generator=g, dtype=torch.float32)


@pytest.mark.parametrize("H,W", SIZES, ids=[f"{h}x{w}" for h, w in SIZES])
def test_spectrum_matches_oracle(H, W):
    img = _image(H, W, H * 7 + W)
    # NaN-filled output: every element must be written.
    out = torch.full((W // 2 + 1, H), float("nan"), dtype=torch.complex64, device="cuda")
    ret = P.image_spectrum(img.cuda(), out)
    assert ret is out
    got = out.cpu().numpy()
    ref = O.image_spectrum_T(img.numpy(), dtype=np.complex128)
    assert np.all(np.isfinite(got.view(np.float32)))
    assert O.rel_l2(ref, got) < 5e-6
    assert np.abs(got - ref).max() < 1e-5 * np.abs(ref).max()


def test_spectrum_agrees_with_cufft():
    img = _image(4096, 4096, 1).cuda()
    ours = P.image_spectrum(img)
    theirs = torch.fft.rfftn(img).transpose(-2, -1).contiguous()
    assert ours.shape == theirs.shape and ours.dtype == theirs.dtype
    rel = (torch.linalg.vector_norm(ours - theirs) / torch.linalg.vector_norm(theirs)).item()
    assert rel < 5e-6


def test_spectrum_on_side_stream_and_repeat():
    img = _image(1024, 2048, 2).cuda()
    ref = P.image_spectrum(img).clone()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        again = P.image_spectrum(img)
    s.synchronize()
    assert torch.equal(ref, again)  # deterministic, stream honoured


def test_correlation_from_own_spectrum():
    """The search pipeline end to end on the GPU: spectrum by the library,
    then correlations, against the oracle correlation of the same inputs."""
    H = W = 4096
    img = _image(H, W, 3)
    g = torch.Generator().manual_seed(4)
    tm = torch.randn((2, 256, 256), generator=g, dtype=torch.float32)
    spec = P.image_spectrum(img.cuda()).cpu()
    out = capi_corr(tm, spec, H, W, full=True)
    ref = O.padded_corr2d_f64(tm.numpy(), O.image_spectrum_T(img.numpy()), H, W, True, True)
    assert_parity(ref, out, what="corr from the library's spectrum")


def test_spectrum_argument_errors():
    img = _image(128, 256, 5).cuda()
    with pytest.raises(RuntimeError, match="must have shape"):
        P.image_spectrum(img, torch.empty(128, 129, dtype=torch.complex64, device="cuda"))
    with pytest.raises(RuntimeError, match="complex64"):
        P.image_spectrum(img, torch.empty(129, 128, dtype=torch.float32, device="cuda"))
    with pytest.raises(RuntimeError, match="2D"):
        P.image_spectrum(img[None])
    with pytest.raises(RuntimeError, match="Unsupported image size"):
        P.image_spectrum(torch.zeros(100, 128, device="cuda"))
