"""The oracle pinned against the definition and the golden fixtures (CPU)."""
import numpy as np
import pytest

from oracle import xcorr_oracle as O


def test_golden_direct_matches_torch_reference_path(golden):
    # The reference test's torch.fft path and the brute-force definition agree.
    for name, c in golden.items():
        assert O.rel_l2(c["direct"], c["torch"]) < 1e-6, name


def test_oracle_matches_golden(golden):
    for name, c in golden.items():
        B, sy, sx, H, W, conj, full = (int(v) for v in c["meta"])
        out = O.padded_corr2d_f64(c["templates"], c["spec_T"], H, W, bool(conj), bool(full))
        assert out.shape == c["torch"].shape, name
        assert O.rel_l2(c["direct"], out) < 1e-6, name
        assert O.rel_l2(c["torch"], out) < 1e-6, name


@pytest.mark.parametrize("conj", [True, False])
@pytest.mark.parametrize("full", [True, False])
def test_oracle_matches_direct_sum(conj, full):
    rng = np.random.default_rng(7)
    img = rng.standard_normal((60, 64))
    t = rng.standard_normal((9, 13))
    spec = np.ascontiguousarray(np.fft.rfft2(img).T)  # exact (complex128) spectrum
    out = O.padded_corr2d_f64(t, spec, 60, 64, conj, full)
    ref = O.direct_corr2d(t, img, conj, full)
    assert np.allclose(out, ref, rtol=1e-10, atol=1e-10)


def test_oracle_known_answer_delta():
    # A unit impulse template at the origin returns the image itself (corr)
    # and a shifted impulse shifts it.
    rng = np.random.default_rng(1)
    img = rng.standard_normal((64, 128))
    spec = np.fft.rfft2(img).T
    t = np.zeros((3, 5))
    t[0, 0] = 1.0
    out = O.padded_corr2d_f64(t, spec, 64, 128, True, True)
    assert np.allclose(out, img, atol=1e-12)
    t2 = np.zeros((3, 5))
    t2[2, 4] = 1.0
    out2 = O.padded_corr2d_f64(t2, spec, 64, 128, True, True)
    assert np.allclose(out2, np.roll(img, shift=(-2, -4), axis=(0, 1)), atol=1e-12)
    conv2 = O.padded_corr2d_f64(t2, spec, 64, 128, False, True)
    assert np.allclose(conv2, np.roll(img, shift=(2, 4), axis=(0, 1)), atol=1e-12)


def test_oracle_valid_crop_is_prefix_of_full():
    rng = np.random.default_rng(3)
    img = rng.standard_normal((64, 64))
    spec = np.fft.rfft2(img).T
    t = rng.standard_normal((2, 10, 7))
    full = O.padded_corr2d_f64(t, spec, 64, 64, True, True)
    valid = O.padded_corr2d_f64(t, spec, 64, 64, True, False)
    assert valid.shape == (2, 55, 58)
    assert np.array_equal(valid, full[:, :55, :58])


def test_torch_cpu_reference_path_matches_f64():
    import torch

    g = torch.Generator().manual_seed(0)
    img = torch.randn((128, 128), generator=g)
    t = torch.randn((2, 32, 32), generator=g)
    image_fft = torch.fft.rfftn(img)
    ref = O.reference_torch_path(t, image_fft, 128, 128, True, True).numpy()
    out = O.padded_corr2d_f64(t.numpy(), image_fft.T.contiguous().numpy(), 128, 128, True, True)
    assert O.rel_l2(out, ref) < 5e-6
