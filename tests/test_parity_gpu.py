"""Parity of the CUDA path with the CPU oracle, through the C ABI.

Seeded inputs, the oracle (oracle/xcorr_oracle.py, float64) on the same
complex64 image spectrum the kernels receive, and the tolerances of the
reference test (rel L2 < 5e-6, test:173-174) and the 2DTM requirement
(max |err| < 1e-4 x peak).  Full-size 2DTM workloads are checked on sampled
templates against the oracle and on all templates through size-independent
properties (linearity in the template, a planted template's correlation peak).
"""
import numpy as np
import pytest
import torch

from oracle import xcorr_oracle as O
from tests.gpu_helpers import assert_parity, capi_corr, make_inputs

pytestmark = pytest.mark.gpu


def test_golden_fixtures_through_capi(golden):
    for name, c in golden.items():
        B, sy, sx, H, W, conj, full = (int(v) for v in c["meta"])
        out = capi_corr(torch.from_numpy(c["templates"]), torch.from_numpy(c["spec_T"]), H, W,
                        bool(full), bool(conj))
        assert_parity(c["torch"], out, what=name + " vs reference torch path")
        assert_parity(c["direct"], out, what=name + " vs direct sum")


SMALL = [
    # B, sy, sx, H, W, conj, full
    (3, 16, 16, 64, 64, True, True),
    (2, 48, 48, 64, 64, False, False),
    (1, 64, 64, 64, 64, True, True),        # no padding at all
    (2, 1, 1, 128, 128, True, True),        # single-pixel template
    (2, 7, 13, 128, 256, True, False),      # odd template sizes
    (2, 31, 9, 256, 512, False, True),
    (1, 200, 100, 512, 256, True, False),
    (2, 100, 100, 1024, 1024, True, True),
    (2, 127, 255, 2048, 1024, True, False),
    (1, 3, 5, 120, 240, True, True),        # radix-3/5 sizes
    (2, 60, 90, 480, 960, False, True),
    (1, 500, 300, 1920, 3840, True, False),
    (1, 256, 128, 4096, 2048, True, True),  # pruned start, nz = 1
    (1, 384, 384, 4096, 4096, True, True),  # pruned start, nz = 2
    (1, 700, 600, 4096, 4096, False, False),  # full start
]


@pytest.mark.parametrize("case", SMALL, ids=[str(c) for c in SMALL])
def test_seeded_parity(case):
    B, sy, sx, H, W, conj, full = case
    _, tm, spec = make_inputs(B, sy, sx, H, W, seed=sum(case[:5]))
    out = capi_corr(tm, spec, H, W, full, conj)
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, conj, full)
    assert_parity(ref, out, what=str(case))


def test_config1_1024_full_maps():
    """1024^2 image, 4 templates 128^2 N(0,1) zero-mean unit-variance, full maps."""
    g = torch.Generator().manual_seed(0)
    img = torch.randn((1024, 1024), generator=g)
    tm = torch.randn((4, 128, 128), generator=g)
    tm = (tm - tm.mean(dim=(1, 2), keepdim=True)) / tm.std(dim=(1, 2), keepdim=True)
    spec = torch.from_numpy(O.image_spectrum_T(img.numpy()))
    out = capi_corr(tm, spec, 1024, 1024, True)
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), 1024, 1024, True, True)
    assert_parity(ref, out, what="1024^2 x 4 x 128^2")


@pytest.mark.parametrize("H,h,B,check", [(4096, 256, 32, (0, 17, 31)), (4096, 512, 8, (0, 7)),
                                         (3840, 384, 8, (0, 5))])
def test_2dtm_sizes_sampled_templates(H, h, B, check):
    _, tm, spec = make_inputs(B, h, h, H, H, seed=H + h)
    out = capi_corr(tm, spec, H, H, True)
    for b in check:
        ref = O.padded_corr2d_f64(tm[b].numpy(), spec.numpy(), H, H, True, True)
        assert_parity(ref, out[b], what=f"{H}^2 / {h}^2 template {b}")


@pytest.mark.parametrize("which", ["soft_mask_256", "gaussian_blob_512"])
def test_baseline_template_content(which):
    """The measured workloads' own template content, not plain N(0,1): 256^2
    templates times the soft circular mask (radius 112 px + 8 px raised
    cosine), and 512^2 Gaussian blobs (sigma 20 px) plus N(0, 0.1) noise,
    each zero-mean unit-variance, in a 4096^2 image; sampled templates
    against the oracle."""
    from bench import gaussian_blob_templates, make_templates

    H = 4096
    if which == "soft_mask_256":
        tm, check = make_templates(8, 1), (0, 5, 7)
    else:
        tm, check = gaussian_blob_templates(4, 512, 20.0, 0.1, 1), (0, 3)
    g = torch.Generator().manual_seed(0)
    spec = torch.from_numpy(O.image_spectrum_T(torch.randn((H, H), generator=g).numpy()))
    out = capi_corr(tm, spec, H, H, True)
    for b in check:
        ref = O.padded_corr2d_f64(tm[b].numpy(), spec.numpy(), H, H, True, True)
        assert_parity(ref, out[b], what=f"{which} template {b}")


def test_linearity_full_size():
    """corr(a T1 + b T2) = a corr(T1) + b corr(T2) at 4096^2 / 256^2."""
    H = 4096
    _, tm, spec = make_inputs(2, 256, 256, H, H, seed=11)
    a, b = 0.75, -1.25
    mix = (a * tm[0] + b * tm[1])[None]
    both = capi_corr(torch.cat([tm, mix]), spec, H, H, True)
    lhs = both[2].astype(np.float64)
    rhs = a * both[0].astype(np.float64) + b * both[1].astype(np.float64)
    assert O.rel_l2(lhs, rhs) < 5e-6


def test_planted_template_peak_full_size():
    """A template added to the image at known offsets gives correlation peaks
    exactly there (the known answer of 2D template matching)."""
    H = 4096
    rng = np.random.default_rng(5)
    img = rng.standard_normal((H, H)).astype(np.float32)
    t = rng.standard_normal((256, 256)).astype(np.float32)
    pos = [(100, 200), (3000, 1500), (4000 - 256, 17)]
    for (y, x) in pos:
        img[y:y + 256, x:x + 256] += 2.0 * t
    spec = torch.from_numpy(O.image_spectrum_T(img))
    out = capi_corr(torch.from_numpy(t)[None], spec, H, H, True)[0]
    flat = np.argsort(out.ravel())[::-1][:3]
    found = sorted((int(i // H), int(i % H)) for i in flat)
    assert found == sorted(pos)


def test_workspace_only_needs_one_slice_and_output_untouched_beyond():
    """The kernels stay inside H * W/2 complex of workspace and the output
    tensor; guard regions around both remain intact."""
    H = W = 1024
    _, tm, spec = make_inputs(3, 64, 64, H, W, seed=3)
    dev = torch.device("cuda", 0)
    nws = H * (W // 2)
    guard = 4096
    ws_all = torch.full((nws + 2 * guard,), complex(7.0, -7.0), dtype=torch.complex64, device=dev)
    ws = ws_all[guard:guard + nws]
    out = capi_corr(tm, spec, H, W, False, ws=ws)
    torch.cuda.synchronize()
    assert torch.all(ws_all[:guard] == complex(7.0, -7.0))
    assert torch.all(ws_all[guard + nws:] == complex(7.0, -7.0))
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, True, False)
    assert_parity(ref, out, what="guarded workspace")


def test_convolution_matches_oracle_large():
    _, tm, spec = make_inputs(2, 256, 256, 4096, 4096, seed=21)
    out = capi_corr(tm, spec, 4096, 4096, True, conj=False)
    ref = O.padded_corr2d_f64(tm[1].numpy(), spec.numpy(), 4096, 4096, False, True)
    assert_parity(ref, out[1], what="conv 4096^2 / 256^2")


def test_results_independent_of_stream_and_repeatable():
    _, tm, spec = make_inputs(4, 96, 96, 512, 512, seed=9)
    s = torch.cuda.Stream()
    a = capi_corr(tm, spec, 512, 512, True)
    with torch.cuda.stream(s):
        b = capi_corr(tm, spec, 512, 512, True, stream=s.cuda_stream)
    assert np.array_equal(a, b)  # deterministic: no atomics, fixed schedule


def test_invalid_device_index_reports_error():
    from zipfft_b200 import _lib

    lib = _lib.load()
    n = torch.cuda.device_count()
    # Correctly sized buffers: even if validation let the call through, every
    # access would stay in bounds.
    x = torch.zeros(16, 16, device="cuda")
    ws = torch.zeros(64 * 33, dtype=torch.complex64, device="cuda")
    cd = torch.zeros(33, 64, dtype=torch.complex64, device="cuda")
    out = torch.zeros(64, 64, device="cuda")
    st = lib.zfft_padded_real_corr_2d(x.data_ptr(), 1, 16, 16, ws.data_ptr(), ws.numel() * 8,
                                      cd.data_ptr(), out.data_ptr(), 64, 64, 64, 64, n + 3, None)
    assert st == _lib.ZFFT_ERROR_INVALID_VALUE
    assert "invalid device index" in _lib.last_error()


@pytest.fixture(autouse=True)
def _device_status_clean():
    """No kernel may have given up on a bounded wait during any test."""
    from zipfft_b200 import _lib

    yield
    assert _lib.check_device_status(0) == 0


def test_bounded_wait_reports_timeout_and_context_survives():
    """A wait that can never complete gives up (~1 ms limit) and reports
    ZFFT_ERROR_TIMEOUT; the CUDA context stays usable afterwards."""
    from zipfft_b200 import _lib

    lib = _lib.load()
    assert _lib.check_device_status(0) == 0
    _lib.check(lib.zfft_selftest_wait_timeout(0, None))
    assert _lib.check_device_status(0) == _lib.ZFFT_ERROR_TIMEOUT
    assert _lib.check_device_status(0) == 0  # cleared by the read
    _, tm, spec = make_inputs(2, 16, 16, 64, 64, seed=1)
    out = capi_corr(tm, spec, 64, 64, True)
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), 64, 64, True, True)
    assert_parity(ref, out, what="after timeout self-test")


@pytest.mark.parametrize("H,h,B", [(4096, 256, 5), (1024, 100, 7), (3840, 384, 3)])
def test_chunked_and_in_place_layouts_agree(H, h, B):
    """A workspace of several whole intermediates (batched groups: one launch
    per kernel for up to 32 templates) gives bit-identical results to the
    minimal in-place workspace (one template per column and inverse-row
    launch)."""
    from zipfft_b200 import _lib

    _, tm, spec = make_inputs(B, h, h, H, H, seed=H + B)
    dev = torch.device("cuda", 0)
    nmin = _lib.load().zfft_workspace_bytes(H, H) // 8
    small = torch.empty(nmin, dtype=torch.complex64, device=dev)
    big = torch.empty(B * H * (H // 2 + 1), dtype=torch.complex64, device=dev)
    a = capi_corr(tm, spec, H, H, True, ws=small)
    b = capi_corr(tm, spec, H, H, True, ws=big)
    assert np.array_equal(a, b)
    ref = O.padded_corr2d_f64(tm[B - 1].numpy(), spec.numpy(), H, H, True, True)
    assert_parity(ref, a[B - 1], what="chunked layout, last template")


@pytest.mark.parametrize("B,sy,sx,H,W,full", [(5, 256, 256, 4096, 4096, True),
                                              (3, 31, 17, 512, 256, False),
                                              (1, 100, 90, 1920, 3840, False)])
def test_corr_peaks_equal_map_maxima(B, sy, sx, H, W, full):
    """corr(..., peaks=): each template's largest output value, folded in by
    the kernel that writes the map, equals the maximum of the stored map bit
    for bit; the maps are the same as without peaks."""
    import zipfft

    _, tm, spec = make_inputs(B, sy, sx, H, W, seed=B + sy + H)
    dev = torch.device("cuda", 0)
    oy, ox = O.out_shape(sy, sx, H, W, full)
    ws = torch.empty((B, H, W // 2 + 1), dtype=torch.complex64, device=dev)
    tm_d, sp_d = tm.to(dev), spec.to(dev)
    out = torch.full((B, oy, ox), float("nan"), device=dev)
    peaks = torch.full((B,), float("nan"), device=dev)
    zipfft.padded_rconv2d.corr(tm_d, ws, sp_d, out, H, W, peaks=peaks)
    ref_out = torch.empty_like(out)
    zipfft.padded_rconv2d.corr(tm_d, ws, sp_d, ref_out, H, W)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    assert torch.equal(peaks, out.reshape(B, -1).amax(dim=1))
    if B == 1:  # 2D input, one peak
        p1 = torch.empty(1, device=dev)
        zipfft.padded_rconv2d.corr(tm_d[0], ws[0], sp_d, out[0], H, W, peaks=p1)
        torch.cuda.synchronize()
        assert torch.equal(p1, peaks)


def test_corr_peaks_propagate_nan_like_amax():
    """A template holding a NaN makes its whole map NaN (every output mixes
    every input); its peak is NaN, as torch.amax of that map is, and the
    other templates' peaks are unaffected."""
    import zipfft

    B, sy, sx, H, W = 3, 16, 16, 256, 256
    _, tm, spec = make_inputs(B, sy, sx, H, W, seed=21)
    tm[1, 3, 5] = float("nan")
    dev = torch.device("cuda", 0)
    ws = torch.empty((B, H, W // 2 + 1), dtype=torch.complex64, device=dev)
    out = torch.empty((B, H, W), device=dev)
    peaks = torch.zeros((B,), device=dev)
    zipfft.padded_rconv2d.corr(tm.to(dev), ws, spec.to(dev), out, H, W, peaks=peaks)
    torch.cuda.synchronize()
    amax = out.reshape(B, -1).amax(dim=1)
    assert torch.isnan(out[1]).all() and torch.isnan(amax[1]) and torch.isnan(peaks[1])
    assert torch.equal(peaks[[0, 2]], amax[[0, 2]])


def test_corr_peaks_argument_errors():
    import zipfft

    _, tm, spec = make_inputs(2, 16, 16, 64, 64, seed=1)
    dev = torch.device("cuda", 0)
    ws = torch.empty((2, 64, 33), dtype=torch.complex64, device=dev)
    out = torch.empty((2, 64, 64), device=dev)
    with pytest.raises(RuntimeError, match="one per template"):
        zipfft.padded_rconv2d.corr(tm.to(dev), ws, spec.to(dev), out, 64, 64,
                                   peaks=torch.empty(3, device=dev))
    with pytest.raises(RuntimeError, match="float32"):
        zipfft.padded_rconv2d.corr(tm.to(dev), ws, spec.to(dev), out, 64, 64,
                                   peaks=torch.empty(2, dtype=torch.float64, device=dev))


def _random_cases(n, seed):
    """Seeded random configurations over every compiled FFT size."""
    sizes = [64, 128, 256, 512, 1024, 2048, 4096, 120, 240, 480, 960, 1920, 3840]
    rng = np.random.default_rng(seed)
    cases = []
    for _ in range(n):
        H, W = (int(x) for x in rng.choice(sizes, 2))
        if H * W > 4096 * 2048:  # keep the float64 oracle quick
            W = 1024
        sy = int(rng.integers(1, H + 1))
        sx = int(rng.integers(1, W + 1))
        if rng.random() < 0.6:  # mostly small templates, as in template matching
            sy, sx = max(1, sy // 8), max(1, sx // 8)
        B = int(rng.integers(1, 5))
        cases.append((B, sy, sx, H, W, bool(rng.random() < 0.7), bool(rng.random() < 0.5)))
    return cases


RANDOM = _random_cases(24, 2026)


@pytest.mark.parametrize("case", RANDOM, ids=[str(c) for c in RANDOM])
def test_random_shapes_match_oracle(case):
    B, sy, sx, H, W, conj, full = case
    _, tm, spec = make_inputs(B, sy, sx, H, W, seed=sy * 7 + sx)
    out = capi_corr(tm, spec, H, W, full, conj)
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, conj, full)
    assert_parity(ref, out, what=str(case))


@pytest.mark.parametrize("B,sy,sx,H,W,full,conj", [(11, 128, 128, 1024, 1024, True, True),
                                                   (7, 48, 33, 512, 256, False, False),
                                                   (9, 20, 30, 120, 480, False, True)])
def test_batched_groups_agree_with_per_template_path(B, sy, sx, H, W, full, conj):
    """Small images with a (B, H, W/2+1) workspace run as batched groups;
    results equal the one-slice workspace's per-template launches bit for bit
    (and the oracle), peaks included."""
    import zipfft
    from zipfft_b200 import _lib

    _, tm, spec = make_inputs(B, sy, sx, H, W, seed=B * 3 + sy)
    dev = torch.device("cuda", 0)
    nmin = _lib.load().zfft_workspace_bytes(H, W) // 8
    a = capi_corr(tm, spec, H, W, full, conj, ws=torch.empty(nmin, dtype=torch.complex64,
                                                             device=dev))
    big = torch.empty((B, H, W // 2 + 1), dtype=torch.complex64, device=dev)
    b = capi_corr(tm, spec, H, W, full, conj, ws=big)
    assert np.array_equal(a, b)
    ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, conj, full)
    assert_parity(ref, b, what="batched groups")
    if conj:
        oy, ox = O.out_shape(sy, sx, H, W, full)
        out = torch.empty((B, oy, ox), device=dev)
        peaks = torch.empty(B, device=dev)
        zipfft.padded_rconv2d.corr(tm.to(dev), big, spec.to(dev), out, H, W, peaks=peaks)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), b)
        assert torch.equal(peaks, out.reshape(B, -1).amax(dim=1))


@pytest.mark.parametrize("H,W,sy,sx", [(512, 256, 48, 33), (4096, 4096, 256, 256)])
def test_valid_crop_with_nan_workspace(H, W, sy, sx):
    """A workspace that starts as NaN (nothing in it needs initialising):
    with an odd valid-crop height the inverse row pass pairs the last output
    row with a row the column pass never wrote, which must not leak in."""
    _, tm, spec = make_inputs(2, sy, sx, H, W, seed=H + sy)
    dev = torch.device("cuda", 0)
    for ws in (torch.full((2, H, W // 2 + 1), complex(float("nan"), float("nan")),
                          dtype=torch.complex64, device=dev),
               torch.full((H * (W // 2),), complex(float("nan"), float("nan")),
                          dtype=torch.complex64, device=dev)):
        out = capi_corr(tm, spec, H, W, False, True, ws=ws)
        ref = O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, True, False)
        assert_parity(ref, out, what=f"NaN workspace {tuple(ws.shape)}")
