"""The CUDA kernels' own source, executed on CPU threads (tests/kernel_emu)
under AddressSanitizer, against the oracle.  Checks index arithmetic (every
access in bounds), the persistent block loops (grids capped at 3 blocks), the
pruned starts (nz = 1, 2) and the radix-3/5 plans before the code reaches a
GPU.  The GPU tests check the compiled kernels themselves."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from oracle import xcorr_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "kernel_emu", "emu_main.cpp")
EXE = os.path.join(ROOT, "_build", "zf_emu")


def _deps():
    files = [SRC] + [os.path.join(ROOT, "zipfft_b200", "csrc", f)
                     for f in ("fft_core.cuh", "xcorr_kernels.cuh", "async_copy.cuh")]
    return max(os.path.getmtime(f) for f in files)


@pytest.fixture(scope="module")
def emu():
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    if not os.path.exists(EXE) or os.path.getmtime(EXE) < _deps():
        os.makedirs(os.path.dirname(EXE), exist_ok=True)
        # Build under a private name and rename: parallel test workers may
        # build at the same time, and none may run a half-written binary.
        tmp = f"{EXE}.{os.getpid()}.tmp"
        subprocess.check_call(["g++", "-std=c++20", "-O1", "-g", "-fsanitize=address,alignment",
                               "-fno-sanitize-recover=alignment", "-fno-omit-frame-pointer",
                               "-pthread", SRC, "-o", tmp])
        os.replace(tmp, EXE)
    return EXE


def first_radix(n):
    p2 = n & -n
    return 16 if p2 >= 16 else (p2 if p2 > 1 else (5 if n % 5 == 0 else 3))


def nz_of(n, length):
    nb0 = n // first_radix(n)
    nz = (length + nb0 - 1) // nb0
    return max(nz, 1) if nz <= 2 else 0


def run_emu(exe, tmp_path, B, sy, sx, H, W, conj, full, nz_col=None, nz_row=None, seed=0,
            chunk=0, max_mode=False, group=0, poison=False, defer=False, sum_batches=False):
    rng = np.random.default_rng(seed)
    img = rng.standard_normal((H, W)).astype(np.float32)
    tm = rng.standard_normal((B, sy, sx)).astype(np.float32)
    spec = O.image_spectrum_T(img)
    oy, ox = O.out_shape(sy, sx, H, W, full)
    nz_col = nz_of(H, sy) if nz_col is None else nz_col
    nz_row = nz_of(W // 2, (sx + 1) // 2) if nz_row is None else nz_row
    fin, fout = str(tmp_path / "in.bin"), str(tmp_path / "out.bin")
    with open(fin, "wb") as f:
        np.array([B, sy, sx, H, W, oy, ox, int(conj), 3, nz_col, nz_row, chunk, int(max_mode),
                  group + (1 << 16 if poison else 0) + (1 << 17 if defer else 0)
                  + (1 << 18 if sum_batches else 0)],
                 np.int32).tofile(f)
        tm.tofile(f)
        spec.tofile(f)
    res = subprocess.run([exe, fin, fout], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-4000:]
    ref = O.padded_corr2d_f64(tm, spec, H, W, conj, full)
    if max_mode in (1, 2, 4):  # True counts as 1; 4: sum of squares without the sum
        raw = np.fromfile(fout, np.uint8)
        n = oy * ox * 4
        mx = raw[:n].view(np.float32).reshape(oy, ox)
        am = raw[n:2 * n].view(np.int32).reshape(oy, ox)
        if max_mode in (2, 4):
            sm = raw[2 * n:3 * n].view(np.float32).reshape(oy, ox)
            sq = raw[3 * n:4 * n].view(np.float32).reshape(oy, ox)
            return (mx, am, sm, sq), ref
        return (mx, am), ref
    raw = np.fromfile(fout, np.float32)
    out = raw[: B * oy * ox].reshape(B, oy, ox)
    if max_mode == 3:
        return (out, raw[B * oy * ox:]), ref
    return out, ref


CASES = [
    # B, sy, sx, H, W, conj, full, nz_col, nz_row, chunk
    (2, 16, 16, 64, 64, True, False, None, None, 0),
    (1, 48, 48, 64, 64, False, False, None, None, 0),
    (2, 12, 20, 64, 128, True, True, None, None, 0),
    (2, 5, 7, 120, 240, True, False, None, None, 0),
    (1, 32, 24, 128, 64, False, True, None, None, 0),
    (1, 16, 16, 256, 256, True, True, 1, 1, 0),
    (1, 30, 30, 256, 256, True, False, 2, 2, 0),
    (1, 17, 32, 256, 256, False, True, 2, 2, 0),
    (1, 100, 90, 240, 120, True, True, None, None, 0),
    (2, 64, 64, 64, 64, True, True, None, None, 0),  # signal == FFT size
    (1, 1, 1, 64, 64, True, True, 1, 1, 0),          # single pixel
    (1, 7, 3, 128, 240, True, False, 1, 1, 0),       # odd widths
    (5, 16, 16, 64, 64, True, True, None, None, 2),  # chunked rows, partial last chunk
    (3, 9, 13, 128, 256, False, False, None, None, 3),  # chunked, odd template
    (4, 30, 30, 256, 256, True, True, 2, 2, 4),
    (2, 100, 20, 2048, 64, True, True, 1, None, 2),   # one column per block: bulk column stores
    (1, 129, 9, 2048, 64, False, False, 2, None, 0),  # valid crop, odd store length
    (2, 10, 100, 64, 2048, True, True, None, None, 2),  # wide rows (W/2 = 1024), chunked
    (1, 33, 300, 128, 2048, False, False, None, None, 0),
]


@pytest.mark.parametrize("case", CASES, ids=[str(c[:7]) for c in CASES])
def test_emulated_kernels_match_oracle(emu, tmp_path, case):
    B, sy, sx, H, W, conj, full, nzc, nzr, chunk = case
    out, ref = run_emu(emu, tmp_path, B, sy, sx, H, W, conj, full, nzc, nzr, chunk=chunk)
    assert O.rel_l2(ref, out) < 1e-6
    assert O.max_abs_over_peak(ref, out) < 1e-5


@pytest.mark.parametrize("chunk,W,sx", [(0, 128, 9), (2, 128, 9), (0, 2048, 9), (0, 256, 10)])
def test_emulated_running_max_argmax(emu, tmp_path, chunk, W, sx):
    """The max / argmax epilogue of the inverse row pass (sx = 10: odd-width
    valid crop, 8-byte accesses on every other row only)."""
    B, H = 5, 64
    (mx, am), ref = run_emu(emu, tmp_path, B, 12, sx, H, W, True, True, chunk=chunk,
                            max_mode=True)
    assert np.allclose(mx, ref.max(axis=0), rtol=0, atol=1e-5 * np.abs(ref).max())
    order = np.sort(ref, axis=0)
    margin = order[-1] - order[-2]
    sure = margin > 1e-4 * np.abs(ref).max()
    assert sure.mean() > 0.99
    assert np.array_equal(am[sure], ref.argmax(axis=0)[sure])
    (mv, av), refv = run_emu(emu, tmp_path, B, 12, sx, H, W, True, False, max_mode=True)
    assert mv.shape == (H - 11, W - sx + 1)
    assert np.allclose(mv, refv.max(axis=0), rtol=0, atol=1e-5 * np.abs(refv).max())


@pytest.mark.parametrize("H,W,defer", [(64, 64, False), (128, 240, False), (240, 120, False),
                                       (2048, 64, False), (256, 512, False), (2048, 64, True),
                                       (128, 240, True)])
def test_emulated_image_spectrum(emu, tmp_path, H, W, defer):
    """zfft_image_spectrum's row and in-place column passes against the
    float64 rfft2 (transposed), including the split of packed column 0 into
    the kx = 0 and kx = W/2 rows; defer: every TMA load lands only when a
    thread polls its barrier."""
    rng = np.random.default_rng(H + W)
    img = rng.standard_normal((H, W)).astype(np.float32)
    fin, fout = str(tmp_path / "in.bin"), str(tmp_path / "out.bin")
    with open(fin, "wb") as f:
        np.array([H, W, 3 + (1 << 17 if defer else 0)], np.int32).tofile(f)
        img.tofile(f)
    res = subprocess.run([emu, "spectrum", fin, fout], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-4000:]
    out = np.fromfile(fout, np.complex64).reshape(W // 2 + 1, H)
    ref = O.image_spectrum_T(img, dtype=np.complex128)
    assert O.rel_l2(ref, out) < 1e-6
    assert np.abs(out - ref).max() < 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("chunk,W,full,sx", [(0, 128, True, 9), (2, 2048, False, 9),
                                             (0, 256, False, 10)])
def test_emulated_running_stats(emu, tmp_path, chunk, W, full, sx):
    """The max / argmax epilogue with per-pixel sum and sum of squares."""
    B, H = 5, 64
    (mx, am, sm, sq), ref = run_emu(emu, tmp_path, B, 12, sx, H, W, True, full, chunk=chunk,
                                    max_mode=2)
    peak = np.abs(ref).max()
    assert np.allclose(mx, ref.max(axis=0), rtol=0, atol=1e-5 * peak)
    assert O.rel_l2(ref.sum(axis=0), sm) < 1e-5
    assert O.rel_l2((ref ** 2).sum(axis=0), sq) < 1e-5


@pytest.mark.parametrize("W,full,sx", [(128, True, 9), (2048, False, 9), (240, False, 9),
                                       (2048, False, 10)])
def test_emulated_peaks(emu, tmp_path, W, full, sx):
    """Maps plus each map's largest value (warp reduction and atomicMax on
    ordered keys): the peaks equal the maxima of the stored maps exactly."""
    B, H = 3, 64
    (out, peaks), ref = run_emu(emu, tmp_path, B, 12, sx, H, W, True, full, max_mode=3)
    assert O.rel_l2(ref, out) < 1e-6
    assert np.array_equal(peaks, out.reshape(B, -1).max(axis=1))


def _random_emu_cases(n, seed):
    sizes = [64, 128, 256, 512, 120, 240]
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        H, W = (int(x) for x in rng.choice(sizes, 2))
        sy, sx = int(rng.integers(1, H // 2 + 1)), int(rng.integers(1, W // 2 + 1))
        B = int(rng.integers(1, 4))
        out.append((B, sy, sx, H, W, bool(rng.random() < 0.7), bool(rng.random() < 0.5),
                    int(rng.choice([0, 2]))))
    return out


RANDOM_EMU = _random_emu_cases(8, 7)


@pytest.mark.parametrize("case", RANDOM_EMU, ids=[str(c) for c in RANDOM_EMU])
def test_emulated_random_shapes(emu, tmp_path, case):
    """Seeded random shapes (sizes, template extents, corr / conv, crop,
    chunked row passes) against the oracle."""
    B, sy, sx, H, W, conj, full, chunk = case
    out, ref = run_emu(emu, tmp_path, B, sy, sx, H, W, conj, full, chunk=chunk,
                       seed=B + sy + sx)
    assert O.rel_l2(ref, out) < 1e-6
    assert O.max_abs_over_peak(ref, out) < 1e-5


@pytest.mark.parametrize("case", [(5, 16, 16, 64, 64, True, True, 2), (3, 30, 45, 128, 256, False, False, 3),
                                  (4, 9, 13, 120, 240, True, False, 4), (2, 100, 20, 2048, 64, True, True, 2)],
                         ids=lambda c: str(c))
def test_emulated_batched_groups(emu, tmp_path, case):
    """Batched groups: one launch of each kernel for a group of templates,
    each in its own Q slice; partial last group."""
    B, sy, sx, H, W, conj, full, group = case
    out, ref = run_emu(emu, tmp_path, B, sy, sx, H, W, conj, full, group=group)
    assert O.rel_l2(ref, out) < 1e-6
    assert O.max_abs_over_peak(ref, out) < 1e-5


def test_emulated_batched_peaks(emu, tmp_path):
    B, H, W = 5, 64, 256
    (out, peaks), ref = run_emu(emu, tmp_path, B, 12, 10, H, W, True, False, max_mode=3, group=2)
    assert O.rel_l2(ref, out) < 1e-6
    assert np.array_equal(peaks, out.reshape(B, -1).max(axis=1))


def test_emulated_pair_kernel_ignores_stale_rows(emu, tmp_path):
    """Odd valid-crop height: the row pair's second row lies past the output
    and was never written by the column pass; a NaN-poisoned workspace must
    not leak into the last output row (the harness fills the workspace with
    NaN in this mode)."""
    # out 81 x 224: odd height, and row 81 lies past the template's rows (48),
    # so nothing ever wrote it
    B, sy, sx, H, W = 2, 48, 33, 128, 256
    out, ref = run_emu(emu, tmp_path, B, sy, sx, H, W, True, False, group=0, poison=True)
    assert np.all(np.isfinite(out))
    assert O.rel_l2(ref, out) < 1e-6


@pytest.mark.parametrize("case", [
    # B, sy, sx, H, W, conj, full, chunk, max_mode, group
    (2, 100, 20, 2048, 64, True, True, 2, 0, 0),    # one column per block, bulk Q stores
    (1, 129, 9, 2048, 64, False, False, 0, 0, 0),   # valid crop: row-pair kernel
    (5, 16, 16, 64, 64, True, True, 2, 0, 0),       # several columns per block, chunked rows
    (2, 10, 100, 64, 2048, True, True, 2, 0, 0),    # wide rows
    (4, 9, 13, 120, 240, True, False, 0, 0, 4),     # batched group
    (3, 12, 9, 128, 128, True, True, 0, 1, 0),      # running max / argmax
    (3, 12, 9, 128, 128, True, False, 0, 2, 0),     # ... with sum / sum of squares
    (3, 12, 10, 64, 256, True, False, 0, 3, 0),     # per-template peaks
    (5, 12, 9, 64, 128, True, True, 0, 1, 2),       # grouped running max / argmax
    (5, 12, 10, 64, 256, True, False, 0, 2, 3),     # ... with sums, valid crop
], ids=lambda c: str(c))
def test_emulated_kernels_with_late_tma_arrival(emu, tmp_path, case):
    """Every TMA load lands only when a thread polls its barrier, the latest
    moment the hardware allows: a read of a double-buffered input before its
    barrier wait would see the previous group's data.  Results must not
    change, and no block may exit with a load in flight."""
    B, sy, sx, H, W, conj, full, chunk, max_mode, group = case
    got, ref = run_emu(emu, tmp_path, B, sy, sx, H, W, conj, full, chunk=chunk,
                       max_mode=max_mode, group=group, defer=True)
    if max_mode in (1, 2):
        mx, am = got[0], got[1]
        peak = np.abs(ref).max()
        assert np.allclose(mx, ref.max(axis=0), rtol=0, atol=1e-5 * peak)
        order = np.sort(ref, axis=0)
        sure = order[-1] - order[-2] > 1e-4 * peak
        assert np.array_equal(am[sure], ref.argmax(axis=0)[sure])
        if max_mode == 2:
            assert O.rel_l2(ref.sum(axis=0), got[2]) < 1e-5
            assert O.rel_l2((ref ** 2).sum(axis=0), got[3]) < 1e-5
        return
    out = got[0] if max_mode == 3 else got
    assert O.rel_l2(ref, out) < 1e-6
    assert O.max_abs_over_peak(ref, out) < 1e-5
    if max_mode == 3:
        assert np.array_equal(got[1], out.reshape(B, -1).max(axis=1))


@pytest.mark.parametrize("group", [0, 2])
def test_emulated_stats_batches_restart_sums_keep_max(emu, tmp_path, group):
    """reset = kResetSums on a batch's first template (the search's per-batch
    partial sums): the sum maps restart there, the maximum and argmax keep
    folding every template.  group = 2: batched groups of two templates per
    launch, each group after the first a new batch."""
    B = 5
    (mx, am, sm, sq), ref = run_emu(emu, tmp_path, B, 12, 9, 64, 128, True, True,
                                    max_mode=2, sum_batches=True, group=group)
    tol = 1e-5 * np.abs(ref).max()
    assert np.allclose(mx, ref.max(axis=0), rtol=0, atol=tol)
    last = ref[4:]  # templates 0-1, 2-3 and 4 form the batches
    assert np.allclose(sm, last.sum(axis=0), rtol=0, atol=tol)
    assert np.allclose(sq, (last ** 2).sum(axis=0), rtol=0, atol=tol * np.abs(ref).max())


@pytest.mark.parametrize("group,W,full,sx,max_mode", [
    (2, 128, True, 9, 1), (3, 128, False, 10, 1), (5, 2048, True, 9, 1),
    (2, 256, True, 9, 2), (4, 240, False, 9, 2)])
def test_emulated_grouped_running_maps(emu, tmp_path, group, W, full, sx, max_mode):
    """Running maps with several templates per launch (batched groups): each
    block folds a row group's templates one after another into the maps, with
    3 blocks for more row groups than that (every block takes several groups).
    Same maxima, argmax (ties excluded) and sums as one template per launch."""
    B, H = 5, 64
    got, ref = run_emu(emu, tmp_path, B, 12, sx, H, W, True, full, max_mode=max_mode,
                       group=group)
    peak = np.abs(ref).max()
    assert np.allclose(got[0], ref.max(axis=0), rtol=0, atol=1e-5 * peak)
    order = np.sort(ref, axis=0)
    sure = order[-1] - order[-2] > 1e-4 * peak
    assert sure.mean() > 0.99
    assert np.array_equal(got[1][sure], ref.argmax(axis=0)[sure])
    if max_mode == 2:
        assert O.rel_l2(ref.sum(axis=0), got[2]) < 1e-5
        assert O.rel_l2((ref ** 2).sum(axis=0), got[3]) < 1e-5
    one, _ = run_emu(emu, tmp_path, B, 12, sx, H, W, True, full, max_mode=max_mode)
    # the same per-pixel arithmetic in the same template order: bit-identical
    for a, b in zip(got, one):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("group", [0, 3])
def test_emulated_sum_of_squares_without_sum(emu, tmp_path, group):
    """kRunningSumSq: the maximum, argmax and sum of squares as kRunningStats
    computes them (bit for bit), no sum map written."""
    B, H, W = 5, 64, 128
    (mx, am, sm, sq), ref = run_emu(emu, tmp_path, B, 12, 9, H, W, True, False, max_mode=4,
                                    group=group)
    (mx2, am2, sm2, sq2), _ = run_emu(emu, tmp_path, B, 12, 9, H, W, True, False, max_mode=2,
                                      group=group)
    assert np.array_equal(mx, mx2) and np.array_equal(am, am2) and np.array_equal(sq, sq2)
    assert not sm.any()
    assert O.rel_l2((ref ** 2).sum(axis=0), sq) < 1e-5
