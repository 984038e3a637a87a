"""The allocation-free cross-correlation entry point.

Some callers of this library cannot allocate device memory themselves: a
host framework whose caching allocator has already reserved the device's
free memory (a new cudaMalloc there fails, or forces the pool to give memory
back), a service that reaches the library through the C ABI and accounts for
every device byte itself, or a real-time pipeline that must not pay
cudaMalloc's implicit device synchronization on its hot path.
zfft_padded_real_corr_2d_noalloc serves them: it takes no workspace and uses a
fixed 16 MiB scratch array inside the library instead.

This file is collected last on purpose, so that a run stopping at the first
failure has run every other test before it.
"""
import numpy as np
import pytest
import torch

from oracle import xcorr_oracle as O
from tests.gpu_helpers import assert_parity, capi_corr, make_inputs
from zipfft_b200 import _lib

pytestmark = pytest.mark.gpu


def noalloc_corr(tm, spec, H, W, full):
    B, sy, sx = tm.shape
    oy, ox = O.out_shape(sy, sx, H, W, full)
    dev = torch.device("cuda", 0)
    tm_d = tm.to(dev).contiguous()
    sp_d = spec.to(dev).contiguous()
    out = torch.full((B, oy, ox), float("nan"), device=dev)
    st = _lib.load().zfft_padded_real_corr_2d_noalloc(
        tm_d.data_ptr(), B, sy, sx, sp_d.data_ptr(), out.data_ptr(), oy, ox, H, W, 0,
        torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st)
    torch.cuda.synchronize(dev)
    return out.cpu().numpy()


# (B, h, w, H, W, full, seed).  The fixed 16 MiB array is laid out by the
# same rules as a caller's workspace of that size, so the cases cover each
# layout it can take: the intermediate alone (2048^2), the row spectra of a
# chunk of templates after it (1920 x 2048: one 15 MiB slice plus 1 MiB), and
# batched groups of several slices (1024 x 2048, 512^2).  The workspace entry
# point is given exactly one slice, so it always runs templates one by one.
NOALLOC_CASES = [
    (3, 100, 80, 2048, 2048, True, 1),
    (2, 37, 53, 1024, 2048, False, 2),
    (4, 37, 29, 1920, 2048, True, 4),
    (8, 48, 48, 512, 512, True, 5),
]


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    # Calls in a row with different shapes and inputs: each runs on the
    # scratch array as the previous call left it.  Results do not depend on
    # the workspace layout, so they equal the workspace entry point's bit for
    # bit; the oracle pins both.
    for (B, h, w, H, W, full, seed) in NOALLOC_CASES:
        _, tm, spec = make_inputs(B, h, w, H, W, seed=seed)
        got = noalloc_corr(tm, spec, H, W, full)
        want = capi_corr(tm, spec, H, W, full, True)
        what = f"no-alloc entry point {(B, h, w, H, W)}"
        assert np.array_equal(want, got), f"{what}: differs from the workspace entry point"
        assert_parity(O.padded_corr2d_f64(tm.numpy(), spec.numpy(), H, W, True, full), got,
                      what=what)
    assert _lib.check_device_status(0) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    _, tm, spec = make_inputs(1, 16, 16, 4096, 4096, seed=3)
    dev = torch.device("cuda", 0)
    out = torch.empty((1, 4096, 4096), device=dev)
    tm_d, sp_d = tm.to(dev), spec.to(dev)
    st = _lib.load().zfft_padded_real_corr_2d_noalloc(
        tm_d.data_ptr(), 1, 16, 16, sp_d.data_ptr(), out.data_ptr(), 4096, 4096, 4096, 4096, 0,
        None)
    assert st == _lib.ZFFT_ERROR_INVALID_VALUE
    assert "fixed" in _lib.last_error() and "scratch" in _lib.last_error()
