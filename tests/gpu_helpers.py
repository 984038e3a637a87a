"""Shared helpers for the GPU tests: seeded inputs and direct C-ABI calls."""
import numpy as np
import torch

from oracle import xcorr_oracle as O
from zipfft_b200 import _lib


def make_inputs(B, sy, sx, H, W, seed, device="cuda:0"):
    g = torch.Generator().manual_seed(seed)
    image = torch.randn((H, W), generator=g, dtype=torch.float32)
    tm = torch.randn((B, sy, sx), generator=g, dtype=torch.float32)
    spec_T = torch.from_numpy(O.image_spectrum_T(image.numpy()))
    return image, tm, spec_T


def capi_corr(tm, spec_T, H, W, full, conj=True, device=0, stream=None, ws=None):
    """Call the C ABI directly with device pointers (no Python validation)."""
    B, sy, sx = tm.shape
    oy, ox = O.out_shape(sy, sx, H, W, full)
    dev = torch.device("cuda", device)
    tm_d = tm.to(dev).contiguous()
    sp_d = spec_T.to(dev).contiguous()
    out = torch.full((B, oy, ox), float("nan"), device=dev)
    lib = _lib.load()
    nbytes = lib.zfft_workspace_bytes(H, W)
    if ws is None:
        ws = torch.empty(nbytes // 8, dtype=torch.complex64, device=dev)
    fn = lib.zfft_padded_real_corr_2d if conj else lib.zfft_padded_real_conv_2d
    s = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    st = fn(tm_d.data_ptr(), B, sy, sx, ws.data_ptr(), ws.numel() * 8, sp_d.data_ptr(),
            out.data_ptr(), oy, ox, H, W, device, s)
    _lib.check(st)
    torch.cuda.synchronize(dev)
    return out.cpu().numpy()


def assert_parity(ref, out, rel=5e-6, peak=1e-4, what=""):
    r = O.rel_l2(ref, out)
    m = O.max_abs_over_peak(ref, out)
    assert np.all(np.isfinite(out)), f"{what}: non-finite output"
    assert r < rel, f"{what}: rel L2 {r:.3e} >= {rel}"
    assert m < peak, f"{what}: max abs / peak {m:.3e} >= {peak}"
