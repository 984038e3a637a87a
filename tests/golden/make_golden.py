"""Generate tests/golden/golden_small.npz (run: python tests/golden/make_golden.py).

Each case holds seeded inputs in the reference test's form and two expected
outputs:
  * `torch`  -- the reference's own oracle, the torch.fft path of
    mgiammar/zipFFT tests/test_real_conv_2d.py:89-127 run on CPU in float32
    (image spectrum from torch.fft.rfftn, transposed like test:127);
  * `direct` -- the definition, a brute-force double sum
    (oracle/direct_corr.c), rounded to float32.
The reference's CUDA path cannot run in this environment (no cuFFTDx, no
sm_100 case), so its test's torch.fft path is the reference output pinned here.
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import xcorr_oracle as O  # noqa: E402

# (name, batch, sig_y, sig_x, fft_y, fft_x, cross_correlate, full_output)
CASES = [
    ("corr_16_64_b2", 2, 16, 16, 64, 64, True, False),
    ("conv_48_64_b1", 1, 48, 48, 64, 64, False, False),
    ("corr_12x20_64x128_full_b3", 3, 12, 20, 64, 128, True, True),
    ("corr_5x7_120x240_b2", 2, 5, 7, 120, 240, True, False),
    ("conv_32x24_128x64_full_b2", 2, 32, 24, 128, 64, False, True),
    ("corr_64_256_b1", 1, 64, 64, 256, 256, True, False),
    ("corr_40x30_120x240_full_b1", 1, 40, 30, 120, 240, True, True),
]


def make_case(seed, B, sy, sx, H, W, conj, full):
    g = torch.Generator().manual_seed(seed)
    image = torch.randn((H, W), generator=g, dtype=torch.float32)
    filt = torch.randn((B, sy, sx), generator=g, dtype=torch.float32)
    image_fft = torch.fft.rfftn(image).contiguous()                      # test:90
    ref = O.reference_torch_path(filt, image_fft, H, W, conj, full)       # test:110-123
    spec_T = image_fft.transpose(-2, -1).contiguous()                    # test:127
    direct = np.stack([O.direct_corr2d(filt[b].numpy(), image.numpy(), conj, full)
                       for b in range(B)])
    return dict(image=image.numpy(), templates=filt.numpy(), spec_T=spec_T.numpy(),
                torch=ref.numpy().astype(np.float32), direct=direct.astype(np.float32),
                meta=np.array([B, sy, sx, H, W, int(conj), int(full)], np.int32))


def main():
    out = {}
    for i, (name, *cfg) in enumerate(CASES):
        case = make_case(1000 + i, *cfg)
        for k, v in case.items():
            out[f"{name}/{k}"] = v
        print(name, "rel_l2(torch, direct) =", O.rel_l2(case["direct"], case["torch"]))
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_small.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
