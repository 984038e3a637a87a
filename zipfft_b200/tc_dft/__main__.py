"""A/B of the column FFT with its 16-point DFTs on the CUDA cores or on the
tensor cores (see the package docstring); prints one JSON line."""
from __future__ import annotations

import argparse
import json
import statistics

import numpy as np
import torch

from zipfft_b200 import tc_dft as T


def rel_l2(got: np.ndarray, ref: np.ndarray) -> float:
    return float(np.linalg.norm(got - ref) / np.linalg.norm(ref))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--columns", type=int, default=4098,
                    help="columns per launch (default 4098 = 2 x 2049, 134 MB)")
    ap.add_argument("--windows", type=int, default=10, help="timed windows per kernel")
    ap.add_argument("--reps", type=int, default=6, help="launches per timed window (<= 8)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tc-blocks-per-sm", type=int, default=0,
                    help="blocks per SM of the tensor-core kernel's grid (0: occupancy calculator)")
    ap.add_argument("--passes", type=int, default=1, choices=(1, 2),
                    help="FFTs per column between its load and store (2: the arithmetic per byte "
                         "of the fused column pass)")
    a = ap.parse_args(argv)
    if not 1 <= a.reps * a.passes <= 8:
        raise SystemExit("--reps x --passes must be 1..8 (each FFT scales the data by ~64)")
    T.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device="cpu").manual_seed(1)
    pristine = torch.complex(torch.randn(a.columns, T.N, generator=g),
                             torch.randn(a.columns, T.N, generator=g)).to(dev)
    x = pristine.clone()

    # Accuracy on the first 64 columns against numpy's float64 FFT (applied
    # `passes` times).
    m = min(64, a.columns)
    ref = pristine[:m].cpu().numpy().astype(np.complex128)
    for _ in range(a.passes):
        ref = np.fft.fft(ref, axis=1)
    err = {}
    for tc in (False, True):
        x.copy_(pristine)
        T.col_fft4096(x, tc, a.passes, a.tc_blocks_per_sm if tc else 0)
        torch.cuda.synchronize()
        err["tensor" if tc else "cuda"] = rel_l2(x[:m].cpu().numpy().astype(np.complex128), ref)
    st = T.status()

    stream = torch.cuda.current_stream(dev)
    for tc in (False, True):
        for _ in range(a.warmup):
            x.copy_(pristine)
            T.col_fft4096(x, tc, a.passes, a.tc_blocks_per_sm if tc else 0)
    torch.cuda.synchronize()
    times = {False: [], True: []}
    for _ in range(a.windows):
        for tc in (False, True):  # interleaved windows
            x.copy_(pristine)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(a.reps):
                T.col_fft4096(x, tc, a.passes, a.tc_blocks_per_sm if tc else 0)
            e1.record(stream)
            e1.synchronize()
            times[tc].append(e0.elapsed_time(e1) * 1e3 / a.reps)
    st |= T.status()

    out = {"what": f"in-place 4096-point forward FFT of {a.columns} contiguous complex64 columns, "
                   f"{a.passes} time(s) per load/store (3 radix-16 stages per FFT, same loads / "
                   "twiddles / exchanges / stores)",
           "passes": a.passes, "tc_blocks_per_sm_requested": a.tc_blocks_per_sm,
           "bytes_per_launch": 2 * a.columns * T.N * 8, "status": st,
           "occupancy_tc_by_smem": {str(b): T.occupancy(True, b) for b in (1024, 33792, 74816)},
           "occupancy_cuda_by_smem": {str(b): T.occupancy(False, b) for b in (1024, 33792)}}
    for tc in (False, True):
        name = "tensor" if tc else "cuda"
        us = statistics.median(times[tc])
        regs, occ = T.kernel_info(tc)
        out[name] = {"us_per_launch": us, "us_per_2049_columns": us * 2049 / a.columns,
                     "achieved_gbs": 2 * a.columns * T.N * 8 / us / 1e3,
                     "rel_l2_vs_float64": err[name], "registers": regs, "blocks_per_sm": occ,
                     "windows_us": [round(t, 2) for t in times[tc]]}
    out["tensor_over_cuda_time"] = out["tensor"]["us_per_launch"] / out["cuda"]["us_per_launch"]
    print(json.dumps(out), flush=True)
    return 0 if st == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
