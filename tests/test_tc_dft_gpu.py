"""The column FFT with its 16-point DFTs on the tensor cores (tcgen05.mma
kind::tf32, 3-pass split) and on the CUDA cores, against numpy's float64 FFT."""
import numpy as np
import pytest
import torch

from zipfft_b200 import tc_dft as T

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("columns", [1, 37, 1000])
@pytest.mark.parametrize("tensor_cores", [False, True])
def test_col_fft4096_matches_float64(columns, tensor_cores):
    g = torch.Generator().manual_seed(columns)
    x = torch.complex(torch.randn(columns, T.N, generator=g), torch.randn(columns, T.N, generator=g))
    ref = np.fft.fft(x.numpy().astype(np.complex128), axis=1)
    y = x.cuda()
    T.col_fft4096(y, tensor_cores)
    torch.cuda.synchronize()
    assert T.status() == 0
    got = y.cpu().numpy().astype(np.complex128)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err < 1e-6, err
    # every column, not only the sum: the worst column stays within 2e-6
    per_col = np.linalg.norm(got - ref, axis=1) / np.linalg.norm(ref, axis=1)
    assert per_col.max() < 2e-6, per_col.max()
