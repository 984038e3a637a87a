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
    # fp32 butterflies ~1.2e-7; the TF32 3-pass GEMM ~1.0e-6 (measured)
    tol = 2e-6 if tensor_cores else 5e-7
    assert err < tol, err
    per_col = np.linalg.norm(got - ref, axis=1) / np.linalg.norm(ref, axis=1)
    assert per_col.max() < 2 * tol, per_col.max()


@pytest.mark.parametrize("tensor_cores", [False, True])
def test_col_fft4096_two_passes_reverse_the_column(tensor_cores):
    """Two forward FFTs give N x[-n mod N]: the second pass starts from the
    first pass's register layout."""
    g = torch.Generator().manual_seed(9)
    x = torch.complex(torch.randn(300, T.N, generator=g), torch.randn(300, T.N, generator=g))
    y = x.cuda()
    T.col_fft4096(y, tensor_cores, passes=2)
    torch.cuda.synchronize()
    assert T.status() == 0
    ref = T.N * np.roll(x.numpy()[:, ::-1], 1, axis=1).astype(np.complex128)
    err = np.linalg.norm(y.cpu().numpy() - ref) / np.linalg.norm(ref)
    assert err < (4e-6 if tensor_cores else 1e-6), err


def test_tensor_core_kernel_with_three_blocks_per_sm():
    """A grid of 3 blocks per SM (each holding 64 TMEM columns) computes the
    same columns as the occupancy-sized grid, bit for bit."""
    g = torch.Generator().manual_seed(3)
    x = torch.complex(torch.randn(1000, T.N, generator=g), torch.randn(1000, T.N, generator=g)).cuda()
    a, b = x.clone(), x.clone()
    T.col_fft4096(a, True)
    T.col_fft4096(b, True, blocks_per_sm=3)
    torch.cuda.synchronize()
    assert T.status() == 0
    assert torch.equal(a, b)
