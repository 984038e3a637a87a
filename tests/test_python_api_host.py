"""The zipfft.padded_rconv2d host-side mirror: module surface and the
reference's validation messages (binding.cu:196-263), checked on CPU tensors."""
import pytest
import torch

import zipfft
import zipfft_b200


def test_package_surface_matches_reference():
    # src/zipfft/__init__.py:25-45
    assert zipfft.is_extension_available("padded_rconv2d")
    assert not zipfft.is_extension_available("cfft1d")
    assert zipfft.get_available_extensions() == ["padded_rconv2d"]
    assert zipfft.get_cuda_architectures() == ["10.0a"]
    assert zipfft.padded_rconv2d is zipfft_b200.padded_rconv2d
    for fn in ("corr", "conv", "get_supported_conv_configs"):
        assert callable(getattr(zipfft.padded_rconv2d, fn))
    import zipfft.padded_rconv2d as sub

    assert sub.corr is zipfft_b200.padded_rconv2d.corr


def tensors(h=16, w=16, H=64, W=64, B=None, dev="cpu"):
    lead = () if B is None else (B,)
    inp = torch.zeros(lead + (h, w), device=dev)
    ws = torch.zeros(lead + (H, W // 2 + 1), dtype=torch.complex64, device=dev)
    cd = torch.zeros((W // 2 + 1, H), dtype=torch.complex64, device=dev)
    out = torch.zeros(lead + (H - h + 1, W - w + 1), device=dev)
    return inp, ws, cd, out


def test_cpu_tensors_rejected_with_reference_messages():
    inp, ws, cd, out = tensors()
    with pytest.raises(RuntimeError, match="Input tensor must be on CUDA device"):
        zipfft.padded_rconv2d.corr(inp, ws, cd, out, 64, 64)
    with pytest.raises(RuntimeError, match="Input tensor must be on CUDA device"):
        zipfft.padded_rconv2d.conv(inp, ws, cd, out, 64, 64)


def test_validation_order_and_messages(monkeypatch):
    # Run the shape checks without a GPU by treating CPU as the device type.
    from zipfft_b200 import padded_rconv2d as P

    class FakeDev:
        type = "cuda"
        index = 0

        def __eq__(self, other):
            return True

    def validate(*a):
        return P._validate(*a)

    inp, ws, cd, out = tensors()

    class Wrap:
        def __init__(self, t):
            self.t = t
            self.device = FakeDev()

        def __getattr__(self, k):
            return getattr(self.t, k)

    def v(i, w, c, o, H=64, W=64):
        return validate(Wrap(i), Wrap(w), Wrap(c), Wrap(o), H, W)

    assert v(inp, ws, cd, out) == (1, 16, 16, 49, 49)
    with pytest.raises(RuntimeError, match="Input tensor must be of type torch.float32"):
        v(inp.double(), ws, cd, out)
    with pytest.raises(RuntimeError, match="FFT workspace tensor must be of type"):
        v(inp, ws.real.contiguous(), cd, out)
    with pytest.raises(RuntimeError, match="Input tensor must be 2D or 3D. Got 4D."):
        v(inp[None, None], ws, cd, out)
    with pytest.raises(RuntimeError, match="last dimension must be fft_size_x/2 \\+ 1"):
        v(inp, ws[:, :-1], cd, out)
    with pytest.raises(RuntimeError, match="second-to-last dimension must be fft_size_y"):
        v(inp, ws[:-1], cd, out)
    with pytest.raises(RuntimeError, match="Convolution data tensor must be 2D. Got 3D."):
        v(inp, ws, cd[None], out)
    with pytest.raises(RuntimeError, match="Output tensor last dimension must be"):
        v(inp, ws, cd, out[:, :-1])
    with pytest.raises(RuntimeError, match="Output tensor second-to-last dimension must be"):
        v(inp, ws, cd, out[:-1])
    # full map accepted
    full = torch.zeros(64, 64)
    assert v(inp, ws, cd, full) == (1, 16, 16, 64, 64)
    # batched: workspace batch must match
    bi, bws, bcd, bout = tensors(B=3)
    assert v(bi, bws, bcd, bout)[0] == 3
    with pytest.raises(RuntimeError, match="first dimension \\(batch\\) must match"):
        v(bi, bws[:2], bcd, bout)
    with pytest.raises(RuntimeError, match="must be contiguous"):
        v(bi.transpose(1, 2), bws, bcd, bout)


def test_expanded_output_rejected_before_launch(monkeypatch):
    """An output expanded over the batch (stride 0) would make the kernels
    write B maps into one map's storage: corr and conv reject it with the
    contiguity error before anything is launched; only corr_max's internal
    shape stand-in skips that check."""
    from zipfft_b200 import _lib
    from zipfft_b200 import padded_rconv2d as P

    class FakeDev:
        type = "cuda"
        index = 0

        def __eq__(self, other):
            return True

    class Wrap:
        def __init__(self, t):
            self.t = t
            self.device = FakeDev()

        def __getattr__(self, k):
            return getattr(self.t, k)

    real_validate = P._validate

    def validate_wrapped(*a, **k):
        return real_validate(*(Wrap(x) if isinstance(x, torch.Tensor) else x for x in a), **k)

    def no_launch():
        raise AssertionError("the library was reached with an invalid output")

    monkeypatch.setattr(P, "_validate", validate_wrapped)
    monkeypatch.setattr(_lib, "load", no_launch)
    bi, bws, bcd, _ = tensors(B=3)
    expanded = torch.zeros(64, 64).expand(3, 64, 64)
    assert expanded.stride(0) == 0
    for fn in (P.corr, P.conv):
        with pytest.raises(RuntimeError, match="Output tensor must be contiguous"):
            fn(bi, bws, bcd, expanded, 64, 64)
    with pytest.raises(RuntimeError, match="Output tensor must be contiguous"):
        P.corr(bi, bws, bcd, expanded, 64, 64, peaks=torch.zeros(3))
    # an overlapping (non-expanded but strided) output is rejected the same way
    base = torch.zeros(3 * 64 + 64, 64)
    overlap = base.as_strided((3, 64, 64), (64, 64, 1))
    with pytest.raises(RuntimeError, match="Output tensor must be contiguous"):
        P.corr(bi, bws, bcd, overlap, 64, 64)
    # corr_max's stand-in (not an output the kernels write) passes the checks
    assert real_validate(Wrap(bi), Wrap(bws), Wrap(bcd), Wrap(expanded), 64, 64,
                         output_is_shape_stand_in=True)[0] == 3
