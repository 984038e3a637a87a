"""C ABI: the library loads, exports every declared symbol, and validates
arguments on the host (no GPU needed for these paths)."""
import ctypes
import os
import re

import pytest

from zipfft_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"ZFFT_API\s+[\w\s\*]+?\b(zfft_\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "zfft_padded_real_corr_2d" in names
    assert "zfft_padded_real_conv_2d" in names
    assert len(names) >= 7


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_sizes():
    lib = _lib.load()
    assert lib.zfft_get_version() >= 100
    for n in (64, 128, 256, 512, 1024, 2048, 4096, 3840, 1920, 120):
        assert lib.zfft_is_fft_size_supported(n) == 1, n
    for n in (0, 32, 100, 8192, 4095, 5000):
        assert lib.zfft_is_fft_size_supported(n) == 0, n
    assert lib.zfft_workspace_bytes(4096, 4096) == 4096 * 2048 * 8
    assert lib.zfft_workspace_bytes(4096, 100) == 0


def test_supported_configs_contain_reference_table():
    from zipfft_b200 import padded_rconv2d as P

    cfgs = P.get_supported_conv_configs()
    assert len(cfgs) == 50
    # spot-check entries of the reference table (binding.cu:55, :83, :105)
    assert (48, 48, 64, 64, 1, False) in cfgs
    assert (16, 16, 64, 64, 1, True) in cfgs
    assert (512, 512, 4096, 4096, 32, True) in cfgs
    assert (256, 256, 4096, 4096, 32, True) in cfgs
    assert all(isinstance(c[5], bool) for c in cfgs)


def call(lib, **kw):
    args = dict(input=None, batch=1, sy=16, sx=16, ws=None, ws_bytes=1 << 30, conv=None,
                out=None, oy=49, ox=49, H=64, W=64, device=0, stream=None)
    args.update(kw)
    return lib.zfft_padded_real_corr_2d(args["input"], args["batch"], args["sy"], args["sx"],
                                        args["ws"], args["ws_bytes"], args["conv"], args["out"],
                                        args["oy"], args["ox"], args["H"], args["W"],
                                        args["device"], args["stream"])


def test_host_validation_codes():
    lib = _lib.load()
    assert call(lib, H=100) == _lib.ZFFT_ERROR_UNSUPPORTED
    assert "Unsupported padded convolution configuration" in _lib.last_error()
    assert call(lib, oy=50) == _lib.ZFFT_ERROR_INVALID_VALUE
    assert "second-to-last dimension" in _lib.last_error()
    assert call(lib, ox=50) == _lib.ZFFT_ERROR_INVALID_VALUE
    assert "last dimension" in _lib.last_error()
    assert call(lib, sy=65) == _lib.ZFFT_ERROR_INVALID_VALUE
    assert call(lib, sy=0) == _lib.ZFFT_ERROR_INVALID_VALUE
    assert call(lib, batch=-1) == _lib.ZFFT_ERROR_INVALID_VALUE
    assert call(lib, ws_bytes=100) == _lib.ZFFT_ERROR_INVALID_VALUE
    assert "workspace too small" in _lib.last_error()
    # empty batch: nothing to do, no device touched
    assert call(lib, batch=0) == _lib.ZFFT_SUCCESS
    assert _lib.last_error() == ""
    # full-map output accepted by validation, then null pointers rejected
    assert call(lib, oy=64, ox=64) == _lib.ZFFT_ERROR_INVALID_VALUE
    assert "null data pointer" in _lib.last_error()


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="not found"):
        _lib.load(str(tmp_path / "libzipfft_b200.so"))


def test_built_library_matches_sources():
    """A stale libzipfft_b200.so (sources changed since the last build) would
    make every GPU result describe old code."""
    from zipfft_b200 import build

    assert build.is_current(), "rebuild with python -m zipfft_b200.build"


def test_image_spectrum_host_validation():
    """zfft_image_spectrum rejects bad sizes and buffers before any device work."""
    lib = _lib.load()
    need = (64 // 2 + 1) * 128 * 8
    assert lib.zfft_image_spectrum(None, 100, 64, None, need, 0, None) == _lib.ZFFT_ERROR_UNSUPPORTED
    assert "Unsupported image size" in _lib.last_error()
    assert lib.zfft_image_spectrum(None, 128, 64, None, need - 8, 0, None) == \
        _lib.ZFFT_ERROR_INVALID_VALUE
    assert "conv_data too small" in _lib.last_error()
    assert lib.zfft_image_spectrum(None, 128, 64, None, need, 0, None) == \
        _lib.ZFFT_ERROR_INVALID_VALUE
    assert "null data pointer" in _lib.last_error()
    buf = (ctypes.c_float * 64)()
    base = ctypes.addressof(buf)
    assert lib.zfft_image_spectrum(base + 2, 128, 64, (base + 15) // 16 * 16, need, 0, None) == \
        _lib.ZFFT_ERROR_INVALID_VALUE
    assert "misaligned" in _lib.last_error()


C_CLIENT = r"""
#include <stdio.h>
#include <string.h>
#include "zipfft_b200.h"

int main(void) {
    int recs[6 * 64];
    int n = zfft_get_supported_conv_configs(recs, 64);
    size_t ws = zfft_workspace_bytes(4096, 4096);
    int bad = zfft_padded_real_corr_2d(NULL, 1, 16, 16, NULL, (size_t)1 << 30, NULL, NULL,
                                       49, 49, 100, 64, 0, NULL);
    int has_msg = strstr(zfft_get_last_error(), "Unsupported") != NULL;
    int empty = zfft_padded_real_corr_2d(NULL, 0, 16, 16, NULL, (size_t)1 << 30, NULL, NULL,
                                         49, 49, 64, 64, 0, NULL);
    printf("%d %d %d %zu %d %d %d %d\n", zfft_get_version(), n,
           zfft_is_fft_size_supported(4096), ws, bad,
           has_msg, empty, (int)strlen(zfft_get_last_error()));
    return 0;
}
"""


def test_header_compiles_as_c_and_links(tmp_path):
    """A plain C11 client (the path a cgo / JNI / FFI binding takes): the
    header compiles warning-free as strict C, the program links against the
    library and calls its host-only entry points (no GPU needed)."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    lib_dir = os.path.join(ROOT, "zipfft_b200")
    src, exe = tmp_path / "client.c", tmp_path / "client"
    src.write_text(C_CLIENT)
    subprocess.check_call(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic",
                           "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                           "-L", lib_dir, "-lzipfft_b200", f"-Wl,-rpath,{lib_dir}"])
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    version, n, ok4096, ws, bad, has_msg, empty, empty_msg = map(int, out.stdout.split())
    assert version == _lib.load().zfft_get_version()
    assert n == 50 and ok4096 == 1 and ws == 4096 * 2048 * 8
    assert bad == _lib.ZFFT_ERROR_UNSUPPORTED and has_msg == 1
    assert empty == _lib.ZFFT_SUCCESS and empty_msg == 0
