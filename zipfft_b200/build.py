"""Build libzipfft_b200.so in-tree for sm_100a.

    python -m zipfft_b200.build [--force] [--jobs N]

Compiles csrc/inst.cu once per FFT size (csrc/zf_sizes.h) plus csrc/capi.cu
with nvcc, in parallel, and links them into zipfft_b200/libzipfft_b200.so with
the CUDA runtime linked statically.  Objects go to _build/ at the repository
root.  Replaces the reference's setuptools/pybind11 build (setup.py:51-153),
which targets sm_80..sm_90 and sm_120 but not sm_100.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import re
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD_DIR = os.path.join(ROOT, "_build")
LIB_PATH = os.path.join(PKG_DIR, "libzipfft_b200.so")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def fft_sizes() -> list[int]:
    text = open(os.path.join(CSRC, "zf_sizes.h")).read()
    body = text.split("#define ZF_FOR_EACH_FFT_SIZE(X)")[1].split("\n\n")[0]
    return [int(s) for s in re.findall(r"X\((\d+)\)", body)]


STAMP_PATH = LIB_PATH + ".stamp"


def sources_hash() -> str:
    """Hash of every input of the library build (sources, headers, flags)."""
    import hashlib

    files = sorted(glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(ROOT, "include", "*.h")))
    hsh = hashlib.sha256()
    for f in files:
        hsh.update(os.path.basename(f).encode())
        with open(f, "rb") as fh:
            hsh.update(fh.read())
    hsh.update(" ".join(NVCC_FLAGS).encode())
    return hsh.hexdigest()


def is_current() -> bool:
    """True if the built library matches the current sources."""
    try:
        with open(STAMP_PATH) as fh:
            return os.path.exists(LIB_PATH) and fh.read().strip() == sources_hash()
    except OSError:
        return False


def _deps_mtime() -> float:
    files = glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    files.append(os.path.abspath(__file__))
    return max(os.path.getmtime(f) for f in files)


def _compile(args: tuple[list[str], str]) -> str:
    cmd, out = args
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {out}:\n{res.stdout}\n{res.stderr}")
    return out


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    """Compile (if stale) and return the path of libzipfft_b200.so."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    deps = _deps_mtime()
    if not force and is_current():
        return LIB_PATH
    cc = nvcc()
    jobs_list = []
    objs = []
    for n in fft_sizes():
        out = os.path.join(BUILD_DIR, f"inst_{n}.o")
        objs.append(out)
        if force or not os.path.exists(out) or os.path.getmtime(out) < deps:
            jobs_list.append(([cc, *NVCC_FLAGS, f"-DZF_SIZE={n}", "-c",
                               os.path.join(CSRC, "inst.cu"), "-o", out], out))
    out = os.path.join(BUILD_DIR, "capi.o")
    objs.append(out)
    if force or not os.path.exists(out) or os.path.getmtime(out) < deps:
        jobs_list.append(([cc, *NVCC_FLAGS, "-c", os.path.join(CSRC, "capi.cu"), "-o", out], out))
    workers = jobs or max(1, os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=workers) as pool:
        for done in pool.map(_compile, jobs_list):
            if verbose:
                print("compiled", os.path.relpath(done, ROOT))
    tmp = LIB_PATH + ".tmp"
    subprocess.check_call([cc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", tmp, *objs])
    os.replace(tmp, LIB_PATH)
    with open(STAMP_PATH, "w") as fh:
        fh.write(sources_hash() + "\n")
    if verbose:
        print("linked", os.path.relpath(LIB_PATH, ROOT))
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--check", action="store_true",
                    help="only report whether the built library matches the sources (exit 1 if not)")
    a = ap.parse_args(argv)
    if a.check:
        ok = is_current()
        print("libzipfft_b200.so is " + ("current" if ok else "STALE: rebuild with python -m zipfft_b200.build"))
        return 0 if ok else 1
    build(force=a.force, jobs=a.jobs, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
