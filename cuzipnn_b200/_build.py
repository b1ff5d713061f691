"""Build the CUDA library libcuzipnn_b200.so in the package folder (sm_100a only).

The library is plain CUDA C++ behind the C ABI of include/cuzipnn_b200.h; nvcc cross-compiles it
without a GPU.  The package loads it with ctypes; there is no JIT cache and no fallback.
"""

from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys
import tempfile

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libcuzipnn_b200.so")
SOURCES = ["zn_api.cu", "zn_planes.cu", "zn_crc32.cu", "zn_encode.cu", "zn_decode.cu"]
HEADERS = ["zn_common.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "-shared", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "cuzipnn_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; returns its path.  The translation
    units compile in parallel into a temporary folder, then link into the package folder."""
    if not force and not _stale():
        return LIB
    nvcc = _nvcc()
    compile_flags = [f for f in FLAGS if f != "-shared"]
    with tempfile.TemporaryDirectory() as tmp:
        cmds = [[nvcc, *ARCH, *compile_flags, "-c", os.path.join(CSRC, f), "-o", os.path.join(tmp, f + ".o")]
                for f in SOURCES]
        if verbose:
            for c in cmds:
                print(" ".join(c), file=sys.stderr)
        with concurrent.futures.ThreadPoolExecutor(len(cmds)) as ex:
            for r in ex.map(lambda c: subprocess.run(c), cmds):
                if r.returncode:
                    raise subprocess.CalledProcessError(r.returncode, r.args)
        link = [nvcc, *ARCH, "-shared", "-o", LIB + ".tmp", *[os.path.join(tmp, f + ".o") for f in SOURCES]]
        if verbose:
            print(" ".join(link), file=sys.stderr)
        subprocess.run(link, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
