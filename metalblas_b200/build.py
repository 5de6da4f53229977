"""Build the sm_100a shared library in-tree (nvcc, no JIT cache).

The library is one CUDA translation unit (``csrc/mb_abi.cu``) exporting the C ABI
declared in ``include/metalblas_b200.h``; a small torch C++ extension
(``csrc/fastpath.cpp``) holds the per-thread descriptor cache of repeated calls.  It links the CUDA runtime statically
so it does not depend on which libcudart torch happened to load, and reaches the
driver (for cuTensorMapEncodeTiled) through cudaGetDriverEntryPoint, so it needs
no libcuda at link time.

    python -m metalblas_b200.build [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_DIR)
SRC = os.path.join(PKG_DIR, "csrc", "mb_abi.cu")
LIB = os.path.join(PKG_DIR, "libmetalblas_b200.so")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def sources() -> list[str]:
    csrc = os.path.join(PKG_DIR, "csrc")
    files = [os.path.join(csrc, f) for f in sorted(os.listdir(csrc)) if f.endswith((".cu", ".cuh"))]
    return files + [os.path.join(REPO, "include", "metalblas_b200.h"), __file__]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [
        nvcc_path(), "-std=c++17", "-O3", ARCH, "-lineinfo",
        "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
        "-I", os.path.join(REPO, "include"),
        "-o", LIB + ".tmp", SRC,
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


FAST_SRC = os.path.join(PKG_DIR, "csrc", "fastpath.cpp")


def fast_lib_path() -> str:
    import sysconfig
    return os.path.join(PKG_DIR, "_mbfast" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_fastpath(force: bool = False, verbose: bool = False) -> str:
    """Compile the host fast path (csrc/fastpath.cpp, a torch C++ extension) in
    tree with g++: torch's headers and libraries, no CUDA device code."""
    import sysconfig

    import torch
    import torch.utils.cpp_extension as ce
    out = fast_lib_path()
    srcs = [FAST_SRC, os.path.join(REPO, "include", "metalblas_b200.h"), __file__]
    if not force and os.path.exists(out) and all(os.path.getmtime(s) <= os.path.getmtime(out) for s in srcs):
        return out
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = ["g++", "-O3", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-DTORCH_EXTENSION_NAME=_mbfast", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-I", sysconfig.get_paths()["include"], "-I", os.path.join(cuda_home, "include"),
           "-I", os.path.join(REPO, "include")]
    for inc in ce.include_paths():
        cmd += ["-I", inc]
    for lib in ce.library_paths():
        cmd += ["-L", lib, f"-Wl,-rpath,{lib}"]
    cmd += [FAST_SRC, "-o", out + ".tmp", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("g++ failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(out + ".tmp", out)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="pass -Xptxas -v (registers, spills)")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    print(build_fastpath(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
