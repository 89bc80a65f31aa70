"""Build ``libsmat_b200.so`` in-tree with nvcc for sm_100a.

    python -m smat_attention_b200.build        # builds if sources are newer

The library is a plain C-ABI shared object (``include/smat_b200.h``) with the
CUDA runtime linked statically, so it loads in any process that has the NVIDIA
driver, with or without torch.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libsmat_b200.so")
SOURCES = ["smat_abi.cu", "noalloc.cu", "selftest.cu", "rows.cu", "lm_ops.cu", "decode.cu",
           "kattn.cu", "kattn_glue.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or add CUDA's bin directory to PATH)")


def _inputs():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)
             if f.endswith((".cu", ".cuh", ".h"))]
    files.append(os.path.join(ROOT, "include", "smat_b200.h"))
    files.append(os.path.join(ROOT, "include", "smat_lm.h"))
    files.append(os.path.join(ROOT, "include", "smat_kattn.h"))
    files.append(os.path.abspath(__file__))
    return files


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(f) > t for f in _inputs())


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    """Compile the library if any source is newer than it; returns its path."""
    if not force and not needs_build():
        return LIB
    cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "--expt-relaxed-constexpr", "-cudart", "static",
           "-I", os.path.join(ROOT, "include"),
           *extra, *[os.path.join(CSRC, s) for s in SOURCES], "-o", LIB + ".tmp"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else [])
    print(LIB)
