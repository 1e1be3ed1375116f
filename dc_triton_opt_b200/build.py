"""Build the in-tree CUDA library ``libdcattn.so`` for sm_100a with nvcc.

    python -m dc_triton_opt_b200.build        # or: import and call build()

The library is the C ABI declared in ``include/dc_attn.h``; the Python layer
loads it with ctypes.  Built artefacts stay in the package directory (they are
git-ignored but travel with the source tree to the GPU host).
"""

from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libdcattn.so")
SOURCES = ["capi.cu", "simt_kernel.cu", "tc_kernel.cu", "tcs_kernel.cu", "tcm_kernel.cu", "bwd_kernel.cu", "proj_kernel.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def nvcc_flags(debug: bool = False):
    flags = [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-std=c++17", "-O3", "-lineinfo",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        "-I", os.path.join(ROOT, "include"),
    ]
    if os.environ.get("DC_PTXAS_VERBOSE"):
        flags += ["-Xptxas", "-v"]
    if debug:
        flags += ["-DDC_DEBUG=1"]
    return flags


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu into an object and link libdcattn.so; returns its path."""
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "dc_attn.h"))
    objs, cmds = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmds.append([NVCC, *nvcc_flags(), "-c", s, "-o", o])
    # the translation units are independent: compile them concurrently
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for cmd in cmds:
            if verbose:
                print(" ".join(cmd), flush=True)
        for f in [ex.submit(subprocess.run, cmd, check=True) for cmd in cmds]:
            f.result()
    if force or _stale(LIB, objs):
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *objs, "-o", LIB,
               "-lcuda", "-Xcompiler", "-fPIC"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
