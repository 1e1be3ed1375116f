"""Build the reference's own CUDA extensions for sm_100a into ``oracle/_ref/``.

TEST AND BENCH INFRASTRUCTURE ONLY: nothing in ``dc_triton_opt_b200`` imports
what this builds.  It compiles, from the sources where they lie in the
reference checkout (never copied into this repository):

  * ``dc_fused_cuda/kernel.cu`` -> module ``dc_fused_cuda``: the reference's
    CUDA port of its one-kernel V4 (``dc_onekernel_v4_cache4_kernel``,
    kernel.cu:1223-1342, binding ``onekernel_v4_forward`` kernel.cu:1350-1431);
    WMMA (mma.sync) tensor cores, fp16, HPG 4/8, BM+W <= 128.
  * ``dc_hopper_cuda/dc_hopper_api.cpp`` + ``dc_hopper_kernel.cu`` -> module
    ``_dc_hopper_cuda``: the HPG=4 wide-window kernels
    (``forward_hpg4_wide_ref`` scalar, ``forward_hpg4_wide_opt`` WMMA,
    dc_hopper_kernel.cu:639-760), BM16/W240 or BM32/W224.

with the reference's own compiler flags (``-O3 --use_fast_math -lineinfo``,
setup.py of each package) and the B200 target in place of sm_80 / sm_90a.
The built ``.so`` files are git-ignored and travel with the tree to the GPU
host, where ``bench.py`` (``repo_best`` block) times them beside this library
and ``tests/test_ref_kernels.py`` checks them against the oracle.  The
reference's Triton kernels are Python sources, which do not travel, so they
are not timed.

    python -m oracle.build_ref [--reference PATH]
"""

from __future__ import annotations

import argparse
import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
DEFAULT_REF = "/root/reference"

MODULES = {
    "dc_fused_cuda": ["dc_fused_cuda/kernel.cu"],
    "_dc_hopper_cuda": ["dc_hopper_cuda/dc_hopper_api.cpp", "dc_hopper_cuda/dc_hopper_kernel.cu"],
}
NVCC_FLAGS = ["-O3", "--use_fast_math", "-lineinfo", "--threads=4",
              "-gencode=arch=compute_100a,code=sm_100a"]


def built(name: str) -> str | None:
    """Path of the built module's directory if its .so exists, else None."""
    d = os.path.join(OUT, name)
    return d if glob.glob(os.path.join(d, f"{name}*.so")) else None


def import_module(name: str):
    """Import a built reference module from oracle/_ref (raises ImportError if absent)."""
    d = built(name)
    if d is None:
        raise ImportError(f"{name} not built (run python -m oracle.build_ref where the reference is present)")
    if d not in sys.path:
        sys.path.insert(0, d)
    import importlib

    import torch  # noqa: F401  (loads libc10 / libtorch the module links against)
    return importlib.import_module(name)


def build(ref: str = DEFAULT_REF, verbose: bool = False) -> list[str]:
    """Compile every module whose sources exist under `ref`; returns the names built."""
    from torch.utils import cpp_extension
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    done = []
    for name, rel in MODULES.items():
        srcs = [os.path.join(ref, r) for r in rel]
        if not all(os.path.exists(s) for s in srcs):
            continue
        bdir = os.path.join(OUT, name)
        os.makedirs(bdir, exist_ok=True)
        cpp_extension.load(name=name, sources=srcs, build_directory=bdir, extra_cflags=["-O3"],
                           extra_cuda_cflags=NVCC_FLAGS, verbose=verbose, is_python_module=True)
        done.append(name)
    return done


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REF)
    a = ap.parse_args()
    print(build(a.reference, verbose=True))
