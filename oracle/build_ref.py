"""Builds oracle/_ref/libafa_ref_ampere.so -- TEST INFRASTRUCTURE ONLY.

Compiles oracle/ref_kernel_shim.cu against the reference's own headers
(<reference>/csrc/include, read in place, never copied) with the reference's
nvcc flags (setup.py:15-51 of the reference) except: PTX only for compute_80
(``-gencode arch=compute_80,code=compute_80``) so the driver JIT-compiles the
Ampere kernel on the B200, and no ``--keep`` (no intermediates are written).
The output is git-ignored and travels to the GPU box as a built file.

Usage: python oracle/build_ref.py [--reference DIR] [--force]
The reference checkout comes from ``--reference`` / the ``reference`` argument,
else the ``AFA_REFERENCE_DIR`` environment variable; with neither given, or
when the directory holds no ``csrc/include``, nothing is built (returns None).
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libafa_ref_ampere.so"


def reference_dir(reference=None):
    """The reference checkout to build from: the argument, else $AFA_REFERENCE_DIR; None if neither."""
    if reference:
        return Path(reference)
    env = os.environ.get("AFA_REFERENCE_DIR")
    return Path(env) if env else None


def build(reference=None, force: bool = False, verbose: bool = False):
    ref = reference_dir(reference)
    if ref is None:
        return None
    inc = ref / "csrc" / "include"
    if not inc.is_dir():
        return None
    src = HERE / "ref_kernel_shim.cu"
    if OUT.exists() and not force and OUT.stat().st_mtime >= src.stat().st_mtime:
        return OUT
    import torch
    from torch.utils import cpp_extension

    OUT.parent.mkdir(parents=True, exist_ok=True)
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    cmd = [
        "/usr/local/cuda/bin/nvcc",
        "-std=c++20",
        "-O3",
        "--use_fast_math",
        "--expt-relaxed-constexpr",
        "-Xcudafe=--diag_suppress=3189",
        "-U__CUDA_NO_HALF_OPERATORS__",
        "-U__CUDA_NO_HALF_CONVERSIONS__",
        "-U__CUDA_NO_HALF2_OPERATORS__",
        "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
        "-gencode",
        "arch=compute_80,code=compute_80",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
        f"-I{inc}",
        *[f"-I{p}" for p in cpp_extension.include_paths()],
        str(src),
        "-o",
        str(OUT) + ".tmp",
        f"-L{torch_lib}",
        "-lc10",
        f"-Xlinker=-rpath,{torch_lib}",
    ]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference kernel build failed:\n{res.stdout}\n{res.stderr}")
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ref = sys.argv[sys.argv.index("--reference") + 1] if "--reference" in sys.argv else None
    out = build(ref, force="--force" in sys.argv, verbose=True)
    if out is None:
        sys.exit("no reference checkout: pass --reference DIR or set AFA_REFERENCE_DIR")
    print(out)
