"""Builds the two native artefacts of the package, in-tree:

* ``libafa_sm100.so``  -- the sm_100a kernels and the C ABI (include/afa_sm100.h),
  compiled by nvcc with ``-gencode arch=compute_100a,code=sm_100a``.  No torch
  dependency; cudart is linked statically so the library loads on machines
  without a GPU or driver.
* ``afa_flash_attention_kernels<EXT_SUFFIX>`` -- the torch extension that
  mirrors the reference binding's ``forward(kernel_cfg, q, k, v, o, benchmark)``
  (csrc/ampere_flash_attention.cu:138-151), compiled by g++ against torch's
  headers and linked to ``libafa_sm100.so`` through an ``$ORIGIN`` rpath.

Replaces the reference's setup.py (setup.py:15-84): sm_100a instead of sm_80,
no ``--keep`` (no compiler intermediates are written), ``-lineinfo`` for
profiling.  Outputs are rebuilt only when a source is newer.

Usage: python -m ampere_flash_attention_from_scratch_b200.build [--force]
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"

LIB_NAME = "libafa_sm100.so"
EXT_NAME = "afa_flash_attention_kernels"

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-warn-spills",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _cxx() -> str:
    # The system g++ is used even when $CXX names a wrapper: a wrapper that swaps
    # in its own libgcc/crt objects (-B...) breaks C++ exceptions thrown through
    # torch's error macros (TORCH_CHECK with formatted messages segfaults).
    return "/usr/bin/g++" if Path("/usr/bin/g++").exists() else os.environ.get("CXX", "g++")


def _stale(out: Path, sources) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(s).stat().st_mtime > t for s in sources)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed ({res.returncode}):\n{' '.join(map(str, cmd))}\n{res.stdout}\n{res.stderr}")
    return res


def generate_presets() -> Path:
    sys.path.insert(0, str(CSRC))
    try:
        import generate_preset_kernels  # noqa: WPS433 (build-time script beside the sources)

        return generate_preset_kernels.main()
    finally:
        sys.path.pop(0)


def library_path() -> Path:
    return PKG / LIB_NAME


def extension_path() -> Path:
    return PKG / (EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def build_library(force: bool = False, verbose: bool = False) -> Path:
    inc = generate_presets()
    out = library_path()
    sources = [
        CSRC / "afa_fwd_sm100.cu",
        CSRC / "afa_fwd_kernel.cuh",
        CSRC / "sm100_ptx.cuh",
        inc,
        INCLUDE / "afa_sm100.h",
    ]
    if force or _stale(out, sources):
        tmp = out.with_suffix(".so.tmp")
        cmd = [_nvcc(), *NVCC_FLAGS, "-shared", f"-I{INCLUDE}", f"-I{CSRC}", "-o", tmp, CSRC / "afa_fwd_sm100.cu"]
        _run(cmd, verbose)
        os.replace(tmp, out)
    return out


def build_extension(force: bool = False, verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    lib = build_library(force=force, verbose=verbose)
    out = extension_path()
    sources = [CSRC / "afa_torch_binding.cpp", INCLUDE / "afa_sm100.h", lib]
    if not (force or _stale(out, sources)):
        return out
    cuda_home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    includes = [*cpp_extension.include_paths(), str(cuda_home / "include"), str(INCLUDE), sysconfig.get_paths()["include"]]
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        _cxx(),
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        "-w",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        *[f"-I{p}" for p in includes],
        CSRC / "afa_torch_binding.cpp",
        "-o",
        out.with_suffix(".tmp"),
        f"-L{PKG}",
        "-l:" + LIB_NAME,
        f"-L{torch_lib}",
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_cuda",
        "-ltorch_python",
        f"-L{cuda_home / 'lib64'}",
        "-lcudart",
        "-Wl,-rpath,$ORIGIN",
        f"-Wl,-rpath,{torch_lib}",
    ]
    _run(cmd, verbose)
    os.replace(out.with_suffix(".tmp"), out)
    return out


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_extension(force=force, verbose=verbose)  # builds the library first


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
