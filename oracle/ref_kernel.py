"""ctypes loader for oracle/_ref/libafa_ref_ampere.so -- TEST INFRASTRUCTURE ONLY.

Runs the reference's own Ampere kernel (PTX JIT-compiled on the B200) so tests
can compare the sm_100a kernel with the reference's output on the same inputs.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB = Path(__file__).resolve().parent / "_ref" / "libafa_ref_ampere.so"

# config ids of ref_kernel_shim.cu: (dtype name, d_head, B_r, B_c)
CONFIGS = {
    0: ("fp16", 128, 64, 32),   # the reference's default AFAForwardKernelConfig()
    1: ("fp16", 128, 128, 64),  # B_r=128, B_c=64, 8 warps
    2: ("bf16", 64, 64, 32),    # same template, bf16 / d=64
}

_lib = None


def available() -> bool:
    return LIB.exists()


def load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(LIB))
        lib.afa_ref_forward.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
        lib.afa_ref_forward.restype = ctypes.c_int
        _lib = lib
    return _lib


def forward(config: int, q, k, v, o, stream=None) -> None:
    """Launch the reference kernel on contiguous CUDA tensors [B, N, H, d]; raises on error."""
    import torch

    for t in (q, k, v, o):
        assert t.is_cuda and t.is_contiguous()
    B, N, H, _ = q.shape
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    rc = load().afa_ref_forward(config, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, N, H, stream)
    if rc != 0:
        raise RuntimeError(f"reference kernel launch failed with code {rc}")
