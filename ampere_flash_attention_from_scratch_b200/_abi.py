"""ctypes view of the C ABI in include/afa_sm100.h (libafa_sm100.so).

This is the binding a non-torch caller would write (cgo / JNI / ctypes all bind
the same ``extern "C"`` symbols); the torch extension is the other caller.  The
structure layout below must match ``AfaFwdArgs`` field for field.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libafa_sm100.so"

AFA_DTYPE_FP16 = 5
AFA_DTYPE_BF16 = 15

AFA_OK = 0
AFA_ERR_INVALID_ARGUMENT = 1
AFA_ERR_UNSUPPORTED_DTYPE = 2
AFA_ERR_NO_KERNEL = 3
AFA_ERR_MISALIGNED = 4
AFA_ERR_NO_DEVICE = 5
AFA_ERR_ARCH = 6
AFA_ERR_TENSOR_MAP = 7
AFA_ERR_LAUNCH = 8
AFA_ERR_DEVICE_TIMEOUT = 9
AFA_ERR_TOO_LARGE = 10
AFA_ERR_SCRATCH_LIMIT = 11
AFA_DEV_TIMEOUT_BASE = 0x100
AFA_NOALLOC_SCRATCH_BYTES = 256
AFA_TEST_PRODUCER_IDLE = 1
AFA_TEST_MMA_IDLE = 2
AFA_TEST_KEEP_SCHED = 4

# Every extern "C" symbol declared in include/afa_sm100.h.
EXPORTED_SYMBOLS = (
    "afa_fwd_sm100",
    "afa_fwd_sm100_noalloc",
    "afa_strerror",
    "afa_status_string",
    "afa_fwd_sm100_supported",
    "afa_fwd_sm100_smem_bytes",
    "afa_fwd_sm100_threads",
    "afa_sm100_version",
)


class AfaFwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("q_strides", ctypes.c_int64 * 3),
        ("k_strides", ctypes.c_int64 * 3),
        ("v_strides", ctypes.c_int64 * 3),
        ("o_strides", ctypes.c_int64 * 3),
        ("batch", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("n_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_uint64),
        ("test_flags", ctypes.c_uint32),
        ("seq_len_kv", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("lse", ctypes.c_void_p),
        ("sched", ctypes.c_void_p),
    ]


_lib = None


def load() -> ctypes.CDLL:
    """Load libafa_sm100.so (raises OSError with the path if it is not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OSError(f"{LIB_PATH} is not built; run `python -m ampere_flash_attention_from_scratch_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.afa_fwd_sm100.argtypes = [ctypes.POINTER(AfaFwdArgs), ctypes.c_void_p]
        lib.afa_fwd_sm100.restype = ctypes.c_int
        lib.afa_fwd_sm100_noalloc.argtypes = [ctypes.POINTER(AfaFwdArgs), ctypes.c_void_p]
        lib.afa_fwd_sm100_noalloc.restype = ctypes.c_int
        lib.afa_strerror.argtypes = [ctypes.c_int]
        lib.afa_strerror.restype = ctypes.c_char_p
        lib.afa_status_string.argtypes = [ctypes.c_int32]
        lib.afa_status_string.restype = ctypes.c_char_p
        lib.afa_fwd_sm100_supported.argtypes = [ctypes.c_int32, ctypes.c_int32]
        lib.afa_fwd_sm100_supported.restype = ctypes.c_int
        lib.afa_fwd_sm100_smem_bytes.argtypes = [ctypes.c_int32, ctypes.c_int32]
        lib.afa_fwd_sm100_smem_bytes.restype = ctypes.c_int
        lib.afa_fwd_sm100_threads.argtypes = []
        lib.afa_fwd_sm100_threads.restype = ctypes.c_int
        lib.afa_sm100_version.argtypes = []
        lib.afa_sm100_version.restype = ctypes.c_int
        _lib = lib
    return _lib


def make_args(q, k, v, o, status=None, scale=0.0, timeout_ns=0, test_flags=0, causal=False,
              lse=None, sched=None) -> AfaFwdArgs:
    """AfaFwdArgs for torch tensors q, o [B, N, H, d] and k, v [B, N_kv, H_kv, d]
    (device memory); lse: optional fp32 [B, H, N] tensor."""
    dt = {"torch.float16": AFA_DTYPE_FP16, "torch.bfloat16": AFA_DTYPE_BF16}.get(str(q.dtype), -1)
    a = AfaFwdArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    for name, t in (("q_strides", q), ("k_strides", k), ("v_strides", v), ("o_strides", o)):
        getattr(a, name)[:] = [t.stride(0), t.stride(1), t.stride(2)]
    a.batch, a.seq_len, a.n_heads, a.head_dim = (int(x) for x in q.shape)
    a.dtype = dt
    a.scale = float(scale)
    a.status = status.data_ptr() if status is not None else None
    a.timeout_ns = int(timeout_ns)
    a.test_flags = int(test_flags)
    a.seq_len_kv, a.n_kv_heads = int(k.shape[1]), int(k.shape[2])
    a.causal = 1 if causal else 0
    a.lse = lse.data_ptr() if lse is not None else None
    a.sched = sched.data_ptr() if sched is not None else None
    return a


def strerror(code: int) -> str:
    return load().afa_strerror(int(code)).decode()
