"""The C ABI of libafa_sm100.so, checked without a GPU.

* every function declared in include/afa_sm100.h is exported;
* the ctypes mirror of AfaFwdArgs has the C layout (compared with a program
  compiled by gcc from the header);
* argument errors come back as AFA_* codes before any CUDA call is made.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from ampere_flash_attention_from_scratch_b200 import _abi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "afa_sm100.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(afa_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected_symbols():
    assert declared_functions() == sorted(_abi.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _abi.load()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_struct_layout_matches_c(tmp_path):
    fields = [f for f, _ in _abi.AfaFwdArgs._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(AfaFwdArgs, {f}));' for f in fields)
    src.write_text(
        f'#include <stdio.h>\n#include <stddef.h>\n#include "afa_sm100.h"\nint main(void) {{\n'
        f'  printf("sizeof %zu\\n", sizeof(AfaFwdArgs));\n{body}\n  return 0;\n}}\n'
    )
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines())
    assert int(out["sizeof"]) == ctypes.sizeof(_abi.AfaFwdArgs)
    for f in fields:
        assert int(out[f]) == getattr(_abi.AfaFwdArgs, f).offset, f


def test_header_compiles_as_cxx(tmp_path):
    src = tmp_path / "h.cpp"
    src.write_text('#include "afa_sm100.h"\nint main() { return afa_sm100_version() > 0 ? 0 : 1; }\n')
    subprocess.run(["g++", "-std=c++17", "-c", f"-I{ROOT / 'include'}", str(src), "-o", str(tmp_path / "h.o")], check=True)


def valid_args(**over):
    a = _abi.AfaFwdArgs()
    a.q = a.k = a.v = a.o = 0x100000
    for name in ("q_strides", "k_strides", "v_strides", "o_strides"):
        getattr(a, name)[:] = [1024 * 4 * 128, 4 * 128, 128]
    a.batch, a.seq_len, a.n_heads, a.head_dim = 2, 1024, 4, 128
    a.dtype = _abi.AFA_DTYPE_FP16
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize(
    "over,code",
    [
        ({"dtype": 7}, _abi.AFA_ERR_UNSUPPORTED_DTYPE),
        ({"head_dim": 96}, _abi.AFA_ERR_NO_KERNEL),
        ({"head_dim": 256}, _abi.AFA_ERR_NO_KERNEL),
        ({"q": None}, _abi.AFA_ERR_INVALID_ARGUMENT),
        ({"o": None}, _abi.AFA_ERR_INVALID_ARGUMENT),
        ({"batch": 0}, _abi.AFA_ERR_INVALID_ARGUMENT),
        ({"seq_len": -1}, _abi.AFA_ERR_INVALID_ARGUMENT),
        ({"n_heads": 0}, _abi.AFA_ERR_INVALID_ARGUMENT),
        ({"k": 0x100008}, _abi.AFA_ERR_MISALIGNED),
        ({"batch": 1 << 20, "n_heads": 1 << 10, "seq_len": 1 << 20}, _abi.AFA_ERR_TOO_LARGE),
        # extension fields
        ({"n_kv_heads": 3}, _abi.AFA_ERR_INVALID_ARGUMENT),  # does not divide n_heads = 4
        ({"n_kv_heads": -1}, _abi.AFA_ERR_INVALID_ARGUMENT),
        ({"seq_len_kv": -5}, _abi.AFA_ERR_INVALID_ARGUMENT),
        ({"causal": 2}, _abi.AFA_ERR_INVALID_ARGUMENT),
        ({"lse": 0x100002}, _abi.AFA_ERR_MISALIGNED),
        ({"sched": 0x100004}, _abi.AFA_ERR_MISALIGNED),
        ({"seq_len_kv": (1 << 31) - 100}, _abi.AFA_ERR_TOO_LARGE),
    ],
)
def test_argument_errors_without_gpu(over, code):
    lib = _abi.load()
    assert lib.afa_fwd_sm100(ctypes.byref(valid_args(**over)), None) == code


def test_misaligned_stride_rejected():
    lib = _abi.load()
    a = valid_args()
    a.v_strides[1] = 4 * 128 + 4
    assert lib.afa_fwd_sm100(ctypes.byref(a), None) == _abi.AFA_ERR_MISALIGNED
    a = valid_args(n_heads=1)
    a.v_strides[2] = 3  # unused stride of a size-1 dimension is ignored
    rc = lib.afa_fwd_sm100(ctypes.byref(a), None)
    assert rc != _abi.AFA_ERR_MISALIGNED


def test_kv_strides_checked_against_kv_shape():
    lib = _abi.load()
    # K/V with one head (GQA): the K head stride is never used, so any value passes
    # the alignment check; a bad K seq stride is still caught.
    a = valid_args(n_kv_heads=1, seq_len_kv=300)
    a.k_strides[:] = [300 * 128, 128, 3]
    a.v_strides[:] = [300 * 128, 128, 3]
    assert lib.afa_fwd_sm100(ctypes.byref(a), None) not in (_abi.AFA_ERR_MISALIGNED, _abi.AFA_ERR_INVALID_ARGUMENT)
    a.k_strides[1] = 130
    assert lib.afa_fwd_sm100(ctypes.byref(a), None) == _abi.AFA_ERR_MISALIGNED


def test_null_args_pointer():
    assert _abi.load().afa_fwd_sm100(None, None) == _abi.AFA_ERR_INVALID_ARGUMENT


def test_strings_and_queries():
    lib = _abi.load()
    assert _abi.strerror(0) == "success"
    assert "not found" in _abi.strerror(_abi.AFA_ERR_NO_KERNEL)
    assert _abi.strerror(12345) == "unknown error"
    assert lib.afa_status_string(0) == b"ok"
    assert b"timeout" in lib.afa_status_string(_abi.AFA_DEV_TIMEOUT_BASE + 8)
    assert lib.afa_fwd_sm100_supported(5, 128) == 1 and lib.afa_fwd_sm100_supported(15, 64) == 1
    assert lib.afa_fwd_sm100_supported(5, 96) == 0
    assert 0 < lib.afa_fwd_sm100_smem_bytes(5, 128) <= 232448
    assert lib.afa_fwd_sm100_smem_bytes(5, 96) == -1
    assert lib.afa_fwd_sm100_threads() in (384, 512)  # 512 with the correction warpgroup
    assert lib.afa_sm100_version() == 300
