"""The torch extension `afa_flash_attention_kernels` on a machine without a GPU:
it imports, exposes the reference's call surface and raises RuntimeError with
the reference's messages for inputs it rejects before launching."""

import pytest
import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig


def test_surface():
    assert callable(fa.forward)
    doc = fa.forward.__doc__
    for kw in ("kernel_cfg", "q", "k", "v", "o", "benchmark"):
        assert kw in doc
    assert sorted(fa.kernel_keys()) == [(5, 64), (5, 128), (15, 64), (15, 128)]


def test_cpu_tensors_rejected():
    q = torch.randn(1, 128, 1, 128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        fa.forward(AFAForwardKernelConfig(), q, q, q, None, False)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        fa.forward(kernel_cfg=AFAForwardKernelConfig(), q=q, k=q, v=q, o=None, benchmark=True)


def test_formatted_errors_cross_the_binding():
    with pytest.raises(RuntimeError, match="formatted error 3 / 4"):
        fa._raise_formatted_error(3, 4)


def test_package_exports_forward():
    import ampere_flash_attention_from_scratch_b200 as pkg

    assert pkg.forward is fa.forward


def test_forward_ext_rejects_host_tensors():
    q = torch.randn(1, 128, 2, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        fa.forward_ext(q, q, q)


def _h(*shape, dtype=torch.float16):
    return torch.zeros(*shape, dtype=dtype)


@pytest.mark.parametrize("args,match", [
    ((_h(1, 64, 2, 64).transpose(1, 2), _h(1, 64, 2, 64), _h(1, 64, 2, 64)), "contiguous"),
    ((_h(1, 64, 2, 64, dtype=torch.float32),) * 3, "Only fp16 and bf16"),
    ((_h(1, 64, 2, 64), _h(1, 64, 2, 64, dtype=torch.bfloat16), _h(1, 64, 2, 64)), "same data type"),
    ((_h(1, 64, 2, 64), _h(1, 64, 2, 64), _h(1, 32, 2, 64)), "key and value tensors must have the same shape"),
    ((_h(1, 64, 2, 64), _h(2, 64, 2, 64), _h(2, 64, 2, 64)), "batch / head_dim differ"),
    ((_h(1, 64, 3, 64), _h(1, 64, 2, 64), _h(1, 64, 2, 64)), "multiple of the number of key/value heads"),
    ((_h(1, 64, 2, 96),) * 3, "no sm_100a kernel for head_dim"),
    ((_h(1, 0, 2, 64),) * 3, "must be positive"),
])
def test_forward_host_rejects_before_any_cuda_call(args, match):
    """forward_host checks its host tensors before touching the device, so the
    same messages appear on a machine without a GPU."""
    with pytest.raises(RuntimeError, match=match):
        fa.forward_host(*args)


def test_forward_host_requires_a_page_locked_output():
    """A copy into pageable memory returns only when it has finished, which would
    serialise the slices' copies behind the kernels: such an `o` is refused."""
    q = _h(1, 64, 2, 64)
    with pytest.raises(RuntimeError, match="o must be page-locked"):
        fa.forward_host(q, q, q, _h(1, 64, 2, 64))


def test_forward_host_rejects_a_mismatched_output():
    q = _h(1, 64, 2, 64)
    with pytest.raises(RuntimeError, match="o must be a contiguous host tensor"):
        fa.forward_host(q, q, q, _h(1, 64, 2, 32))
    with pytest.raises(RuntimeError, match="o must be a contiguous host tensor"):
        fa.forward_host(q, q, q, _h(1, 64, 2, 64, dtype=torch.bfloat16))
