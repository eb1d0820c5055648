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
