"""The sm_100a kernel against the reference's own kernel on the B200.

The reference kernel (oracle/_ref, JIT-compiled from compute_80 PTX) and the
sm_100a kernel run on the same inputs; both are checked against the fp32
oracle and against each other with the fp16 tolerance of the north star.
"""

import pytest
import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig, DType
from oracle import ref_kernel
from oracle.attention_oracle import attention_fp32, error_stats

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not ref_kernel.available(), reason="oracle/_ref not built")]


@pytest.mark.parametrize("config,dtype,d,sigma", [(0, torch.float16, 128, 1.0), (1, torch.float16, 128, 1.0), (2, torch.bfloat16, 64, 3.0)])
def test_against_reference_kernel(config, dtype, d, sigma):
    g = torch.Generator().manual_seed(7 + config)
    B, N, H = 2, 1024, 4
    q = (torch.randn(B, N, H, d, generator=g) * sigma).to(dtype)
    k = (torch.randn(B, N, H, d, generator=g) * sigma).to(dtype)
    v = torch.randn(B, N, H, d, generator=g).to(dtype)
    qd, kd, vd = (t.cuda() for t in (q, k, v))
    o_ref = torch.empty_like(qd)
    ref_kernel.forward(config, qd, kd, vd, o_ref)
    cfg = AFAForwardKernelConfig(dtype=DType.FP16 if dtype == torch.float16 else DType.BF16, d_head=d)
    o_new, _ = fa.forward(cfg, qd, kd, vd, None, False)
    torch.cuda.synchronize()
    fa.check_status(0)
    oracle = attention_fp32(q, k, v)
    tol = (1e-2, 1e-3) if dtype == torch.float16 else (2e-2, 2e-3)
    for name, out in (("reference kernel", o_ref), ("sm_100a kernel", o_new)):
        mx, mean = error_stats(out, oracle)
        assert mx <= tol[0] and mean <= tol[1], f"{name} vs oracle: max {mx:.3e} mean {mean:.3e}"
    mx, mean = error_stats(o_new, o_ref)
    assert mx <= tol[0] and mean <= tol[1], f"sm_100a vs reference kernel: max {mx:.3e} mean {mean:.3e}"
