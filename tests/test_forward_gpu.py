"""GPU parity of the sm_100a forward kernel against the CPU fp32 oracle.

Calls go through the reference-facing API (afa_flash_attention_kernels.forward,
which calls the C ABI afa_fwd_sm100 in libafa_sm100.so).  Tolerances, written
per dtype below, are the north star's for fp16 (max-abs <= 1e-2, mean-abs
<= 1e-3, demo.py:61-72 of the reference uses the same max-abs bound) and twice
that for bf16 (bf16 rounding of P and O is 8x coarser than fp16's).
"""

import math

import pytest
import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig, DType
from ampere_flash_attention_from_scratch_b200.workloads import WORKLOADS, make_inputs
from oracle.attention_oracle import attention_fp32, error_stats

pytestmark = pytest.mark.gpu

TOL = {torch.float16: (1e-2, 1e-3), torch.bfloat16: (2e-2, 2e-3)}


def cfg_for(dtype, d):
    return AFAForwardKernelConfig(dtype=DType.FP16 if dtype == torch.float16 else DType.BF16, d_head=d)


def rand_qkv(B, N, H, d, dtype, sigma_qk=1.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, N, H, d, generator=g) * sigma_qk).to(dtype)
    k = (torch.randn(B, N, H, d, generator=g) * sigma_qk).to(dtype)
    v = torch.randn(B, N, H, d, generator=g).to(dtype)
    return q, k, v


def run_forward(q, k, v, o=None, benchmark=False):
    dev = torch.device("cuda:0")
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    out, ms = fa.forward(cfg_for(q.dtype, q.shape[-1]), qd, kd, vd, o, benchmark)
    torch.cuda.synchronize()
    fa.check_status(0)
    return out, ms


def assert_close(out, ref, dtype, what=""):
    mx, mean = error_stats(out, ref)
    tmax, tmean = TOL[dtype]
    assert mx <= tmax and mean <= tmean, f"{what} max-abs {mx:.3e} (tol {tmax}), mean-abs {mean:.3e} (tol {tmean})"


SMALL = [
    (1, 128, 1, 128, torch.float16),
    (1, 256, 2, 64, torch.bfloat16),
    (2, 384, 3, 128, torch.float16),
    (2, 512, 2, 64, torch.float16),
    (1, 1024, 2, 128, torch.bfloat16),
]


@pytest.mark.parametrize("B,N,H,d,dtype", SMALL)
def test_small_shapes(B, N, H, d, dtype):
    q, k, v = rand_qkv(B, N, H, d, dtype, seed=B * 1000 + N + d)
    out, _ = run_forward(q, k, v)
    assert out.shape == q.shape and out.dtype == dtype
    assert_close(out, attention_fp32(q, k, v), dtype)


@pytest.mark.parametrize("N", [1, 7, 100, 129, 200, 255, 257, 1000])
@pytest.mark.parametrize("d,dtype", [(128, torch.float16), (64, torch.bfloat16)])
def test_ragged_seq_len(N, d, dtype):
    """seq_len not a multiple of the 128-row tiles (TMA zero-fill + column mask)."""
    q, k, v = rand_qkv(2, N, 2, d, dtype, seed=N)
    out, _ = run_forward(q, k, v)
    assert_close(out, attention_fp32(q, k, v), dtype, f"N={N}")


def test_cfg1_full():
    wl = WORKLOADS["cfg1"]
    q, k, v = make_inputs(wl, seed=42)
    out, _ = run_forward(q, k, v)
    assert_close(out, attention_fp32(q, k, v), wl.dtype, "cfg1")


def test_cfg2_sampled_slices():
    wl = WORKLOADS["cfg2"]
    q, k, v = make_inputs(wl, seed=42)
    out, _ = run_forward(q, k, v)
    g = torch.Generator().manual_seed(1)
    pairs = [(int(torch.randint(wl.batch, (1,), generator=g)), int(torch.randint(wl.n_heads, (1,), generator=g))) for _ in range(6)]
    ref = attention_fp32(q, k, v, slices=pairs)
    got = torch.stack([out[b, :, h, :].cpu() for b, h in pairs])
    assert_close(got, ref, wl.dtype, "cfg2 slices")


def test_wide_softmax_bf16_d64():
    """cfg5's value distribution (Q, K ~ N(0, 3)) at a CPU-checkable size."""
    q, k, v = rand_qkv(2, 2048, 2, 64, torch.bfloat16, sigma_qk=3.0, seed=5)
    out, _ = run_forward(q, k, v)
    assert_close(out, attention_fp32(q, k, v), torch.bfloat16, "wide softmax")


@pytest.mark.parametrize("dtype,d", [(torch.float16, 128), (torch.bfloat16, 64)])
def test_strided_views(dtype, d):
    """Head-sliced views of a wider tensor and a [B, H, N, d] tensor viewed as [B, N, H, d]."""
    B, N, H = 2, 320, 3
    big = torch.randn(B, N, 2 * H, d).to(dtype)
    q = big[:, :, H:]
    bhnd = torch.randn(B, H, N, d).to(dtype)
    k = bhnd.transpose(1, 2)
    v = torch.randn(B, N, H, d).to(dtype)
    dev = torch.device("cuda:0")
    qd = big.to(dev)[:, :, H:]
    kd = bhnd.to(dev).transpose(1, 2)
    vd = v.to(dev)
    assert not qd.is_contiguous() and not kd.is_contiguous()
    out, _ = fa.forward(cfg_for(dtype, d), qd, kd, vd, None, False)
    torch.cuda.synchronize()
    fa.check_status(0)
    assert_close(out, attention_fp32(q, k, v), dtype, "strided")


def test_output_buffer_in_place_and_strided():
    q, k, v = rand_qkv(1, 256, 2, 128, torch.float16, seed=3)
    dev = torch.device("cuda:0")
    big = torch.full((1, 256, 4, 128), 7.0, dtype=torch.float16, device=dev)
    o = big[:, :, 1:3]
    out, _ = fa.forward(cfg_for(torch.float16, 128), q.to(dev), k.to(dev), v.to(dev), o, False)
    torch.cuda.synchronize()
    assert out.data_ptr() == o.data_ptr()
    assert_close(o, attention_fp32(q, k, v), torch.float16, "strided o")
    assert torch.all(big[:, :, 0] == 7.0) and torch.all(big[:, :, 3] == 7.0), "wrote outside o"


def test_benchmark_timing_and_default_config():
    """The reference's call pattern: default config, benchmark=True returns a positive ms."""
    q, k, v = rand_qkv(2, 1024, 4, 128, torch.float16, seed=9)
    dev = torch.device("cuda:0")
    o = torch.empty_like(q, device=dev)
    out, ms = fa.forward(AFAForwardKernelConfig(), q.to(dev), k.to(dev), v.to(dev), o, True)
    assert ms > 0.0 and math.isfinite(ms)
    out2, ms2 = fa.forward(AFAForwardKernelConfig(), q.to(dev), k.to(dev), v.to(dev), None, False)
    torch.cuda.synchronize()
    assert ms2 == 0.0
    assert torch.equal(out, out2), "not deterministic"


def test_config_mismatch_errors():
    q = torch.randn(1, 128, 1, 128, device="cuda:0").to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="dtype does not match"):
        fa.forward(AFAForwardKernelConfig(), q, q, q, None, False)
    q16 = q.to(torch.float16)
    with pytest.raises(RuntimeError, match="not found"):
        fa.forward(AFAForwardKernelConfig(d_head=96), q16, q16, q16, None, False)
    k = torch.randn(1, 256, 1, 128, device="cuda:0").to(torch.float16)
    with pytest.raises(RuntimeError, match="same shape"):
        fa.forward(AFAForwardKernelConfig(), q16, k, q16, None, False)
