"""Shapes that give every CTA of the persistent grid several work items.

The MMA warp issues the next item's first S = QK^T before the current item's
last PV (the unmasked kernel at both head dims, the causal kernel at head_dim
64, where the next item is read once from the dynamic queue and carried over),
and the softmax warps decode an unmasked item while they wait for its final O.
These paths only run when a CTA has a next item, which the small randomised
shapes never give (at most ~120 items for 148 CTAs).  Here: single-tile items
(N_kv <= 128, where the early S0 also releases Q tile 0's buffer), ragged key
lengths, GQA, head-major storage, and causal items whose Q tile 0 sees one
K/V tile; O and lse against the fp32 oracle."""

import pytest
import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig, DType
from oracle.attention_oracle import attention_fp32, error_stats

pytestmark = pytest.mark.gpu

TOL = {torch.float16: (1e-2, 1e-3), torch.bfloat16: (2e-2, 2e-3)}

# (B, N, N_kv, H, H_kv, d, dtype, causal, head_major); work items = B * H * ceil(N / 256)
CASES = [
    (2, 128, 128, 160, 160, 128, torch.float16, False, False),   # 320 single-tile items
    (1, 300, 77, 100, 100, 64, torch.bfloat16, False, False),    # 200 items, one ragged K/V tile
    (3, 256, 200, 64, 16, 64, torch.float16, False, True),       # 192 items, GQA 4:1, head-major
    (1, 1000, 1500, 64, 8, 128, torch.bfloat16, False, True),    # 256 items, 12 K/V tiles, GQA 8:1
    (2, 700, 700, 64, 64, 64, torch.float16, True, False),       # 384 causal items, d = 64
    (1, 520, 520, 96, 32, 64, torch.bfloat16, True, True),       # 288 causal items, GQA, head-major
    (1, 520, 520, 96, 96, 128, torch.float16, True, False),      # 288 causal items, d = 128
]


def _tensor(B, N, H, d, dtype, head_major, g):
    if head_major:  # storage [B, H, N, d], viewed as [B, N, H, d]
        return torch.randn(B, H, N, d, generator=g, device="cuda").to(dtype).transpose(1, 2)
    return torch.randn(B, N, H, d, generator=g, device="cuda").to(dtype)


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}N{}K{}H{}/{}d{}{}{}{}".format(
    c[0], c[1], c[2], c[3], c[4], c[5], "bf16" if c[6] == torch.bfloat16 else "fp16",
    "causal" if c[7] else "", "hm" if c[8] else ""))
def test_several_items_per_cta(case):
    B, N, NK, H, HK, d, dtype, causal, head_major = case
    assert B * H * ((N + 255) // 256) > 148  # more items than SMs
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + N + H)
    q = _tensor(B, N, H, d, dtype, head_major, g)
    k = _tensor(B, NK, HK, d, dtype, head_major, g)
    v = _tensor(B, NK, HK, d, dtype, head_major, g)
    out, lse = fa.forward_ext(q, k, v, None, causal, None, True)
    torch.cuda.synchronize()
    fa.check_status(0)
    ref, ref_lse = attention_fp32(q, k, v, causal=causal, return_lse=True)
    mx, mean = error_stats(out, ref)
    tmax, tmean = TOL[dtype]
    assert mx <= tmax and mean <= tmean, f"max-abs {mx:.3e} mean-abs {mean:.3e}"
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse), fin)
    if fin.any():
        assert (lse[fin] - ref_lse[fin]).abs().max().item() <= 1e-3
    # The reference entry point (non-causal, equal shapes) runs the same kernel.
    if not causal and N == NK and H == HK and not head_major:
        cfg = AFAForwardKernelConfig(dtype=DType.FP16 if dtype == torch.float16 else DType.BF16, d_head=d)
        o2, _ = fa.forward(cfg, q, k, v, None, False)
        torch.cuda.synchronize()
        assert torch.equal(o2, out)
