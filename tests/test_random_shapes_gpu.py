"""Randomised differential test of the kernel against the fp32 oracle.

40 configurations drawn from a fixed seed: batch 1-3, query and key lengths
1-1100 (independently), 1-8 query heads with a random divisor as K/V heads,
head_dim 64/128, fp16/bf16, causal or not, contiguous [B, N, H, d] tensors or
head-major storage viewed as [B, N, H, d] (non-contiguous strides).  O within
the tolerances of the other parity tests, lse within 1e-3 where finite and
-inf exactly where the oracle has -inf."""

import random

import pytest
import torch

import afa_flash_attention_kernels as fa
from oracle.attention_oracle import attention_fp32, error_stats

pytestmark = pytest.mark.gpu

TOL = {torch.float16: (1e-2, 1e-3), torch.bfloat16: (2e-2, 2e-3)}


def _configs(n=40, seed=2024):
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        h = rng.randint(1, 8)
        divisors = [x for x in range(1, h + 1) if h % x == 0]
        out.append(dict(B=rng.randint(1, 3), N=rng.choice([1, 7, 128, 129, 255, 256, 257, rng.randint(1, 1100)]),
                        NK=rng.choice([1, 64, 128, 300, rng.randint(1, 1100)]), H=h, HK=rng.choice(divisors),
                        d=rng.choice([64, 128]), dtype=rng.choice([torch.float16, torch.bfloat16]),
                        causal=rng.random() < 0.5, head_major=rng.random() < 0.4, seed=rng.randint(0, 10 ** 6)))
    return out


def _tensor(B, N, H, d, dtype, head_major, g):
    if head_major:  # storage [B, H, N, d], viewed as [B, N, H, d]
        return torch.randn(B, H, N, d, generator=g, device="cuda").to(dtype).transpose(1, 2)
    return torch.randn(B, N, H, d, generator=g, device="cuda").to(dtype)


@pytest.mark.parametrize("cfg", _configs(), ids=lambda c: "B{B}N{N}K{NK}H{H}/{HK}d{d}{causal}{head_major}".format(**c))
def test_random_configuration(cfg):
    g = torch.Generator(device="cuda").manual_seed(cfg["seed"])
    q = _tensor(cfg["B"], cfg["N"], cfg["H"], cfg["d"], cfg["dtype"], cfg["head_major"], g)
    k = _tensor(cfg["B"], cfg["NK"], cfg["HK"], cfg["d"], cfg["dtype"], cfg["head_major"], g)
    v = _tensor(cfg["B"], cfg["NK"], cfg["HK"], cfg["d"], cfg["dtype"], cfg["head_major"], g)
    out, lse = fa.forward_ext(q, k, v, None, cfg["causal"], None, True)
    torch.cuda.synchronize()
    fa.check_status(0)
    ref, ref_lse = attention_fp32(q, k, v, causal=cfg["causal"], return_lse=True)
    mx, mean = error_stats(out, ref)
    tmax, tmean = TOL[cfg["dtype"]]
    assert mx <= tmax and mean <= tmean, f"max-abs {mx:.3e} mean-abs {mean:.3e}"
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse), fin)
    if fin.any():
        assert (lse[fin] - ref_lse[fin]).abs().max().item() <= 1e-3
