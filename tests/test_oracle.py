"""Pins the CPU oracle (oracle/attention_oracle.py) before it is trusted.

* fp32 oracle vs float64 numpy and vs torch's SDPA math backend;
* the blockwise restatement of the reference kernel vs the reference kernel's
  own outputs on the B200 (tests/golden/ref_kernel_*.npz, written by
  tests/golden/make_reference_golden.py): within 1 ulp of the output type;
* the fp32 oracle vs those outputs within the parity tolerance;
* a planted mistake in the oracle (wrong softmax scale) is caught.
"""

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.attention_oracle import attention_blockwise, attention_fp32, attention_fp64, error_stats

GOLDEN = Path(__file__).resolve().parent / "golden"
GOLDEN_FILES = sorted(GOLDEN.glob("ref_kernel_*.npz"))
TOL = {torch.float16: (1e-2, 1e-3), torch.bfloat16: (2e-2, 2e-3)}


def rand_qkv(B, N, H, d, dtype, sigma_qk=1.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, N, H, d, generator=g) * sigma_qk).to(dtype)
    k = (torch.randn(B, N, H, d, generator=g) * sigma_qk).to(dtype)
    v = torch.randn(B, N, H, d, generator=g).to(dtype)
    return q, k, v


def ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of the spacing of a's dtype at max(|a|, |b|)."""
    mant = {torch.float16: 10, torch.bfloat16: 7}[a.dtype]
    emin = {torch.float16: -14, torch.bfloat16: -126}[a.dtype]
    af, bf = a.float(), b.float()
    mag = torch.maximum(af.abs(), bf.abs())
    _, e = torch.frexp(mag)
    e = torch.clamp(e - 1, min=emin)
    spacing = torch.pow(2.0, (e - mant).float())
    return (af - bf).abs() / spacing


def load_golden(path):
    z = np.load(path)
    B, N, H, d = (int(x) for x in z["shape"])
    dtype = getattr(torch, str(z["dtype"]).split(".")[-1])
    q, k, v = rand_qkv(B, N, H, d, dtype, float(z["sigma_qk"]), int(z["seed"]))
    out = torch.from_numpy(z["out_bits"]).view(dtype)
    cid = int(z["config"])
    br, bc = (128, 64) if cid == 1 else (64, 32)
    return q, k, v, out, br, bc


@pytest.mark.parametrize("dtype,d", [(torch.float16, 128), (torch.bfloat16, 64), (torch.float16, 64)])
def test_fp32_matches_fp64(dtype, d):
    q, k, v = rand_qkv(2, 96, 3, d, dtype, seed=d)
    o32 = attention_fp32(q, k, v)
    o64 = attention_fp64(q, k, v)
    assert np.abs(o32.numpy() - o64).max() < 2e-6


def test_fp32_matches_sdpa_math():
    q, k, v = rand_qkv(2, 200, 2, 128, torch.float16, seed=1)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float().transpose(1, 2), k.float().transpose(1, 2), v.float().transpose(1, 2), scale=1 / math.sqrt(128)
    ).transpose(1, 2)
    assert (attention_fp32(q, k, v) - ref).abs().max() < 2e-6


def test_fp32_chunking_and_slices():
    q, k, v = rand_qkv(2, 300, 2, 64, torch.bfloat16, seed=2)
    full = attention_fp32(q, k, v)
    chunked = attention_fp32(q, k, v, max_scores=300 * 7)
    assert torch.equal(full, chunked) or (full - chunked).abs().max() < 1e-6
    sl = attention_fp32(q, k, v, slices=[(1, 0), (0, 1)])
    assert torch.equal(sl[0], full[1, :, 0]) and torch.equal(sl[1], full[0, :, 1])


def test_blockwise_close_to_exact():
    q, k, v = rand_qkv(1, 128, 2, 128, torch.float16, seed=3)
    mx, mean = error_stats(attention_blockwise(q, k, v), attention_fp32(q, k, v))
    assert mx < 1e-3 and mean < 1e-4


def test_blockwise_rejects_ragged_like_reference():
    q, k, v = rand_qkv(1, 100, 1, 64, torch.float16)
    with pytest.raises(ValueError):
        attention_blockwise(q, k, v)


@pytest.mark.parametrize("path", GOLDEN_FILES, ids=lambda p: p.stem)
def test_blockwise_restates_reference_kernel(path):
    """Near bit-level agreement with the reference kernel's own output: >= 98% of
    elements bit-identical, every element within 1 ulp of the output type or
    2^-15 absolute (outputs close to 0 come from cancellation in the fp32 PV sum,
    where the tensor core's summation order shows)."""
    q, k, v, out, br, bc = load_golden(path)
    ours = attention_blockwise(q, k, v, br, bc)
    ulps = ulp_distance(ours, out)
    absdiff = (ours.float() - out.float()).abs()
    assert bool(((ulps <= 1.0) | (absdiff <= 2.0 ** -15)).all())
    assert float((ulps == 0).float().mean()) > 0.98


@pytest.mark.parametrize("path", GOLDEN_FILES, ids=lambda p: p.stem)
def test_fp32_oracle_vs_reference_kernel(path):
    q, k, v, out, _, _ = load_golden(path)
    mx, mean = error_stats(out, attention_fp32(q, k, v))
    tmax, tmean = TOL[out.dtype]
    assert mx <= tmax and mean <= tmean


def test_planted_scale_mistake_is_caught():
    """An oracle with the wrong softmax scale (1 instead of 1/sqrt(d)) must fail the golden check."""
    q, k, v, out, _, _ = load_golden(GOLDEN / "ref_kernel_fp16_d128_default.npz")
    mx, mean = error_stats(out, attention_fp32(q, k, v, scale=1.0))
    assert mx > 1e-2 or mean > 1e-3


def test_golden_fixtures_present():
    assert len(GOLDEN_FILES) >= 3
