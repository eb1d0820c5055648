"""The oracle's extensions beyond the reference: K/V of their own length and
head count (GQA), the bottom-right causal mask and the log-sum-exp output.

Pinned on CPU against float64 and against torch's SDPA math path, whose
``causal_lower_right`` bias and ``enable_gqa`` flag state the same conventions
independently of this repository's code.
"""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel
from torch.nn.attention.bias import causal_lower_right

from oracle.attention_oracle import attention_fp32, attention_fp64

CASES = [
    # B, N, N_kv, H, H_kv, d
    (2, 37, 53, 4, 2, 64),
    (1, 64, 64, 8, 1, 128),
    (2, 100, 19, 4, 4, 64),
    (1, 1, 77, 2, 1, 64),
]


def _qkv(B, N, NK, H, HK, d, seed=0, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, N, H, d, generator=g).to(dtype)
    k = torch.randn(B, NK, HK, d, generator=g).to(dtype)
    v = torch.randn(B, NK, HK, d, generator=g).to(dtype)
    return q, k, v


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("causal", [False, True])
def test_fp32_against_fp64(case, causal):
    q, k, v = _qkv(*case)
    o, lse = attention_fp32(q, k, v, causal=causal, return_lse=True)
    o64, lse64 = attention_fp64(q, k, v, causal=causal, return_lse=True)
    assert np.abs(o.double().numpy() - o64).max() < 1e-5
    fin = np.isfinite(lse64)
    assert np.array_equal(np.isfinite(lse.numpy()), fin)
    assert np.abs(lse.double().numpy()[fin] - lse64[fin]).max() < 1e-5


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("causal", [False, True])
def test_against_sdpa_lower_right_and_gqa(case, causal):
    B, N, NK, H, HK, d = case
    if causal and N > NK:
        pytest.skip("rows that see no key: SDPA returns NaN there (tested below)")
    q, k, v = _qkv(*case)
    o = attention_fp32(q, k, v, causal=causal)
    qt, kt, vt = (t.float().transpose(1, 2) for t in (q, k, v))
    with sdpa_kernel(SDPBackend.MATH):
        ref = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=causal_lower_right(N, NK) if causal else None,
                                             enable_gqa=True).transpose(1, 2)
    assert (ref - o).abs().max().item() < 1e-5


def test_lse_is_logsumexp_of_scaled_scores():
    q, k, v = _qkv(1, 33, 41, 2, 1, 64, seed=3)
    _, lse = attention_fp32(q, k, v, return_lse=True)
    s = torch.einsum("bnhd,bmhd->bhnm", q.double(), k.double().expand(-1, -1, 2, -1)) / math.sqrt(64)
    assert (lse.double() - torch.logsumexp(s, dim=-1)).abs().max().item() < 1e-5


def test_rows_that_see_no_key():
    # N > N_kv with the bottom-right causal mask: query rows i < N - N_kv see no key.
    q, k, v = _qkv(1, 50, 20, 2, 2, 64, seed=5)
    o, lse = attention_fp32(q, k, v, causal=True, return_lse=True)
    assert torch.all(o[:, :30] == 0)
    assert torch.all(torch.isneginf(lse[:, :, :30]))
    assert torch.all(torch.isfinite(lse[:, :, 30:]))
    # row 30 sees exactly key 0: O = v[0], lse = s_00
    assert torch.allclose(o[0, 30, 0], v[0, 0, 0].float(), atol=1e-6)
    s00 = (q[0, 30, 0].float() @ k[0, 0, 0].float()) / 8.0
    assert abs(lse[0, 0, 30].item() - s00.item()) < 1e-5


def test_slices_match_full():
    q, k, v = _qkv(2, 40, 60, 4, 2, 64, seed=9)
    o, lse = attention_fp32(q, k, v, causal=True, return_lse=True)
    pairs = [(1, 3), (0, 0)]
    os_, ls_ = attention_fp32(q, k, v, causal=True, return_lse=True, slices=pairs, max_scores=500)
    for i, (b, h) in enumerate(pairs):
        assert torch.equal(os_[i], o[b, :, h, :])
        assert torch.equal(ls_[i], lse[b, h])
