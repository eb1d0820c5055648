"""GPU parity of the extensions beyond the reference (forward_ext): K/V of
their own length and head count (GQA), the bottom-right causal mask and the
fp32 log-sum-exp, against the fp32 oracle (tests/test_oracle_ext.py pins the
oracle's conventions against float64 and torch SDPA).

Tolerances: O as the reference's (fp16 max-abs 1e-2 / mean-abs 1e-3, bf16
2e-2 / 2e-3); lse within 1e-3 absolute -- the kernel forms it from fp32 scores,
an fp32 running max and an fp32 sum of ex2.approx terms (relative error of a
few 1e-7 each), so its error is far below that bound.
"""

import math

import pytest
import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig, DType
from oracle.attention_oracle import attention_fp32, error_stats

pytestmark = pytest.mark.gpu

TOL = {torch.float16: (1e-2, 1e-3), torch.bfloat16: (2e-2, 2e-3)}
LSE_TOL = 1e-3


def _qkv(B, N, NK, H, HK, d, dtype, seed=0, sigma=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, N, H, d, generator=g) * sigma).to(dtype)
    k = (torch.randn(B, NK, HK, d, generator=g) * sigma).to(dtype)
    v = torch.randn(B, NK, HK, d, generator=g).to(dtype)
    dev = torch.device("cuda:0")
    return q.to(dev), k.to(dev), v.to(dev)


def _run(q, k, v, causal, lse=True, scale=None):
    out, l = fa.forward_ext(q, k, v, None, causal, scale, lse)
    torch.cuda.synchronize()
    fa.check_status(0)
    return out, l


def _check(out, l, ref, ref_lse, dtype, what):
    mx, mean = error_stats(out, ref)
    tmax, tmean = TOL[dtype]
    assert mx <= tmax and mean <= tmean, f"{what}: O max-abs {mx:.3e} mean-abs {mean:.3e}"
    if l is not None:
        fin = torch.isfinite(ref_lse)
        assert torch.equal(torch.isfinite(l), fin), f"{what}: -inf pattern of lse differs"
        err = (l[fin] - ref_lse[fin]).abs().max().item() if fin.any() else 0.0
        assert err <= LSE_TOL, f"{what}: lse max-abs {err:.3e}"
        assert torch.all(torch.isneginf(l[~fin]))


CASES = [
    # B, N, N_kv, H, H_kv, d, dtype
    (2, 300, 300, 4, 4, 128, torch.float16),
    (1, 1000, 1000, 4, 1, 64, torch.bfloat16),
    (2, 257, 513, 8, 2, 128, torch.bfloat16),
    (1, 700, 129, 2, 2, 64, torch.float16),  # N > N_kv: causal rows that see no key
    (1, 1, 4096, 4, 4, 128, torch.float16),  # one query row (decode-like)
    (1, 2048, 2048, 8, 8, 128, torch.float16),
    (2, 640, 384, 6, 3, 64, torch.float16),
    (1, 129, 1, 2, 1, 128, torch.bfloat16),  # one key
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(str(x) for x in c[:6]) + f"-{str(c[6])[6:]}")
@pytest.mark.parametrize("causal", [False, True])
def test_against_oracle(case, causal):
    B, N, NK, H, HK, d, dtype = case
    q, k, v = _qkv(B, N, NK, H, HK, d, dtype, seed=N + NK)
    out, l = _run(q, k, v, causal)
    ref, ref_lse = attention_fp32(q, k, v, causal=causal, return_lse=True)
    _check(out, l, ref, ref_lse, dtype, f"{case} causal={causal}")


def test_equal_shapes_match_reference_entry_bit_for_bit():
    q, k, v = _qkv(2, 1000, 1000, 4, 4, 128, torch.float16, seed=1)
    cfg = AFAForwardKernelConfig(dtype=DType.FP16, d_head=128)
    a, _ = fa.forward(cfg, q, k, v, None, False)
    b, lse = _run(q, k, v, False)
    assert torch.equal(a, b)
    assert lse.shape == (2, 4, 1000) and lse.dtype == torch.float32
    _, none = fa.forward_ext(q, k, v, None, False, None, False)
    assert none is None


def test_gqa_equals_repeated_heads():
    # Grouped K/V heads give exactly the output of the same heads repeated.
    q, k, v = _qkv(1, 777, 901, 8, 2, 64, torch.bfloat16, seed=2)
    a, la = _run(q, k, v, True)
    kr, vr = (t.repeat_interleave(4, dim=2).contiguous() for t in (k, v))
    b, lb = _run(q, kr, vr, True)
    assert torch.equal(a, b) and torch.equal(la, lb)


def test_causal_diagonal_row_sees_prefix_only():
    # Changing keys/values after row i's last visible key leaves row i unchanged.
    q, k, v = _qkv(1, 512, 512, 2, 2, 128, torch.float16, seed=4)
    a, la = _run(q, k, v, True)
    k2, v2 = k.clone(), v.clone()
    k2[:, 300:] = torch.randn_like(k2[:, 300:].float()).to(k2.dtype)
    v2[:, 300:] = 7.0
    b, lb = _run(q, k2, v2, True)
    assert torch.equal(a[:, :300], b[:, :300]) and torch.equal(la[:, :, :300], lb[:, :, :300])


def test_softmax_scale_argument():
    q, k, v = _qkv(1, 256, 384, 2, 1, 64, torch.float16, seed=6)
    out, l = _run(q, k, v, False, scale=0.05)
    ref, ref_lse = attention_fp32(q, k, v, scale=0.05, return_lse=True)
    _check(out, l, ref, ref_lse, torch.float16, "scale=0.05")


def test_wide_softmax_range_causal_bf16():
    q, k, v = _qkv(1, 1536, 1536, 4, 2, 64, torch.bfloat16, seed=8, sigma=3.0)
    out, l = _run(q, k, v, True)
    ref, ref_lse = attention_fp32(q, k, v, causal=True, return_lse=True)
    _check(out, l, ref, ref_lse, torch.bfloat16, "sigma 3 causal")


@pytest.mark.slow
def test_large_causal_sampled_slices():
    # [4, 8192, 32, 128] fp16 causal with GQA 4:1; three (b, h) slices against the oracle on the GPU.
    q, k, v = _qkv(4, 8192, 8192, 32, 8, 128, torch.float16, seed=10)
    out, l = _run(q, k, v, True)
    pairs = [(0, 0), (3, 31), (2, 13)]
    ref, ref_lse = attention_fp32(q, k, v, causal=True, return_lse=True, slices=pairs, max_scores=1 << 26)
    got = torch.stack([out[b, :, h, :] for b, h in pairs]).float()
    got_l = torch.stack([l[b, h] for b, h in pairs])
    _check(got, got_l, ref, ref_lse, torch.float16, "large causal")


def test_dynamic_schedule_matches_static_and_resets_words():
    # The causal kernel with scheduler words hands out work items dynamically;
    # every item is computed the same way on whichever SM takes it, so the output
    # is bit-identical to the static schedule, and the words are 0 afterwards.
    import ctypes
    from ampere_flash_attention_from_scratch_b200 import _abi
    lib = _abi.load()
    q, k, v = _qkv(2, 3000, 3000, 8, 2, 128, torch.float16, seed=12)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    sched = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = []
    for words in (None, sched, sched):  # static, then dynamic twice (words reused)
        o = torch.empty_like(q)
        lse = torch.empty(2, 8, 3000, device="cuda")
        a = _abi.make_args(q, k, v, o, status=status, causal=True, lse=lse, sched=words)
        assert lib.afa_fwd_sm100(ctypes.byref(a), stream) == _abi.AFA_OK
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert sched.tolist() == [0, 0]
        outs.append((o, lse))
    for o, lse in outs[1:]:
        assert torch.equal(o, outs[0][0]) and torch.equal(lse, outs[0][1])


def test_error_messages():
    q, k, v = _qkv(1, 128, 128, 4, 4, 64, torch.float16)
    with pytest.raises(RuntimeError, match="multiple of the number of key/value heads"):
        fa.forward_ext(q, k[:, :, :3].contiguous(), v[:, :, :3].contiguous())
    with pytest.raises(RuntimeError, match="same shape"):
        fa.forward_ext(q, k, v[:, :64].contiguous())
    with pytest.raises(RuntimeError, match="softmax_scale"):
        fa.forward_ext(q, k, v, None, False, -1.0)
