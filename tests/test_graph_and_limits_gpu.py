"""CUDA-graph capture of the forward calls, a very long sequence, and the
host-side cost of a launch.

The launch path makes no host synchronisation and no allocation beyond the
torch output tensor, so forward / forward_ext can be captured in a CUDA graph
and replayed; the causal kernel's scheduler words return to zero at the end of
every launch, so replays need no reset.  The long-sequence case checks
indexing beyond the benchmark shapes against the fp32 oracle on sampled rows.
"""

import time

import pytest
import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig, DType
from oracle.attention_oracle import attention_fp32

pytestmark = pytest.mark.gpu


def _qkv(B, N, H, d, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B, N, H, d, generator=g, device="cuda").to(dtype) for _ in range(3)]


def test_cuda_graph_capture_and_replay():
    q, k, v = _qkv(2, 1500, 4, 128, torch.float16, seed=1)
    cfg = AFAForwardKernelConfig(dtype=DType.FP16, d_head=128)
    o1 = torch.empty_like(q)
    o2 = torch.empty_like(q)
    lse = None
    ref1, _ = fa.forward(cfg, q, k, v, None, False)
    ref2, ref_lse = fa.forward_ext(q, k, v, None, True, None, True)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up on the capture stream (scheduler words for it exist)
        fa.forward(cfg, q, k, v, o1, False)
        fa.forward_ext(q, k, v, o2, True, None, False)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):  # the stream whose scheduler words exist
        fa.forward(cfg, q, k, v, o1, False)
        _, lse = fa.forward_ext(q, k, v, o2, True, None, True)
    for _ in range(3):
        o1.zero_()
        o2.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(o1, ref1)
        assert torch.equal(o2, ref2)
        assert torch.equal(lse, ref_lse)
    fa.check_status(0)


@pytest.mark.slow
def test_very_long_sequence():
    # N = 131072 (512 K/V tiles per work item), bf16 d=64, causal and not.
    q, k, v = _qkv(1, 131072, 2, 64, torch.bfloat16, seed=2)
    for causal in (False, True):
        out, lse = fa.forward_ext(q, k, v, None, causal, None, True)
        torch.cuda.synchronize()
        fa.check_status(0)
        rows = torch.tensor([0, 1, 4097, 65535, 131071], device="cuda")
        qs = q[:, rows]
        # The oracle on the sampled rows: with the causal mask row r sees keys <= r.
        for i, r in enumerate(rows.tolist()):
            kk = k[:, : r + 1] if causal else k
            vv = v[:, : r + 1] if causal else v
            ref, ref_lse = attention_fp32(qs[:, i:i + 1], kk, vv, return_lse=True)
            assert (out[:, r:r + 1].float() - ref).abs().max().item() <= 2e-2
            assert (lse[:, :, r] - ref_lse[:, :, 0]).abs().max().item() <= 1e-3


def test_host_launch_cost_is_small():
    # A tiny forward is dominated by host work: argument checks, three TMA
    # descriptors and the launch.  Bound it loosely so a regression shows.
    q, k, v = _qkv(1, 128, 1, 64, torch.float16, seed=3)
    cfg = AFAForwardKernelConfig(dtype=DType.FP16, d_head=64)
    o = torch.empty_like(q)
    for _ in range(10):
        fa.forward(cfg, q, k, v, o, False)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    n = 200
    for _ in range(n):
        fa.forward(cfg, q, k, v, o, False)
    t1 = time.perf_counter()
    torch.cuda.synchronize()
    per_call_us = (t1 - t0) / n * 1e6
    print(f"host time per forward call: {per_call_us:.1f} us")
    assert per_call_us < 200.0
