"""forward_host: host-resident Q/K/V/O, batch slices copied in, computed and
copied out on three overlapping streams.  Must equal the device path bit for
bit (each batch slice is an independent launch of the same kernel)."""

import pytest
import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig, DType

pytestmark = pytest.mark.gpu


def _host(B, N, NK, H, HK, d, dtype, seed, pinned):
    g = torch.Generator().manual_seed(seed)
    ts = [torch.randn(B, N, H, d, generator=g).to(dtype), torch.randn(B, NK, HK, d, generator=g).to(dtype),
          torch.randn(B, NK, HK, d, generator=g).to(dtype)]
    return [t.pin_memory() if pinned else t for t in ts]


@pytest.mark.parametrize("B,N,NK,H,HK,d,dtype,causal,chunks,pinned", [
    (5, 1000, 1000, 4, 4, 128, torch.float16, False, 2, True),     # odd batch, 2 slices
    (3, 700, 700, 4, 2, 64, torch.bfloat16, True, 0, True),        # default slices (3), causal + GQA
    (8, 513, 257, 2, 1, 128, torch.float16, True, 8, False),       # pageable host memory, one batch per slice
    (1, 300, 300, 2, 2, 64, torch.float16, False, 4, True),        # more slices asked than batches
])
def test_matches_device_path(B, N, NK, H, HK, d, dtype, causal, chunks, pinned):
    q, k, v = _host(B, N, NK, H, HK, d, dtype, seed=B * N, pinned=pinned)
    o = fa.forward_host(q, k, v, None, causal, chunks)
    torch.cuda.synchronize()
    fa.check_status(0)
    assert o.device.type == "cpu" and o.shape == q.shape and o.dtype == q.dtype
    ref, _ = fa.forward_ext(q.cuda(), k.cuda(), v.cuda(), None, causal)
    assert torch.equal(o, ref.cpu())


def test_output_buffer_and_reference_entry_agree():
    q, k, v = _host(4, 1024, 1024, 4, 4, 128, torch.float16, seed=3, pinned=True)
    o = torch.empty_like(q).pin_memory()
    ret = fa.forward_host(q, k, v, o)
    torch.cuda.synchronize()
    assert ret.data_ptr() == o.data_ptr()
    ref, _ = fa.forward(AFAForwardKernelConfig(dtype=DType.FP16, d_head=128), q.cuda(), k.cuda(), v.cuda(), None, False)
    assert torch.equal(o, ref.cpu())


def test_rejects_device_tensors():
    q = torch.randn(1, 128, 2, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="host"):
        fa.forward_host(q, q, q)


def test_temporary_pinned_inputs_survive_until_copied():
    """Inputs passed as temporaries (``q.pin_memory()``) are released when the call
    returns, while their copies are still queued behind earlier work on the stream.
    Page-locked tensors allocated right after (and filled with NaN) must not be
    given that memory before the copies have read it."""
    B, N, H, d = 8, 4096, 16, 128
    q, k, v = _host(B, N, N, H, H, d, torch.float16, seed=11, pinned=False)
    # Three page-locked blocks of this size left in the allocator's cache: the
    # temporaries below take them without page-locking anew (fast), so the call
    # is made while the spin still holds its copies back.
    warm = [torch.empty_like(q).pin_memory() for _ in range(3)]
    del warm
    torch.cuda.synchronize()
    torch.cuda._sleep(2_000_000_000)  # a fixed-length spin (~1 s) keeps the copies queued
    o = fa.forward_host(q.pin_memory(), k.pin_memory(), v.pin_memory())
    junk = [torch.full_like(q, float("nan")).pin_memory() for _ in range(3)]
    torch.cuda.synchronize()
    fa.check_status(0)
    ref, _ = fa.forward_ext(q.cuda(), k.cuda(), v.cuda())
    assert torch.equal(o, ref.cpu())
    del junk
