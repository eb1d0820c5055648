"""Device-side failure detection without faulting the GPU.

With AFA_TEST_PRODUCER_IDLE the kernel's TMA producer loads nothing, so the
MMA issuer's bounded wait for Q runs out after a short timeout_ns: the kernel
must report AFA_DEV_TIMEOUT_BASE + site in the status word and return (no hang,
no fault, nothing left in flight), and the next normal call on the same
context must still produce the right answer.  With AFA_TEST_MMA_IDLE the MMA
issuer issues nothing: the producer fills the K/V ring, its wait for a free
slot runs out with its loads in flight or landed, and it waits for them before
the CTA exits -- same checks.
"""

import ctypes

import pytest
import torch

from ampere_flash_attention_from_scratch_b200 import _abi
from oracle.attention_oracle import attention_fp32, error_stats

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("flag", [_abi.AFA_TEST_PRODUCER_IDLE, _abi.AFA_TEST_MMA_IDLE])
def test_bounded_wait_runs_out_and_context_survives(flag):
    lib = _abi.load()
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(2, 384, 2, 128, generator=g).to(torch.float16) for _ in range(3))
    qd, kd, vd = (t.to(dev) for t in (q, k, v))
    o = torch.zeros_like(qd)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream

    a = _abi.make_args(qd, kd, vd, o, status=status, timeout_ns=20_000_000,
                       test_flags=flag)
    assert lib.afa_fwd_sm100(ctypes.byref(a), stream) == _abi.AFA_OK
    torch.cuda.synchronize()
    st = int(status.item())
    assert _abi.AFA_DEV_TIMEOUT_BASE < st < _abi.AFA_DEV_TIMEOUT_BASE + 32, hex(st)
    assert b"timeout" in lib.afa_status_string(st)

    status.zero_()
    a = _abi.make_args(qd, kd, vd, o, status=status)
    assert lib.afa_fwd_sm100(ctypes.byref(a), stream) == _abi.AFA_OK
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    mx, mean = error_stats(o, attention_fp32(q, k, v))
    assert mx <= 1e-2 and mean <= 1e-3
