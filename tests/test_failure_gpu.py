"""Device-side failure detection without faulting the GPU.

With AFA_TEST_PRODUCER_IDLE the kernel's TMA producer loads nothing, so the
MMA issuer's bounded wait for Q runs out after a short timeout_ns: the kernel
must report AFA_DEV_TIMEOUT_BASE + site in the status word and return (no hang,
no fault, nothing left in flight), and the next normal call on the same
context must still produce the right answer.  With AFA_TEST_MMA_IDLE the MMA
issuer issues nothing: the producer fills the K/V ring, its wait for a free
slot runs out with its loads in flight or landed, and it waits for them before
the CTA exits -- same checks.

Through the torch binding the status word sits in mapped page-locked host
memory: a launch that aborted is raised by the next call on the device, without
check_status(), naming the wait site.
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


def _torch_inputs(seed, d=128, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(2, 384, 2, d, generator=g).to(dtype) for _ in range(3)]


@pytest.mark.parametrize("entry", ["forward", "forward_ext"])
def test_torch_path_raises_on_the_next_call(entry):
    import afa_flash_attention_kernels as fa
    from afa_py.afa_config import AFAForwardKernelConfig, DType

    cfg = AFAForwardKernelConfig(dtype=DType.FP16, d_head=128)
    q, k, v = _torch_inputs(6)
    qd, kd, vd = (t.cuda() for t in (q, k, v))
    fa.check_status(0)  # nothing pending from earlier tests
    fa._set_test_flags(_abi.AFA_TEST_PRODUCER_IDLE, 20_000_000)
    if entry == "forward":
        fa.forward(cfg, qd, kd, vd)  # returns at once; the kernel aborts after 20 ms
    else:
        fa.forward_ext(qd, kd, vd)
    torch.cuda.synchronize()  # the aborted launch has finished (no check_status)
    with pytest.raises(RuntimeError, match=r"earlier launch on cuda:0.*timeout: .*waiting"):
        fa.forward_ext(qd, kd, vd)
    # Raised once: the word was cleared, and the flags applied to one launch only.
    o, _ = fa.forward_ext(qd, kd, vd)
    fa.check_status(0)
    mx, mean = error_stats(o, attention_fp32(q, k, v))
    assert mx <= 1e-2 and mean <= 1e-3


def test_torch_path_benchmark_call_raises_for_its_own_launch():
    import afa_flash_attention_kernels as fa
    from afa_py.afa_config import AFAForwardKernelConfig, DType

    q, k, v = (t.cuda() for t in _torch_inputs(8, d=64, dtype=torch.bfloat16))
    fa.check_status(0)
    fa._set_test_flags(_abi.AFA_TEST_MMA_IDLE, 20_000_000)
    with pytest.raises(RuntimeError, match="attention kernel reported: timeout"):
        fa.forward(AFAForwardKernelConfig(dtype=DType.BF16, d_head=64), q, k, v, None, True)
    fa.check_status(0)


def test_check_status_raises_after_an_abort():
    import afa_flash_attention_kernels as fa

    q, k, v = (t.cuda() for t in _torch_inputs(9))
    fa.check_status(0)
    fa._set_test_flags(_abi.AFA_TEST_PRODUCER_IDLE, 20_000_000)
    fa.forward_ext(q, k, v, None, True)  # causal kernel, dynamic schedule
    with pytest.raises(RuntimeError, match="attention kernel reported: timeout"):
        fa.check_status(0)
    fa.check_status(0)  # cleared
    # The scheduler words came back to zero on the abort path: a normal causal call is complete.
    o, _ = fa.forward_ext(q, k, v, None, True)
    fa.check_status(0)
    mx, mean = error_stats(o, attention_fp32(*(t.cpu() for t in (q, k, v)), causal=True))
    assert mx <= 1e-2 and mean <= 1e-3
