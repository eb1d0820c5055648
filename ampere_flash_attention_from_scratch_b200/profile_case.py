"""A small, self-contained forward workload for profiler captures.

    python -m ampere_flash_attention_from_scratch_b200.profile_case d128|d64

Runs a few launches on a problem larger than L2 (so DRAM counters mean
something) but small enough for a full `ncu --set full` capture to finish in
about a minute: d128 = [4, 4096, 32, 128] fp16, d64 = [2, 8192, 32, 64] bf16
(Q, K ~ N(0, 3) as in the [8, 16384, 32, 64] workload).  Prints the
event-timed duration of the last launch.
"""

import sys

import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig, DType

CASES = {
    "d128": (4, 4096, 32, 128, torch.float16, 1.0),
    "d64": (2, 8192, 32, 64, torch.bfloat16, 3.0),
}


def main(which: str = "d128", launches: int = 3) -> float:
    B, N, H, d, dt, sig = CASES[which]
    g = torch.Generator(device="cuda").manual_seed(42)
    q = (torch.randn(B, N, H, d, generator=g, device="cuda") * sig).to(dt)
    k = (torch.randn(B, N, H, d, generator=g, device="cuda") * sig).to(dt)
    v = torch.randn(B, N, H, d, generator=g, device="cuda").to(dt)
    o = torch.empty_like(q)
    cfg = AFAForwardKernelConfig(dtype=DType.FP16 if dt == torch.float16 else DType.BF16, d_head=d)
    for _ in range(launches):
        fa.forward(cfg, q, k, v, o, False)
    torch.cuda.synchronize()
    fa.check_status(0)
    _, ms = fa.forward(cfg, q, k, v, o, True)
    print(f"{which}: [{B},{N},{H},{d}] {ms:.3f} ms  {4 * B * H * N * N * d / ms / 1e9:.1f} TFLOP/s")
    return ms


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "d128")
