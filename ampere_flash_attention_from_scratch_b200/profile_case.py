"""A small, self-contained forward workload for profiler captures.

    python -m ampere_flash_attention_from_scratch_b200.profile_case d128|d64|d128c

Runs a few launches on a problem larger than L2 (so DRAM counters mean
something) but small enough for a full `ncu --set full` capture to finish in
about a minute: d128 = [4, 4096, 32, 128] fp16, d64 = [2, 8192, 32, 64] bf16
(Q, K ~ N(0, 3) as in the [8, 16384, 32, 64] workload), d128c = the d128
shape with the causal mask (forward_ext; half the FLOPs counted).  Prints the
event-timed duration of the last launch.
"""

import sys

import torch

import afa_flash_attention_kernels as fa
from afa_py.afa_config import AFAForwardKernelConfig, DType

CASES = {
    "d128": (4, 4096, 32, 128, torch.float16, 1.0, False),
    "d64": (2, 8192, 32, 64, torch.bfloat16, 3.0, False),
    "d128c": (4, 4096, 32, 128, torch.float16, 1.0, True),
}


def main(which: str = "d128", launches: int = 3) -> float:
    B, N, H, d, dt, sig, causal = CASES[which]
    g = torch.Generator(device="cuda").manual_seed(42)
    q = (torch.randn(B, N, H, d, generator=g, device="cuda") * sig).to(dt)
    k = (torch.randn(B, N, H, d, generator=g, device="cuda") * sig).to(dt)
    v = torch.randn(B, N, H, d, generator=g, device="cuda").to(dt)
    o = torch.empty_like(q)
    cfg = AFAForwardKernelConfig(dtype=DType.FP16 if dt == torch.float16 else DType.BF16, d_head=d)

    def launch():
        if causal:
            fa.forward_ext(q, k, v, o, True)
        else:
            fa.forward(cfg, q, k, v, o, False)

    for _ in range(launches):
        launch()
    torch.cuda.synchronize()
    fa.check_status(0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    launch()
    e1.record()
    e1.synchronize()
    fa.check_status(0)
    ms = e0.elapsed_time(e1)
    flops = 4 * B * H * N * N * d * (0.5 if causal else 1.0)
    print(f"{which}: [{B},{N},{H},{d}]{' causal' if causal else ''} {ms:.3f} ms  {flops / ms / 1e9:.1f} TFLOP/s")
    return ms


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "d128")
