"""Benchmark / parity workloads: the five configurations the attention forward
is measured and checked on, and their seeded synthetic inputs.

Inputs follow the reference's harness (demo.py:16-26,
benchmarks/afa_fwd_kernel_benchmarks_by_seqlen.py:79-105): ``torch.manual_seed``
then q, k, v drawn in that order with ``torch.randn``, here in fp32, scaled by
sigma and cast to the compute dtype.  Layout [B, N, H, d].  There is no public
dataset behind these numbers; the data is synthetic by construction.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    seq_len: int
    n_heads: int
    d_head: int
    dtype: torch.dtype
    sigma_qk: float
    sigma_v: float

    @property
    def shape(self):
        return (self.batch, self.seq_len, self.n_heads, self.d_head)

    @property
    def flops(self) -> int:
        """4*B*H*N^2*d: two N x N x d GEMMs (QK^T and PV) per (b, h)."""
        return 4 * self.batch * self.n_heads * self.seq_len * self.seq_len * self.d_head

    @property
    def hbm_bytes(self) -> int:
        """Algorithmic HBM bytes: read Q, K, V and write O once (2 bytes each)."""
        return 4 * self.batch * self.seq_len * self.n_heads * self.d_head * 2

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.d_head)

    def dtype_name(self) -> str:
        return {torch.float16: "fp16", torch.bfloat16: "bf16"}[self.dtype]


WORKLOADS = {
    "cfg1": Workload("cfg1", 1, 1024, 8, 128, torch.float16, 1.0, 1.0),
    "cfg2": Workload("cfg2", 16, 1024, 32, 128, torch.float16, 1.0, 1.0),
    "cfg3": Workload("cfg3", 16, 4096, 32, 128, torch.float16, 1.0, 1.0),
    "cfg4": Workload("cfg4", 16, 8192, 32, 128, torch.float16, 1.0, 1.0),
    "cfg5": Workload("cfg5", 8, 16384, 32, 64, torch.bfloat16, 3.0, 1.0),
}


def make_inputs(wl: Workload, seed: int = 42, device="cpu", batch_slice: slice | None = None):
    """Seeded q, k, v for a workload: randn fp32 * sigma, cast to wl.dtype.

    Drawn on ``device`` (CPU and CUDA generators give different streams; all
    ranks of one run draw on the same kind of device, so every rank sees the
    same full tensors and ``batch_slice`` selects its shard).
    """
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = []
    for sigma in (wl.sigma_qk, wl.sigma_qk, wl.sigma_v):
        t = torch.randn(wl.shape, generator=g, device=device, dtype=torch.float32)
        t.mul_(sigma)
        t = t.to(wl.dtype)
        if batch_slice is not None:
            t = t[batch_slice].contiguous()
        out.append(t)
    return tuple(out)
