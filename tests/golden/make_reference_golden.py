"""Generates tests/golden/ref_kernel_*.npz from the reference's own CUDA kernel.

Runs on a machine with a GPU and oracle/_ref/libafa_ref_ampere.so built (see
oracle/build_ref.py; the reference kernel is JIT-compiled from PTX).  Inputs
are drawn on the CPU from a fixed seed (torch.Generator), so the test side can
regenerate them without storing them; each file holds the shape, dtype, seed,
sigmas, reference-kernel config id and the reference kernel's fp16/bf16 output.

Usage: python tests/golden/make_reference_golden.py [OUTDIR]
"""

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import ref_kernel  # noqa: E402

CASES = [
    # name, config id, B, N, H, d, dtype, sigma_qk, seed
    ("ref_kernel_fp16_d128_default", 0, 1, 256, 2, 128, torch.float16, 1.0, 42),
    ("ref_kernel_fp16_d128_br128", 1, 1, 256, 2, 128, torch.float16, 1.0, 43),
    ("ref_kernel_bf16_d64_wide", 2, 1, 256, 2, 64, torch.bfloat16, 3.0, 44),
]


def inputs(B, N, H, d, dtype, sigma_qk, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, N, H, d, generator=g) * sigma_qk).to(dtype)
    k = (torch.randn(B, N, H, d, generator=g) * sigma_qk).to(dtype)
    v = torch.randn(B, N, H, d, generator=g).to(dtype)
    return q, k, v


def main(outdir: Path):
    outdir.mkdir(parents=True, exist_ok=True)
    for name, cid, B, N, H, d, dtype, sig, seed in CASES:
        q, k, v = inputs(B, N, H, d, dtype, sig, seed)
        qd, kd, vd = (t.cuda() for t in (q, k, v))
        o = torch.empty_like(qd)
        ref_kernel.forward(cid, qd, kd, vd, o)
        torch.cuda.synchronize()
        bits = o.cpu().view(torch.int16).numpy()
        np.savez_compressed(outdir / f"{name}.npz", out_bits=bits, shape=np.array([B, N, H, d]),
                            dtype=np.array(str(dtype)), seed=np.array(seed), sigma_qk=np.array(sig),
                            config=np.array(cid))
        print(f"wrote {outdir / (name + '.npz')}")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent)
