"""Sequence-length sweep of the forward kernel, with the reference's command line.

Same arguments and summary format as the reference's
benchmarks/afa_fwd_kernel_benchmarks_by_seqlen.py (:24-75 arguments, :81-128
timing through ``forward(cfg, q, k, v, o, True)``, :180-195 summary); usage::

    python -m ampere_flash_attention_from_scratch_b200.seqlen_sweep \\
        --config_string "(FP16, 128, 64, 32, 4): async+eager+swizzled+load_2_2_2_tiles" \\
        --batch_size 16 --n_heads 32 --seq_lens 1024 2048 4096 8192

Differences, by design:
* throughput is 4*B*H*N^2*d FLOPs per forward (both GEMMs, 2 FLOPs per
  multiply-add), the metric this package is measured on; the reference
  script printed 2*B*H*N^2*d.  ``--flops_formula 2bhn2d`` prints that one;
* ``--causal`` and ``--n_kv_heads`` time the extensions through
  ``forward_ext`` (a causal forward is counted as half the FLOPs);
* ``--json PATH`` writes the results for ``result_table``.
"""

from __future__ import annotations

import argparse
import json
import sys

import torch

from .afa_config import AFAForwardKernelConfig, is_valid_config


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Benchmark the sm_100a forward kernel across sequence lengths",
                                formatter_class=argparse.RawDescriptionHelpFormatter, epilog=__doc__)
    p.add_argument("--config_string", type=str,
                   default="(FP16, 128, 64, 32, 4): async+eager+swizzled+load_2_2_2_tiles",
                   help="configuration string, e.g. '(FP16, 128, 64, 32, 4): async+eager+swizzled+load_2_2_2_tiles'")
    p.add_argument("--batch_size", type=int, default=16, help="batch size")
    p.add_argument("--seq_lens", type=int, nargs="+", default=[1024, 2048, 4096, 8192],
                   help="sequence lengths to benchmark")
    p.add_argument("--n_heads", type=int, default=32, help="number of (query) heads")
    p.add_argument("--warmup", type=int, default=2, help="warm-up iterations (default: 2)")
    p.add_argument("--repeats", type=int, default=10, help="timed iterations (default: 10)")
    p.add_argument("--seed", type=int, default=42, help="random seed (default: 42)")
    p.add_argument("--causal", action="store_true", help="causal mask (forward_ext)")
    p.add_argument("--n_kv_heads", type=int, default=0, help="K/V heads for grouped attention (forward_ext); 0 = n_heads")
    p.add_argument("--flops_formula", choices=("4bhn2d", "2bhn2d"), default="4bhn2d",
                   help="FLOPs per forward: 4*B*H*N^2*d (default) or the reference script's 2*B*H*N^2*d")
    p.add_argument("--label", type=str, default="sm_100a kernel", help="row label for result_table")
    p.add_argument("--json", type=str, default=None, help="write the results as JSON to this path")
    return p.parse_args(argv)


def flops_per_forward(batch: int, n_heads: int, seq_len: int, d_head: int, causal: bool = False,
                      formula: str = "4bhn2d") -> float:
    """FLOPs of one forward: 4*B*H*N^2*d (or 2*B*H*N^2*d), halved under the causal mask."""
    f = (4.0 if formula == "4bhn2d" else 2.0) * batch * n_heads * seq_len * seq_len * d_head
    return f * (0.5 if causal else 1.0)


def benchmark_kernel(fa, cfg: AFAForwardKernelConfig, batch_size: int, seq_len: int, n_heads: int,
                     warmup: int = 2, repeats: int = 10, seed: int = 42, causal: bool = False,
                     n_kv_heads: int = 0) -> float:
    """Mean runtime in ms of one forward on fresh seeded N(0,1) inputs [B, N, H, d]."""
    torch.manual_seed(seed)
    dev = torch.device("cuda")
    dtype = cfg.dtype.to_torch_dtype()
    hk = n_kv_heads or n_heads
    q = torch.randn(batch_size, seq_len, n_heads, cfg.d_head, device=dev, dtype=dtype)
    k = torch.randn(batch_size, seq_len, hk, cfg.d_head, device=dev, dtype=dtype)
    v = torch.randn(batch_size, seq_len, hk, cfg.d_head, device=dev, dtype=dtype)
    o = torch.empty_like(q)
    ext = causal or hk != n_heads

    def once() -> float:
        if not ext:
            return fa.forward(cfg, q, k, v, o, True)[1]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fa.forward_ext(q, k, v, o, causal)
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1)

    for _ in range(warmup):
        once()
    torch.cuda.synchronize()
    runtimes = [once() for _ in range(repeats)]
    fa.check_status(dev.index or 0)
    return sum(runtimes) / len(runtimes)


def run(args: argparse.Namespace, fa=None, out=sys.stdout) -> dict:
    if fa is None:
        import afa_flash_attention_kernels as fa  # noqa: F811  (built extension; raises if missing)
    cfg = AFAForwardKernelConfig.from_string_config(args.config_string)
    if not is_valid_config(cfg):
        print(f"Warning: Configuration may not be valid: {cfg}", file=out)
    cap = torch.cuda.get_device_capability()
    print("=" * 80, file=out)
    print("AFA Forward Kernel Benchmark by Sequence Length (sm_100a)", file=out)
    print("=" * 80, file=out)
    print(f"Config: {cfg}", file=out)
    print(f"Batch Size: {args.batch_size}", file=out)
    print(f"Number of Heads: {args.n_heads}" + (f" (K/V heads {args.n_kv_heads})" if args.n_kv_heads else ""), file=out)
    print(f"Head Dimension: {cfg.d_head}", file=out)
    print(f"Causal: {args.causal}", file=out)
    print(f"GPU: {torch.cuda.get_device_name(0)}", file=out)
    print(f"SM Version: {cap[0]}{cap[1]}", file=out)
    print(f"Warmup iterations: {args.warmup}", file=out)
    results = []
    for n in args.seq_lens:
        try:
            ms = benchmark_kernel(fa, cfg, args.batch_size, n, args.n_heads, args.warmup, args.repeats, args.seed,
                                  args.causal, args.n_kv_heads)
            tf = flops_per_forward(args.batch_size, args.n_heads, n, cfg.d_head, args.causal,
                                   args.flops_formula) / (ms * 1e-3) / 1e12
            results.append({"seq_len": n, "ms": ms, "tflops": tf})
        except Exception as e:  # a failed size is reported, the sweep goes on (as the reference script)
            results.append({"seq_len": n, "ms": None, "tflops": None, "error": str(e)})
    print("=" * 80, file=out)
    print("\nSummary:", file=out)
    print(f"{'Seq Len':<10} {'Runtime (ms)':<15} {'Throughput (TFLOPS, ' + args.flops_formula + ')':<20}", file=out)
    print("-" * 80, file=out)
    for r in results:
        if r["ms"] is not None:
            print(f"{r['seq_len']:<10} [{r['ms']:0.2f}, {r['tflops']:<0.2f}]", file=out)
        else:
            print(f"{r['seq_len']:<10} {'FAILED':<15} {r.get('error', '')}", file=out)
    doc = {
        "label": args.label, "config_string": args.config_string, "batch_size": args.batch_size,
        "n_heads": args.n_heads, "n_kv_heads": args.n_kv_heads or args.n_heads, "d_head": cfg.d_head,
        "causal": args.causal, "flops_formula": args.flops_formula, "gpu": torch.cuda.get_device_name(0),
        "results": results,
    }
    if args.json:
        with open(args.json, "w") as f:
            json.dump(doc, f, indent=1)
    return doc


def main(argv=None) -> int:
    args = parse_args(argv)
    try:
        import afa_flash_attention_kernels as fa
    except ImportError as e:
        print(f"Error: could not import afa_flash_attention_kernels ({e}).")
        print("Build it first: python -m ampere_flash_attention_from_scratch_b200.build")
        return 1
    try:
        AFAForwardKernelConfig.from_string_config(args.config_string)
    except Exception as e:
        print(f"Error: Failed to parse config string: {e}")
        return 1
    run(args, fa)
    return 0


if __name__ == "__main__":
    sys.exit(main())
