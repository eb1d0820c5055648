"""Markdown comparison table of seq-len sweep results.

Counterpart of the reference's tools/kernel_benchmark_result_show.py (:45-66:
one row per kernel, one column per shape, cells "[ms, TFLOPs], ratio %" against
the first row).  Instead of a table pasted into the source it reads the JSON
files written by ``seqlen_sweep --json``; the reference's bar chart needs
matplotlib, which this environment does not provide, so only the table is
produced.

    python -m ampere_flash_attention_from_scratch_b200.result_table base.json new.json [--baseline 0]
"""

from __future__ import annotations

import argparse
import json
import sys


def shape_label(doc: dict, seq_len: int) -> str:
    return f"[{doc['batch_size']}, {seq_len}, {doc['n_heads']}, {doc['d_head']}]"


def make_table(docs: list[dict], baseline: int = 0) -> str:
    """Rows = runs, columns = the union of shapes in order of first appearance;
    each cell "[ms, TFLOPs], ratio%" with the ratio of TFLOPs to the baseline
    run's at that shape ("-" where a run lacks the shape or failed)."""
    cols: list[str] = []
    cells: list[dict] = []
    for d in docs:
        row = {}
        for r in d["results"]:
            key = shape_label(d, r["seq_len"])
            if key not in cols:
                cols.append(key)
            row[key] = r
        cells.append(row)
    base = cells[baseline] if docs else {}
    lines = ["| Kernel | " + " | ".join(cols) + " |", "|---" * (len(cols) + 1) + "|"]
    for d, row in zip(docs, cells):
        out = []
        for c in cols:
            r = row.get(c)
            if r is None or r.get("ms") is None:
                out.append("-")
                continue
            b = base.get(c)
            ratio = (f", {100.0 * r['tflops'] / b['tflops']:.2f}%"
                     if b is not None and b.get("tflops") else "")
            out.append(f"[{r['ms']:.2f}, {r['tflops']:.2f}]{ratio}")
        lines.append(f"| {d.get('label', '?')} | " + " | ".join(out) + " |")
    return "\n".join(lines)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("files", nargs="+", help="JSON files written by seqlen_sweep --json")
    p.add_argument("--baseline", type=int, default=0, help="index of the run the ratios refer to (default 0)")
    a = p.parse_args(argv)
    docs = []
    for f in a.files:
        with open(f) as fh:
            docs.append(json.load(fh))
    print(make_table(docs, a.baseline))
    return 0


if __name__ == "__main__":
    sys.exit(main())
