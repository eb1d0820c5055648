"""The seq-len sweep CLI and the results table (the reference's
benchmarks/afa_fwd_kernel_benchmarks_by_seqlen.py and
tools/kernel_benchmark_result_show.py counterparts)."""

import io
import json

import pytest
import torch

from ampere_flash_attention_from_scratch_b200 import result_table, seqlen_sweep


def test_reference_command_line_parses():
    a = seqlen_sweep.parse_args(["--config_string", "(FP16, 128, 64, 32, 4): async+eager+swizzled+load_2_2_2_tiles",
                                 "--batch_size", "16", "--n_heads", "16", "--seq_lens", "512", "1024", "2048"])
    assert a.batch_size == 16 and a.n_heads == 16 and a.seq_lens == [512, 1024, 2048]
    assert a.warmup == 2 and a.repeats == 10 and a.seed == 42 and not a.causal and a.n_kv_heads == 0


def test_flops_formula():
    assert seqlen_sweep.flops_per_forward(16, 32, 8192, 128) == 4.0 * 16 * 32 * 8192 ** 2 * 128
    assert seqlen_sweep.flops_per_forward(16, 32, 8192, 128, formula="2bhn2d") == 2.0 * 16 * 32 * 8192 ** 2 * 128
    assert seqlen_sweep.flops_per_forward(1, 1, 100, 64, causal=True) == 0.5 * 4 * 100 * 100 * 64


def _doc(label, pts):
    return {"label": label, "batch_size": 16, "n_heads": 32, "d_head": 128,
            "results": [{"seq_len": n, "ms": ms, "tflops": tf} for n, ms, tf in pts]}


def test_table_ratios_and_missing_cells(tmp_path):
    a = _doc("reference", [(1024, 5.0, 30.0), (2048, 20.0, 30.0)])
    b = _doc("sm100", [(1024, 0.5, 300.0), (2048, None, None), (4096, 1.0, 400.0)])
    t = result_table.make_table([a, b])
    lines = t.splitlines()
    assert lines[0] == "| Kernel | [16, 1024, 32, 128] | [16, 2048, 32, 128] | [16, 4096, 32, 128] |"
    assert lines[2] == "| reference | [5.00, 30.00], 100.00% | [20.00, 30.00], 100.00% | - |"
    assert lines[3] == "| sm100 | [0.50, 300.00], 1000.00% | - | [1.00, 400.00] |"
    fa, fb = tmp_path / "a.json", tmp_path / "b.json"
    fa.write_text(json.dumps(a))
    fb.write_text(json.dumps(b))
    assert result_table.main([str(fa), str(fb), "--baseline", "1"]) == 0


def test_main_reports_bad_config(capsys):
    assert seqlen_sweep.main(["--config_string", "not a config", "--seq_lens", "128"]) == 1


@pytest.mark.gpu
def test_sweep_runs_on_gpu(tmp_path):
    import afa_flash_attention_kernels as fa
    out = io.StringIO()
    a = seqlen_sweep.parse_args(["--batch_size", "2", "--n_heads", "4", "--seq_lens", "256", "1000",
                                 "--repeats", "3", "--json", str(tmp_path / "r.json")])
    doc = seqlen_sweep.run(a, fa, out)
    assert [r["seq_len"] for r in doc["results"]] == [256, 1000]
    assert all(r["ms"] > 0 and r["tflops"] > 0 for r in doc["results"])
    assert "Summary:" in out.getvalue()
    a = seqlen_sweep.parse_args(["--batch_size", "1", "--n_heads", "4", "--n_kv_heads", "2", "--causal",
                                 "--seq_lens", "512", "--repeats", "2"])
    doc = seqlen_sweep.run(a, fa, io.StringIO())
    assert doc["results"][0]["ms"] > 0 and doc["causal"] and doc["n_kv_heads"] == 2
    assert "[16, 256" not in result_table.make_table([json.loads((tmp_path / "r.json").read_text())])
