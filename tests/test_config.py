"""The config API (afa_py.afa_config) behaves like the reference's.

Compared with records of the reference module itself
(tests/golden/config_golden.json, written by tests/golden/make_config_golden.py):
defaults, string and C++ forms, parsing, rejected strings, the validity rule
over the whole tiling grid, and the preset / progressive lists.
"""

import dataclasses
import json
from pathlib import Path

import pytest

from afa_py.afa_config import (
    AFAForwardKernelConfig,
    DType,
    get_preset_kernel_configs,
    get_progressive_configs,
    get_sm100_preset_configs,
    is_valid_config,
    sm100_kernel_key,
)

G = json.loads((Path(__file__).resolve().parent / "golden" / "config_golden.json").read_text())


def rec(cfg):
    d = dataclasses.asdict(cfg)
    d["dtype"] = int(cfg.dtype)
    return {"fields": d, "string": cfg.string_config(), "cpp": cfg.to_cpp_struct()}


def test_default_config():
    assert rec(AFAForwardKernelConfig()) == G["default"]
    assert str(AFAForwardKernelConfig()) == G["default"]["string"]


def test_dtype_values_are_torch_scalar_types():
    import torch

    assert int(DType.FP16) == 5 and int(DType.BF16) == 15
    assert DType.FP16.to_torch_dtype() == torch.float16
    assert DType.from_torch_dtype(torch.bfloat16) == DType.BF16


def test_presets_and_progressive():
    assert [rec(c) for c in get_preset_kernel_configs()] == G["presets"]
    assert [rec(c) for c in get_progressive_configs()] == G["progressive"]


@pytest.mark.parametrize("text", sorted(G["parse"]))
def test_parse(text):
    cfg = AFAForwardKernelConfig.from_string_config(text)
    assert rec(cfg) == G["parse"][text]
    assert AFAForwardKernelConfig.from_string_config(cfg.string_config()) == cfg


@pytest.mark.parametrize("text", sorted(G["bad"]))
def test_bad_strings(text):
    if G["bad"][text] == "ValueError":
        with pytest.raises(ValueError):
            AFAForwardKernelConfig.from_string_config(text)
    else:
        AFAForwardKernelConfig.from_string_config(text)


def test_validity_grid():
    for entry in G["valid_grid"]:
        br, bc, nw, asy, eag, qf, kf, vf = entry["args"]
        cfg = AFAForwardKernelConfig(DType.FP16, 128, br, bc, nw, asy, eag, True, True, True, qf, kf, vf)
        assert is_valid_config(cfg) == entry["valid"], entry


def test_sm100_presets_cover_dtype_and_head_dim():
    keys = sorted(sm100_kernel_key(c) for c in get_sm100_preset_configs())
    assert keys == [(5, 64), (5, 128), (15, 64), (15, 128)]


def test_generated_kernel_table_is_current():
    """csrc/afa_preset_kernels.inc matches what the generator renders from the presets."""
    import importlib.util
    import sys

    csrc = Path(__file__).resolve().parents[1] / "ampere_flash_attention_from_scratch_b200" / "csrc"
    spec = importlib.util.spec_from_file_location("_gen_presets", csrc / "generate_preset_kernels.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    from ampere_flash_attention_from_scratch_b200 import afa_config

    text = mod.render(afa_config.get_sm100_preset_configs(), afa_config.SM100_STAGES)
    assert (csrc / "afa_preset_kernels.inc").read_text() == text
