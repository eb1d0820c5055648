"""Generates tests/golden/config_golden.json from the reference's Python config
module (afa_py/afa_config.py), imported from a reference checkout.

Records, for the reference implementation: the preset and progressive config
lists (string form and C++ struct form), the parse of a set of config strings,
and is_valid_config over the full tiling grid.  tests/test_config.py compares
ampere_flash_attention_from_scratch_b200.afa_config with these records.

Usage: python tests/golden/make_config_golden.py REFERENCE_DIR
(or with AFA_REFERENCE_DIR set in the environment instead of the argument).
"""

import dataclasses
import itertools
import json
import sys
from pathlib import Path

PARSE_CASES = [
    "(FP16, 128, 64, 32, 4): async+eager+swizzled+buffer+opt_softmax+load_2_2_2_tiles",
    "(BF16, 64, 128, 64, 8): async+swizzled+load_0_2_0_tiles",
    "(FP16, 128, 64, 32, 4): ",
    "(FP16,128,64,64,4):eager+opt_softmax",
    "(BF16, 128, 64, 32, 4): load_2_2_tiles+async",
    "(FP16, 128, 64, 32, 4): load_1_2_3_tiles+load_2_2_2_tiles",
]
BAD_CASES = ["FP16, 128, 64, 32, 4", "(FP16, 128, 64, 32): async", "(FP32, 128, 64, 32, 4): async", "[FP16, 128, 64, 32, 4]: async"]


def main(ref_dir: Path, out: Path):
    sys.path.insert(0, str(ref_dir))
    from afa_py import afa_config as ac  # the reference module

    def rec(cfg):
        d = dataclasses.asdict(cfg)
        d["dtype"] = int(cfg.dtype)
        return {"fields": d, "string": cfg.string_config(), "cpp": cfg.to_cpp_struct()}

    grid = []
    for combo in itertools.product([64, 128], [32, 64], [4, 8], [False, True], [False, True], [0, 2], [0, 2], [0, 2]):
        br, bc, nw, asy, eag, qf, kf, vf = combo
        cfg = ac.AFAForwardKernelConfig(ac.DType.FP16, 128, br, bc, nw, asy, eag, True, True, True, qf, kf, vf)
        grid.append({"args": list(combo), "valid": bool(ac.is_valid_config(cfg))})
    bad = {}
    for s in BAD_CASES:
        try:
            ac.AFAForwardKernelConfig.from_string_config(s)
            bad[s] = "ok"
        except ValueError:
            bad[s] = "ValueError"
    data = {
        "default": rec(ac.AFAForwardKernelConfig()),
        "presets": [rec(c) for c in ac.get_preset_kernel_configs()],
        "progressive": [rec(c) for c in ac.get_progressive_configs()],
        "parse": {s: rec(ac.AFAForwardKernelConfig.from_string_config(s)) for s in PARSE_CASES},
        "bad": bad,
        "valid_grid": grid,
    }
    out.write_text(json.dumps(data, indent=1, sort_keys=True))
    print(f"wrote {out}")


if __name__ == "__main__":
    import os

    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AFA_REFERENCE_DIR")
    if not arg:
        sys.exit("usage: make_config_golden.py REFERENCE_DIR (or set AFA_REFERENCE_DIR)")
    ref = Path(arg)
    main(ref, Path(__file__).resolve().parent / "config_golden.json")
