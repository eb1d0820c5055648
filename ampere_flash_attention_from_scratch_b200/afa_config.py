"""Kernel configuration object of the attention-forward API.

Mirrors the reference's Python config module (afa_py/afa_config.py): the same
``DType`` values, the same ``AFAForwardKernelConfig`` fields and defaults, the
same string form ``"(FP16, 128, 64, 32, 4): async+eager+swizzled+buffer+
opt_softmax+load_2_2_2_tiles"``, the same validity rules and preset lists, so
code written against the reference keeps working unchanged.

On sm_100a one kernel exists per (dtype, head_dim); the Ampere tiling knobs
(B_r, B_c, n_warps, async/eager/swizzled/buffer/opt_softmax, load_x_y_z) are
accepted and carried along but do not select a different kernel.
``get_sm100_preset_configs`` lists the configurations the sm_100a library is
compiled for, with the tile sizes it really uses.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass
from enum import IntEnum

import torch

__all__ = [
    "DType",
    "AFAForwardKernelConfig",
    "is_valid_config",
    "get_preset_kernel_configs",
    "get_progressive_configs",
    "get_sm100_preset_configs",
    "sm100_kernel_key",
]


class DType(IntEnum):
    """Element type; the values are torch ScalarType codes (afa_py/afa_config.py:8-28)."""

    FP16 = 5
    BF16 = 15

    def to_cpp_str(self) -> str:
        names = {DType.FP16: "torch::kFloat16", DType.BF16: "torch::kBFloat16"}
        if self not in names:
            raise ValueError(f"Invalid DType: {self}")
        return names[self]

    def to_torch_dtype(self):
        table = {DType.FP16: torch.float16, DType.BF16: torch.bfloat16}
        if self not in table:
            raise ValueError(f"Invalid DType: {self}")
        return table[self]

    @classmethod
    def from_torch_dtype(cls, dt) -> "DType":
        if dt == torch.float16:
            return cls.FP16
        if dt == torch.bfloat16:
            return cls.BF16
        raise ValueError(f"Only fp16 and bf16 are supported, got {dt}")


# The optional-feature flags in the order the string form lists them
# (afa_py/afa_config.py:61-75): (attribute name, token).
_FLAG_TOKENS = (
    ("async_copy", "async"),
    ("eager_load_blocks", "eager"),
    ("swizzled", "swizzled"),
    ("mma_double_buffer_loads", "buffer"),
    ("optimized_softmax", "opt_softmax"),
)


@dataclass
class AFAForwardKernelConfig:
    """Kernel selection key passed to ``afa_flash_attention_kernels.forward``.

    Field names, order and defaults follow afa_py/afa_config.py:33-48.
    """

    dtype: DType = DType(5)
    d_head: int = 128
    B_r: int = 64
    B_c: int = 32
    n_warps: int = 4
    async_copy: bool = True
    eager_load_blocks: bool = True
    swizzled: bool = True
    mma_double_buffer_loads: bool = True
    optimized_softmax: bool = True

    Q_col_fragments_per_warp_gemm: int = 2
    K_col_fragments_per_warp_gemm: int = 2
    V_col_fragments_per_warp_gemm: int = 2

    def to_torch_dtype(self):
        # The reference returns the DType itself (afa_py/afa_config.py:50-51);
        # its binding casts that IntEnum to a torch ScalarType.
        return self.dtype

    def __str__(self):
        return self.string_config()

    def string_config(self) -> str:
        head = f"({self.dtype.name}, {self.d_head}, {self.B_r}, {self.B_c}, {self.n_warps}): "
        tokens = [tok for attr, tok in _FLAG_TOKENS if getattr(self, attr)]
        tokens.append(
            "load_{}_{}_{}_tiles".format(
                self.Q_col_fragments_per_warp_gemm,
                self.K_col_fragments_per_warp_gemm,
                self.V_col_fragments_per_warp_gemm,
            )
        )
        return head + "+".join(tokens)

    def to_cpp_struct(self) -> str:
        def lit(v):
            return str(v).lower() if isinstance(v, bool) else str(v)

        fields = [
            self.dtype.to_cpp_str(),
            self.d_head,
            self.B_r,
            self.B_c,
            self.n_warps,
            self.async_copy,
            self.eager_load_blocks,
            self.swizzled,
            self.mma_double_buffer_loads,
            self.optimized_softmax,
            self.Q_col_fragments_per_warp_gemm,
            self.K_col_fragments_per_warp_gemm,
            self.V_col_fragments_per_warp_gemm,
        ]
        return "AFAForwardKernelConfig{" + ", ".join(lit(f) for f in fields) + "}"

    @classmethod
    def from_string_config(cls, config_str: str) -> "AFAForwardKernelConfig":
        """Parse the string form (afa_py/afa_config.py:95-179).

        ``"(FP16, 128, 64, 32, 4): async+eager+swizzled+buffer+opt_softmax+load_2_2_2_tiles"``
        Flags that are absent are False; a missing ``load_x_y_z_tiles`` token
        means 0/0/0.  Malformed strings raise ``ValueError``.
        """
        if ":" not in config_str:
            raise ValueError(f"Invalid config string format: {config_str}")
        base, flags = (part.strip() for part in config_str.split(":", 1))
        if not (base.startswith("(") and base.endswith(")")):
            raise ValueError(f"Invalid base part format: {base}")
        values = [v.strip() for v in base[1:-1].split(",")]
        if len(values) != 5:
            raise ValueError(f"Expected 5 values in base part, got {len(values)}")
        try:
            dtype = DType[values[0]]
        except KeyError:
            raise ValueError(f"Invalid dtype: {values[0]}") from None
        d_head, B_r, B_c, n_warps = (int(v) for v in values[1:])

        tokens = [t.strip() for t in flags.split("+")]
        kwargs = {attr: (tok in tokens) for attr, tok in _FLAG_TOKENS}
        frags = (0, 0, 0)
        for tok in tokens:
            if tok.startswith("load_") and tok.endswith("_tiles"):
                parts = tok[len("load_") : -len("_tiles")].split("_")
                if len(parts) == 3:
                    frags = tuple(int(x) for x in parts)
                break
        return cls(
            dtype=dtype,
            d_head=d_head,
            B_r=B_r,
            B_c=B_c,
            n_warps=n_warps,
            Q_col_fragments_per_warp_gemm=frags[0],
            K_col_fragments_per_warp_gemm=frags[1],
            V_col_fragments_per_warp_gemm=frags[2],
            **kwargs,
        )


def is_valid_config(cfg: AFAForwardKernelConfig) -> bool:
    """Validity rules of the reference's Ampere tiling (afa_py/afa_config.py:183-205)."""
    if cfg.eager_load_blocks and not cfg.async_copy:
        return False
    q, k = cfg.Q_col_fragments_per_warp_gemm, cfg.K_col_fragments_per_warp_gemm
    if q != 0 and q != k:
        return False
    if cfg.B_r == 64:
        if cfg.n_warps == 8:
            return False
        if cfg.B_c == 32 and q == 0:
            return False
        if cfg.B_c == 64 and q != 0:
            return False
    elif cfg.B_r == 128 and q == 0:
        return False
    return True


def get_preset_kernel_configs() -> list[AFAForwardKernelConfig]:
    """The reference's preset enumeration (afa_py/afa_config.py:208-243): the
    valid members of FP16 x d128 x B_r{64,128} x B_c{32,64} x warps{4,8} x
    fragments{0,2}^3 with every optimisation switched on."""
    axes = (
        [DType.FP16],
        [128],
        [64, 128],
        [32, 64],
        [4, 8],
        [True],
        [True],
        [True],
        [True],
        [True],
        [0, 2],
        [0, 2],
        [0, 2],
    )
    out = []
    for combo in itertools.product(*axes):
        cfg = AFAForwardKernelConfig(*combo)
        if is_valid_config(cfg):
            out.append(cfg)
    return out


def get_progressive_configs() -> list[AFAForwardKernelConfig]:
    """The reference's ablation ladder (afa_py/afa_config.py:246-266)."""
    steps = (
        "",
        "async",
        "async+eager",
        "async+eager+swizzled",
        "async+eager+swizzled+load_2_2_2_tiles",
        "async+eager+swizzled+buffer+load_2_2_2_tiles",
    )
    out = []
    for opts in steps:
        text = f"(FP16, 128, 64, 32, 4): {opts}" if opts else "(FP16, 128, 64, 32, 4): "
        try:
            out.append(AFAForwardKernelConfig.from_string_config(text))
        except ValueError:
            continue
    return out


# Tiling of the sm_100a kernel: 256 query rows per CTA (two 128-row Q tiles),
# 128-row K/V tiles, 12 warps (TMA, MMA, TMEM-alloc, spare, 2 softmax warpgroups).
SM100_B_R = 256
SM100_B_C = 128
SM100_N_WARPS = 12
# K/V ring depth per head_dim (shared memory: 2 Q tiles + stages x one K/V tile).
SM100_STAGES = {64: 8, 128: 4}


def get_sm100_preset_configs() -> list[AFAForwardKernelConfig]:
    """Configurations the sm_100a library is compiled for: {FP16, BF16} x {64, 128}."""
    out = []
    for dtype in (DType.FP16, DType.BF16):
        for d in (128, 64):
            out.append(
                AFAForwardKernelConfig(
                    dtype=dtype,
                    d_head=d,
                    B_r=SM100_B_R,
                    B_c=SM100_B_C,
                    n_warps=SM100_N_WARPS,
                    Q_col_fragments_per_warp_gemm=0,
                    K_col_fragments_per_warp_gemm=0,
                    V_col_fragments_per_warp_gemm=0,
                )
            )
    return out


def sm100_kernel_key(cfg: AFAForwardKernelConfig) -> tuple[int, int]:
    """(dtype code, head_dim): the key of the sm_100a kernel table."""
    return int(DType(cfg.dtype)), int(cfg.d_head)
