"""Reference import path ``afa_py.afa_config`` (afa_py/afa_config.py of the
reference), re-exported from ampere_flash_attention_from_scratch_b200.afa_config."""

from ampere_flash_attention_from_scratch_b200.afa_config import *  # noqa: F401,F403
from ampere_flash_attention_from_scratch_b200.afa_config import (  # noqa: F401
    SM100_B_C,
    SM100_B_R,
    SM100_N_WARPS,
    SM100_STAGES,
)
