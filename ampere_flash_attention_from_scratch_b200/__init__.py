"""B200 (sm_100a) FlashAttention forward behind the reference's API.

Drop-in surface (same names as the reference):

    import afa_flash_attention_kernels as fa          # or: from ampere_flash_attention_from_scratch_b200 import forward
    from afa_py.afa_config import AFAForwardKernelConfig
    O, ms = fa.forward(AFAForwardKernelConfig(), q, k, v, o, benchmark)

``forward`` runs the hand-written tcgen05/TMA kernel in ``libafa_sm100.so``;
there is no other implementation behind it.  If the native extension is not
built, importing ``forward`` raises ImportError (build with
``python -m ampere_flash_attention_from_scratch_b200.build``).
"""

from .afa_config import (  # noqa: F401
    AFAForwardKernelConfig,
    DType,
    get_preset_kernel_configs,
    get_progressive_configs,
    get_sm100_preset_configs,
    is_valid_config,
    sm100_kernel_key,
)


def _load_extension():
    try:
        from . import afa_flash_attention_kernels as ext  # native torch extension
    except ImportError as e:  # pragma: no cover - exercised only when unbuilt
        raise ImportError(
            "the sm_100a extension afa_flash_attention_kernels is not built: run "
            "`python -m ampere_flash_attention_from_scratch_b200.build` (" + str(e) + ")"
        ) from e
    return ext


def __getattr__(name):
    if name in ("forward", "forward_ext", "forward_host", "check_status", "kernel_keys"):
        return getattr(_load_extension(), name)
    raise AttributeError(name)
