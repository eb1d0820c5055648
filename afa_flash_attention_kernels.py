"""Reference import path of the torch extension (``import afa_flash_attention_kernels as fa``).

Re-exports the sm_100a extension built inside ampere_flash_attention_from_scratch_b200;
``forward(kernel_cfg, q, k, v, o, benchmark=False) -> (O, runtime_ms)`` as in the
reference binding (csrc/ampere_flash_attention.cu:138-141), plus
``forward_ext(q, k, v, o=None, causal=False, softmax_scale=None, return_lse=False)
-> (O, lse)`` for K/V of their own length and head count, the causal mask and
the log-sum-exp output, and ``forward_host(q, k, v, o=None, causal=False, chunks=0) -> O``
for host-resident tensors (copies in, compute and copies out overlapped per batch slice).
"""

from ampere_flash_attention_from_scratch_b200.afa_flash_attention_kernels import (  # noqa: F401
    _raise_formatted_error,
    _set_test_flags,
    check_status,
    forward,
    forward_ext,
    forward_host,
    kernel_keys,
)
