"""B200-native (sm_100a) DeepSeek sparse attention over a paged MLA latent cache.

Drop-in for the reference operator `kernel(q_nope, q_pe, ckv_cache, kpe_cache,
sparse_indices, sm_scale) -> (output, lse)` (solution/triton/kernel.py:138-182)
plus the FP8 lightning indexer and exact top-k that feed it.  All compute runs
in libdsa_b200.so (hand-written CUDA for sm_100a, C ABI in include/dsa_b200.h).
"""
from .kernel import (get_options, kernel, kernel_splitk, kernel_splitk_v2, options,  # noqa: F401
                     read_device_error, set_options, workspace_size)

__all__ = ["kernel", "kernel_splitk", "kernel_splitk_v2", "read_device_error", "options",
           "set_options", "get_options", "workspace_size"]
