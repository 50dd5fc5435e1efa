"""TVM-FFI registration of the operator: fills the slot the reference leaves
empty (`@register_func("flashinfer.kernel")`, solution/cuda/binding.py:14-25;
the template imports `tvm.ffi`, the installed package is `tvm_ffi`).

    from flashinfer_repo_b200.binding import register
    register()                      # "flashinfer.kernel" -> kernel()
    f = tvm_ffi.get_global_func("flashinfer.kernel")
    output, lse = f(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale)

Arguments arrive as TVM-FFI tensors and are viewed as torch tensors through
DLPack (no copy); the work is the same sm_100a kernel.
"""
from __future__ import annotations

import torch

from .kernel import kernel


def _as_torch(t):
    return t if isinstance(t, torch.Tensor) else torch.from_dlpack(t)


def register(name: str = "flashinfer.kernel"):
    import tvm_ffi

    def ffi_kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale):
        out, lse = kernel(_as_torch(q_nope), _as_torch(q_pe), _as_torch(ckv_cache),
                          _as_torch(kpe_cache), _as_torch(sparse_indices), float(sm_scale))
        return out, lse

    tvm_ffi.register_global_func(name, ffi_kernel, override=True)
    return tvm_ffi.get_global_func(name)
