"""Drop-in `kernel` for the DSA sparse-attention operator.

Same name, arguments, return values and shape checks as the reference entry
point `kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale)
-> (output, lse)` (solution/triton/kernel.py:138-182, entry point named in
config.toml:8, destination_passing_style = false).  The work runs in the
sm_100a CUDA kernel of libdsa_b200.so, called through its C ABI on torch's
current stream.  There is no Triton, no dispatch and no CPU fallback: CPU
tensors or a missing library raise.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading

import torch

from . import _lib

NUM_HEADS = 16
HEAD_DIM_CKV = 512
HEAD_DIM_KPE = 64
PAGE_SIZE = 64
TOPK = 2048


class _Workspace:
    """Per-device persistent workspace: the device error word (zeroed when
    allocated, cleared by read_device_error) followed by split-K partials."""

    def __init__(self):
        self.buf = None
        self.lock = threading.Lock()

    def get(self, device, nbytes):
        with self.lock:
            if self.buf is None or self.buf.numel() < nbytes:
                self.buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            return self.buf


_workspaces: dict[int, _Workspace] = {}
_ws_size_cache: dict[tuple, int] = {}


def workspace_for(device: torch.device) -> _Workspace:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None:
        ws = _workspaces.setdefault(idx, _Workspace())
    return ws


def _rowmajor(t: torch.Tensor, align_elems: int) -> torch.Tensor:
    """Keep strided views when the last dim is contiguous and rows are aligned."""
    ok = t.stride(-1) == 1 and all(s % align_elems == 0 for s in t.stride()[:-1])
    ok = ok and (t.data_ptr() % (2 * align_elems) == 0)
    return t if ok else t.contiguous()


def _check_inputs(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices):
    num_tokens, num_qo_heads, head_dim_ckv = q_nope.shape
    num_pages, page_size, _ = ckv_cache.shape
    head_dim_kpe = q_pe.shape[-1]
    topk = sparse_indices.shape[-1]
    # the reference's static assertions (kernel.py:147-151); heads may be any
    # multiple of 16 here (independent 16-head groups sharing the indices)
    assert num_qo_heads % NUM_HEADS == 0 and num_qo_heads > 0
    assert head_dim_ckv == HEAD_DIM_CKV
    assert head_dim_kpe == HEAD_DIM_KPE
    assert page_size == PAGE_SIZE
    assert topk % 32 == 0 and topk > 0
    assert q_pe.shape[:2] == q_nope.shape[:2]
    assert kpe_cache.shape == (num_pages, page_size, head_dim_kpe)
    assert sparse_indices.shape[0] == num_tokens
    for name, t in (("q_nope", q_nope), ("q_pe", q_pe), ("ckv_cache", ckv_cache),
                    ("kpe_cache", kpe_cache), ("sparse_indices", sparse_indices)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor (no CPU path)")
    for name, t in (("q_nope", q_nope), ("q_pe", q_pe), ("ckv_cache", ckv_cache),
                    ("kpe_cache", kpe_cache)):
        assert t.dtype == torch.bfloat16, f"{name} must be bfloat16"
    return num_tokens, num_qo_heads, num_pages, topk


def kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, *, output=None,
           lse=None, workspace=None):
    """DSA sparse attention; returns (output [T,H,512] bf16, lse [T,H] fp32 base-2).

    output/lse may be passed to write into existing tensors (same shapes);
    by default they are allocated, like the reference (kernel.py:156-157).
    workspace: optional uint8 CUDA tensor of at least workspace_size(T, H,
    topk) bytes, 256-byte aligned, zeroed before its first use (its first
    word is the device error word); calls that may run concurrently (on
    different streams) each need their own.  Default: the device's shared
    workspace, so such calls must not overlap.
    """
    num_tokens, heads, num_pages, topk = _check_inputs(q_nope, q_pe, ckv_cache, kpe_cache,
                                                       sparse_indices)
    device = q_nope.device
    if output is None:
        output = torch.empty((num_tokens, heads, HEAD_DIM_CKV), dtype=torch.bfloat16, device=device)
    if lse is None:
        lse = torch.empty((num_tokens, heads), dtype=torch.float32, device=device)
    if num_tokens == 0:
        return output, lse
    assert output.stride(-1) == 1 and lse.stride(-1) == 1

    _launch("dsa_sparse_attention", q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale,
            num_tokens, heads, num_pages, topk,
            (output.data_ptr(), output.stride(0), output.stride(1),
             lse.data_ptr(), lse.stride(0), lse.stride(1)), workspace=workspace)
    return output, lse


def workspace_size(num_tokens: int, heads: int = NUM_HEADS, topk: int = 2048, device=None) -> int:
    """Bytes of the attention workspace a call of this shape needs on `device`
    (default: the current device) under the current options."""
    device = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    with torch.cuda.device(device):
        return _workspace_bytes(device, num_tokens, heads, topk)


_OPTION_FIELDS = [f for f, _ in _lib.Options._fields_]
_options_generation = [0]  # bumped by set_options: cached workspace sizes depend on the plan


def get_options() -> dict:
    """The library's current tuning options (struct dsa_options) as a dict."""
    o = _lib.Options()
    _lib.call("dsa_get_options", ctypes.byref(o))
    return {f: getattr(o, f) for f in _OPTION_FIELDS}


def set_options(**fields) -> None:
    """Set tuning/profiling options of the native library (process-wide).
    Unnamed fields keep their defaults; set_options() restores all defaults.
    Nothing is read from the environment."""
    unknown = set(fields) - set(_OPTION_FIELDS)
    if unknown:
        raise TypeError(f"unknown option(s) {sorted(unknown)}")
    o = _lib.Options(merge_pdl=1)
    for f, v in fields.items():
        setattr(o, f, int(v))
    _lib.call("dsa_set_options", ctypes.byref(o))
    _options_generation[0] += 1


@contextlib.contextmanager
def options(**fields):
    """`with options(attention_ctas=7): ...` -- options for the block, the
    previous set restored afterwards (for tests and profiling)."""
    prev = get_options()
    set_options(**fields)
    try:
        yield
    finally:
        set_options(**prev)


def _workspace_bytes(device, num_tokens, heads, topk):
    # the plan (and so the size) also depends on the tuning options
    key = (device.index, num_tokens, heads, topk, _options_generation[0])
    nbytes = _ws_size_cache.get(key)
    if nbytes is None:
        n = ctypes.c_size_t(0)
        _lib.call("dsa_sparse_attention_workspace_size", num_tokens, heads, topk, ctypes.byref(n))
        nbytes = _ws_size_cache[key] = n.value
    return nbytes


def _launch(fn, q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, num_tokens, heads,
            num_pages, topk, out_args, workspace=None):
    if sparse_indices.dtype != torch.int32:
        sparse_indices = sparse_indices.to(torch.int32)
    if sparse_indices.stride(-1) != 1:
        sparse_indices = sparse_indices.contiguous()
    q_nope = _rowmajor(q_nope, 2)
    q_pe = _rowmajor(q_pe, 2)
    ckv_cache = _rowmajor(ckv_cache, 8)
    kpe_cache = _rowmajor(kpe_cache, 8)
    device = q_nope.device
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        nbytes = _workspace_bytes(device, num_tokens, heads, topk)
        if workspace is not None:
            if not (workspace.is_cuda and workspace.device == device and workspace.dtype == torch.uint8
                    and workspace.is_contiguous()):
                raise ValueError("workspace must be a contiguous uint8 tensor on the inputs' device")
            ws = workspace  # the library checks its size and alignment
        else:
            ws = workspace_for(device).get(device, nbytes)
        _lib.call(
            fn,
            q_nope.data_ptr(), q_nope.stride(0), q_nope.stride(1),
            q_pe.data_ptr(), q_pe.stride(0), q_pe.stride(1),
            ckv_cache.data_ptr(), ckv_cache.stride(0), ckv_cache.stride(1),
            kpe_cache.data_ptr(), kpe_cache.stride(0), kpe_cache.stride(1),
            sparse_indices.data_ptr(), sparse_indices.stride(0),
            num_tokens, heads, num_pages, PAGE_SIZE, topk, float(sm_scale),
            *out_args, ws.data_ptr(), ws.numel(), ctypes.c_void_p(stream.cuda_stream))


def kernel_scatter(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, out_ptrs,
                   lse_ptrs, out_strides, lse_strides, sync=None):
    """`kernel` whose results are stored into every (out_ptrs[k], lse_ptrs[k])
    target (device addresses, peer GPUs' included, each offset to where these
    heads belong; up to 8) with the given (token, head) element strides,
    instead of into freshly allocated tensors.  Returns nothing.  Without
    `sync` the caller orders the stores (e.g. with a peer barrier); with
    sync = (flags, rank, world) -- flags a ctypes array of the ranks' flag
    buffers as mapped here -- the operator ends with that cross-GPU barrier
    itself (dsa_sparse_attention_scatter_sync)."""
    num_tokens, heads, num_pages, topk = _check_inputs(q_nope, q_pe, ckv_cache, kpe_cache,
                                                       sparse_indices)
    n = len(out_ptrs)
    assert n == len(lse_ptrs) and 1 <= n <= 8
    if num_tokens == 0:
        return
    outs = (ctypes.c_void_p * n)(*out_ptrs)
    lses = (ctypes.c_void_p * n)(*lse_ptrs)
    targets = (ctypes.cast(outs, ctypes.c_void_p), int(out_strides[0]), int(out_strides[1]),
               ctypes.cast(lses, ctypes.c_void_p), int(lse_strides[0]), int(lse_strides[1]), n)
    if sync is None:
        _launch("dsa_sparse_attention_scatter", q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices,
                sm_scale, num_tokens, heads, num_pages, topk, targets)
    else:
        flags, rank, world = sync
        _launch("dsa_sparse_attention_scatter_sync", q_nope, q_pe, ckv_cache, kpe_cache,
                sparse_indices, sm_scale, num_tokens, heads, num_pages, topk,
                targets + (ctypes.cast(flags, ctypes.c_void_p), int(rank), int(world)))


def kernel_splitk(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, SPLIT_K=None):
    """Same signature as the reference's kernel_splitk (kernel.py:496).  The
    split of the top-k dimension is chosen by occupancy inside the library,
    so SPLIT_K is accepted for compatibility and ignored."""
    return kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale)


kernel_splitk_v2 = kernel_splitk


def read_device_error(device=None, clear=True) -> int:
    """Synchronise and return the DSA_DEVERR_* bits raised by kernels that
    used this device's workspace (bad indices, timed-out waits)."""
    device = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    ws = workspace_for(device).buf
    if ws is None:
        return 0
    bits = ctypes.c_int(0)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        _lib.call("dsa_read_device_error", ws.data_ptr(), int(clear), ctypes.byref(bits),
                  ctypes.c_void_p(stream.cuda_stream))
    return bits.value
