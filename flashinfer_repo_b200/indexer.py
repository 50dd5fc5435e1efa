"""FP8 lightning indexer + exact top-k (the step that produces `sparse_indices`).

Replaces the reference's `run_indexer_and_topk` (solution/triton/indexer_kernel.py:
345-433: indexer_kernel + topk_kernel) with the sm_100a kernels of
libdsa_b200.so.  Differences from the reference, all deliberate:
  * keys are fp8 rows of 128 bytes with an fp32 per-token scale (the layout of
    BASELINE cfg4: keys [P,64,128] + scales [P,64], or the page-packed format
    via byte strides); the reference reads a single fp8 byte as the scale from
    a 129-byte interleaved row (indexer_kernel.py:186-197);
  * selection is exact with a total order (descending score, ties toward the
    lower position); the reference's replace-the-minimum loop duplicates ids
    on ties (indexer_kernel.py:335-339);
  * it returns token positions and the physical slot ids that `kernel()`
    consumes; the reference returns logical concatenated ids (:317);
  * no device-to-host synchronisation (the reference calls .item() twice,
    :371, :384): the score buffer is sized from the block-table width.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

NUM_INDEX_HEADS = 64
INDEX_HEAD_DIM = 128
PAGE_SIZE = 64


def _u8(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.uint8:
        return t
    if t.dtype == getattr(torch, "float8_e4m3fn", None):
        return t.view(torch.uint8)
    raise AssertionError(f"expected fp8 e4m3 (or its uint8 bits), got {t.dtype}")


def indexer_scores(q_fp8, k_cache_fp8, k_scale, weights, seq_lens, block_table, *, max_len=None,
                   num_pages=None, k_page_stride=None, scale_page_stride=None, out=None,
                   device_error=None):
    """Indexer scores [B, max_len] fp32: scores[b, t] = scale_t * sum_h w[b,h] *
    ReLU(q[b,h] . k8_t) for t < seq_lens[b]; entries past seq_lens[b] are left
    as they were (zero when `out` is allocated here).

    q_fp8 [B,64,128] and k_cache_fp8 [P,64,128] are float8_e4m3fn (or uint8
    bits); k_scale [P,64] fp32.  For the page-packed format pass the byte
    strides and num_pages explicitly.
    """
    q = _u8(q_fp8).contiguous()
    kc = _u8(k_cache_fp8)
    B, H, D = q.shape
    assert H == NUM_INDEX_HEADS and D == INDEX_HEAD_DIM
    for name, t in (("q", q), ("k_cache", kc), ("k_scale", k_scale), ("weights", weights),
                    ("seq_lens", seq_lens), ("block_table", block_table)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor (no CPU path)")
    assert weights.dtype == torch.float32 and weights.shape == (B, H)
    weights = weights.contiguous()
    seq_lens = seq_lens.to(torch.int32).contiguous()
    block_table = block_table.to(torch.int32)
    assert block_table.stride(-1) == 1
    if max_len is None:
        max_len = block_table.shape[1] * PAGE_SIZE
    if num_pages is None:
        num_pages = kc.shape[0]
    if k_page_stride is None:
        assert kc.stride(-1) == 1 and kc.stride(-2) == INDEX_HEAD_DIM
        k_page_stride = kc.stride(0)
    if scale_page_stride is None:
        assert k_scale.dtype == torch.float32 and k_scale.stride(-1) == 1
        scale_page_stride = k_scale.stride(0) * 4
    if out is None:
        out = torch.zeros((B, max_len), dtype=torch.float32, device=q.device)
    err_ptr = device_error.data_ptr() if device_error is not None else None
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.call("dsa_indexer_scores", q.data_ptr(), kc.data_ptr(), int(k_page_stride),
                  k_scale.data_ptr(), int(scale_page_stride), weights.data_ptr(),
                  block_table.data_ptr(), block_table.stride(0), seq_lens.data_ptr(), B, H, D,
                  int(num_pages), int(max_len), out.data_ptr(), out.stride(0), err_ptr,
                  ctypes.c_void_p(stream))
    return out


def topk_select(scores, seq_lens, block_table=None, topk=2048, order="score", out=None):
    """Exact top-k per row of `scores` [B, L] over the first seq_lens[b] entries
    (ties toward the lower position).  Returns (positions [B, topk] int32,
    slots [B, topk] int32 or None), -1 padded; order "score" emits descending
    score (ties by ascending position), "position" emits ascending position
    (skips the sort).  out: optional (positions, slots) int32 [B, topk] row-major
    tensors to write into (slots None when block_table is None)."""
    assert order in ("score", "position")
    assert scores.dtype == torch.float32 and scores.stride(-1) == 1 and scores.is_cuda
    B = scores.shape[0]
    seq_lens = seq_lens.to(torch.int32).contiguous()
    if out is not None:
        pos, slots = out
        for t in (pos, slots):
            assert t is None or (t.dtype == torch.int32 and t.shape == (B, topk) and t.is_contiguous())
        assert (slots is None) == (block_table is None)
    else:
        pos = torch.empty((B, topk), dtype=torch.int32, device=scores.device)
        slots = None
    bt_ptr, bt_stride = None, 0
    if block_table is not None:
        block_table = block_table.to(torch.int32)
        if slots is None:
            slots = torch.empty_like(pos)
        bt_ptr, bt_stride = block_table.data_ptr(), block_table.stride(0)
    with torch.cuda.device(scores.device):
        stream = torch.cuda.current_stream(scores.device).cuda_stream
        _lib.call("dsa_topk_select", scores.data_ptr(), scores.stride(0), seq_lens.data_ptr(), bt_ptr,
                  bt_stride, B, int(topk), pos.data_ptr(),
                  slots.data_ptr() if slots is not None else None, 0 if order == "score" else 1,
                  ctypes.c_void_p(stream))
    return pos, slots


def indexer_topk(q_fp8, k_cache_fp8, k_scale, weights, seq_lens, block_table, topk=2048,
                 order="score", **kw):
    """Indexer scores then exact top-k; returns (positions, slots).  `slots`
    can be passed straight to `kernel()` as `sparse_indices` (one row per
    request / decode token)."""
    scores = indexer_scores(q_fp8, k_cache_fp8, k_scale, weights, seq_lens, block_table, **kw)
    return topk_select(scores, seq_lens, block_table, topk, order)


def index_cache_append(keys, slot_ids, k_cache_fp8, k_scale, *, num_pages=None, k_page_stride=None,
                       scale_page_stride=None, device_error=None):
    """Quantise `keys` [N,128] (bf16) to e4m3 with a per-token scale max|k|/448
    and write them at flat slot ids `slot_ids` [N] (-1 = skip) of the paged
    index-key cache (k_cache_fp8 [P,64,128] + k_scale [P,64], or the page-packed
    layout via byte strides)."""
    assert keys.dtype == torch.bfloat16 and keys.shape[-1] == INDEX_HEAD_DIM and keys.is_cuda
    keys = keys.contiguous()
    slot_ids = slot_ids.to(torch.int32).contiguous()
    kc = _u8(k_cache_fp8)
    if num_pages is None:
        num_pages = kc.shape[0]
    if k_page_stride is None:
        k_page_stride = kc.stride(0)
    if scale_page_stride is None:
        scale_page_stride = k_scale.stride(0) * 4
    err_ptr = device_error.data_ptr() if device_error is not None else None
    with torch.cuda.device(keys.device):
        stream = torch.cuda.current_stream(keys.device).cuda_stream
        _lib.call("dsa_index_cache_append", keys.data_ptr(), keys.shape[0], slot_ids.data_ptr(),
                  kc.data_ptr(), int(k_page_stride), k_scale.data_ptr(), int(scale_page_stride),
                  int(num_pages), err_ptr, ctypes.c_void_p(stream))
