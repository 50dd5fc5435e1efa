"""ctypes front end of the C oracle (oracle/dsa_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the flashinfer_repo_b200 package.

`build()` compiles dsa_oracle.c with gcc + OpenMP into oracle/_build/.
The attention function restates the reference golden `run`
(solution/triton/indexer_kernel.py:436-497); the indexer/top-k functions are
PARITY UNPINNED (the reference has no oracle for them), see dsa_oracle.c.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "dsa_oracle.c")
_OUT = os.path.join(_HERE, "_build", "libdsa_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle shared library (gcc -O2 -fopenmp)."""
    os.makedirs(os.path.dirname(_OUT), exist_ok=True)
    if force or not os.path.exists(_OUT) or os.path.getmtime(_OUT) < os.path.getmtime(_SRC):
        subprocess.check_call(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-std=c11",
                               "-o", _OUT, _SRC, "-lm"])
    return _OUT


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        P = ctypes.c_void_p
        I = ctypes.c_int64
        _lib.oracle_dsa_attention.argtypes = [P, P, P, P, P, I, I, I, ctypes.c_float, P, P,
                                              ctypes.c_int]
        _lib.oracle_indexer_scores.argtypes = [P, P, I, P, I, P, P, I, P, I, I, I, P,
                                               ctypes.c_int]
        _lib.oracle_topk.argtypes = [P, I, I, P, P, I, I, P, P, ctypes.c_int]
        for f in (_lib.oracle_dsa_attention, _lib.oracle_indexer_scores, _lib.oracle_topk):
            f.restype = ctypes.c_int
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _threads(n):
    return int(n if n else (os.cpu_count() or 1))


def dsa_attention(q_nope, q_pe, ckv, kpe, idx, sm_scale, nthreads=None):
    """fp64-accurate restatement of the reference `run`.

    q_nope [T,16,512], q_pe [T,16,64], ckv [P,64,512], kpe [P,64,64] are bf16
    bit patterns (uint16); idx [T,topk] int32.  Returns (out uint16 bf16 bits
    [T,16,512], lse float32 [T,16], base 2).
    """
    q_nope, q_pe, ckv, kpe = (np.ascontiguousarray(a, dtype=np.uint16)
                              for a in (q_nope, q_pe, ckv, kpe))
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    T, topk = idx.shape
    P = ckv.shape[0]
    out = np.zeros((T, 16, 512), np.uint16)
    lse = np.zeros((T, 16), np.float32)
    rc = lib().oracle_dsa_attention(_p(q_nope), _p(q_pe), _p(ckv), _p(kpe), _p(idx), T, P, topk,
                                    float(sm_scale), _p(out), _p(lse), _threads(nthreads))
    if rc != 0:
        raise ValueError("oracle_dsa_attention: index out of range")
    return out, lse


def indexer_scores(q, k_cache, k_page_stride, scale_base, s_page_stride, w, block_table,
                   seq_lens, max_len, nthreads=None):
    """Indexer scores [B, max_len] fp32 (-inf past each request's length).

    q: uint8 e4m3 bits [B,H,128]; k_cache / scale_base: uint8 byte buffers with
    per-page byte strides; w float32 [B,H]; block_table int32 [B, maxP].
    """
    q = np.ascontiguousarray(q, dtype=np.uint8)
    k_cache = np.ascontiguousarray(k_cache).view(np.uint8)
    scale_base = np.ascontiguousarray(scale_base).view(np.uint8)
    w = np.ascontiguousarray(w, dtype=np.float32)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    B, H, _ = q.shape
    out = np.empty((B, max_len), np.float32)
    lib().oracle_indexer_scores(_p(q), _p(k_cache), int(k_page_stride), _p(scale_base),
                                int(s_page_stride), _p(w), _p(bt), bt.shape[1], _p(sl), B, H,
                                int(max_len), _p(out), _threads(nthreads))
    return out


def topk(scores, seq_lens, block_table, k, nthreads=None, order="score"):
    """Exact top-k (ties -> lower position).  Returns (positions int32 [B,k],
    slots int32 [B,k]), -1 padded; order "score": descending score, ties by
    ascending position; "position": the same set in ascending position."""
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    B, L = scores.shape
    pos = np.empty((B, k), np.int32)
    slots = np.empty((B, k), np.int32)
    lib().oracle_topk(_p(scores), B, L, _p(sl), _p(bt), bt.shape[1], int(k), _p(pos), _p(slots),
                      _threads(nthreads))
    if order == "position":
        for b in range(B):
            n = int((pos[b] >= 0).sum())
            perm = np.argsort(pos[b, :n], kind="stable")
            pos[b, :n] = pos[b, :n][perm]
            slots[b, :n] = slots[b, :n][perm]
    return pos, slots


def index_cache_append(keys_bf16_bits, slot_ids, k_cache, scales):
    """Restatement of the FP8 index-key writer (no reference counterpart: the
    reference only reads this cache): per token scale = max|k|/448 in fp32
    (1 for an all-zero row), e4m3 = round-to-nearest-even(k/scale), saturating.
    Writes into k_cache [P,64,128] uint8 and scales [P,64] float32 in place."""
    from flashinfer_repo_b200.workloads import bf16_bits_to_f32, f32_to_e4m3_bits
    k = bf16_bits_to_f32(keys_bf16_bits).reshape(-1, 128)
    for i, sid in enumerate(np.asarray(slot_ids)):
        if sid < 0:
            continue
        amax = np.float32(np.abs(k[i]).max())
        sc = np.float32(amax / np.float32(448.0)) if amax > 0 else np.float32(1.0)
        k_cache[sid >> 6, sid & 63] = f32_to_e4m3_bits((k[i] / sc).astype(np.float32))
        scales[sid >> 6, sid & 63] = sc
