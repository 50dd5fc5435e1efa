"""Golden attention cases: the seeded inputs behind tests/golden/*.npz.

The fixtures hold only the reference's outputs plus a digest of the inputs;
the inputs themselves are regenerated from the parameters here (numpy PCG64,
bit-reproducible), so the fixture files stay small.
"""
from __future__ import annotations

import hashlib

import numpy as np

from flashinfer_repo_b200 import workloads as W


def _edge_case():
    """Edge cases the reference operator has to handle (kernel.py:97,118-136;
    indexer_kernel.py:469-475): tail padding (context < 2048), interior -1,
    an all-padding token, duplicate indices, a single valid index."""
    case = W.make_attention_case(11, [3000, 1000, 3000, 3000, 3000, 3000, 2048, 5000])
    rng = np.random.default_rng(12)
    idx = case.idx
    idx[2, rng.random(W.TOPK) < 0.3] = -1                 # interior padding
    idx[3, :] = -1                                       # nothing valid
    dup = idx[4, :16].copy()
    idx[4, :] = np.tile(dup, W.TOPK // 16)               # 128 copies of 16 rows
    idx[5, 1:] = -1                                      # one valid row
    idx[6, :1024] = -1                                   # leading padding
    return case


def _big_logits_case():
    return W.make_attention_case(21, [4096, 4096], kv_std=2.0, shared_cache=True)


def _alt_scale_case():
    return W.make_attention_case(31, [4096, 8192, 2500], kv_std=1.0,
                                 sm_scale=0.1352337788608801)


def _cfg2_small_case():
    """cfg2's shape (T=64 tokens of independent requests, shuffled page
    tables, 2048 distinct positions, -1 padded) with contexts drawn from
    U[1024, 4096] instead of U[1024, 65536], so that the host can regenerate
    the inputs in about a second."""
    return W.make_attention_case(51, W.cfg2_ctx_lens(51, 64, 1024, 4096))


CASES = {
    "cfg1_seed0": lambda: W.cfg1_case(0),
    "edge": _edge_case,
    "big_logits": _big_logits_case,
    "alt_scale": _alt_scale_case,
    "cfg2_small": _cfg2_small_case,
}

# Indexer inputs for the reference's own indexer / top-k kernels: exact by
# construction (every score exact in fp16 products and fp32 sums, in any
# order), power-of-two batches, contexts short enough for the reference's
# unrolled top-k loop.
INDEXER_CASES = {
    "exact_b4": lambda: W.make_indexer_case(61, [1024, 777, 1000, 512], exact=True),
    "exact_b2": lambda: W.make_indexer_case(62, [1500, 333], exact=True),
}


def digest(case: W.AttentionCase) -> str:
    h = hashlib.sha256()
    for a in (case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx):
        h.update(np.ascontiguousarray(a).tobytes())
    h.update(np.float32(case.sm_scale).tobytes())
    return h.hexdigest()


def indexer_digest(case: W.IndexerCase) -> str:
    h = hashlib.sha256()
    for a in (case.q, case.k, case.scale, case.w, case.block_table, case.seq_lens):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()
