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


CASES = {
    "cfg1_seed0": lambda: W.cfg1_case(0),
    "edge": _edge_case,
    "big_logits": _big_logits_case,
    "alt_scale": _alt_scale_case,
}


def digest(case: W.AttentionCase) -> str:
    h = hashlib.sha256()
    for a in (case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx):
        h.update(np.ascontiguousarray(a).tobytes())
    h.update(np.float32(case.sm_scale).tobytes())
    return h.hexdigest()
