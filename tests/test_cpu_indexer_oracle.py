"""CPU checks of the indexer/top-k oracle (PARITY UNPINNED by the reference:
it has no indexer oracle).  The oracle is checked against a direct numpy
evaluation of the formula and against hand-built tie cases."""
from __future__ import annotations

import numpy as np

from flashinfer_repo_b200 import workloads as W
from oracle import oracle as O
from tests.helpers import oracle_indexer


def _numpy_scores(case, max_len):
    q = W.e4m3_bits_to_f32(case.q).astype(np.float64)
    out = np.full((len(case.seq_lens), max_len), -np.inf)
    for b, L in enumerate(case.seq_lens):
        t = np.arange(L)
        pages = case.block_table[b, t // 64]
        k = W.e4m3_bits_to_f32(case.k[pages, t % 64]).astype(np.float64)
        logits = k @ q[b].T
        out[b, :L] = case.scale[pages, t % 64] * (np.maximum(logits, 0) @ case.w[b].astype(np.float64))
    return out.astype(np.float32)


def test_oracle_scores_match_numpy():
    case = W.make_indexer_case(5, [300, 64, 1, 1000])
    max_len = case.block_table.shape[1] * 64
    got = oracle_indexer(case, max_len)
    ref = _numpy_scores(case, max_len)
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin)
    assert np.allclose(got[fin], ref[fin], rtol=1e-6, atol=1e-6)


def test_exact_case_is_exact():
    case = W.make_indexer_case(6, [700, 200], exact=True)
    max_len = case.block_table.shape[1] * 64
    assert np.array_equal(oracle_indexer(case, max_len), _numpy_scores(case, max_len))


def test_topk_order_and_ties():
    scores = np.array([[1.0, 3.0, 3.0, 2.0, 3.0, -np.inf, 0.5, 2.0]], np.float32)
    bt = np.array([[7]], np.int32)
    pos, slots = O.topk(scores, np.array([8], np.int32), bt, 5)
    assert pos.tolist() == [[1, 2, 4, 3, 7]]
    assert slots.tolist() == [[7 * 64 + 1, 7 * 64 + 2, 7 * 64 + 4, 7 * 64 + 3, 7 * 64 + 7]]
    pos, _ = O.topk(scores, np.array([3], np.int32), bt, 5)
    assert pos.tolist() == [[1, 2, 0, -1, -1]]
    pos, slots = O.topk(scores, np.array([8], np.int32), bt, 5, order="position")
    assert pos.tolist() == [[1, 2, 3, 4, 7]]
    assert slots.tolist() == [[7 * 64 + 1, 7 * 64 + 2, 7 * 64 + 3, 7 * 64 + 4, 7 * 64 + 7]]


def test_e4m3_exact_generator_values():
    case = W.make_indexer_case(7, [100], exact=True)
    v = W.e4m3_bits_to_f32(case.q)
    assert np.array_equal(v, np.round(v)) and np.abs(v).max() <= 3
