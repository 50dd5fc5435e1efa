"""Parity against the reference's OWN GPU kernels.

tests/golden/ref_triton_attn_*.npz hold the outputs of the reference Triton
operator `kernel` (solution/triton/kernel.py:138-182) and of `kernel_splitk`
with SPLIT_K=16 (kernel.py:496-567), produced on a B200 by
tests/golden/make_ref_gpu_golden.py from the unmodified reference sources, on
the inputs tests/golden/cases.py regenerates from seeds.  The CPU tests pin
the oracle to them; the GPU tests pin this library's operator to them, with
the reference's tolerances (atol = rtol = 1e-2 on the output, 1e-3 on LSE).

One reference defect is recorded rather than matched: `kernel` returns NaN
for a token whose first 64 indices are all -1 (every score of its first
block is -inf, so p = exp(-inf - -inf) = NaN at kernel.py:101-102 and the
NaN survives every later rescale).  The golden `run` (indexer_kernel.py:
436-497) and `kernel_splitk` give a finite result for that token; for it this
library is compared with `kernel_splitk`.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from flashinfer_repo_b200 import workloads as W
from tests.golden.cases import CASES, digest
from tests.helpers import ATOL, LSE_ATOL, RTOL

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAMES = [n for n in CASES if os.path.exists(os.path.join(GOLDEN, f"ref_triton_attn_{n}.npz"))]
# token -> why the reference's single-pass kernel is not the comparison there
NAN_TOKENS = {"edge": [6]}


def _fixture(name):
    g = np.load(os.path.join(GOLDEN, f"ref_triton_attn_{name}.npz"))
    case = CASES[name]()
    assert str(g["digest"]) == digest(case), "input generator drifted from the fixture"
    return case, g


def _reference_outputs(name, g):
    """(out bits, lse) of the reference kernels to compare with: `kernel`,
    with `kernel_splitk` rows for the tokens where `kernel` returns NaN."""
    out, lse = g["out"].copy(), g["lse"].copy()
    for t in NAN_TOKENS.get(name, []):
        out[t], lse[t] = g["out_splitk16"][t], g["lse_splitk16"][t]
    return out, lse


def _close(got_bits, got_lse, ref_bits, ref_lse):
    a, b = W.bf16_bits_to_f32(got_bits), W.bf16_bits_to_f32(ref_bits)
    assert not np.isnan(a).any() and not np.isnan(b).any()
    err = np.abs(a - b)
    bad = (err > ATOL) & (err / np.maximum(np.abs(b), 1e-30) > RTOL)
    assert not bad.any(), f"{bad.sum()} elements out of tolerance (max abs err {err.max():.3g})"
    assert np.array_equal(np.isneginf(got_lse), np.isneginf(ref_lse))
    fin = ~np.isneginf(ref_lse)
    if fin.any():
        assert np.abs(got_lse[fin] - ref_lse[fin]).max() <= LSE_ATOL
    return float(err.max())


def test_fixtures_present():
    assert set(NAMES) == set(CASES), "missing ref_triton_attn fixtures"


@pytest.mark.parametrize("name", NAMES)
def test_reference_kernel_nan_defect_is_where_recorded(name):
    """The reference `kernel` output is finite everywhere except the recorded
    tokens; its split-K variant is finite everywhere."""
    _, g = _fixture(name)
    nan_tok = np.where(np.isnan(W.bf16_bits_to_f32(g["out"])).any(axis=(1, 2)))[0]
    assert list(nan_tok) == NAN_TOKENS.get(name, [])
    assert not np.isnan(W.bf16_bits_to_f32(g["out_splitk16"])).any()


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_triton_kernels(name):
    from oracle import oracle as O
    case, g = _fixture(name)
    out, lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx, case.sm_scale)
    _close(out, lse, *_reference_outputs(name, g))
    _close(out, lse, g["out_splitk16"], g["lse_splitk16"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_operator_matches_reference_triton_kernels(cuda_device, name):
    import torch

    from flashinfer_repo_b200 import kernel, read_device_error
    from tests.helpers import case_to_device, out_bits
    case, g = _fixture(name)
    out, lse = kernel(*case_to_device(case, cuda_device), case.sm_scale)
    torch.cuda.synchronize()
    assert read_device_error(cuda_device) == 0
    got, got_lse = out_bits(out), lse.cpu().numpy()
    _close(got, got_lse, *_reference_outputs(name, g))
    _close(got, got_lse, g["out_splitk16"], g["lse_splitk16"])


# ------------------------------------------------------------------ indexer + top-k
# tests/golden/ref_triton_indexer_*.npz: scores of the reference indexer_kernel
# (indexer_kernel.py:4-287) on exact-by-construction inputs, stored as its
# concatenated per-request array (score of request b, position p at
# seq_offsets[b] + p, :283-287), and the output of run_indexer_and_topk
# (:345-433) for k = 2048 and k = 64 (logical ids seq_offsets[b] + p).
#
# The reference top-k is recorded, not matched: topk_kernel (:289-343) keeps K
# running slots initialised to -1e9 and, for every new score above the
# smallest slot, overwrites EVERY slot equal to that minimum (:333-339).  All
# slots start equal, so each accepted score overwrites all of them and the
# result is the arg-max position repeated K times (the first among equal
# maxima, since only a strictly larger score replaces).  What is pinned is the
# part both agree on: this library's first selected position (score order,
# ties to the lower position) equals the reference's, and the reference's
# selection is contained in this library's top-k set.
from tests.golden.cases import INDEXER_CASES, indexer_digest  # noqa: E402

IDX_NAMES = list(INDEXER_CASES)


def _indexer_fixture(name):
    g = np.load(os.path.join(GOLDEN, f"ref_triton_indexer_{name}.npz"))
    case = INDEXER_CASES[name]()
    assert str(g["digest"]) == indexer_digest(case), "input generator drifted from the fixture"
    return case, g


def _ref_scores_2d(case, g):
    L = case.block_table.shape[1] * 64
    out = np.full((len(case.seq_lens), L), np.nan, np.float32)
    for b, n in enumerate(case.seq_lens):
        o = int(g["seq_offsets"][b])
        out[b, :n] = g["scores"][o:o + n]
    return out


def _check_topk_against_reference(case, g, pos_score_order, sets):
    offs = g["seq_offsets"].astype(np.int64)
    for k in (2048, 64):
        ref = g[f"topk{k}"].astype(np.int64) - offs[:, None]  # logical ids -> positions
        for b in range(len(case.seq_lens)):
            assert len(set(ref[b].tolist())) == 1  # the recorded degenerate output
            assert pos_score_order[b, 0] == ref[b, 0]
            assert set(ref[b].tolist()) <= sets[b]


@pytest.mark.parametrize("name", IDX_NAMES)
def test_oracle_matches_reference_indexer(name):
    from oracle import oracle as O
    from tests.helpers import oracle_indexer
    case, g = _indexer_fixture(name)
    L = case.block_table.shape[1] * 64
    ours = oracle_indexer(case, L)
    ref = _ref_scores_2d(case, g)
    m = ~np.isnan(ref)
    assert np.array_equal(ours[m], ref[m]), "indexer scores differ from the reference kernel's"
    pos, _ = O.topk(ours, case.seq_lens, case.block_table, 2048)
    _check_topk_against_reference(case, g, pos, [set(p[p >= 0].tolist()) for p in pos])


@pytest.mark.gpu
@pytest.mark.parametrize("name", IDX_NAMES)
def test_indexer_kernel_matches_reference_indexer(cuda_device, name):
    import torch

    from flashinfer_repo_b200 import indexer as IX
    from tests.helpers import indexer_case_to_device
    case, g = _indexer_fixture(name)
    args = indexer_case_to_device(case, cuda_device)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    scores = IX.indexer_scores(*args, device_error=err)
    pos, _ = IX.topk_select(scores, args[4], args[5], 2048)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = _ref_scores_2d(case, g)
    m = ~np.isnan(ref)
    assert np.array_equal(scores.cpu().numpy()[:, :ref.shape[1]][m], ref[m])
    pos = pos.cpu().numpy()
    _check_topk_against_reference(case, g, pos, [set(p[p >= 0].tolist()) for p in pos])
