"""GPU parity of the FP8 indexer (tcgen05) and the exact top-k against the C
oracle.  Parity here is unpinned by the reference (it has no indexer oracle);
exactness is shown with inputs whose scores are exact in fp32 in any
summation order (small-integer e4m3 values, power-of-two scales, weights in
sixteenths), and on random inputs by re-selecting the kernel's own scores."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from flashinfer_repo_b200 import indexer as IX
from flashinfer_repo_b200 import workloads as W
from oracle import oracle as O
from tests.helpers import indexer_case_to_device, oracle_indexer

pytestmark = pytest.mark.gpu
RAGGED = [5000, 2048, 100, 4096, 1, 130, 0, 64, 8191]


def _run(case, dev, topk=2048):
    args = indexer_case_to_device(case, dev)
    max_len = case.block_table.shape[1] * 64
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    scores = IX.indexer_scores(*args, device_error=err)
    pos, slots = IX.topk_select(scores, args[4], args[5], topk)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return scores.cpu().numpy(), pos.cpu().numpy(), slots.cpu().numpy(), max_len


def _valid_mask(case, max_len):
    return np.arange(max_len)[None, :] < case.seq_lens[:, None]


@pytest.mark.parametrize("tie_heavy", [False, True])
def test_exact_inputs_bit_exact(cuda_device, tie_heavy):
    case = W.make_indexer_case(1, RAGGED, exact=True, tie_heavy=tie_heavy)
    scores, pos, slots, max_len = _run(case, cuda_device)
    ref = oracle_indexer(case, max_len)
    m = _valid_mask(case, max_len)
    assert np.array_equal(scores[m], ref[m]), "exact-by-construction scores differ"
    rpos, rslots = O.topk(ref, case.seq_lens, case.block_table, 2048)
    assert np.array_equal(pos, rpos) and np.array_equal(slots, rslots)
    if tie_heavy:  # the case really has ties at the selection boundary
        b = 0
        kth = ref[b, rpos[b, 2047]]
        assert (ref[b, : case.seq_lens[b]] == kth).sum() > 1


@pytest.mark.parametrize("topk", [2048, 512, 7])
def test_random_inputs(cuda_device, topk):
    case = W.make_indexer_case(2, RAGGED)
    scores, pos, slots, max_len = _run(case, cuda_device, topk)
    ref = oracle_indexer(case, max_len)
    m = _valid_mask(case, max_len)
    scale = np.abs(ref).max(axis=1, keepdims=True) + 1e-30
    assert (np.abs(scores - ref)[m] <= (1e-5 * np.broadcast_to(scale, ref.shape))[m]).all()
    # selection is exact given the kernel's own scores
    own_scores = np.where(m, scores, -np.inf).astype(np.float32)
    rpos, rslots = O.topk(own_scores, case.seq_lens, case.block_table, topk)
    assert np.array_equal(pos, rpos) and np.array_equal(slots, rslots)


def test_page_packed_layout(cuda_device):
    """Each page = 64x128 key bytes followed by 64 fp32 scales (byte strides)."""
    case = W.make_indexer_case(3, [3000, 777, 6400], exact=True)
    P = case.k.shape[0]
    packed = np.zeros((P, 64 * 128 + 256), np.uint8)
    packed[:, : 64 * 128] = case.k.reshape(P, -1)
    packed[:, 64 * 128:] = case.scale.view(np.uint8).reshape(P, -1)
    q, _, _, w, sl, bt = indexer_case_to_device(case, cuda_device)
    buf = torch.from_numpy(packed).to(cuda_device)
    k = buf[:, : 64 * 128].view(P, 64, 128)
    sc = buf[:, 64 * 128:].view(torch.float32)
    scores = IX.indexer_scores(q, k, sc, w, sl, bt)
    max_len = case.block_table.shape[1] * 64
    ref = oracle_indexer(case, max_len)
    m = _valid_mask(case, max_len)
    assert np.array_equal(scores.cpu().numpy()[m], ref[m])


def test_full_size_cfg4(cuda_device):
    """BASELINE cfg4 size: 128 requests x 32768 tokens.  Top-k is checked
    exactly against the kernel's own scores for every request, and scores
    against the oracle on a sample of requests."""
    case = W.make_indexer_case(4, [32768] * 128, fast=True)
    scores, pos, slots, max_len = _run(case, cuda_device)
    rpos, rslots = O.topk(scores, case.seq_lens, case.block_table, 2048)
    assert np.array_equal(pos, rpos) and np.array_equal(slots, rslots)
    pick = [0, 57, 127]
    sub = W.IndexerCase(case.q[pick], case.k, case.scale, case.w[pick], case.block_table[pick],
                        case.seq_lens[pick])
    ref = oracle_indexer(sub, max_len)
    scale = np.abs(ref).max(axis=1, keepdims=True)
    assert (np.abs(scores[pick] - ref) <= 1e-5 * scale).all()


@pytest.mark.parametrize("L", [40960, 40961, 65536, 2049])
def test_topk_long_and_tied_rows(cuda_device, L):
    """Rows longer than the shared-memory cache take the streaming path; heavy
    ties (values on a coarse grid) exercise the lower-position rule."""
    rng = np.random.default_rng(L)
    B = 3
    scores = np.round(rng.standard_normal((B, L)) * 4).astype(np.float32) / 4
    scores[1] = 1.0  # every score equal
    lens = np.array([L, L, L // 2], np.int32)
    bt = rng.permutation(B * ((L + 63) // 64)).astype(np.int32).reshape(B, -1)
    pos, slots = IX.topk_select(torch.from_numpy(scores).to(cuda_device), torch.from_numpy(lens).to(cuda_device),
                                torch.from_numpy(bt).to(cuda_device), 2048)
    rpos, rslots = O.topk(scores, lens, bt, 2048)
    assert np.array_equal(pos.cpu().numpy(), rpos) and np.array_equal(slots.cpu().numpy(), rslots)
    assert rpos[1].tolist() == list(range(2048))


@pytest.mark.parametrize("L", [32768, 40961, 3000])
def test_topk_position_order(cuda_device, L):
    """order="position" returns the same set as the score order, in ascending
    position (tie-heavy rows and an all-equal row included)."""
    rng = np.random.default_rng(L + 7)
    B = 3
    scores = rng.standard_normal((B, L)).astype(np.float32)
    scores[1] = np.round(scores[1] * 2) / 2  # heavy ties
    scores[2] = 0.5                           # all equal
    lens = np.array([L, L - 5, L], np.int32)
    bt = rng.permutation(B * ((L + 63) // 64)).astype(np.int32).reshape(B, -1)

    def dev(a):
        return torch.from_numpy(a).to(cuda_device)
    pos, slots = IX.topk_select(dev(scores), dev(lens), dev(bt), 2048, order="position")
    rpos, rslots = O.topk(scores, lens, bt, 2048, order="position")
    assert np.array_equal(pos.cpu().numpy(), rpos) and np.array_equal(slots.cpu().numpy(), rslots)
    spos, _ = IX.topk_select(dev(scores), dev(lens), dev(bt), 2048)
    for b in range(B):
        assert sorted(spos[b].cpu().tolist()) == sorted(rpos[b].tolist())
