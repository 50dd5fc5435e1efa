"""FP8 index-key cache writer: bit-exact against the numpy restatement, in
the split and page-packed layouts, and round-tripped through the indexer."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from flashinfer_repo_b200 import indexer as IX
from flashinfer_repo_b200 import workloads as W
from oracle import oracle as O
from tests.helpers import bf16_tensor

pytestmark = pytest.mark.gpu


def _inputs(seed, n, P):
    rng = np.random.default_rng(seed)
    keys = W.f32_to_bf16_bits(rng.standard_normal((n, 128), dtype=np.float32) * rng.uniform(0.01, 30, (n, 1)).astype(np.float32))
    keys[3] = 0  # all-zero row -> scale 1
    slots = rng.choice(P * 64, n, replace=False).astype(np.int32)
    slots[5] = -1  # skipped
    return keys, slots


def test_append_split_layout_bit_exact(cuda_device):
    P, n = 40, 700
    keys, slots = _inputs(1, n, P)
    kc = torch.zeros((P, 64, 128), dtype=torch.uint8, device=cuda_device)
    sc = torch.zeros((P, 64), dtype=torch.float32, device=cuda_device)
    IX.index_cache_append(bf16_tensor(keys, cuda_device), torch.from_numpy(slots).to(cuda_device), kc, sc)
    rk = np.zeros((P, 64, 128), np.uint8)
    rs = np.zeros((P, 64), np.float32)
    O.index_cache_append(keys, slots, rk, rs)
    assert np.array_equal(kc.cpu().numpy(), rk) and np.array_equal(sc.cpu().numpy(), rs)


def test_append_page_packed_layout(cuda_device):
    P, n = 16, 300
    keys, slots = _inputs(2, n, P)
    buf = torch.zeros((P, 64 * 128 + 256), dtype=torch.uint8, device=cuda_device)
    kc = buf[:, : 64 * 128].view(P, 64, 128)
    sc = buf[:, 64 * 128:].view(torch.float32)
    IX.index_cache_append(bf16_tensor(keys, cuda_device), torch.from_numpy(slots).to(cuda_device), kc, sc)
    rk = np.zeros((P, 64, 128), np.uint8)
    rs = np.zeros((P, 64), np.float32)
    O.index_cache_append(keys, slots, rk, rs)
    assert np.array_equal(kc.cpu().numpy(), rk) and np.array_equal(sc.cpu().numpy(), rs)


def test_append_then_index(cuda_device):
    """Keys written for a whole request are scored by the indexer as the
    oracle scores the same quantised cache."""
    L = 3000
    ic = W.make_indexer_case(9, [L])
    P = ic.k.shape[0]
    rng = np.random.default_rng(10)
    keys = W.f32_to_bf16_bits(rng.standard_normal((L, 128), dtype=np.float32))
    t = np.arange(L)
    slots = (ic.block_table[0, t // 64] * 64 + t % 64).astype(np.int32)
    kc = torch.zeros((P, 64, 128), dtype=torch.uint8, device=cuda_device)
    sc = torch.ones((P, 64), dtype=torch.float32, device=cuda_device)
    IX.index_cache_append(bf16_tensor(keys, cuda_device), torch.from_numpy(slots).to(cuda_device), kc, sc)
    q = torch.from_numpy(ic.q).to(cuda_device).view(torch.float8_e4m3fn)
    scores = IX.indexer_scores(q, kc, sc, torch.from_numpy(ic.w).to(cuda_device),
                               torch.from_numpy(ic.seq_lens).to(cuda_device),
                               torch.from_numpy(ic.block_table).to(cuda_device))
    rk = np.zeros((P, 64, 128), np.uint8)
    rs = np.ones((P, 64), np.float32)
    O.index_cache_append(keys, slots, rk, rs)
    ref = O.indexer_scores(ic.q, rk.reshape(P, -1), 8192, rs.reshape(P, -1), 256, ic.w, ic.block_table,
                           ic.seq_lens, ic.block_table.shape[1] * 64)
    got = scores.cpu().numpy()[0, :L]
    assert np.abs(got - ref[0, :L]).max() <= 1e-5 * np.abs(ref[0, :L]).max()
