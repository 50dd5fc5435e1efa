"""End-to-end DSA step (indexer -> top-k -> attention) against the oracle
composition, and its CUDA-graph capture."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from flashinfer_repo_b200 import workloads as W
from flashinfer_repo_b200.pipeline import DecodeStepGraph, run_sparse_attention_pipeline
from oracle import oracle as O
from tests.helpers import (assert_attention_close, bf16_tensor, indexer_case_to_device,
                           oracle_indexer, out_bits)

pytestmark = pytest.mark.gpu


def _setup(dev, seq_lens, tokens_per_request=1):
    ic = W.make_indexer_case(21, seq_lens, exact=True)
    P = ic.k.shape[0]
    rng = np.random.default_rng(22)
    B = len(seq_lens)
    T = B * tokens_per_request
    ckv = W.f32_to_bf16_bits(rng.standard_normal((P, 64, 512), dtype=np.float32) * 0.5)
    kpe = W.f32_to_bf16_bits(rng.standard_normal((P, 64, 64), dtype=np.float32) * 0.5)
    qn = W.f32_to_bf16_bits(rng.standard_normal((T, 16, 512), dtype=np.float32))
    qp = W.f32_to_bf16_bits(rng.standard_normal((T, 16, 64), dtype=np.float32))
    dev_args = indexer_case_to_device(ic, dev) + tuple(bf16_tensor(x, dev) for x in (qn, qp, ckv, kpe))
    return ic, (qn, qp, ckv, kpe), dev_args


def _oracle(ic, host, query_request):
    max_len = ic.block_table.shape[1] * 64
    scores = oracle_indexer(ic, max_len)
    _, slots = O.topk(scores, ic.seq_lens, ic.block_table, 2048, order="position")
    qn, qp, ckv, kpe = host
    out, lse = O.dsa_attention(qn, qp, ckv, kpe, slots[query_request], W.SM_SCALE)
    return slots, out, lse


def test_pipeline_matches_oracle_composition(cuda_device):
    ic, host, a = _setup(cuda_device, [3000, 700, 5000, 64])
    out, lse, slots = run_sparse_attention_pipeline(*a, W.SM_SCALE)
    rslots, rout, rlse = _oracle(ic, host, np.arange(4))
    assert np.array_equal(slots.cpu().numpy(), rslots)
    assert_attention_close(out, lse, rout, rlse, "pipeline")


def test_multiple_queries_per_request(cuda_device):
    ic, host, a = _setup(cuda_device, [2500, 4100, 900], tokens_per_request=2)
    qr = np.array([0, 0, 1, 1, 2, 2], np.int64)
    out, lse, _ = run_sparse_attention_pipeline(*a, W.SM_SCALE,
                                                query_request=torch.from_numpy(qr).to(cuda_device))
    _, rout, rlse = _oracle(ic, host, qr)
    assert_attention_close(out, lse, rout, rlse, "query_request")


def test_cuda_graph_step(cuda_device):
    ic, host, a = _setup(cuda_device, [3000, 1200, 4096])
    step = DecodeStepGraph(*a, W.SM_SCALE)
    out, lse, slots = step.replay()
    eo, el, es = run_sparse_attention_pipeline(*a, W.SM_SCALE)
    torch.cuda.synchronize()
    assert torch.equal(out, eo) and torch.equal(lse, el) and torch.equal(slots, es)
    a[6].mul_(-1)  # new queries in place (q_nope), replay sees them
    out2, lse2, _ = step.replay()
    eo2, el2, _ = run_sparse_attention_pipeline(*a, W.SM_SCALE)
    torch.cuda.synchronize()
    assert torch.equal(out2, eo2) and torch.equal(lse2, el2)
    assert not torch.equal(out2, eo)
    _ = out_bits


def test_private_workspace_and_topk_out(cuda_device):
    """kernel(workspace=) with a caller-owned workspace and topk_select(out=)
    into caller-owned tensors give the same results as the defaults."""
    from flashinfer_repo_b200 import indexer as IX
    from flashinfer_repo_b200.kernel import kernel, workspace_size
    ic, host, a = _setup(cuda_device, [3000, 1200, 4096])
    scores = IX.indexer_scores(*a[:6])
    pos, slots = IX.topk_select(scores, a[4], a[5], 2048, order="position")
    pos2 = torch.empty_like(pos)
    slots2 = torch.empty_like(slots)
    IX.topk_select(scores, a[4], a[5], 2048, order="position", out=(pos2, slots2))
    assert torch.equal(pos, pos2) and torch.equal(slots, slots2)
    o1, l1 = kernel(*a[6:10], slots, W.SM_SCALE)
    ws = torch.zeros(workspace_size(3, 16, 2048, cuda_device), dtype=torch.uint8, device=cuda_device)
    o2, l2 = kernel(*a[6:10], slots, W.SM_SCALE, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    assert int(ws[:4].view(torch.int32).item()) == 0  # the error word of this workspace
    with pytest.raises(Exception):
        kernel(*a[6:10], slots, W.SM_SCALE, workspace=ws[:64])  # too small: the library refuses
