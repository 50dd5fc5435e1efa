"""GPU parity of the cluster plan: each (token, 16-head group) split over a
thread-block cluster of C CTAs that merge their split-K partials through
distributed shared memory inside the attention grid (no merge grid).  Checked
against the C oracle (restating the reference `run`, indexer_kernel.py:436-497)
and against the stream-K plan with the same partition of the top-k dimension,
whose partials the merge grid combines (LSE merge of kernel.py:437-493)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from flashinfer_repo_b200 import kernel, options, read_device_error
from flashinfer_repo_b200 import workloads as W
from oracle import oracle as O
from tests.golden.cases import CASES
from tests.helpers import assert_attention_close, case_to_device

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(autouse=True)
def _default_options():
    with options():
        yield


def _vs_oracle_and_stream_k(case, device, c, heads=16):
    args = case_to_device(case, device)
    with options(attention_cluster=c):
        out, lse = kernel(*args, case.sm_scale)
    # the same partition (tpt/C tiles per CTA) through the merge grid
    vt = case.idx.shape[0] * (heads // 16)
    with options(attention_ctas=vt * c, attention_min_tiles=1, attention_cluster=1):
        out_s, lse_s = kernel(*args, case.sm_scale)
    torch.cuda.synchronize()
    assert read_device_error(device) == 0
    ref_out, ref_lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx,
                                       case.sm_scale)
    assert_attention_close(out, lse, ref_out, ref_lse, f"cluster {c}")
    # same partials, same merge arithmetic: at most one bf16 rounding apart
    d = (out.float() - out_s.float()).abs().max().item()
    assert d <= 2 ** -6 * max(1.0, out_s.float().abs().max().item()), d
    assert torch.allclose(lse, lse_s, atol=1e-5, rtol=0, equal_nan=True)
    assert torch.equal(torch.isinf(lse), torch.isinf(lse_s))
    return out, lse


@pytest.mark.parametrize("c", [2, 4, 8])
def test_cluster_sizes_ragged(cuda_device, c):
    """Ragged contexts, including one shorter than a cluster part (parts with
    no valid row: m = -inf partials)."""
    case = W.make_attention_case(21, [5000, 40, 1500, 4096, 2048, 300])
    _vs_oracle_and_stream_k(case, cuda_device, c)


@pytest.mark.parametrize("c", [2, 8])
def test_cluster_golden_edge(cuda_device, c):
    """The reference `run` outputs of the edge case (padding-only tokens,
    -1 runs) through the cluster plan."""
    case = CASES["edge"]()
    g = np.load(os.path.join(HERE, "golden", "attn_edge.npz"))
    with options(attention_cluster=c):
        out, lse = kernel(*case_to_device(case, cuda_device), case.sm_scale)
    torch.cuda.synchronize()
    assert_attention_close(out, lse, g["out"], g["lse"], f"edge cluster {c}")


def test_cluster_128_heads(cuda_device):
    """8 head groups per token: the clusters are (token, group) pairs."""
    case = W.make_attention_case(22, [20000] * 3, heads=128, clustered=True, shared_cache=True)
    qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
    with options(attention_cluster=4):
        out, lse = kernel(qn, qp, ckv, kpe, idx, case.sm_scale)
    for g in (0, 3, 7):
        sl = slice(16 * g, 16 * g + 16)
        ref_out, ref_lse = O.dsa_attention(case.q_nope[:, sl], case.q_pe[:, sl], case.ckv, case.kpe,
                                           case.idx, case.sm_scale)
        assert_attention_close(out[:, sl], lse[:, sl], ref_out, ref_lse, f"group {g}")


def test_cfg2_sized_batch(cuda_device):
    """A cfg2-sized batch (64 tokens) through C = 4 (256 CTAs): deterministic,
    equal to the oracle, and the default plan (stream-K) agrees with it."""
    ctx = np.random.default_rng(23).integers(1024, 9000, size=64)
    case = W.make_attention_case(23, ctx)
    args = case_to_device(case, cuda_device)
    with options(attention_cluster=4):
        o1, l1 = kernel(*args, case.sm_scale)
        o2, l2 = kernel(*args, case.sm_scale)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    o3, l3 = kernel(*args, case.sm_scale)
    ref_out, ref_lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx,
                                       case.sm_scale)
    assert_attention_close(o1, l1, ref_out, ref_lse, "cluster 4")
    assert_attention_close(o3, l3, ref_out, ref_lse, "stream-K")


def test_forced_size_that_does_not_fit_falls_back(cuda_device):
    """A forced cluster size whose grid would exceed the resident slots runs
    the stream-K plan instead (same answer)."""
    case = W.make_attention_case(24, [3000] * 80)  # 80 x 8 CTAs > slots
    args = case_to_device(case, cuda_device)
    with options(attention_cluster=8):
        out, lse = kernel(*args, case.sm_scale)
    ref_out, ref_lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx,
                                       case.sm_scale)
    assert_attention_close(out, lse, ref_out, ref_lse)
