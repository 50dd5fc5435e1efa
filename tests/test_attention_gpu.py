"""GPU parity of the sm_100a sparse-attention kernel (through the C ABI via
flashinfer_repo_b200.kernel) against the reference's golden outputs and the
C oracle."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from flashinfer_repo_b200 import kernel, options, read_device_error
from flashinfer_repo_b200 import workloads as W
from oracle import oracle as O
from tests.golden.cases import CASES, digest
from tests.helpers import assert_attention_close, case_to_device, out_bits

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(autouse=True)
def _default_options():
    with options():
        yield


@pytest.mark.parametrize("name", list(CASES))
def test_golden_reference_outputs(cuda_device, name):
    """Same seeded inputs as the reference `run` fixtures (tests/golden)."""
    case = CASES[name]()
    g = np.load(os.path.join(HERE, "golden", f"attn_{name}.npz"))
    assert str(g["digest"]) == digest(case)
    out, lse = kernel(*case_to_device(case, cuda_device), case.sm_scale)
    torch.cuda.synchronize()
    assert_attention_close(out, lse, g["out"], g["lse"], name)
    assert read_device_error(cuda_device) == 0


def _oracle_check(case, device, **kw):
    out, lse = kernel(*case_to_device(case, device), case.sm_scale, **kw)
    ref_out, ref_lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx,
                                       case.sm_scale)
    return assert_attention_close(out, lse, ref_out, ref_lse), out, lse


@pytest.mark.parametrize("seed", [1, 2])
def test_batched_ragged_contexts(cuda_device, seed):
    """cfg2-like batch at oracle-friendly size: ragged contexts incl. < 2048."""
    ctx = np.random.default_rng(seed).integers(300, 9000, size=12)
    case = W.make_attention_case(100 + seed, ctx)
    _oracle_check(case, cuda_device)


@pytest.mark.parametrize("ctas", [1, 3, 7, 64, 500])
def test_split_counts_agree(cuda_device, ctas):
    """Any partition of the top-k dimension over CTAs gives the oracle's answer
    (split-K equivalence, cf. test_splitk_correctness.py:20-26)."""
    case = W.make_attention_case(7, [5000, 3000, 1500, 4096, 2048])
    with options(attention_ctas=ctas, attention_min_tiles=1):
        _oracle_check(case, cuda_device)


@pytest.mark.parametrize("ctas", [16, 37])
def test_more_tokens_than_ctas(cuda_device, ctas):
    """More tokens than CTAs (the prefill-sized plan): only tokens straddling a
    CTA boundary are split, and the merge grid runs one row per boundary."""
    rng = np.random.default_rng(17)
    case = W.make_attention_case(17, rng.integers(1500, 5000, size=40))
    case.idx[3, :700] = -1
    with options(attention_ctas=ctas, attention_min_tiles=1):
        _oracle_check(case, cuda_device)


@pytest.mark.parametrize("T", [37, 48, 64, 100])
def test_token_aligned_plans(cuda_device, T):
    """Batches with fewer tokens than resident CTAs: each token split over the
    same number of CTAs, also when that number does not divide its 64 tiles
    (T=37: 8 CTAs per token, T=48: 6), or the stream-K plan (T=100), agree
    with the oracle and with an explicit stream-K partition."""
    ctx = np.random.default_rng(T).integers(300, 5000, size=T)
    case = W.make_attention_case(300 + T, ctx)
    _, out, lse = _oracle_check(case, cuda_device)
    with options(attention_ctas=296):
        o2, l2 = kernel(*case_to_device(case, cuda_device), case.sm_scale)
    torch.cuda.synchronize()
    assert (out.float() - o2.float()).abs().max().item() <= 2 ** -6
    assert torch.allclose(lse, l2, atol=1e-5, rtol=0)
    assert read_device_error(cuda_device) == 0


@pytest.mark.parametrize("stages", [2, 3, 4])
def test_pipeline_depths(cuda_device, stages):
    case = W.make_attention_case(8, [5000, 2100, 4096])
    with options(attention_stages=stages):
        _oracle_check(case, cuda_device)


def test_environment_is_not_read(cuda_device, monkeypatch):
    """Leftover variables of the old profiling knobs change nothing: a stray
    DSA_ATTN_STAGE=2 once made kernel() run the merge grid alone."""
    case = W.make_attention_case(16, [5000, 3000, 4096])
    args = case_to_device(case, cuda_device)
    ref_out, ref_lse = kernel(*args, case.sm_scale)
    for k, v in (("DSA_ATTN_STAGE", "2"), ("DSA_ATTN_IMPL", "1"), ("DSA_ATTN_CTAS", "3"),
                 ("DSA_ATTN_PDL", "0"), ("DSA_ATTN_STAGES", "4"), ("DSA_ATTN_MIN_TILES", "1")):
        monkeypatch.setenv(k, v)
    out, lse = kernel(*args, case.sm_scale)
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)


def test_deterministic(cuda_device):
    case = W.make_attention_case(9, [6000] * 6)
    args = case_to_device(case, cuda_device)
    o1, l1 = kernel(*args, case.sm_scale)
    o2, l2 = kernel(*args, case.sm_scale)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_128_heads_as_groups(cuda_device):
    """cfg3 shape on one GPU: 128 heads = 8 groups of 16 sharing the indices;
    each group must equal the 16-head operator on its slice."""
    case = W.make_attention_case(10, [20000] * 3, heads=128, clustered=True, shared_cache=True)
    qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
    out, lse = kernel(qn, qp, ckv, kpe, idx, case.sm_scale)
    for g in (0, 5, 7):
        sl = slice(16 * g, 16 * g + 16)
        ref_out, ref_lse = O.dsa_attention(case.q_nope[:, sl], case.q_pe[:, sl], case.ckv, case.kpe,
                                           case.idx, case.sm_scale)
        assert_attention_close(out[:, sl], lse[:, sl], ref_out, ref_lse, f"group {g}")


def test_strided_views(cuda_device):
    """Non-contiguous q / cache views (the reference passes all strides)."""
    case = W.make_attention_case(12, [3000, 5000])
    qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
    qn_big = torch.zeros((qn.shape[0], 32, 512), dtype=qn.dtype, device=cuda_device)
    qn_big[:, ::2] = qn
    ckv_big = torch.zeros((ckv.shape[0], 64, 520), dtype=ckv.dtype, device=cuda_device)
    ckv_big[:, :, :512] = ckv
    out, lse = kernel(qn_big[:, ::2], qp, ckv_big[:, :, :512], kpe, idx, case.sm_scale)
    ref_out, ref_lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx,
                                       case.sm_scale)
    assert_attention_close(out, lse, ref_out, ref_lse)


def test_bad_index_flagged_not_faulting(cuda_device):
    case = W.make_attention_case(13, [3000])
    qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
    read_device_error(cuda_device)
    idx[0, 5] = ckv.shape[0] * 64 + 100  # out of range: skipped and flagged
    kernel(qn, qp, ckv, kpe, idx, case.sm_scale)
    assert read_device_error(cuda_device) & 1
    assert read_device_error(cuda_device) == 0


def test_empty_batch(cuda_device):
    case = W.make_attention_case(14, [3000])
    qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
    out, lse = kernel(qn[:0], qp[:0], ckv, kpe, idx[:0], case.sm_scale)
    assert out.shape == (0, 16, 512) and lse.shape == (0, 16)


def test_full_size_cfg2_against_oracle(cuda_device):
    """BASELINE cfg2 at full size (T=64, contexts U[1024,65536], 2.3 GB cache)
    built on the device; the rows each token selected are compacted into a
    small cache so the oracle can check every token."""
    from flashinfer_repo_b200.bench_inputs import make_cfg2_device
    qn, qp, ckv, kpe, idx, scale = make_cfg2_device(seed=3, device=cuda_device)
    out, lse = kernel(qn, qp, ckv, kpe, idx, scale)
    valid = idx >= 0
    rows = idx[valid].long()
    uniq, inv = torch.unique(rows, return_inverse=True)
    small_idx = torch.full_like(idx, -1)
    small_idx[valid] = inv.to(torch.int32)
    npg = (uniq.numel() + 63) // 64
    def compact(cache, d):
        flat = cache.reshape(-1, d)[uniq]
        pad = torch.zeros((npg * 64 - uniq.numel(), d), dtype=cache.dtype, device=cache.device)
        return torch.cat([flat, pad]).reshape(npg, 64, d)
    c_ckv, c_kpe = compact(ckv, 512), compact(kpe, 64)
    ref_out, ref_lse = O.dsa_attention(out_bits(qn), out_bits(qp), out_bits(c_ckv), out_bits(c_kpe),
                                       small_idx.cpu().numpy(), scale)
    assert_attention_close(out, lse, ref_out, ref_lse, "cfg2 full")
    assert read_device_error(cuda_device) == 0


def test_causal_prefill_against_oracle(cuda_device):
    """cfg5 shape at oracle-friendly size: 96 queries at the end of an
    8192-token context, causal top-2048 (positions <= the query's own)."""
    from flashinfer_repo_b200.bench_inputs import make_prefill_device
    qn, qp, ckv, kpe, idx, scale = make_prefill_device(seed=4, device=cuda_device, queries=96, ctx=8192)
    out, lse = kernel(qn, qp, ckv, kpe, idx, scale)
    ref_out, ref_lse = O.dsa_attention(out_bits(qn), out_bits(qp), out_bits(ckv), out_bits(kpe),
                                       idx.cpu().numpy(), scale)
    assert_attention_close(out, lse, ref_out, ref_lse, "prefill")


def test_full_size_cfg5_subsample_against_oracle(cuda_device):
    """BASELINE cfg5 at full size: 4096 causal queries over one 65536-token
    sequence, the whole grid launched as in the bench (tokens outnumber CTAs:
    boundary-row merge plan); 40 tokens spread over the batch (the first and
    last, CTA-boundary neighbourhoods included by the spread) are checked
    against the oracle, plus the -inf-free LSE of every token."""
    from flashinfer_repo_b200.bench_inputs import make_prefill_device
    qn, qp, ckv, kpe, idx, scale = make_prefill_device(seed=6, device=cuda_device)
    out, lse = kernel(qn, qp, ckv, kpe, idx, scale)
    torch.cuda.synchronize()
    assert read_device_error(cuda_device) == 0
    T = idx.shape[0]
    assert T == 4096 and torch.isfinite(lse).all()
    sel = np.unique(np.concatenate([[0, 1, T - 2, T - 1],
                                    np.random.default_rng(6).choice(T, 36, replace=False)]))
    st = torch.from_numpy(sel).to(cuda_device)
    ref_out, ref_lse = O.dsa_attention(out_bits(qn[st]), out_bits(qp[st]), out_bits(ckv), out_bits(kpe),
                                       idx[st].cpu().numpy(), scale)
    assert_attention_close(out[st], lse[st], ref_out, ref_lse, "cfg5 full, subsample")


def test_tvm_ffi_entry_point(cuda_device):
    """Called through the TVM-FFI global `flashinfer.kernel` (the reference's
    CUDA binding slot), the operator returns the same result."""
    pytest.importorskip("tvm_ffi")
    from flashinfer_repo_b200.binding import register
    f = register()
    case = W.cfg1_case(0)
    args = case_to_device(case, cuda_device)
    out, lse = f(*args, case.sm_scale)
    out, lse = torch.from_dlpack(out), torch.from_dlpack(lse)
    ref_out, ref_lse = kernel(*args, case.sm_scale)
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)


@pytest.mark.parametrize("name", list(CASES))
def test_tcgen05_variant_golden(cuda_device, name):
    """The tcgen05 kernel (64-row tiles, TMEM accumulators) on the reference's
    golden outputs."""
    case = CASES[name]()
    g = np.load(os.path.join(HERE, "golden", f"attn_{name}.npz"))
    with options(attention_kernel=2):
        out, lse = kernel(*case_to_device(case, cuda_device), case.sm_scale)
    assert_attention_close(out, lse, g["out"], g["lse"], name)


@pytest.mark.parametrize("ctas", [1, 5, 64])
def test_tcgen05_variant_ragged_and_splits(cuda_device, ctas):
    case = W.make_attention_case(15, [5000, 300, 3000, 64, 9000, 2048])
    case.idx[2, 100:900] = -1
    case.idx[3, :] = -1
    with options(attention_kernel=2, attention_ctas=ctas, attention_min_tiles=1):
        _oracle_check(case, cuda_device)
