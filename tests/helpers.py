"""Shared test helpers: numpy cases -> torch tensors, reference tolerances."""
from __future__ import annotations

import numpy as np
import torch

from flashinfer_repo_b200.workloads import bf16_bits_to_f32

# Tolerances of the reference's evaluation (docs/CORRECTNESS.md:23-42): an
# output element fails only if it exceeds BOTH atol and rtol; every element
# must pass.  LSE tolerance from the build target: 1e-3 absolute.
ATOL = 1e-2
RTOL = 1e-2
LSE_ATOL = 1e-3


def bf16_tensor(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def case_to_device(case, device):
    return (bf16_tensor(case.q_nope, device), bf16_tensor(case.q_pe, device),
            bf16_tensor(case.ckv, device), bf16_tensor(case.kpe, device),
            torch.from_numpy(case.idx).to(device))


def out_bits(out: torch.Tensor) -> np.ndarray:
    return out.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def assert_attention_close(out, lse, ref_out_bits, ref_lse, what=""):
    """out/lse: torch results; ref_out_bits: uint16 bf16 bits; ref_lse: float32."""
    got = bf16_bits_to_f32(out_bits(out))
    ref = bf16_bits_to_f32(ref_out_bits)
    assert got.shape == ref.shape, what
    abs_err = np.abs(got - ref)
    rel_err = abs_err / np.maximum(np.abs(ref), 1e-30)
    bad = (abs_err > ATOL) & (rel_err > RTOL)
    assert not np.isnan(got).any(), f"{what}: NaN in output"
    assert not bad.any(), (f"{what}: {bad.sum()} output elements out of tolerance, "
                           f"max abs err {abs_err.max():.4g}")
    got_lse = lse.detach().cpu().numpy()
    ref_lse = np.asarray(ref_lse, dtype=np.float32)
    inf_ref = np.isneginf(ref_lse)
    assert np.array_equal(np.isneginf(got_lse), inf_ref), f"{what}: -inf LSE pattern differs"
    if (~inf_ref).any():
        err = np.abs(got_lse[~inf_ref] - ref_lse[~inf_ref]).max()
        assert err <= LSE_ATOL, f"{what}: LSE max abs err {err:.3g}"
    return float(abs_err.max())


def indexer_case_to_device(case, device):
    """IndexerCase -> (q fp8, k fp8, scale, w, seq_lens, block_table) on `device`."""
    f8 = torch.float8_e4m3fn
    return (torch.from_numpy(case.q).to(device).view(f8), torch.from_numpy(case.k).to(device).view(f8),
            torch.from_numpy(case.scale).to(device), torch.from_numpy(case.w).to(device),
            torch.from_numpy(case.seq_lens).to(device), torch.from_numpy(case.block_table).to(device))


def oracle_indexer(case, max_len):
    from oracle import oracle as O
    P = case.k.shape[0]
    return O.indexer_scores(case.q, case.k.reshape(P, -1), 64 * 128, case.scale.reshape(P, -1), 64 * 4,
                            case.w, case.block_table, case.seq_lens, max_len)
