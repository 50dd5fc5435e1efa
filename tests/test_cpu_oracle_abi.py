"""CPU tests: oracle pinned to the reference's golden vectors, workload
generators, C-ABI library loads and exports every declared symbol, host-side
argument checks.  No GPU needed."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from flashinfer_repo_b200 import _lib
from flashinfer_repo_b200 import workloads as W
from oracle import oracle as O
from tests.golden.cases import CASES, digest
from tests.helpers import ATOL, LSE_ATOL, RTOL

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_matches_reference_golden(name):
    """The C oracle reproduces the reference `run` outputs
    (solution/triton/indexer_kernel.py:436-497) on the committed fixtures."""
    case = CASES[name]()
    g = np.load(os.path.join(ROOT, "tests", "golden", f"attn_{name}.npz"))
    assert str(g["digest"]) == digest(case), "input generator drifted from the fixture"
    out, lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx, case.sm_scale)
    a, b = W.bf16_bits_to_f32(out), W.bf16_bits_to_f32(g["out"])
    # oracle (fp64) vs reference (fp32): at most one bf16 ulp apart
    err = np.abs(a - b)
    assert (err <= np.maximum(np.abs(b), 1e-3) * 2 ** -7 + 1e-6).all()
    assert not ((err > ATOL) & (err / np.maximum(np.abs(b), 1e-30) > RTOL)).any()
    fin = np.isfinite(g["lse"])
    assert np.array_equal(fin, np.isfinite(lse))
    assert np.abs(lse[fin] - g["lse"][fin]).max() <= LSE_ATOL / 100


def test_edge_case_semantics():
    """All-padding token -> output 0, lse -inf (kernel.py:118-136)."""
    case = CASES["edge"]()
    out, lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx, case.sm_scale)
    assert (out[3] == 0).all() and np.isneginf(lse[3]).all()
    assert np.isfinite(lse[[0, 1, 2, 4, 5, 6, 7]]).all()


def test_oracle_rejects_out_of_range_index():
    case = W.cfg1_case(0)
    idx = case.idx.copy()
    idx[0, 0] = case.ckv.shape[0] * 64
    with pytest.raises(ValueError):
        O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, idx, case.sm_scale)


def test_cfg1_generator_matches_spec():
    case = W.cfg1_case(0)
    assert case.q_nope.shape == (1, 16, 512) and case.ckv.shape == (64, 64, 512)
    idx = case.idx[0]
    assert len(np.unique(idx)) == 2048 and idx.min() >= 0 and idx.max() < 4096


def test_ragged_generator_pads_tail():
    case = W.make_attention_case(3, [100, 5000])
    assert (case.idx[0, 100:] == -1).all() and (case.idx[0, :100] >= 0).all()
    assert len(np.unique(case.idx[1])) == 2048


def test_bf16_conversion_round_trip():
    x = np.array([1.0, -2.5, 3.14159, 1e-20, 65504.0, np.inf, -np.inf], np.float32)
    b = W.f32_to_bf16_bits(x)
    assert np.array_equal(W.bf16_bits_to_f32(b)[[0, 1, 5, 6]], x[[0, 1, 5, 6]])
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(b, ref)


def test_e4m3_conversion_matches_torch():
    x = np.random.default_rng(0).standard_normal(4096).astype(np.float32) * 50
    x[:4] = [500.0, -1000.0, 0.0, 448.0]
    b = W.f32_to_e4m3_bits(x)
    ref = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(b, ref)
    codes = np.arange(256, dtype=np.uint8)
    ours = W.e4m3_bits_to_f32(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(ours), np.isnan(theirs))
    assert np.array_equal(ours[~np.isnan(ours)], theirs[~np.isnan(theirs)])


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "dsa_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dsa_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = _declared_symbols()
    assert "dsa_sparse_attention" in syms
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/dsa_b200.h but not exported"


def test_signatures_cover_declarations():
    assert set(_declared_symbols()) == set(_lib.SIGNATURES) | {"dsa_last_error_message"}


def test_signature_argument_counts_match_header():
    """Every ctypes argtypes list has as many entries as the header declaration
    has parameters (guards against an ABI change on one side only)."""
    src = open(os.path.join(ROOT, "include", "dsa_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    decls = dict(re.findall(r"\b(dsa_[a-z0-9_]+)\s*\(([^;]*?)\)\s*;", src, flags=re.S))
    for name, argtypes in _lib.SIGNATURES.items():
        params = decls[name].strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert n == len(argtypes), f"{name}: header has {n} parameters, ctypes table {len(argtypes)}"


def test_abi_argument_validation_without_gpu():
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    assert lib.dsa_sparse_attention_workspace_size(1, 20, 2048, ctypes.byref(n)) == 1
    assert b"multiple of 16" in lib.dsa_last_error_message()
    rc = lib.dsa_sparse_attention(None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, None, 0,
                                  1, 16, 64, 32, 2048, 0.1, None, 0, 0, None, 0, 0, None, 0, None)
    assert rc == 2 and b"page_size" in lib.dsa_last_error_message()
    rc = lib.dsa_sparse_attention(None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, None, 0,
                                  0, 16, 64, 64, 2048, 0.1, None, 0, 0, None, 0, 0, None, 0, None)
    assert rc == 0  # zero tokens: nothing to do


def test_kernel_rejects_cpu_tensors_and_bad_shapes():
    from flashinfer_repo_b200 import kernel
    case = W.cfg1_case(0)
    bf = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)  # noqa: E731
    args = [bf(case.q_nope), bf(case.q_pe), bf(case.ckv), bf(case.kpe), torch.from_numpy(case.idx)]
    with pytest.raises(RuntimeError, match="CUDA"):
        kernel(*args, case.sm_scale)
    bad = list(args)
    bad[0] = bad[0][:, :, :256]
    with pytest.raises(AssertionError):
        kernel(*bad, case.sm_scale)


def test_tvm_ffi_slot_registered_and_routes_to_kernel():
    """The reference's empty `flashinfer.kernel` TVM-FFI slot is filled; CPU
    tensors reach the operator and are refused (no CPU path)."""
    pytest.importorskip("tvm_ffi")
    from flashinfer_repo_b200.binding import register
    f = register()
    bf = torch.bfloat16
    with pytest.raises(Exception, match="CUDA"):
        f(torch.zeros(1, 16, 512, dtype=bf), torch.zeros(1, 16, 64, dtype=bf),
          torch.zeros(2, 64, 512, dtype=bf), torch.zeros(2, 64, 64, dtype=bf),
          torch.zeros(1, 2048, dtype=torch.int32), 0.1)


def test_options_struct_round_trip_and_validation():
    """dsa_set_options / dsa_get_options (host only): the ctypes struct has the
    header's field count, values round-trip, out-of-range fields (a cluster
    size other than 2, 4 or 8) are rejected and leave the options unchanged."""
    hdr = open(os.path.join(ROOT, "include", "dsa_b200.h")).read()
    body = re.search(r"typedef struct dsa_options \{(.*?)\} dsa_options;", hdr, re.S).group(1)
    assert len(re.findall(r"\bint \w+;", body)) == len(_lib.Options._fields_)
    lib = _lib.load()
    lib.dsa_set_options.argtypes = [ctypes.POINTER(_lib.Options)]
    lib.dsa_get_options.argtypes = [ctypes.POINTER(_lib.Options)]
    try:
        assert lib.dsa_set_options(ctypes.byref(_lib.Options(merge_pdl=1, attention_cluster=4))) == 0
        got = _lib.Options()
        assert lib.dsa_get_options(ctypes.byref(got)) == 0 and got.attention_cluster == 4
        for bad in (3, -1, 16):
            assert lib.dsa_set_options(ctypes.byref(_lib.Options(merge_pdl=1, attention_cluster=bad))) != 0
        assert lib.dsa_get_options(ctypes.byref(got)) == 0 and got.attention_cluster == 4
    finally:
        lib.dsa_set_options(None)
