"""GPU test of dsa_sparse_attention_noalloc, the entry point for callers that
cannot allocate device memory at call time (engines whose memory pool owns
all free HBM, plugin hosts that pass only inputs and outputs).  It must give
the same results as dsa_sparse_attention, called through the C ABI, and as the
CPU oracle, on two consecutive calls (the static scratch keeps the previous
call's contents); it must report device errors through its own getter, refuse
plans larger than its scratch, and take no device memory after its first call.

The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from flashinfer_repo_b200 import _lib, options
from flashinfer_repo_b200 import workloads as W
from tests.helpers import ATOL, LSE_ATOL, RTOL, assert_attention_close, case_to_device

pytestmark = pytest.mark.gpu


def _strides(qn, qp, ckv, kpe, idx, out, lse):
    return (qn.data_ptr(), qn.stride(0), qn.stride(1), qp.data_ptr(), qp.stride(0), qp.stride(1),
            ckv.data_ptr(), ckv.stride(0), ckv.stride(1), kpe.data_ptr(), kpe.stride(0),
            kpe.stride(1), idx.data_ptr(), idx.stride(0), idx.shape[0], qn.shape[1], ckv.shape[0],
            64, idx.shape[1])


def _call_with_workspace(lib, args, scale, out, lse, stream):
    n = ctypes.c_size_t(0)
    assert lib.dsa_sparse_attention_workspace_size(args[14], args[15], args[18], ctypes.byref(n)) == 0
    ws = torch.zeros(n.value, dtype=torch.uint8, device=out.device)
    rc = lib.dsa_sparse_attention(*args, scale, out.data_ptr(), out.stride(0), out.stride(1),
                                  lse.data_ptr(), lse.stride(0), lse.stride(1), ws.data_ptr(),
                                  ws.numel(), stream)
    assert rc == 0, lib.dsa_last_error_message()
    return ws


def _call_noalloc(lib, args, scale, out, lse, stream):
    rc = lib.dsa_sparse_attention_noalloc(*args, scale, out.data_ptr(), out.stride(0),
                                          out.stride(1), lse.data_ptr(), lse.stride(0),
                                          lse.stride(1), stream)
    assert rc == 0, lib.dsa_last_error_message()


def _assert_same(out, lse, ref_out, ref_lse):
    a, b = out.float().cpu().numpy(), ref_out.float().cpu().numpy()
    err = np.abs(a - b)
    assert not ((err > ATOL) & (err / np.maximum(np.abs(b), 1e-30) > RTOL)).any()
    la, lb = lse.cpu().numpy(), ref_lse.cpu().numpy()
    assert np.array_equal(np.isneginf(la), np.isneginf(lb))
    fin = ~np.isneginf(lb)
    assert np.abs(la[fin] - lb[fin]).max() <= LSE_ATOL


def _read_error(lib, stream, clear=1):
    bits = ctypes.c_int(-1)
    assert lib.dsa_sparse_attention_noalloc_read_error(clear, ctypes.byref(bits), stream) == 0
    return bits.value


def test_noalloc_matches_workspace_entry_point(cuda_device):
    lib = _lib.load()
    torch.cuda.set_device(cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    cases = [W.make_attention_case(41, [5000, 1500, 3000, 9000, 2048, 700]),
             W.make_attention_case(42, [4096, 12000, 64])]
    for case in cases:  # two calls in a row, different shapes: scratch is reused
        qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
        idx[1, 100:300] = -1
        T = idx.shape[0]
        args = _strides(qn, qp, ckv, kpe, idx, None, None)
        ref_out = torch.empty((T, 16, 512), dtype=torch.bfloat16, device=cuda_device)
        ref_lse = torch.empty((T, 16), dtype=torch.float32, device=cuda_device)
        _call_with_workspace(lib, args, case.sm_scale, ref_out, ref_lse, stream)
        from oracle import oracle as O
        o_out, o_lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe,
                                       idx.cpu().numpy(), case.sm_scale)
        for _ in range(2):
            out = torch.full_like(ref_out, float("nan"))
            lse = torch.full_like(ref_lse, float("nan"))
            _call_noalloc(lib, args, case.sm_scale, out, lse, stream)
            torch.cuda.synchronize()
            _assert_same(out, lse, ref_out, ref_lse)
            assert_attention_close(out, lse, o_out, o_lse, "noalloc vs oracle")
    assert _read_error(lib, stream) == 0


def test_noalloc_largest_grid_and_no_new_memory(cuda_device):
    """A batch large enough for the full default grid (2 x 148 CTAs, 592 of the
    640 partial slots), twice; device free memory is unchanged by the calls
    after the first."""
    lib = _lib.load()
    torch.cuda.set_device(cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    case = W.make_attention_case(43, [4096] * 1024, shared_cache=True)
    qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
    args = _strides(qn, qp, ckv, kpe, idx, None, None)
    T = idx.shape[0]
    ref_out = torch.empty((T, 16, 512), dtype=torch.bfloat16, device=cuda_device)
    ref_lse = torch.empty((T, 16), dtype=torch.float32, device=cuda_device)
    _call_with_workspace(lib, args, case.sm_scale, ref_out, ref_lse, stream)
    out = torch.empty_like(ref_out)
    lse = torch.empty_like(ref_lse)
    _call_noalloc(lib, args, case.sm_scale, out, lse, stream)  # first call: module + address set-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(cuda_device)[0]
    for _ in range(2):
        out.fill_(float("nan"))
        lse.fill_(float("nan"))
        _call_noalloc(lib, args, case.sm_scale, out, lse, stream)
        torch.cuda.synchronize()
        _assert_same(out, lse, ref_out, ref_lse)
    assert torch.cuda.mem_get_info(cuda_device)[0] == free0


def test_noalloc_reports_device_errors(cuda_device):
    """An out-of-range index is skipped and flagged; the flag stays set across
    calls until the getter clears it."""
    lib = _lib.load()
    torch.cuda.set_device(cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    case = W.make_attention_case(44, [3000, 5000])
    qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
    idx[0, 5] = ckv.shape[0] * 64 + 3  # past the last slot
    args = _strides(qn, qp, ckv, kpe, idx, None, None)
    out = torch.empty((2, 16, 512), dtype=torch.bfloat16, device=cuda_device)
    lse = torch.empty((2, 16), dtype=torch.float32, device=cuda_device)
    _read_error(lib, stream)  # start clean
    _call_noalloc(lib, args, case.sm_scale, out, lse, stream)
    assert _read_error(lib, stream, clear=0) == 1  # DSA_DEVERR_BAD_INDEX
    idx[0, 5] = -1
    _call_noalloc(lib, args, case.sm_scale, out, lse, stream)
    assert _read_error(lib, stream, clear=1) == 1  # still set: accumulated
    _call_noalloc(lib, args, case.sm_scale, out, lse, stream)
    assert _read_error(lib, stream) == 0


def test_noalloc_rejects_plans_larger_than_its_scratch(cuda_device):
    """A grid forced past the 320 CTAs the static scratch holds is refused
    before anything is launched."""
    lib = _lib.load()
    torch.cuda.set_device(cuda_device)
    case = W.make_attention_case(45, [4096] * 8, shared_cache=True)
    qn, qp, ckv, kpe, idx = case_to_device(case, cuda_device)
    args = _strides(qn, qp, ckv, kpe, idx, None, None)
    out = torch.empty((8, 16, 512), dtype=torch.bfloat16, device=cuda_device)
    lse = torch.empty((8, 16), dtype=torch.float32, device=cuda_device)
    with options(attention_ctas=321, attention_min_tiles=1):
        rc = lib.dsa_sparse_attention_noalloc(*args, case.sm_scale, out.data_ptr(), out.stride(0),
                                              out.stride(1), lse.data_ptr(), lse.stride(0),
                                              lse.stride(1), None)
    assert rc == 2
    assert b"320" in lib.dsa_last_error_message()
