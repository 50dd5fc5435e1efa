"""Peer-memory runtime of the fused head-sharded gather on one GPU: the
bounded cross-GPU barrier completes for a single rank and reports a timeout
(without hanging or faulting) when a rank never arrives.  Two ranks that wait
for each other are only ever run on two GPUs (test_parallel_gpu.py), never as
two launches on one GPU."""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

from flashinfer_repo_b200 import _lib

pytestmark = pytest.mark.gpu

FLAG_INTS = 16  # >= 1 + 8


def _barrier(flag_ptrs, rank, world, err):
    arr = (ctypes.c_void_p * world)(*flag_ptrs)
    _lib.call("dsa_peer_barrier", ctypes.cast(arr, ctypes.c_void_p), rank, world, err.data_ptr(),
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_barrier_world1_and_epochs(cuda_device):
    flags = torch.zeros(FLAG_INTS, dtype=torch.int32, device=cuda_device)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for _ in range(3):
        _barrier([flags.data_ptr()], 0, 1, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert flags[0].item() == 3 and flags[1].item() == 3  # epoch counter and own arrival


def test_barrier_missing_rank_times_out(cuda_device):
    """Rank 1 never arrives: the wait gives up after its bound (~2 s), sets
    DSA_DEVERR_TIMEOUT and the context stays usable."""
    mine = torch.zeros(FLAG_INTS, dtype=torch.int32, device=cuda_device)
    absent = torch.zeros(FLAG_INTS, dtype=torch.int32, device=cuda_device)  # nobody writes it
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    t0 = time.time()
    _barrier([mine.data_ptr(), absent.data_ptr()], 0, 2, err)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert err.item() & 2, "timeout bit not set"
    assert dt < 30
    x = torch.ones(4, device=cuda_device) * 2  # context still usable
    assert x.sum().item() == 8


def _scatter_sync(case, dev, flag_ptrs, rank, world, out, lse):
    """The operator with its epilogues storing into `out`/`lse` and the
    cross-GPU barrier inside its last grid (dsa_sparse_attention_scatter_sync)."""
    from flashinfer_repo_b200.kernel import kernel_scatter
    from tests.helpers import case_to_device
    qn, qp, ckv, kpe, idx = case_to_device(case, dev)
    flags = (ctypes.c_void_p * world)(*flag_ptrs)
    H = qn.shape[1]
    kernel_scatter(qn, qp, ckv, kpe, idx, case.sm_scale, [out.data_ptr()], [lse.data_ptr()],
                   (H * 512, 512), (H, 1), sync=(flags, rank, world))
    return qn, qp, ckv, kpe, idx


@pytest.mark.parametrize("ctas", [0, 1])
def test_scatter_sync_world1(cuda_device, ctas):
    """One rank: the in-operator barrier completes (in the merge grid when
    tokens are split, in the attention grid when one CTA does everything),
    bumps the epoch once per call, and the stored result equals kernel()'s."""
    from flashinfer_repo_b200 import kernel, options, read_device_error
    from flashinfer_repo_b200 import workloads as W
    case = W.make_attention_case(71, [5000, 3000, 2048])
    flags = torch.zeros(FLAG_INTS, dtype=torch.int32, device=cuda_device)
    out = torch.empty((3, 16, 512), dtype=torch.bfloat16, device=cuda_device)
    lse = torch.empty((3, 16), dtype=torch.float32, device=cuda_device)
    with options(attention_ctas=ctas):
        for _ in range(3):
            args = _scatter_sync(case, cuda_device, [flags.data_ptr()], 0, 1, out, lse)
        ref_out, ref_lse = kernel(*args, case.sm_scale)
    torch.cuda.synchronize()
    assert read_device_error(cuda_device) == 0
    assert flags[0].item() == 3 and flags[1].item() == 3 and flags[9].item() == 0
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)


def test_scatter_sync_missing_rank_times_out(cuda_device):
    """Rank 1 never arrives: the barrier at the end of the operator gives up
    after its bound, the results are stored all the same, the timeout bit is
    set in the workspace error word and the context stays usable."""
    from flashinfer_repo_b200 import kernel, read_device_error
    from flashinfer_repo_b200 import workloads as W
    case = W.make_attention_case(72, [4096, 2500])
    mine = torch.zeros(FLAG_INTS, dtype=torch.int32, device=cuda_device)
    absent = torch.zeros(FLAG_INTS, dtype=torch.int32, device=cuda_device)  # nobody writes it
    out = torch.empty((2, 16, 512), dtype=torch.bfloat16, device=cuda_device)
    lse = torch.empty((2, 16), dtype=torch.float32, device=cuda_device)
    read_device_error(cuda_device)
    t0 = time.time()
    args = _scatter_sync(case, cuda_device, [mine.data_ptr(), absent.data_ptr()], 0, 2, out, lse)
    torch.cuda.synchronize()
    assert time.time() - t0 < 30
    assert read_device_error(cuda_device) & 2, "timeout bit not set"
    ref_out, ref_lse = kernel(*args, case.sm_scale)
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
