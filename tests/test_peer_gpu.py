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
