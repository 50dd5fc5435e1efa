"""Head-sharded cfg3 attention over 2 GPUs with an NCCL all-gather must equal
the 128-head operator on one GPU (skipped with fewer than 2 GPUs)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from flashinfer_repo_b200 import kernel
    from flashinfer_repo_b200.bench_inputs import make_paged_batch
    from flashinfer_repo_b200.parallel import head_sharded_attention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    qn, qp, ckv, kpe, idx, scale = make_paged_batch([20000, 9000, 131072], 5, dev, heads=64,
                                                    clustered=True, shared_cache=True)
    out, lse = head_sharded_attention(qn, qp, ckv, kpe, idx, scale)
    ref_out, ref_lse = kernel(qn, qp, ckv, kpe, idx, scale)
    torch.cuda.synchronize()
    q.put((rank, torch.equal(out, ref_out), torch.equal(lse, ref_lse)))
    dist.destroy_process_group()


def test_head_sharded_nccl_equals_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] and r[2] for r in res), res


def _peer_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from flashinfer_repo_b200 import kernel
    from flashinfer_repo_b200.bench_inputs import make_paged_batch
    from flashinfer_repo_b200.kernel import read_device_error
    from flashinfer_repo_b200.parallel import PeerHeadShardedAttention, head_sharded_attention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    res = []
    peer = None
    for step in range(4):  # both buffers, twice; inputs change every step
        qn, qp, ckv, kpe, idx, scale = make_paged_batch([20000, 9000, 131072], 100 + step, dev,
                                                        heads=64, clustered=True,
                                                        shared_cache=True)
        if peer is None:
            peer = PeerHeadShardedAttention(qn.shape[0], 64, dev)
        out, lse = peer(qn, qp, ckv, kpe, idx, scale)
        out, lse = out.clone(), lse.clone()  # read before the next call
        g_out, g_lse = head_sharded_attention(qn, qp, ckv, kpe, idx, scale)
        r_out, r_lse = kernel(qn, qp, ckv, kpe, idx, scale)
        torch.cuda.synchronize()
        res.append((torch.equal(out, g_out), torch.equal(lse, g_lse),
                    float((out.float() - r_out.float()).abs().max()),
                    float((lse - r_lse).abs().max())))
    err = read_device_error(dev)
    dist.barrier()
    peer.close()
    q.put((rank, res, err))
    dist.destroy_process_group()


def test_peer_scatter_equals_all_gather():
    """The fused peer-store path equals the NCCL all-gather path bit for bit
    (same per-rank kernel call), and the single-GPU 64-head result within the
    split-K rounding (a different split of the top-k dimension)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for rank, steps, err in res:
        assert err == 0, (rank, err)
        for eq_o, eq_l, d_o, d_l in steps:
            assert eq_o and eq_l, (rank, steps)
            assert d_o <= 1e-2 and d_l <= 1e-3, (rank, steps)
