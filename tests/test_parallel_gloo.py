"""Multi-process host logic on CPU (gloo, world sizes 2-4): request sharding,
head sharding with the packed all-gather, and failure detection (a rank that
leaves before the collective makes the others fail within the process-group
timeout instead of hanging).  The local 16-head operator is the C oracle
here; on GPUs it is the sm_100a kernel (same function)."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashinfer_repo_b200 import workloads as W
from flashinfer_repo_b200.parallel import head_sharded_attention, shard_range
from oracle import oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _oracle_fn(qn, qp, ckv, kpe, idx, scale):
    out, lse = O.dsa_attention(_bits(qn), _bits(qp), _bits(ckv), _bits(kpe), idx.numpy(), scale,
                               nthreads=2)
    return torch.from_numpy(out.view(np.int16)).view(torch.bfloat16), torch.from_numpy(lse)


def _to_t(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if mode == "heads":
            case = W.make_attention_case(77, [5000, 3000, 9000], heads=16 * world, shared_cache=True)
            out, lse = head_sharded_attention(_to_t(case.q_nope), _to_t(case.q_pe), _to_t(case.ckv),
                                              _to_t(case.kpe), torch.from_numpy(case.idx),
                                              case.sm_scale, local_fn=_oracle_fn)
            q.put((rank, _bits(out), lse.numpy()))
        elif mode == "requests":
            case = W.make_attention_case(78, [4000, 2500, 700, 5000, 3300])
            a, b = shard_range(case.T, rank, world)
            out, lse = _oracle_fn(_to_t(case.q_nope[a:b]), _to_t(case.q_pe[a:b]), _to_t(case.ckv),
                                  _to_t(case.kpe), torch.from_numpy(case.idx[a:b]), case.sm_scale)
            q.put((rank, (a, b), _bits(out), lse.numpy()))
        elif mode == "rank_leaves":
            if rank == 1:
                q.put((rank, "left"))
                return  # leaves between steps, before the collective
            t = torch.zeros(4)
            try:
                dist.all_reduce(t)
                q.put((rank, "no error"))
            except Exception as e:  # noqa: BLE001
                q.put((rank, "error:" + type(e).__name__))
    finally:
        if mode != "rank_leaves":
            dist.destroy_process_group()


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(res, key=lambda r: r[0])


def test_shard_range_covers_everything():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            parts = [shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_all_gather_matches_full_operator(world):
    res = _run("heads", world)
    case = W.make_attention_case(77, [5000, 3000, 9000], heads=16 * world, shared_cache=True)
    for g in range(world):
        sl = slice(16 * g, 16 * g + 16)
        ref_out, ref_lse = O.dsa_attention(case.q_nope[:, sl], case.q_pe[:, sl], case.ckv, case.kpe,
                                           case.idx, case.sm_scale)
        for _, out, lse in res:
            assert np.array_equal(out[:, sl], ref_out)
            assert np.array_equal(lse[:, sl], ref_lse)


@pytest.mark.parametrize("world", [2, 3])
def test_request_sharding_is_exact_partition(world):
    res = _run("requests", world)
    case = W.make_attention_case(78, [4000, 2500, 700, 5000, 3300])
    ref_out, ref_lse = O.dsa_attention(case.q_nope, case.q_pe, case.ckv, case.kpe, case.idx,
                                       case.sm_scale)
    for _, (a, b), out, lse in res:
        assert np.array_equal(out, ref_out[a:b]) and np.array_equal(lse, ref_lse[a:b])


def test_rank_leaving_is_detected_not_hung():
    res = _run("rank_leaves")
    assert res[1][1] == "left"
    assert res[0][1].startswith("error:")
