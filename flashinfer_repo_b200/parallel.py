"""Multi-GPU layouts of the DSA decode operator (one process per GPU).

Two ways to spread the work over the GPUs of one node:

* Request sharding (BASELINE cfg1/2/4/5): query tokens are independent, so
  rank r takes a contiguous block of requests (`shard_range`) with their
  pages resident on its GPU and calls `kernel()` on them.  No collective is
  on the data path; aggregate throughput = all tokens / slowest rank.
* Head sharding (BASELINE cfg3, 128 heads): rank g computes heads
  [16g, 16g+16) -- exactly the reference's 16-head operator
  (solution/triton/kernel.py:138-182) -- over a replicated latent cache, then
  one all-gather of a packed per-rank buffer (output bf16 + LSE fp32,
  T*16*(512*2+4) bytes) assembles [T, 16*world, 512] and [T, 16*world].
  The payload is small (131.6 KB per rank at T=8), so the collective is
  latency-bound; it is issued on torch's current stream (NCCL over NVLink on
  the B200 node, gloo on CPU for the host-side tests).

The reference itself is single-GPU and has no collective (its only parallel
decomposition is split-K inside one GPU, kernel.py:343-567).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

HEADS_PER_RANK = 16
DC = 512


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block of [0, n) owned by `rank`: the first n % world ranks
    take one extra item."""
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def pack_out_lse(out: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
    """[T,h,512] bf16 + [T,h] fp32 -> one flat uint8 buffer (out bytes, then lse bytes)."""
    T, h, _ = out.shape
    buf = torch.empty(T * h * (DC * 2 + 4), dtype=torch.uint8, device=out.device)
    nb = T * h * DC * 2
    buf[:nb].view(torch.bfloat16).view(T, h, DC).copy_(out)
    buf[nb:].view(torch.float32).view(T, h).copy_(lse)
    return buf


def unpack_gathered(gathered: torch.Tensor, world: int, T: int, h: int = HEADS_PER_RANK):
    """[world, bytes] -> (out [T, h*world, 512] bf16, lse [T, h*world] fp32),
    rank g's heads at [h*g, h*g+h)."""
    nb = T * h * DC * 2
    outs = gathered[:, :nb].contiguous().view(torch.bfloat16).view(world, T, h, DC)
    lses = gathered[:, nb:].contiguous().view(torch.float32).view(world, T, h)
    out = outs.permute(1, 0, 2, 3).reshape(T, world * h, DC)
    lse = lses.permute(1, 0, 2).reshape(T, world * h)
    return out, lse


def head_sharded_attention(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale,
                           group=None, local_fn=None):
    """cfg3 head sharding.  q_nope/q_pe hold ALL heads [T, H, *] with H a
    multiple of 16*world; this rank computes its H/world heads with `local_fn`
    (default: the sm_100a `kernel`) and all-gathers the packed results.
    Returns the full (output [T, H, 512], lse [T, H])."""
    if local_fn is None:
        from .kernel import kernel as local_fn
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T, H, _ = q_nope.shape
    assert H % (HEADS_PER_RANK * world) == 0, f"{H} heads do not split into {world} x 16k"
    h = H // world
    sl = slice(h * rank, h * (rank + 1))
    out, lse = local_fn(q_nope[:, sl], q_pe[:, sl], ckv_cache, kpe_cache, sparse_indices, sm_scale)
    mine = pack_out_lse(out, lse)
    gathered = torch.empty((world, mine.numel()), dtype=torch.uint8, device=mine.device)
    if mine.is_cuda:
        dist.all_gather_into_tensor(gathered, mine, group=group)
    else:  # gloo (host-side tests)
        dist.all_gather(list(gathered.unbind(0)), mine, group=group)
    return unpack_gathered(gathered, world, T, h)
