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

import ctypes

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


class _DeviceBytes:
    """A raw device allocation seen by torch through __cuda_array_interface__
    (no copy; the owner keeps the allocation alive)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerHeadShardedAttention:
    """cfg3 head sharding with the gather fused into the attention epilogues.

    Every rank holds a peer buffer (CUDA IPC, mapped by all ranks of the node)
    with two [T, H, 512] bf16 outputs, two [T, H] fp32 LSE arrays and the
    barrier flags.  A call computes this rank's H/world heads with
    `dsa_sparse_attention_scatter`, whose epilogues store each result row
    into the same place of EVERY rank's buffer (plain stores over NVLink), and
    its last grid ends with the cross-GPU barrier
    (`dsa_sparse_attention_scatter_sync`); after it the local buffer holds all
    H heads.
    Calls alternate between the two buffers.  Rule for the caller: read the
    returned tensors on the current stream before issuing the next call.
    Then the barrier of call n+1 follows every rank's reads of call n's
    results, and call n+2, the next writer of that buffer, follows the barrier.

    Replaces the all-gather + pack/unpack of `head_sharded_attention`; the
    payload crossing NVLink is the same (each rank's slice to every peer).
    """

    def __init__(self, num_tokens: int, num_heads: int, device=None, group=None):
        from . import _lib
        self._lib = _lib
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert 1 <= self.world <= 8, "one node: at most 8 ranks"
        assert num_heads % (HEADS_PER_RANK * self.world) == 0
        self.T, self.H = num_tokens, num_heads
        self.h = num_heads // self.world
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())

        def al(n):
            return (n + 255) // 256 * 256

        ob, lb = al(num_tokens * num_heads * DC * 2), al(num_tokens * num_heads * 4)
        self.off_out = (0, ob)
        self.off_lse = (2 * ob, 2 * ob + lb)
        self.off_flags = 2 * ob + 2 * lb
        self.nbytes = self.off_flags + 256
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            _lib.call("dsa_peer_alloc", self.nbytes, ctypes.byref(ptr), handle)
        self.local = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.ptrs = []
        self.opened = []
        with torch.cuda.device(self.device):
            for q, hq in enumerate(handles):
                if q == self.rank:
                    self.ptrs.append(self.local)
                    continue
                p = ctypes.c_void_p()
                _lib.call("dsa_peer_open", ctypes.create_string_buffer(hq, 64), ctypes.byref(p))
                self.ptrs.append(p.value)
                self.opened.append(p.value)
        raw = torch.as_tensor(_DeviceBytes(self.local, self.nbytes), device=self.device)
        self._raw = raw
        n_out, n_lse = num_tokens * num_heads * DC, num_tokens * num_heads
        self.out = [raw[o:o + 2 * n_out].view(torch.bfloat16).view(num_tokens, num_heads, DC)
                    for o in self.off_out]
        self.lse = [raw[o:o + 4 * n_lse].view(torch.float32).view(num_tokens, num_heads)
                    for o in self.off_lse]
        self._flags = (ctypes.c_void_p * self.world)(*[p + self.off_flags for p in self.ptrs])
        self.step = 0
        dist.barrier(group=group)  # every rank mapped every buffer before the first store

    def __call__(self, q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale):
        from .kernel import kernel_scatter
        T, H, _ = q_nope.shape
        assert (T, H) == (self.T, self.H), "shapes are fixed at construction"
        b = self.step & 1
        sl = slice(self.h * self.rank, self.h * (self.rank + 1))
        head0 = self.h * self.rank
        outs = [p + self.off_out[b] + head0 * DC * 2 for p in self.ptrs]
        lses = [p + self.off_lse[b] + head0 * 4 for p in self.ptrs]
        # one operator call: epilogues store into every rank's buffer, and the
        # grid that stores last ends with the cross-GPU barrier
        kernel_scatter(q_nope[:, sl], q_pe[:, sl], ckv_cache, kpe_cache, sparse_indices, sm_scale,
                       outs, lses, (H * DC, DC), (H, 1), sync=(self._flags, self.rank, self.world))
        self.step += 1
        return self.out[b], self.lse[b]

    def barrier(self):
        """A bare cross-GPU barrier on the current stream (dsa_peer_barrier),
        e.g. to line the ranks up on the device before timing a step."""
        from .kernel import workspace_for
        ws = workspace_for(self.device).buf
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            self._lib.call("dsa_peer_barrier", ctypes.cast(self._flags, ctypes.c_void_p), self.rank,
                           self.world, ws.data_ptr() if ws is not None else None,
                           ctypes.c_void_p(stream))

    def close(self):
        """Unmap the peers' buffers and free this rank's (after a host sync;
        every rank must have finished using them: call after a dist.barrier)."""
        if self.local is None:
            return
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self.opened:
                self._lib.call("dsa_peer_close", ctypes.c_void_p(p))
            self._raw = self.out = self.lse = None
            self._lib.call("dsa_peer_free", ctypes.c_void_p(self.local))
        self.local = None
        self.opened = []
