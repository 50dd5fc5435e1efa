"""Device-side generators of the full-size benchmark inputs (multi-GB caches).

Same structure and distributions as flashinfer_repo_b200.workloads (which is
the bit-reproducible host version used for fixtures), but generated with
torch on the GPU because the cfg2 cache alone is ~2.3 GB.
"""
from __future__ import annotations

import torch

from .workloads import DC, DP, PS, SM_SCALE, TOPK


def _gen(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn_bf16(shape, g, device, std=1.0, chunk_rows=4096):
    """bf16 N(0, std^2) without materialising an fp32 copy of the whole tensor."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=device)
    flat = out.view(shape[0], -1)
    for r in range(0, shape[0], chunk_rows):
        blk = torch.randn(flat[r: r + chunk_rows].shape, generator=g, device=device)
        flat[r: r + chunk_rows] = (blk * std).to(torch.bfloat16)
    return out


def make_paged_batch(ctx_lens, seed, device, heads=16, topk=TOPK, kv_std=0.5, clustered=False,
                     shared_cache=False):
    """Tokens t with contexts ctx_lens[t]; pages of all requests drawn from one
    global permutation (shuffled page tables).  Returns
    (q_nope, q_pe, ckv, kpe, sparse_indices, sm_scale)."""
    g = _gen(seed, device)
    ctx = [int(c) for c in ctx_lens]
    T = len(ctx)
    npg = [(c + PS - 1) // PS for c in ctx]
    P = max(npg) if shared_cache else sum(npg)
    perm = torch.randperm(P, generator=g, device=device).to(torch.int64)
    ckv = _randn_bf16((P, PS, DC), g, device, kv_std)
    kpe = _randn_bf16((P, PS, DP), g, device, kv_std)
    q_nope = _randn_bf16((T, heads, DC), g, device)
    q_pe = _randn_bf16((T, heads, DP), g, device)
    idx = torch.full((T, topk), -1, dtype=torch.int32, device=device)
    off = 0
    for t, c in enumerate(ctx):
        table = perm[: npg[t]] if shared_cache else perm[off: off + npg[t]]
        off += npg[t]
        if c <= topk:
            pos = torch.randperm(c, generator=g, device=device)
        elif clustered and c > 4096 + topk:
            half = topk // 2
            recent = c - 4096 + torch.randperm(4096, generator=g, device=device)[:half]
            rest = torch.randperm(c - 4096, generator=g, device=device)[: topk - half]
            pos = torch.cat([recent, rest])
            pos = pos[torch.randperm(topk, generator=g, device=device)]
        else:
            pos = torch.randperm(c, generator=g, device=device)[:topk]
        idx[t, : pos.numel()] = (table[pos // PS] * PS + pos % PS).to(torch.int32)
    return q_nope, q_pe, ckv, kpe, idx, SM_SCALE


def cfg2_ctx(seed, T=64, lo=1024, hi=65536):
    g = torch.Generator()
    g.manual_seed(seed + 7919)
    return torch.randint(lo, hi + 1, (T,), generator=g).tolist()


def make_cfg2_device(seed=0, device="cuda", T=64):
    """BASELINE cfg2: T=64 decode tokens, contexts U[1024, 65536], page size 64,
    shuffled page tables, 2048 distinct positions per token (-1 padded)."""
    return make_paged_batch(cfg2_ctx(seed, T), seed, device)


def make_cfg3_device(seed=0, device="cuda", heads=128):
    """BASELINE cfg3: T=8, 128 heads, context 131072, clustered top-k, shared
    latent cache (replicated on every GPU when heads are sharded)."""
    return make_paged_batch([131072] * 8, seed, device, heads=heads, kv_std=1.0, clustered=True,
                            shared_cache=True)


def attention_bytes(idx: torch.Tensor, heads: int = 16) -> int:
    """Algorithmic HBM bytes of one call: per token n_valid*(512+64)*2 gathered
    + topk*4 indices + heads*576*2 q + heads*512*2 out + heads*4 lse."""
    T, topk = idx.shape
    n_valid = int((idx >= 0).sum().item())
    return n_valid * (DC + DP) * 2 + T * (topk * 4 + heads * (DC + DP) * 2 + heads * DC * 2
                                          + heads * 4)


def attention_flops(idx: torch.Tensor, heads: int = 16) -> int:
    n_valid = int((idx >= 0).sum().item())
    return 2 * heads * n_valid * (DC + DP) + 2 * heads * n_valid * DC



def make_cfg4_device(seed=0, device="cuda", T=128, ctx=32768, heads=16):
    """BASELINE cfg4: T=128 requests of context 32768; index keys e4m3
    [P,64,128] (uniform finite codes), fp32 scales U(0.5,2), index queries e4m3
    [T,64,128] from N(0,1), head weights N(0,1)/8; the latent cache for the
    16-head attention over the same pages.  Returns a dict of tensors."""
    g = _gen(seed, device)
    npg = (ctx + PS - 1) // PS
    P = T * npg
    perm = torch.randperm(P, generator=g, device=device).to(torch.int32)
    block_table = perm.view(T, npg).contiguous()
    k8 = torch.randint(0, 256, (P, PS, 128), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    k8 = torch.where((k8 & 0x7F) == 0x7F, k8 ^ 1, k8)
    scale = torch.rand((P, PS), generator=g, device=device) * 1.5 + 0.5
    q8 = torch.randn((T, 64, 128), generator=g, device=device).clamp(-448, 448).to(torch.float8_e4m3fn)
    w = torch.randn((T, 64), generator=g, device=device) / 8
    seq_lens = torch.full((T,), ctx, dtype=torch.int32, device=device)
    ckv = _randn_bf16((P, PS, DC), g, device, 0.5)
    kpe = _randn_bf16((P, PS, DP), g, device, 0.5)
    q_nope = _randn_bf16((T, heads, DC), g, device)
    q_pe = _randn_bf16((T, heads, DP), g, device)
    return dict(q8=q8, k8=k8, scale=scale, w=w, seq_lens=seq_lens, block_table=block_table,
                ckv=ckv, kpe=kpe, q_nope=q_nope, q_pe=q_pe, sm_scale=SM_SCALE)


def indexer_bytes(seq_lens, heads=64, topk=TOPK) -> int:
    """Algorithmic HBM bytes of the indexer per call: per request
    ctx*(128+4) keys+scales, 64*128 q, 64*4 weights, plus topk*4*2 outputs."""
    ctx = int(seq_lens.sum().item())
    B = seq_lens.numel()
    return ctx * 132 + B * (heads * 128 + heads * 4 + topk * 8)


def make_prefill_device(seed=0, device="cuda", queries=4096, ctx=65536, heads=16, topk=TOPK):
    """BASELINE cfg5 (one sequence per GPU): `queries` query tokens at absolute
    positions ctx-queries .. ctx-1, each selecting `topk` distinct positions
    <= its own position (causal), over one request of `ctx` tokens with a
    shuffled page table."""
    g = _gen(seed, device)
    npg = (ctx + PS - 1) // PS
    perm = torch.randperm(npg, generator=g, device=device).to(torch.int64)
    ckv = _randn_bf16((npg, PS, DC), g, device, 0.5)
    kpe = _randn_bf16((npg, PS, DP), g, device, 0.5)
    q_nope = _randn_bf16((queries, heads, DC), g, device)
    q_pe = _randn_bf16((queries, heads, DP), g, device)
    idx = torch.empty((queries, topk), dtype=torch.int32, device=device)
    pos0 = ctx - queries
    for r0 in range(0, queries, 256):  # random keys, causal mask, top-k -> distinct positions
        r1 = min(queries, r0 + 256)
        keys = torch.rand((r1 - r0, ctx), generator=g, device=device)
        allowed = torch.arange(ctx, device=device)[None, :] <= (pos0 + torch.arange(r0, r1, device=device))[:, None]
        keys = torch.where(allowed, keys, torch.full_like(keys, -1.0))
        pos = keys.topk(topk, dim=1).indices
        idx[r0:r1] = (perm[pos // PS] * PS + pos % PS).to(torch.int32)
    return q_nope, q_pe, ckv, kpe, idx, SM_SCALE
