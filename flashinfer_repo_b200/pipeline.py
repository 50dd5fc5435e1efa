"""DSA decode step: FP8 indexer -> exact top-k -> sparse MLA attention.

Replaces `run_sparse_attention_pipeline` (solution/triton/kernel.py:184-332),
which calls run_indexer_and_topk (two device-to-host .item() syncs,
indexer_kernel.py:371,384), gets logical concatenated ids back, and
`repeat_interleave`s them by the KV sequence lengths (kernel.py:308-311) --
i.e. it assumes one query per KV token.  Here:
  * the indexer/top-k emit physical slot ids that the attention operator
    consumes directly;
  * query tokens map to requests through `query_request` (default: one
    decode token per request, token b <-> request b);
  * nothing synchronises with the host, so the whole step can be captured in
    a CUDA graph (`DecodeStepGraph`).
"""
from __future__ import annotations

import torch

from . import indexer as IX
from .kernel import kernel


def run_sparse_attention_pipeline(q_index_fp8, k_index_cache_fp8, k_scale, weights, seq_lens,
                                  block_table, q_nope, q_pe, ckv_cache, kpe_cache, sm_scale,
                                  topk=2048, query_request=None, scores_out=None, output=None,
                                  lse=None):
    """One DSA step.  Index tensors are per request ([B,...]); q_nope/q_pe are
    per query token ([T,16k,*]).  Returns (output [T,H,512] bf16, lse [T,H]
    fp32 base 2, slots [B,topk] int32 in ascending token position)."""
    scores = IX.indexer_scores(q_index_fp8, k_index_cache_fp8, k_scale, weights, seq_lens,
                               block_table, out=scores_out)
    # position order: the attention operator does not need score order
    _, slots = IX.topk_select(scores, seq_lens, block_table, topk, order="position")
    sparse_indices = slots if query_request is None else slots.index_select(0, query_request)
    out, lse = kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output=output,
                      lse=lse)
    return out, lse, slots


class DecodeStepGraph:
    """The pipeline captured once in a CUDA graph for fixed shapes and tensor
    addresses; `replay()` reruns it on the current contents of the captured
    input tensors (refresh them in place between steps)."""

    def __init__(self, q_index_fp8, k_index_cache_fp8, k_scale, weights, seq_lens, block_table,
                 q_nope, q_pe, ckv_cache, kpe_cache, sm_scale, topk=2048):
        self.args = (q_index_fp8, k_index_cache_fp8, k_scale, weights, seq_lens, block_table,
                     q_nope, q_pe, ckv_cache, kpe_cache, sm_scale)
        dev = q_nope.device
        T, H, _ = q_nope.shape
        self.scores = torch.zeros((seq_lens.numel(), block_table.shape[1] * 64),
                                  dtype=torch.float32, device=dev)
        self.output = torch.empty((T, H, 512), dtype=torch.bfloat16, device=dev)
        self.lse = torch.empty((T, H), dtype=torch.float32, device=dev)
        self.topk = topk
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            # warm-up outside capture: first-call set-up (workspace, attributes)
            _, _, self.slots = self._step()
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                _, _, self.slots = self._step()
        torch.cuda.current_stream(dev).wait_stream(side)

    def _step(self):
        return run_sparse_attention_pipeline(*self.args, topk=self.topk, scores_out=self.scores,
                                             output=self.output, lse=self.lse)

    def replay(self):
        self.graph.replay()
        return self.output, self.lse, self.slots
