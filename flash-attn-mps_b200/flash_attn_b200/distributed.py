"""KV-sequence-sharded long-context decode across GPUs (one process per GPU).

Each rank owns a contiguous slice of every request's KV sequence in its own
paged cache (``kv_shard``). A decode step is:

1. local split-KV decode over the rank's slice into an fp32 partial
   ``(out [B,Hq,Dv], lse [Hq,B])`` -- the tensor-core decode kernel plus its
   split merge;
2. ``gather_partials``: one NCCL all-gather of the partials over NVLink /
   NVSwitch into ``[N,B,Hq,Dv]`` and ``[N,Hq,B]``;
3. the N-way LSE merge kernel (the same one that combines split-KV partials)
   writes the final output in the caller's dtype on every rank.

Sinks are seeded on rank 0 only, so they are counted once (the reference's
"sink counted once" contract, tests/test_vllm.py:130-149). The reference has
no distributed code (flash_attn_mps/vllm.py:5); this composes its split-KV
merge semantics (kernels/merge.metal:30-58) across ranks.
"""

import torch
import torch.distributed as dist


def kv_shard(length, rank, world):
    """Token range [start, end) of a length-``length`` sequence owned by ``rank``."""
    return length * rank // world, length * (rank + 1) // world


def gather_partials(partial_out, partial_lse, group=None, out=None, out_lse=None):
    """All-gather per-rank partial states: [B,Hq,Dv] and [Hq,B] -> [N,...]."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world, *partial_out.shape), dtype=partial_out.dtype, device=partial_out.device)
    if out_lse is None:
        out_lse = torch.empty((world, *partial_lse.shape), dtype=partial_lse.dtype, device=partial_lse.device)
    dist.all_gather_into_tensor(out.view(-1), partial_out.contiguous().view(-1), group=group)
    dist.all_gather_into_tensor(out_lse.view(-1), partial_lse.contiguous().view(-1), group=group)
    return out, out_lse


class ShardedDecoder:
    """Reusable buffers for KV-sharded decode steps of a fixed batch shape."""

    def __init__(self, batch, q_heads, head_dim, out_dtype, device, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.partial = torch.empty(batch, q_heads, head_dim, dtype=torch.float32, device=device)
        self.gathered = torch.empty(self.world, batch, q_heads, head_dim, dtype=torch.float32, device=device)
        self.gathered_lse = torch.empty(self.world, q_heads, batch, dtype=torch.float32, device=device)
        self.out = torch.empty(batch, q_heads, head_dim, dtype=out_dtype, device=device)
        self.out_lse = torch.empty(q_heads, batch, dtype=torch.float32, device=device)

    def step(self, q, k_cache, v_cache, *, cu_seqlens_q, seqused_k, max_seqlen_k, block_table,
             k_descale=None, v_descale=None, s_aux=None, softmax_scale=None):
        """One decode step over this rank's slice; returns the merged (out, lse)."""
        from ._attention import attention
        from ._merge import _merge_partials
        o, l = attention(q, k_cache, v_cache, cu_seqlens_q=cu_seqlens_q, seqused_k=seqused_k,
                         max_seqlen_q=1, max_seqlen_k=max_seqlen_k, block_table=block_table,
                         k_descale=k_descale, v_descale=v_descale, softmax_scale=softmax_scale,
                         s_aux=s_aux if self.rank == 0 else None, out=self.partial)
        gathered, gathered_lse = gather_partials(o, l, self.group, self.gathered, self.gathered_lse)
        return _merge_partials(gathered, gathered_lse, out=self.out, out_lse=self.out_lse)
