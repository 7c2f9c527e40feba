"""KV-sequence-sharded long-context decode across GPUs (one process per GPU).

Each rank owns a contiguous slice of every request's KV sequence in its own
paged cache (``kv_shard``). A decode step is:

1. local split-KV decode over the rank's slice into an fp32 partial
   ``(out [B,Hq,Dv], lse [Hq,B])`` -- the tensor-core decode kernel plus its
   split merge;
2. one NCCL all-gather over NVLink / NVSwitch: each rank's out and lse sit in
   one flat fp32 buffer (out first, then lse), so a step issues a single
   collective and the N-way merge reads the gathered rows through strides;
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


def packed_views(flat, batch, heads, dim):
    """Split ``[..., B*Hq*Dv + Hq*B]`` fp32 rows into (out [..., B,Hq,Dv], lse [..., Hq,B]) views."""
    n_out = batch * heads * dim
    if flat.shape[-1] != n_out + heads * batch:
        raise ValueError("packed row length does not match the state shape")
    return (flat[..., :n_out].unflatten(-1, (batch, heads, dim)),
            flat[..., n_out:].unflatten(-1, (heads, batch)))


def gather_partials(partial_out, partial_lse, group=None):
    """All-gather per-rank partial states with ONE collective.

    ``[B,Hq,Dv]`` and ``[Hq,B]`` fp32 are packed into one row, all-gathered into
    ``[N, row]`` and returned as strided ``[N,B,Hq,Dv]`` / ``[N,Hq,B]`` views.
    """
    world = dist.get_world_size(group)
    batch, heads, dim = partial_out.shape
    row = torch.cat([partial_out.float().reshape(-1), partial_lse.float().reshape(-1)])
    gathered = torch.empty(world, row.numel(), dtype=torch.float32, device=row.device)
    dist.all_gather_into_tensor(gathered.view(-1), row, group=group)
    return packed_views(gathered, batch, heads, dim)


class ShardedDecoder:
    """Reusable buffers for KV-sharded decode steps of a fixed batch shape.

    ``packed`` holds this rank's partial state as one fp32 row
    ``[B*Hq*Dv | Hq*B]``; ``gathered`` is ``[N, row]`` after the all-gather and
    the merge reads its out/lse parts as strided views.
    """

    def __init__(self, batch, q_heads, head_dim, out_dtype, device, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        row = batch * q_heads * head_dim + q_heads * batch
        self.packed = torch.empty(row, dtype=torch.float32, device=device)
        self.partial, self.partial_lse = packed_views(self.packed, batch, q_heads, head_dim)
        self.gathered_flat = torch.empty(self.world, row, dtype=torch.float32, device=device)
        self.gathered, self.gathered_lse = packed_views(self.gathered_flat, batch, q_heads, head_dim)
        self.out = torch.empty(batch, q_heads, head_dim, dtype=out_dtype, device=device)
        self.out_lse = torch.empty(q_heads, batch, dtype=torch.float32, device=device)

    def step(self, q, k_cache, v_cache, *, cu_seqlens_q, seqused_k, max_seqlen_k, block_table,
             k_descale=None, v_descale=None, s_aux=None, softmax_scale=None):
        """One decode step over this rank's slice; returns the merged (out, lse)."""
        from ._attention import attention
        from ._merge import _merge_partials
        attention(q, k_cache, v_cache, cu_seqlens_q=cu_seqlens_q, seqused_k=seqused_k,
                  max_seqlen_q=1, max_seqlen_k=max_seqlen_k, block_table=block_table,
                  k_descale=k_descale, v_descale=v_descale, softmax_scale=softmax_scale,
                  s_aux=s_aux if self.rank == 0 else None, out=self.partial, lse=self.partial_lse)
        dist.all_gather_into_tensor(self.gathered_flat.view(-1), self.packed, group=self.group)
        return _merge_partials(self.gathered, self.gathered_lse, out=self.out, out_lse=self.out_lse)
