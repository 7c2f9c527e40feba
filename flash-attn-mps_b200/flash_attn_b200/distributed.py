"""KV-sequence-sharded long-context decode across GPUs (one process per GPU).

Each rank owns a contiguous slice of every request's KV sequence in its own
paged cache (``kv_shard``). A decode step is:

1. local split-KV decode over the rank's slice into an fp32 partial
   ``(out [B,Hq,Dv], lse [Hq,B])`` -- the tensor-core decode kernel plus its
   split merge -- written as one flat fp32 row (out first, then lse);
2. the exchange of the rows: by default over peer memory (``exchange="p2p"``):
   the row is decoded straight into this rank's slot of a gather buffer in
   symmetric memory, the push kernel copies it into the same slot of every
   peer's buffer and raises a per-rank flag there, and a one-warp kernel waits
   (bounded) for every peer's flag (``fa_shard_push`` / ``fa_shard_wait``);
   or (``exchange="nccl"``) one NCCL all-gather of the rows over NVLink /
   NVSwitch;
3. the N-way LSE merge kernel (the same one that combines split-KV partials)
   reads the gathered rows through strides and writes the final output in the
   caller's dtype on every rank.

Sinks are seeded on rank 0 only, so they are counted once (the reference's
"sink counted once" contract, tests/test_vllm.py:130-149). The reference has
no distributed code (flash_attn_mps/vllm.py:5); this composes its split-KV
merge semantics (kernels/merge.metal:30-58) across ranks.
"""

import ctypes
import os

import torch
import torch.distributed as dist

from . import _capi


def _symmetric_memory_available():
    """torch's symmetric memory (the peer-memory exchange's buffer) is importable."""
    try:
        import torch.distributed._symmetric_memory  # noqa: F401
    except ImportError:
        return False
    return True


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

    ``exchange="p2p"`` (the default on CUDA devices with ``world > 1``;
    ``FAB_SHARD_EXCHANGE`` overrides it): a gather buffer in symmetric memory
    -- two parities x N slots of the packed row ``[B*Hq*Dv | Hq*B]`` plus a
    flag array -- mapped into every rank; step e decodes into this rank's slot
    of parity e & 1, pushes it to every peer over NVLink and waits for the
    peers' flags before the merge (8 ranks, config 4: 0.439 ms per step
    against 0.459 with the NCCL all-gather).
    ``exchange="nccl"`` (and every CPU / single-rank group): the row is
    all-gathered with NCCL (or gloo) into ``[N, row]``.
    The merge reads the gathered out/lse parts as strided views either way.
    """

    def __init__(self, batch, q_heads, head_dim, out_dtype, device, group=None, exchange=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shape = (batch, q_heads, head_dim)
        self.row = batch * q_heads * head_dim + q_heads * batch
        self.out = torch.empty(batch, q_heads, head_dim, dtype=out_dtype, device=device)
        self.out_lse = torch.empty(q_heads, batch, dtype=torch.float32, device=device)
        if exchange is None:
            exchange = os.environ.get("FAB_SHARD_EXCHANGE", "p2p")
        if self.world < 2 or torch.device(device).type != "cuda" or not _symmetric_memory_available():
            exchange = "nccl"
        self.exchange = exchange
        if exchange == "p2p":
            self._init_p2p(device)
        else:
            self.packed = torch.empty(self.row, dtype=torch.float32, device=device)
            self.partial, self.partial_lse = packed_views(self.packed, batch, q_heads, head_dim)
            self.gathered_flat = torch.empty(self.world, self.row, dtype=torch.float32, device=device)
            self.gathered, self.gathered_lse = packed_views(self.gathered_flat, batch, q_heads, head_dim)

    def _init_p2p(self, device):
        # Plain peer loads and stores only: no NVSwitch-side object is bound
        # to the buffer.
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem
        n, row = self.world, self.row
        if n > _capi.FA_MAX_PEERS:
            raise ValueError(f"the peer-memory exchange supports at most {_capi.FA_MAX_PEERS} ranks")
        row_padded = (row + 63) // 64 * 64          # 256-byte aligned slots
        data = 2 * n * row_padded
        # The flag array (2 * FA_MAX_PEERS uint32: per-rank flags, then the push
        # kernel's CTA counter) follows the slots in 256 spare bytes.
        self.symm = symm_mem.empty(data + 64, dtype=torch.float32, device=device)
        self.symm.zero_()
        handle = symm_mem.rendezvous(self.symm, self.group if self.group is not None else dist.group.WORLD)
        self._handle = handle
        elem = self.symm.element_size()
        peers = _capi.PeerBuffers()
        for p in range(n):
            base = handle.buffer_ptrs[p] + handle.offset
            peers.slots[p] = base
            peers.flags[p] = base + data * elem
        self.peers = peers
        self.row_padded = row_padded
        self.epoch = 0
        # Slot views of this rank's buffer: [parity, rank] rows and the merge views.
        slots = self.symm[:data].view(2, n, row_padded)
        self.slots = slots
        handle.barrier()
        torch.cuda.synchronize(device)

    def step(self, q, k_cache, v_cache, *, cu_seqlens_q, seqused_k, max_seqlen_k, block_table,
             k_descale=None, v_descale=None, s_aux=None, softmax_scale=None):
        """One decode step over this rank's slice; returns the merged (out, lse)."""
        from ._attention import attention
        from ._merge import _merge_partials
        batch, heads, dim = self.shape
        if self.exchange == "p2p":
            self.epoch += 1
            par = self.epoch & 1
            mine = self.slots[par, self.rank, :self.row]
            partial, partial_lse = packed_views(mine, batch, heads, dim)
        else:
            partial, partial_lse = self.partial, self.partial_lse
        attention(q, k_cache, v_cache, cu_seqlens_q=cu_seqlens_q, seqused_k=seqused_k,
                  max_seqlen_q=1, max_seqlen_k=max_seqlen_k, block_table=block_table,
                  k_descale=k_descale, v_descale=v_descale, softmax_scale=softmax_scale,
                  s_aux=s_aux if self.rank == 0 else None, out=partial, lse=partial_lse)
        if self.exchange == "p2p":
            lib = _capi.library()
            stream = _capi.stream_of(q.device)
            row = self.slots[par, self.rank, :self.row_padded]
            _capi.check(lib.fa_shard_push(_capi.ref(_capi.tensor(row)), _capi.ref(self.peers), self.world,
                                          self.rank, ctypes.c_uint32(self.epoch), stream))
            _capi.check(lib.fa_shard_wait(_capi.ref(self.peers), self.world, self.rank,
                                          ctypes.c_uint32(self.epoch), stream))
            gathered, gathered_lse = packed_views(self.slots[par, :, :self.row], batch, heads, dim)
        else:
            dist.all_gather_into_tensor(self.gathered_flat.view(-1), self.packed, group=self.group)
            gathered, gathered_lse = self.gathered, self.gathered_lse
        return _merge_partials(gathered, gathered_lse, out=self.out, out_lse=self.out_lse)
