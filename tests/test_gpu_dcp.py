"""Context parallelism (vLLM DCP) through the vLLM entry point.

Each simulated rank r of N holds KV tokens r, r+N, r+2N, ... of every sequence,
runs attention with cp_world_size/cp_rank/cp_tot_seqused_k, and the ranks'
partial (out, lse) merged with the N-way LSE merge must equal attention over
the whole KV (oracle): causal prefill chunks, decode with sliding windows,
sinks counted once, bf16 and FP8 K/V, packed and paged caches.
"""

import pytest
import torch

from flash_attn_b200._merge import _merge_partials
from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


def _shard_paged(kv, lengths, world, rank, page, device):
    """Rank's strided share of each sequence in a paged cache + table + local lengths."""
    local = [x[rank::world] for x in kv]
    counts = [int(l.shape[0]) for l in local]
    cols = max((c + page - 1) // page for c in counts) + 1
    B = len(counts)
    cache = torch.zeros(B * cols, page, *kv[0].shape[1:], dtype=kv[0].dtype)
    for b, l in enumerate(local):
        for i in range(l.shape[0]):
            cache[b * cols + i // page, i % page] = l[i]
    table = torch.arange(B * cols, dtype=torch.int32).reshape(B, cols)
    return cache.to(device), table.to(device), torch.tensor(counts, dtype=torch.int32, device=device)


def _run_ranks(q, keys, vals, qlens, klens, world, paged, device, **kw):
    cq = cu(qlens, device)
    tot = torch.tensor(klens, dtype=torch.int32, device=device)
    outs, lses = [], []
    for rank in range(world):
        if paged:
            kc, table, used = _shard_paged(keys, klens, world, rank, 16, device)
            vc, _, _ = _shard_paged(vals, klens, world, rank, 16, device)
            args = dict(seqused_k=used, block_table=table)
            k, v = kc, vc
            max_k = int(used.max())
        else:
            local_k = [x[rank::world] for x in keys]
            local_v = [x[rank::world] for x in vals]
            counts = [int(x.shape[0]) for x in local_k]
            k = torch.cat(local_k).to(device)
            v = torch.cat(local_v).to(device)
            args = dict(cu_seqlens_k=cu(counts, device))
            max_k = max(counts)
        out = torch.empty(q.shape[0], q.shape[1], v.shape[-1], dtype=torch.float32, device=device)
        o, l = vllm_attention(q, k, v, max(qlens), cq, max_k, out=out, return_softmax_lse=True,
                              cp_world_size=world, cp_rank=rank, cp_tot_seqused_k=tot, **args, **kw)
        outs.append(o)
        lses.append(l)
    return _merge_partials(torch.stack(outs), torch.stack(lses))


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("paged", [False, True])
def test_dcp_causal_prefill_chunks(device, world, paged):
    g = torch.Generator().manual_seed(71)
    qlens, klens = [1, 40, 130], [300, 40, 777]
    keys = [torch.randn(n, 2, 128, generator=g).to(torch.bfloat16) for n in klens]
    vals = [torch.randn(n, 2, 128, generator=g).to(torch.bfloat16) for n in klens]
    q = torch.randn(sum(qlens), 8, 128, generator=g).to(torch.bfloat16).to(device)
    out, lse = _run_ranks(q, keys, vals, qlens, klens, world, paged, device, causal=True)
    k_full, v_full = torch.cat(keys).to(device), torch.cat(vals).to(device)
    ref, refl = reference(q, k_full, v_full, cu(qlens, device), cu(klens, device), causal=True)
    assert_attention_close(out, ref, torch.float32)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_dcp_decode_window_and_sinks(device, world, kv):
    g = torch.Generator().manual_seed(72)
    klens = [1, 600, 2049, 33]
    qlens = [1] * len(klens)
    dtype = torch.bfloat16 if kv == "bf16" else torch.float8_e4m3fn
    keys = [torch.randn(n, 2, 128, generator=g).to(dtype) for n in klens]
    vals = [torch.randn(n, 2, 128, generator=g).to(dtype) for n in klens]
    q = torch.randn(len(klens), 8, 128, generator=g).to(torch.bfloat16).to(device)
    sinks = torch.linspace(-1, 1, 8, device=device)
    out, lse = _run_ranks(q, keys, vals, qlens, klens, world, True, device, causal=True,
                          window_size=[255, 0], s_aux=sinks)
    k_full, v_full = torch.cat(keys).to(device), torch.cat(vals).to(device)
    ref, refl = reference(q, k_full, v_full, cu(qlens, device), cu(klens, device), causal=True,
                          window=(255, 0), sinks=sinks)
    assert_attention_close(out, ref, torch.float32)
    assert_lse_close(lse, refl, atol=1e-3 if kv == "fp8" else 1e-4)
