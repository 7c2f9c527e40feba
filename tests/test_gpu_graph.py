"""The library's launches inside CUDA graphs (capture once, replay per step).

A serving loop captures its decode step (store the new token, attend over the
paged cache) into a CUDA graph and replays it with new inputs copied into the
captured buffers. Every entry point runs on the caller's current stream, plans
on the host from shapes only and allocates its workspace through PyTorch (the
graph's private pool), so capture works; the replayed results must equal an
eager call on the same inputs.
"""

import pytest
import torch

from flash_attn_b200 import flash_attn_varlen_func, flash_attn_with_kvcache, store_kvcache
from flash_attn_b200._decode import decode_attention

pytestmark = pytest.mark.gpu


def _capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        result = fn()
    return graph, result


def test_paged_decode_step_with_append_replays(device):
    g = torch.Generator().manual_seed(21)
    B, H, HK, D, page, pages = 8, 16, 4, 128, 16, 64
    kc = torch.randn(B * pages, page, HK, D, generator=g).to(torch.bfloat16).to(device)
    vc = torch.randn_like(kc)
    table = torch.randperm(B * pages, generator=g).int().reshape(B, pages).to(device)
    lens = torch.randint(100, pages * page - 2, (B,), generator=g).int().to(device)
    q = torch.empty(B, 1, H, D, dtype=torch.bfloat16, device=device)
    k = torch.empty(B, 1, HK, D, dtype=torch.bfloat16, device=device)
    v = torch.empty_like(k)

    def step():
        return flash_attn_with_kvcache(q, kc, vc, k, v, cache_seqlens=lens, block_table=table, causal=True)

    graph, out = _capture(step)
    for trial in range(3):
        q.copy_(torch.randn(q.shape, generator=g).to(torch.bfloat16))
        k.copy_(torch.randn(k.shape, generator=g).to(torch.bfloat16))
        v.copy_(torch.randn(v.shape, generator=g).to(torch.bfloat16))
        graph.replay()
        expected = step()
        torch.cuda.synchronize()
        assert torch.equal(out, expected), trial


def test_fp8_store_and_split_decode_replay(device):
    g = torch.Generator().manual_seed(22)
    B, H, HK, D, page, pages = 4, 32, 8, 128, 16, 256
    kc = torch.zeros(B * pages, page, HK, D, dtype=torch.float8_e4m3fn, device=device)
    vc = torch.zeros_like(kc)
    table = torch.randperm(B * pages, generator=g).int().reshape(B, pages).to(device)
    ctx = pages * page
    scale = ((1 + 3 * torch.rand(HK, generator=g)) / 448).to(device)
    rows = torch.randn(B * ctx, HK, D, generator=g).to(torch.bfloat16).to(device)
    slots = (table.long()[:, :, None] * page + torch.arange(page, device=device)).reshape(-1)
    store_kvcache(rows, rows, kc, vc, slots, k_scale=scale, v_scale=scale)
    used = torch.full((B,), ctx - 5, dtype=torch.int32, device=device)
    cu = torch.arange(B + 1, dtype=torch.int32, device=device)
    descale = scale.reshape(1, HK).expand(B, HK)
    q = torch.empty(B, H, D, dtype=torch.bfloat16, device=device)
    new = torch.empty(B, HK, D, dtype=torch.bfloat16, device=device)
    new_slots = (table.long()[torch.arange(B), (ctx - 5) // page] * page + (ctx - 5) % page).to(device)

    def step():
        store_kvcache(new, new, kc, vc, new_slots, k_scale=scale, v_scale=scale)
        return decode_attention(q, kc, vc, cu_seqlens_q=cu, seqused_k=used + 1, max_seqlen_k=ctx,
                                block_table=table, k_descale=descale, v_descale=descale)

    graph, (out, lse) = _capture(step)
    for trial in range(3):
        q.copy_(torch.randn(q.shape, generator=g).to(torch.bfloat16))
        new.copy_(torch.randn(new.shape, generator=g).to(torch.bfloat16))
        graph.replay()
        expected, expected_lse = step()
        torch.cuda.synchronize()
        assert torch.equal(out, expected) and torch.equal(lse, expected_lse), trial


def test_varlen_prefill_replays(device):
    g = torch.Generator().manual_seed(23)
    lens = [300, 1000, 77, 513]
    total = sum(lens)
    q = torch.empty(total, 16, 128, dtype=torch.bfloat16, device=device)
    k = torch.empty(total, 4, 128, dtype=torch.bfloat16, device=device)
    v = torch.empty_like(k)
    cu = torch.tensor([0, 300, 1300, 1377, 1890], dtype=torch.int32, device=device)

    def step():
        return flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), causal=True,
                                      return_softmax_lse=True)

    graph, (out, lse) = _capture(step)
    for trial in range(2):
        for t in (q, k, v):
            t.copy_(torch.randn(t.shape, generator=g).to(torch.bfloat16))
        graph.replay()
        expected, expected_lse = step()
        torch.cuda.synchronize()
        assert torch.equal(out, expected) and torch.equal(lse, expected_lse), trial


def test_launch_counter_counts_captures_not_replays(device):
    from flash_attn_b200 import _capi
    k = torch.randn(32, 2, 128, device=device).to(torch.bfloat16)
    cache = torch.zeros(4, 16, 2, 128, dtype=torch.bfloat16, device=device)
    slots = torch.arange(32, device=device)
    before = _capi.kernel_launches()
    store_kvcache(k, k, cache, cache.clone(), slots)
    assert _capi.kernel_launches() - before == 1
    graph, _ = _capture(lambda: store_kvcache(k, k, cache, cache.clone(), slots))
    captured = _capi.kernel_launches()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert _capi.kernel_launches() == captured
