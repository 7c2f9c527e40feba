"""Varlen prefill on the tcgen05 kernel (bf16/f16, head_dim 128) vs the oracle.

Covers ragged lengths around the 128-row/128-key tile edges, q_len != k_len
(lower-right causal), GQA ratios, non-causal, and the benchmark's config 2
(32 sequences, lengths U[64, 4096], 32/8 heads) checked on sampled rows.
"""

import numpy as np
import pytest
import torch

from flash_attn_b200 import flash_attn_varlen_func
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


def _run(device, dtype, qlens, klens, hq, hk, causal, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sum(qlens), hq, 128, generator=g).to(dtype).to(device)
    k = torch.randn(sum(klens), hk, 128, generator=g).to(dtype).to(device)
    v = torch.randn(sum(klens), hk, 128, generator=g).to(dtype).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    out, lse = flash_attn_varlen_func(q, k, v, cq, ck, max(qlens), max(klens), causal=causal,
                                      return_softmax_lse=True)
    return q, k, v, cq, ck, out, lse


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("causal", [True, False])
def test_tile_edges(device, dtype, causal):
    lens = [1, 7, 127, 128, 129, 255, 256, 300, 513]
    q, k, v, cq, ck, out, lse = _run(device, dtype, lens, lens, 8, 2, causal)
    ref, refl = reference(q, k, v, cq, ck, causal=causal)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("causal", [True, False])
def test_query_shorter_than_keys(device, causal):
    qlens = [1, 5, 100, 128, 200, 0, 64]
    klens = [300, 5, 1000, 129, 700, 17, 64]
    q, k, v, cq, ck, out, lse = _run(device, torch.bfloat16, qlens, klens, 4, 4, causal, seed=3)
    ref, refl = reference(q, k, v, cq, ck, causal=causal)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_queries_longer_than_keys_mask_whole_rows(device):
    # Lower-right causal: the first q_len - k_len rows see no key at all.
    qlens, klens = [300, 130], [100, 0]
    q, k, v, cq, ck, out, lse = _run(device, torch.float16, qlens, klens, 4, 1, True, seed=5)
    ref, refl = reference(q, k, v, cq, ck, causal=True)
    assert_attention_close(out, ref)
    assert_lse_close(lse, refl)
    assert torch.isneginf(lse[:, :200]).all() and torch.count_nonzero(out[:200]) == 0


@pytest.mark.parametrize("hq,hk", [(32, 8), (16, 16), (8, 1)])
def test_gqa_ratios(device, hq, hk):
    lens = [64, 1000, 333]
    q, k, v, cq, ck, out, lse = _run(device, torch.bfloat16, lens, lens, hq, hk, True, seed=hq)
    ref, refl = reference(q, k, v, cq, ck, causal=True)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def _sample_rows_reference(q, k, v, cq, ck, b, rows, causal):
    """Oracle on selected query rows of request b (lower-right causal positions kept)."""
    q0, q1 = int(cq[b]), int(cq[b + 1])
    k0, k1 = int(ck[b]), int(ck[b + 1])
    qlen, klen = q1 - q0, k1 - k0
    outs, lses = [], []
    for r in rows:
        kend = min(klen, r + 1 + klen - qlen) if causal else klen
        qq = q[q0 + r:q0 + r + 1]
        kk, vv = k[k0:k0 + kend], v[k0:k0 + kend]
        o, l = reference(qq, kk, vv, torch.tensor([0, 1], dtype=torch.int32),
                         torch.tensor([0, kend], dtype=torch.int32), causal=causal)
        outs.append(o)
        lses.append(l)
    return torch.cat(outs), torch.cat(lses, dim=1)


def test_benchmark_config2_sampled_rows(device):
    # Config 2: 32 sequences, L ~ U[64, 4096] (seeded), 32 q / 8 kv heads, D=128, causal.
    rng = np.random.default_rng(2)
    lens = rng.integers(64, 4097, size=32).tolist()
    q, k, v, cq, ck, out, lse = _run(device, torch.bfloat16, lens, lens, 32, 8, True, seed=2)
    cqc, ckc = cq.cpu(), ck.cpu()
    for b in (0, int(np.argmax(lens)), 17):
        L = lens[b]
        rows = sorted(set([0, 1, 127, 128, L // 2, L - 129, L - 2, L - 1]) & set(range(L)))
        ref, refl = _sample_rows_reference(q, k, v, cqc, ckc, b, rows, True)
        got = out[int(cqc[b]) + torch.tensor(rows, device=device)]
        got_lse = lse[:, int(cqc[b]) + torch.tensor(rows, device=device)]
        assert_attention_close(got, ref, torch.bfloat16)
        assert_lse_close(got_lse, refl)
    assert torch.isfinite(out).all() and torch.isfinite(lse).all()


@pytest.mark.parametrize("window,causal", [((1024, 0), True), ((0, 0), True), ((15, 2), False),
                                           ((-1, 7), False), ((127, -1), True), ((300, 40), False)])
def test_windows_on_tensor_core_path(device, window, causal):
    from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
    lens = [1, 200, 700, 1500, 129]
    g = torch.Generator().manual_seed(7)
    q = torch.randn(sum(lens), 8, 128, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(sum(lens), 2, 128, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn(sum(lens), 2, 128, generator=g).to(torch.bfloat16).to(device)
    c = cu(lens, device)
    sinks = torch.linspace(-2, 2, 8, device=device)
    out, lse = vllm_attention(q, k, v, max(lens), c, max(lens), cu_seqlens_k=c, causal=causal,
                              window_size=list(window), s_aux=sinks, return_softmax_lse=True)
    ref, refl = reference(q, k, v, c, c, causal=causal, window=window, sinks=sinks)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("cap", [0.25, 1.0, 50.0])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_softcap_on_tensor_core_path(device, cap, dtype):
    lens = [100, 333, 1024]
    g = torch.Generator().manual_seed(11)
    q = (torch.randn(sum(lens), 4, 128, generator=g) * 3).to(dtype).to(device)
    k = (torch.randn(sum(lens), 4, 128, generator=g) * 3).to(dtype).to(device)
    v = torch.randn(sum(lens), 4, 128, generator=g).to(dtype).to(device)
    c = cu(lens, device)
    out, lse = flash_attn_varlen_func(q, k, v, c, c, max(lens), max(lens), causal=True, softcap=cap,
                                      window_size=(1024, 0) if cap == 50.0 else (-1, -1),
                                      return_softmax_lse=True)
    ref, refl = reference(q, k, v, c, c, causal=True, softcap=cap,
                          window=(1024, 0) if cap == 50.0 else (-1, -1))
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


def test_dynamic_causal_and_descales_on_tensor_core_path(device):
    from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
    qlens, klens = [5, 300, 257], [400, 300, 600]
    g = torch.Generator().manual_seed(13)
    q = torch.randn(sum(qlens), 8, 128, generator=g).to(torch.float16).to(device)
    k = torch.randn(sum(klens), 4, 128, generator=g).to(torch.float16).to(device)
    v = torch.randn(sum(klens), 4, 128, generator=g).to(torch.float16).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    dyn = torch.tensor([True, False, True], device=device)
    qs = torch.tensor([[.5], [.75], [1.]], device=device).expand(3, 4)
    ks = torch.tensor([[.4, .6, 1.1, .9]], device=device).expand(3, 4)
    vs = torch.tensor([[.2, .9, 1., 1.5]], device=device).expand(3, 4)
    out, lse = vllm_attention(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=True,
                              dynamic_causal=dyn, q_descale=qs, k_descale=ks, v_descale=vs,
                              return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=dyn, q_descale=qs, k_descale=ks, v_descale=vs)
    assert_attention_close(out, ref)
    assert_lse_close(lse, refl)


def _paged_kv(device, dtype, klens, page, hk, seed, columns_extra=1):
    """K/V in a paged cache [pages, page, hk, 128] with NaN-poisoned slots past
    each sequence and -1 table entries for pages wholly past it."""
    g = torch.Generator().manual_seed(seed)
    B = len(klens)
    columns = max((n + page - 1) // page for n in klens) + columns_extra
    n_pages = B * columns + 1
    table = torch.randperm(n_pages, generator=g)[:B * columns].int().reshape(B, columns)
    raw = [torch.randn(n_pages, page, hk, 128, generator=g) for _ in range(2)]
    for b, n in enumerate(klens):
        for col in range(columns):
            lo = col * page
            for pos in range(max(lo, n), lo + page):
                for r in raw:
                    r[int(table[b, col]), pos - lo] = float("nan")
            if lo >= n:
                table[b, col] = -1
    k, v = (r.to(dtype).to(device) for r in raw)
    return k, v, table.to(device)


@pytest.mark.parametrize("page", [16, 64, 256])
@pytest.mark.parametrize("causal", [True, False])
def test_paged_prefill_chunks_over_cached_prefix(device, page, causal):
    # Chunked prefill: new query tokens attend over a paged cache holding the
    # prefix plus themselves (q_len <= k_len, lower-right causal).
    from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
    qlens, klens = [1, 130, 300, 64], [700, 130, 1025, 2000]
    k, v, table = _paged_kv(device, torch.bfloat16, klens, page, 4, seed=page)
    g = torch.Generator().manual_seed(31)
    q = torch.randn(sum(qlens), 16, 128, generator=g).to(torch.bfloat16).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    out, lse = vllm_attention(q, k, v, max(qlens), cq, max(klens), seqused_k=used, block_table=table,
                              causal=causal, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, used_k=used, block_table=table, causal=causal)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_paged_prefill_features(device, dtype):
    from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
    qlens, klens = [200, 513, 33], [200, 900, 400]
    k, v, table = _paged_kv(device, dtype, klens, 32, 2, seed=8)
    g = torch.Generator().manual_seed(32)
    q = (torch.randn(sum(qlens), 8, 128, generator=g) * 2).to(dtype).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    sinks = torch.linspace(-1, 1, 8, device=device)
    kd = torch.tensor([[.5, 1.25]], device=device).expand(3, 2)
    vd = torch.tensor([[2., .75]], device=device).expand(3, 2)
    out, lse = vllm_attention(q, k, v, max(qlens), cq, max(klens), seqused_k=used, block_table=table,
                              causal=True, window_size=[255, 0], softcap=20.0, s_aux=sinks,
                              k_descale=kd, v_descale=vd, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, used_k=used, block_table=table, causal=True, window=(255, 0),
                          softcap=20.0, sinks=sinks, k_descale=kd, v_descale=vd)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("causal", [True, False])
def test_head_dim_64_on_tensor_core_path(device, dtype, causal):
    qlens, klens = [1, 127, 128, 129, 700, 5], [1, 127, 300, 129, 1000, 64]
    g = torch.Generator().manual_seed(41)
    q = torch.randn(sum(qlens), 8, 64, generator=g).to(dtype).to(device)
    k = torch.randn(sum(klens), 2, 64, generator=g).to(dtype).to(device)
    v = torch.randn(sum(klens), 2, 64, generator=g).to(dtype).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    out, lse = flash_attn_varlen_func(q, k, v, cq, ck, max(qlens), max(klens), causal=causal,
                                      return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=causal)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


def test_head_dim_64_paged_softcap_window_sinks(device):
    from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
    qlens, klens = [64, 400], [300, 1100]
    g = torch.Generator().manual_seed(42)
    columns = 1100 // 16 + 2
    table = torch.randperm(2 * columns, generator=g)[:2 * columns].int().reshape(2, columns).to(device)
    k = torch.randn(2 * columns, 16, 4, 64, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn_like(k)
    q = (torch.randn(sum(qlens), 16, 64, generator=g) * 2).to(torch.bfloat16).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    sinks = torch.linspace(-1, 1, 16, device=device)
    out, lse = vllm_attention(q, k, v, max(qlens), cq, max(klens), seqused_k=used, block_table=table,
                              causal=True, window_size=[200, 0], softcap=10.0, s_aux=sinks,
                              return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, used_k=used, block_table=table, causal=True, window=(200, 0),
                          softcap=10.0, sinks=sinks)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)
