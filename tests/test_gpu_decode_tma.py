"""Paged decode through the TMA page-gather pipeline vs the oracle.

Paged K/V with power-of-two pages of at least 8 tokens reach the decode kernel
whose producer warp loads whole pages (or page slices) as TMA boxes into a
swizzled shared-memory ring. These cases cover page sizes below, equal to and
above the kernel's token tile (64 tokens for bf16/f16, 128 for FP8), tiles that
start before the visible range (leftpad, sliding windows, splits), unused
block-table columns set to -1, NaN-poisoned slots outside the visible range,
and a cache whose token and head strides are permuted.
"""

import pytest
import torch

from flash_attn_b200._decode import decode_attention
from flash_attn_b200._capi import library
from helpers import assert_attention_close, assert_lse_close, reference

pytestmark = pytest.mark.gpu


def _paged_case(device, page, kv_dtype, lengths, pads, kvh=2, d=128, permuted=False, seed=0):
    """K/V caches [pages, page, kv_heads, d] (a permuted view if asked) and a block table.

    Slots outside each request's [pad, pad + length) are NaN; table columns that
    lie wholly past the request are -1.
    """
    g = torch.Generator().manual_seed(seed)
    B = len(lengths)
    columns = max((p + n + page - 1) // page for p, n in zip(pads, lengths)) + 1
    n_pages = B * columns + 2
    table = torch.randperm(n_pages, generator=g)[:B * columns].int().reshape(B, columns)
    shape = (n_pages, kvh, page, d) if permuted else (n_pages, page, kvh, d)
    raw = [torch.randn(shape, generator=g) for _ in range(2)]
    views = [r.transpose(1, 2) if permuted else r for r in raw]
    for b, (n, p) in enumerate(zip(lengths, pads)):
        for col in range(columns):
            lo, hi = col * page, (col + 1) * page
            physical = int(table[b, col])
            for pos in range(lo, hi):
                if pos < p or pos >= p + n:
                    for view in views:
                        view[physical, pos - lo] = float("nan")
            if lo >= p + n:
                table[b, col] = -1
    k, v = (r.to(kv_dtype).to(device) for r in raw)
    if permuted:
        k, v = k.transpose(1, 2), v.transpose(1, 2)
    return k, v, table.to(device)


@pytest.mark.parametrize("page", [8, 32, 64, 128, 256])
@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_decode_tma_page_sizes_leftpad_and_poison(device, page, kv):
    lengths, pads = [1, 200, 777, 1500], [0, 5, 300, 17]
    kv_dtype = torch.bfloat16 if kv == "bf16" else torch.float8_e4m3fn
    k, v, table = _paged_case(device, page, kv_dtype, lengths, pads, seed=page)
    q = torch.randn(4, 8, 128, device=device).to(torch.bfloat16)
    cq = torch.arange(5, device=device, dtype=torch.int32)
    used = torch.tensor(lengths, device=device, dtype=torch.int32)
    left = torch.tensor(pads, device=device, dtype=torch.int32)
    kws = {}
    if kv == "fp8":
        kws = dict(k_descale=torch.tensor([[.5, .75]], device=device).expand(4, 2),
                   v_descale=torch.tensor([[1.25, .5]], device=device).expand(4, 2))
    expected, el = reference(q, k, v, cq, used_k=used, block_table=table, leftpad=pads, **kws)
    for splits in (0, 3):
        for out_dtype in (torch.bfloat16, torch.float32):
            out = torch.empty(4, 8, 128, device=device, dtype=out_dtype)
            actual, lse = decode_attention(q, k, v, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=1500,
                                           block_table=table, leftpad_k=left, num_splits=splits, out=out,
                                           **kws)
            if out_dtype == torch.float32 and kv == "bf16":
                torch.testing.assert_close(actual.cpu().double(), expected, atol=2e-5, rtol=2e-4)
            else:
                assert_attention_close(actual, expected, torch.bfloat16)
            assert_lse_close(lse, el, atol=1e-3 if kv == "fp8" else 1e-4)
    assert library().fa_pipeline_timeouts(1) == 0


@pytest.mark.parametrize("window", [(100, 0), (0, 0), (1023, -1)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_tma_windows_sinks_softcap(device, window, dtype):
    lengths, pads = [64, 65, 1000, 3000], [3, 0, 64, 1]
    k, v, table = _paged_case(device, 16, dtype, lengths, pads, kvh=4, seed=7)
    q = torch.randn(4, 16, 128, device=device).to(dtype)
    cq = torch.arange(5, device=device, dtype=torch.int32)
    used = torch.tensor(lengths, device=device, dtype=torch.int32)
    left = torch.tensor(pads, device=device, dtype=torch.int32)
    sinks = torch.linspace(-2, 2, 16, device=device)
    expected, el = reference(q, k, v, cq, used_k=used, block_table=table, leftpad=pads, window=window,
                             sinks=sinks, softcap=.9)
    for splits in (0, 1, 5):
        actual, lse = decode_attention(q, k, v, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=3000,
                                       block_table=table, leftpad_k=left, num_splits=splits,
                                       window_size=window, s_aux=sinks, softcap=.9)
        assert_attention_close(actual, expected, dtype)
        assert_lse_close(lse, el, atol=1e-4)


@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_decode_tma_permuted_cache_strides(device, kv):
    # Cache stored [pages, kv_heads, page, d] and viewed as [pages, page, kv_heads, d].
    kv_dtype = torch.bfloat16 if kv == "bf16" else torch.float8_e4m3fn
    lengths, pads = [500, 31, 129], [0, 1, 32]
    k, v, table = _paged_case(device, 32, kv_dtype, lengths, pads, kvh=4, permuted=True, seed=3)
    assert k.stride(1) == 128 and k.stride(2) == 32 * 128
    q = torch.randn(3, 32, 128, device=device).to(torch.bfloat16)
    cq = torch.arange(4, device=device, dtype=torch.int32)
    used = torch.tensor(lengths, device=device, dtype=torch.int32)
    left = torch.tensor(pads, device=device, dtype=torch.int32)
    expected, el = reference(q, k, v, cq, used_k=used, block_table=table, leftpad=pads)
    actual, lse = decode_attention(q, k, v, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=500,
                                   block_table=table, leftpad_k=left)
    assert_attention_close(actual, expected, torch.bfloat16)
    assert_lse_close(lse, el, atol=1e-3 if kv == "fp8" else 1e-4)


def test_decode_tma_head_dim_64(device):
    lengths, pads = [10, 300, 2049], [0, 9, 0]
    k, v, table = _paged_case(device, 64, torch.float16, lengths, pads, kvh=1, d=64, seed=5)
    q = torch.randn(3, 8, 64, device=device).to(torch.float16)
    cq = torch.arange(4, device=device, dtype=torch.int32)
    used = torch.tensor(lengths, device=device, dtype=torch.int32)
    left = torch.tensor(pads, device=device, dtype=torch.int32)
    expected, el = reference(q, k, v, cq, used_k=used, block_table=table, leftpad=pads)
    for splits in (0, 2, 7):
        actual, lse = decode_attention(q, k, v, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=2049,
                                       block_table=table, leftpad_k=left, num_splits=splits)
        assert_attention_close(actual, expected)
        assert_lse_close(lse, el, atol=1e-4)
