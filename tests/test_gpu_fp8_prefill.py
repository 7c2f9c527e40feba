"""Prefill over FP8 E4M3 K/V on the tcgen05 kernel (exact 16-bit copy of the
K/V rows first) against the oracle: packed and paged caches, bf16/f16 queries,
head dims 64 and 128, descales, softcap + window, sinks. Calls whose longest
query chunk is below one 128-row tile stay on the mma.sync kernel; the launch
counter tells the two routes apart (dequant + prefill = 2 launches)."""

import pytest
import torch

from flash_attn_b200 import _capi
from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


def _paged(rows_per_seq, page, g, device, heads, dim, pages_extra=3):
    counts = [int(r.shape[0]) for r in rows_per_seq]
    cols = max((c + page - 1) // page for c in counts) + 1
    n_pages = len(counts) * cols + pages_extra
    cache = torch.zeros(n_pages, page, heads, dim, dtype=torch.float8_e4m3fn)
    perm = torch.randperm(n_pages, generator=g)[:len(counts) * cols].int().reshape(len(counts), cols)
    for b, r in enumerate(rows_per_seq):
        for i in range(r.shape[0]):
            cache[perm[b, i // page], i % page] = r[i]
    return cache.to(device), perm.to(device)


def _launches(fn):
    before = _capi.kernel_launches()
    result = fn()
    return result, _capi.kernel_launches() - before


@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dim", [128, 64])
@pytest.mark.parametrize("causal", [True, False])
def test_packed_fp8_prefill_on_tensor_cores(device, qdtype, dim, causal):
    g = torch.Generator().manual_seed(81)
    qlens, klens = [200, 1, 640, 129], [330, 40, 640, 129]
    q = torch.randn(sum(qlens), 8, dim, generator=g).to(qdtype).to(device)
    k = (torch.randn(sum(klens), 2, dim, generator=g) * 2).to(torch.float8_e4m3fn).to(device)
    v = (torch.randn(sum(klens), 2, dim, generator=g) * 2).to(torch.float8_e4m3fn).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    kd = torch.tensor([[.5, 1.5]], device=device).expand(4, 2)
    vd = torch.tensor([[2., .25]], device=device).expand(4, 2)
    (out, lse), n = _launches(lambda: vllm_attention(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck,
                                                      causal=causal, k_descale=kd, v_descale=vd,
                                                      return_softmax_lse=True))
    assert n == 2, "expected the dequant + tcgen05 prefill route"
    ref, refl = reference(q, k, v, cq, ck, causal=causal, k_descale=kd, v_descale=vd)
    assert_attention_close(out, ref, qdtype)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("page", [16, 32])
def test_paged_fp8_prefill_with_softcap_window_sinks(device, page):
    g = torch.Generator().manual_seed(82)
    qlens, klens = [150, 300, 7], [900, 300, 1000]
    keys = [(torch.randn(n, 4, 128, generator=g) * 3).to(torch.float8_e4m3fn) for n in klens]
    vals = [(torch.randn(n, 4, 128, generator=g) * 3).to(torch.float8_e4m3fn) for n in klens]
    kc, table = _paged(keys, page, g, device, 4, 128)
    vc = torch.zeros_like(kc)
    vcpu = vc.cpu()
    for b, r in enumerate(vals):
        for i in range(r.shape[0]):
            vcpu[table[b, i // page].item(), i % page] = r[i]
    vc = vcpu.to(device)
    q = torch.randn(sum(qlens), 16, 128, generator=g).to(torch.bfloat16).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    sinks = torch.linspace(-1, 1, 16, device=device)
    kd = torch.full((3, 4), 0.25, device=device)
    (out, lse), n = _launches(lambda: vllm_attention(
        q, kc, vc, max(qlens), cq, max(klens), seqused_k=used, block_table=table, causal=True,
        window_size=[400, 0], softcap=20.0, s_aux=sinks, k_descale=kd, return_softmax_lse=True))
    assert n == 2
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, causal=True, window=(400, 0),
                          softcap=20.0, sinks=sinks, k_descale=kd)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_short_query_chunks_stay_on_mma_kernel(device):
    g = torch.Generator().manual_seed(83)
    qlens, klens = [64, 100, 3], [500, 100, 80]
    q = torch.randn(sum(qlens), 8, 128, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(sum(klens), 2, 128, generator=g).to(torch.float8_e4m3fn).to(device)
    v = torch.randn(sum(klens), 2, 128, generator=g).to(torch.float8_e4m3fn).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    (out, lse), n = _launches(lambda: vllm_attention(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck,
                                                      causal=True, return_softmax_lse=True))
    assert n == 1, "expected the mma.sync kernel (one launch, no split merge)"
    ref, refl = reference(q, k, v, cq, ck, causal=True)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_page_outside_cache_reads_as_zeros(device):
    g = torch.Generator().manual_seed(84)
    page, klen = 16, 256
    k = (torch.randn(klen, 2, 128, generator=g)).to(torch.float8_e4m3fn)
    v = (torch.randn(klen, 2, 128, generator=g)).to(torch.float8_e4m3fn)
    kc, table = _paged([k], page, g, device, 2, 128)
    vc = torch.zeros_like(kc).cpu()
    for i in range(klen):
        vc[table[0, i // page].item(), i % page] = v[i]
    vc = vc.to(device)
    bad = table.clone()
    bad[0, 3] = -1  # tokens 48..63 come from no page
    q = torch.randn(200, 8, 128, generator=g).to(torch.bfloat16).to(device)
    cq = cu([200], device)
    used = torch.tensor([klen], dtype=torch.int32, device=device)
    out, lse = vllm_attention(q, kc, vc, 200, cq, klen, seqused_k=used, block_table=bad, causal=True,
                              return_softmax_lse=True)
    # Expected: the same cache with those 16 tokens zeroed (score 0, value 0).
    kz, vz = kc.clone(), vc.clone()
    kz.view(torch.uint8)[table[0, 3]] = 0  # E4M3 code 0x00 = +0
    vz.view(torch.uint8)[table[0, 3]] = 0
    ref, refl = reference(q, kz, vz, cq, used_k=used, block_table=table, causal=True)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_oversized_copy_falls_back_to_mma(device):
    # max_seqlen_k bounds the paged copy (B * max_k rows): past the copy-size
    # cap the call stays on the mma.sync kernel, which reads the FP8 bytes.
    g = torch.Generator().manual_seed(85)
    page, klens = 16, [100, 37]
    keys = [torch.randn(n, 2, 128, generator=g).to(torch.float8_e4m3fn) for n in klens]
    vals = [torch.randn(n, 2, 128, generator=g).to(torch.float8_e4m3fn) for n in klens]
    kc, table = _paged(keys, page, g, device, 2, 128)
    vc = torch.zeros_like(kc).cpu()
    for b, r in enumerate(vals):
        for i in range(r.shape[0]):
            vc[table[b, i // page].item(), i % page] = r[i]
    vc = vc.to(device)
    q = torch.randn(300, 8, 128, generator=g).to(torch.bfloat16).to(device)
    cq = cu([150, 150], device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    (out, lse), n = _launches(lambda: vllm_attention(q, kc, vc, 150, cq, 1 << 26, seqused_k=used, block_table=table,
                                                      causal=True, return_softmax_lse=True))
    assert n == 1, "expected the mma.sync kernel past the copy-size cap"
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, causal=True)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)
