"""The mma.sync tensor-core kernel: f16/bf16 cases outside the tcgen05 prefill
and the paged-decode kernel (FP8 K/V in prefill, head dims 96/256, DiffKV
192->128, ALiBi, leftpad, explicit splits) against the oracle."""

import pytest
import torch

from flash_attn_b200 import flash_attn_varlen_func
from flash_attn_b200._decode import decode_attention
from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


def _qkv(device, dtype, qlens, klens, hq, hk, dq, dv, kv_dtype=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sum(qlens), hq, dq, generator=g).to(dtype).to(device)
    kv_dtype = kv_dtype or dtype
    k = torch.randn(sum(klens), hk, dq, generator=g).to(kv_dtype).to(device)
    v = torch.randn(sum(klens), hk, dv, generator=g).to(kv_dtype).to(device)
    return q, k, v


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("causal", [True, False])
def test_fp8_kv_prefill_with_descales(device, dtype, causal):
    qlens, klens = [1, 100, 300, 64], [130, 100, 700, 64]
    q, k, v = _qkv(device, dtype, qlens, klens, 8, 2, 128, 128, torch.float8_e4m3fn, seed=1)
    cq, ck = cu(qlens, device), cu(klens, device)
    kd = torch.tensor([[.5, 1.5]], device=device).expand(4, 2)
    vd = torch.tensor([[2., .25]], device=device).expand(4, 2)
    out, lse = vllm_attention(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=causal,
                              k_descale=kd, v_descale=vd, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=causal, k_descale=kd, v_descale=vd)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


def test_fp8_paged_prefill(device):
    qlens, klens, page = [64, 257], [300, 1000], 16
    g = torch.Generator().manual_seed(2)
    cols = max(klens) // page + 1
    raw = torch.randn(2 * cols, page, 4, 256, generator=g)
    packed = raw.to(torch.float8_e4m3fn).to(device)
    k, v = packed.split(128, dim=-1)
    table = torch.randperm(2 * cols, generator=g).int().reshape(2, cols).to(device)
    q = torch.randn(sum(qlens), 16, 128, generator=g).to(torch.bfloat16).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    out, lse = vllm_attention(q, k, v, max(qlens), cq, max(klens), seqused_k=used, block_table=table,
                              causal=True, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, used_k=used, block_table=table, causal=True)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("dims", [(96, 96), (256, 256), (192, 128), (64, 64)])
@pytest.mark.parametrize("causal", [True, False])
def test_head_dims_and_diffkv(device, dims, causal):
    qlens, klens = [1, 65, 200], [40, 65, 333]
    q, k, v = _qkv(device, torch.bfloat16, qlens, klens, 8, 4, dims[0], dims[1], seed=3)
    cq, ck = cu(qlens, device), cu(klens, device)
    # Head dim 64 with ALiBi (taken by the tcgen05 kernel since it gained ALiBi).
    slopes = torch.linspace(.01, .1, 8, device=device) if dims == (64, 64) else None
    out, lse = flash_attn_varlen_func(q, k, v, cq, ck, max(qlens), max(klens), causal=causal,
                                      alibi_slopes=slopes, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=causal, alibi=slopes)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_alibi_softcap_window_sinks(device, dtype):
    qlens, klens = [5, 129, 400], [5, 300, 400]
    q, k, v = _qkv(device, dtype, qlens, klens, 8, 2, 128, 128, seed=4)
    q = q * 2
    cq, ck = cu(qlens, device), cu(klens, device)
    slopes = torch.linspace(.02, .3, 8, device=device)
    sinks = torch.linspace(-1, 1, 8, device=device)
    out, lse = vllm_attention(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=True,
                              window_size=[100, 0], softcap=3.0, alibi_slopes=slopes, s_aux=sinks,
                              return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=True, window=(100, 0), softcap=3.0, alibi=slopes,
                          sinks=sinks)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


def test_leftpad_prefill_over_cache(device):
    from flash_attn_b200 import flash_attn_with_kvcache
    g = torch.Generator().manual_seed(5)
    B, S, H, HK, D, cap = 3, 40, 8, 2, 128, 512
    kc = torch.randn(B, cap, HK, D, generator=g).to(torch.bfloat16).to(device)
    vc = torch.randn_like(kc)
    q = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(device)
    lens = torch.tensor([100, 300, 512], dtype=torch.int32, device=device)
    left = torch.tensor([0, 17, 200], dtype=torch.int32, device=device)
    out = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=lens, cache_leftpad=left, causal=True)
    for b in range(B):
        n, lp = int(lens[b]), int(left[b])
        kk, vv = kc[b, lp:n], vc[b, lp:n]
        ref, _ = reference(q[b], kk, vv, torch.tensor([0, S], dtype=torch.int32),
                           torch.tensor([0, n - lp], dtype=torch.int32), causal=True)
        assert_attention_close(out[b], ref, torch.bfloat16)


@pytest.mark.parametrize("splits", [0, 1, 5])
def test_head_dim_256_decode_splits(device, splits):
    g = torch.Generator().manual_seed(6)
    B, H, HK, D, page = 3, 8, 2, 256, 16
    lens = [17, 700, 1500]
    cols = max(lens) // page + 1
    kc = torch.randn(B * cols, page, HK, D, generator=g).to(torch.bfloat16).to(device)
    vc = torch.randn_like(kc)
    table = torch.randperm(B * cols, generator=g).int().reshape(B, cols).to(device)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16).to(device)
    cq = torch.arange(B + 1, dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    out, lse = decode_attention(q, kc, vc, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=max(lens),
                                block_table=table, num_splits=splits)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)
