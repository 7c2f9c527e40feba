"""Head dims other than 64/128 on the tcgen05 prefill (zero-padded through the
tensor maps' true extent): 32, 48, 80, 96 and 112 against the oracle, packed
and paged, plus FP8 E4M3 K/V through the dequant copy."""

import pytest
import torch

from flash_attn_b200 import flash_attn_varlen_func
from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dim", [32, 48, 80, 96, 112])
@pytest.mark.parametrize("causal", [True, False])
def test_varlen_prefill_head_dims(device, dim, causal):
    g = torch.Generator().manual_seed(101)
    qlens, klens = [130, 1, 300, 64], [200, 50, 300, 64]
    q = torch.randn(sum(qlens), 8, dim, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(sum(klens), 2, dim, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn(sum(klens), 2, dim, generator=g).to(torch.bfloat16).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    out, lse = flash_attn_varlen_func(q, k, v, cq, ck, max(qlens), max(klens), causal=causal,
                                      return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=causal)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("kv_fp8", [False, True])
@pytest.mark.parametrize("dim", [96, 80])
def test_paged_prefill_head_dims(device, kv_fp8, dim):
    g = torch.Generator().manual_seed(102)
    qlens, klens, page = [200, 129], [600, 129], 16
    cols = max(klens) // page + 1
    kv_dtype = torch.float8_e4m3fn if kv_fp8 else torch.bfloat16
    kc = torch.randn(2 * cols, page, 2, dim, generator=g).to(kv_dtype).to(device)
    vc = torch.randn(2 * cols, page, 2, dim, generator=g).to(kv_dtype).to(device)
    table = torch.randperm(2 * cols, generator=g).int().reshape(2, cols).to(device)
    q = torch.randn(sum(qlens), 8, dim, generator=g).to(torch.bfloat16).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    sinks = torch.linspace(-1, 1, 8, device=device)
    out, lse = vllm_attention(q, kc, vc, max(qlens), cq, max(klens), seqused_k=used, block_table=table,
                              causal=True, window_size=[256, 0], s_aux=sinks, return_softmax_lse=True)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, causal=True, window=(256, 0),
                          sinks=sinks)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)
