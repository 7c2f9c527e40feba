"""Paged decode for head dims other than 64/128 on the tensor-core decode
kernel (Q tail and K/V columns past the true dim read as zero): bf16 through
the TMA gather (page 16), the cp.async gather (page 48) and packed K/V, FP8
E4M3 with descales, automatic and explicit split counts, against the oracle."""

import pytest
import torch

from flash_attn_b200._decode import decode_attention
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


def _paged(g, device, lens, page, hk, dim, dtype):
    cols = max(lens) // page + 1
    kc = torch.randn(len(lens) * cols, page, hk, dim, generator=g).to(dtype).to(device)
    vc = torch.randn(len(lens) * cols, page, hk, dim, generator=g).to(dtype).to(device)
    table = torch.randperm(len(lens) * cols, generator=g).int().reshape(len(lens), cols).to(device)
    return kc, vc, table


@pytest.mark.parametrize("dim", [32, 48, 80, 96])
@pytest.mark.parametrize("page", [16, 48])
@pytest.mark.parametrize("splits", [0, 3])
def test_bf16_paged_decode_head_dims(device, dim, page, splits):
    g = torch.Generator().manual_seed(111)
    lens = [1, 700, 2000, 35]
    kc, vc, table = _paged(g, device, lens, page, 2, dim, torch.bfloat16)
    q = torch.randn(len(lens), 8, dim, generator=g).to(torch.bfloat16).to(device)
    cq = torch.arange(len(lens) + 1, dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    out, lse = decode_attention(q, kc, vc, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=max(lens),
                                block_table=table, num_splits=splits)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("dim", [48, 80, 96, 112])
def test_fp8_paged_decode_head_dims(device, dim):
    g = torch.Generator().manual_seed(112)
    lens = [5, 1500, 3000]
    kc, vc, table = _paged(g, device, lens, 16, 2, dim, torch.float8_e4m3fn)
    q = torch.randn(len(lens), 8, dim, generator=g).to(torch.bfloat16).to(device)
    cq = torch.arange(len(lens) + 1, dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    kd = torch.tensor([[.5, 1.5]], device=device).expand(3, 2)
    vd = torch.tensor([[2., .25]], device=device).expand(3, 2)
    out, lse = decode_attention(q, kc, vc, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=max(lens),
                                block_table=table, k_descale=kd, v_descale=vd)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, k_descale=kd, v_descale=vd)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl, atol=1e-3)


@pytest.mark.parametrize("dim", [80, 96])
def test_packed_decode_head_dims(device, dim):
    g = torch.Generator().manual_seed(113)
    klens = [300, 1, 900]
    k = torch.randn(sum(klens), 2, dim, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn(sum(klens), 2, dim, generator=g).to(torch.bfloat16).to(device)
    q = torch.randn(len(klens), 8, dim, generator=g).to(torch.bfloat16).to(device)
    cq = torch.arange(len(klens) + 1, dtype=torch.int32, device=device)
    ck = cu(klens, device)
    out, lse = decode_attention(q, k, v, cu_seqlens_q=cq, cu_seqlens_k=ck, max_seqlen_k=max(klens))
    ref, refl = reference(q, k, v, cq, ck)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)
