"""Paged decode for head dims other than 64/128 on the tensor-core decode
kernel (Q tail and K/V columns past the true dim read as zero): bf16 through
the TMA gather (page 16), the cp.async gather (page 48) and packed K/V, FP8
E4M3 with descales up to head dim 256 (8- and 16-head tiles, bf16 and f16
queries, sinks, softcap, windows, fp32 outputs), automatic and explicit split
counts, against the oracle."""

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


def _poisoned_fp8_cache(g, device, lens, page, hk, dim):
    # Pages in use by the sequences come from a permutation; every table entry
    # past a sequence points at one page of NaN codes.
    cols = max(lens) // page + 1
    n = len(lens) * cols
    raw = torch.randn(n + 1, page, hk, 2 * dim, generator=g)
    raw[n] = float("nan")
    packed = raw.to(torch.float8_e4m3fn).to(device)
    kc, vc = packed.split(dim, dim=-1)
    table = torch.randperm(n, generator=g).int().reshape(len(lens), cols)
    for b, length in enumerate(lens):
        table[b, (length + page - 1) // page:] = n
    return kc, vc, table.to(device)


@pytest.mark.parametrize("dim", [256, 144])
@pytest.mark.parametrize("group", [4, 16])
@pytest.mark.parametrize("page", [16, 48])
@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float16])
def test_fp8_paged_decode_wide_head_dims(device, dim, group, page, qdtype):
    # FP8 E4M3 K/V at head dims 129..256 on the 256-wide instantiation: GQA
    # groups of 4 (8-head tiles) and 16 (16-head tiles), TMA page gathers
    # (page 16) and cp.async gathers (page 48), bf16 queries (scale folded into
    # f16 fragments) and f16 queries, descales, sinks and a softcap.
    g = torch.Generator().manual_seed(114 + dim + group)
    lens = [5, 1500, 3000]
    hk = 2
    kc, vc, table = _poisoned_fp8_cache(g, device, lens, page, hk, dim)
    q = torch.randn(len(lens), hk * group, dim, generator=g).to(qdtype).to(device)
    cq = torch.arange(len(lens) + 1, dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    kd = torch.tensor([[.5, 1.5]], device=device).expand(3, 2)
    vd = torch.tensor([[2., .25]], device=device).expand(3, 2)
    sinks = torch.linspace(-2, 2, hk * group, device=device)
    out, lse = decode_attention(q, kc, vc, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=max(lens),
                                block_table=table, k_descale=kd, v_descale=vd, s_aux=sinks, softcap=5.0)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, k_descale=kd, v_descale=vd,
                          sinks=sinks, softcap=5.0)
    assert torch.isfinite(out).all()
    assert_attention_close(out, ref, qdtype)
    assert_lse_close(lse, refl, atol=1e-3)


@pytest.mark.parametrize("splits", [1, 5])
@pytest.mark.parametrize("window", [(-1, -1), (300, 0)])
def test_fp8_decode_head_dim_256_fp32_out_splits_window(device, splits, window):
    # fp32 output (the multi-GPU partial's precision path), explicit split
    # counts and a sliding window at head dim 256 over FP8 K/V.
    g = torch.Generator().manual_seed(115)
    lens = [700, 2500]
    kc, vc, table = _poisoned_fp8_cache(g, device, lens, 16, 2, 256)
    q = torch.randn(len(lens), 16, 256, generator=g).to(torch.float16).to(device)
    cq = torch.arange(len(lens) + 1, dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    kd = torch.full((2, 2), .75, device=device)
    vd = torch.full((2, 2), 1.25, device=device)
    out = torch.empty(len(lens), 16, 256, device=device, dtype=torch.float32)
    res, lse = decode_attention(q, kc, vc, cu_seqlens_q=cq, seqused_k=used, max_seqlen_k=max(lens),
                                block_table=table, k_descale=kd, v_descale=vd, num_splits=splits,
                                window_size=window, out=out)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, k_descale=kd, v_descale=vd,
                          window=window)
    assert res.data_ptr() == out.data_ptr()
    torch.testing.assert_close(res.cpu().double(), ref, atol=2e-5, rtol=2e-4)
    assert_lse_close(lse, refl, atol=1e-4)
