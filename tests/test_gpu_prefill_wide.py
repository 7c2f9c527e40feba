"""Prefill with head dims above 128 on the one-tile tcgen05 kernel.

The reference's fast path covers head dim 256 (flash_attn_mps/_attention.py:
149-158) and its generic kernels any dq != dv (DiffKV); here QK head dims
129..256 with V head dims up to 256 run on prefill_wide_sm100.cu. Every case
is checked against the float64 oracle (reference tests/reference.py:6-90)
with the reference's tolerances (max-abs 1e-2 on 16-bit outputs, LSE 1e-3):
several key tiles, causal and not, q_len != k_len, GQA, windows, softcap,
sinks, descales, padded dims, FP8 K/V (exact 16-bit copy in front of the
kernel), paged caches (pages of 16..256 tokens through a permuted block table)
and the batch-invariant mode.
"""

import pytest
import torch

from flash_attn_b200 import flash_attn_varlen_func
from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_varlen
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


def _qkv(device, dtype, qlens, klens, hq, hk, dq, dv, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sum(qlens), hq, dq, generator=g)
    k = torch.randn(sum(klens), hk, dq, generator=g)
    v = torch.randn(sum(klens), hk, dv, generator=g)
    return q.to(dtype).to(device), k.to(dtype).to(device), v.to(dtype).to(device)


@pytest.mark.parametrize("dims", [(256, 256), (192, 128), (256, 128), (160, 160), (200, 96)])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_wide_head_dims_against_oracle(device, dims, causal, dtype):
    dq, dv = dims
    qlens, klens = [1, 129, 300, 513], [1, 129, 420, 513]
    q, k, v = _qkv(device, dtype, qlens, klens, 8, 2, dq, dv, seed=dq + dv)
    cq, ck = cu(qlens, device), cu(klens, device)
    out, lse = flash_attn_varlen_func(q, k, v, cq, ck, max(qlens), max(klens), causal=causal,
                                      return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=causal)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("dims", [(256, 256), (192, 128)])
def test_wide_softcap_window_sinks_descales(device, dims):
    dq, dv = dims
    qlens, klens = [77, 260, 640], [300, 260, 900]
    q, k, v = _qkv(device, torch.bfloat16, qlens, klens, 8, 4, dq, dv, seed=11)
    q = q * 2
    cq, ck = cu(qlens, device), cu(klens, device)
    sinks = torch.linspace(-1, 1, 8, device=device)
    g = torch.Generator().manual_seed(12)
    qd = (0.5 + torch.rand(3, 4, generator=g)).to(device)
    kd = (0.5 + torch.rand(3, 4, generator=g)).to(device)
    vd = (0.5 + torch.rand(3, 4, generator=g)).to(device)
    out, lse = vllm_varlen(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=True,
                           window_size=[200, 0], softcap=30.0, s_aux=sinks, q_descale=qd, k_descale=kd,
                           v_descale=vd, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=True, window=(200, 0), softcap=30.0, sinks=sinks,
                          q_descale=qd, k_descale=kd, v_descale=vd)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_wide_dynamic_causal_and_seqused(device):
    qlens, klens = [130, 5, 256], [400, 300, 256]
    q, k, v = _qkv(device, torch.bfloat16, qlens, klens, 4, 1, 256, 256, seed=13)
    cq = cu(qlens, device)
    ck = cu(klens, device)
    flags = torch.tensor([True, False, True], device=device)
    out, lse = vllm_varlen(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=True,
                           dynamic_causal=flags, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=flags)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_wide_fp8_kv_through_the_exact_copy(device):
    # FP8 E4M3 K/V with per-(request, KV head) descales and a full 128-row
    # query tile: the K/V rows are decoded exactly to bf16 and the one-tile
    # kernel runs on the copy.
    qlens, klens = [256, 300], [400, 300]
    q, k, v = _qkv(device, torch.bfloat16, qlens, klens, 8, 2, 256, 256, seed=14)
    k8, v8 = (k * 8).to(torch.float8_e4m3fn), (v * 8).to(torch.float8_e4m3fn)
    kd = torch.full((2, 2), 1 / 8, device=device)
    vd = torch.full((2, 2), 1 / 8, device=device)
    cq, ck = cu(qlens, device), cu(klens, device)
    out, lse = vllm_varlen(q, k8, v8, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=True,
                           k_descale=kd, v_descale=vd, return_softmax_lse=True)
    ref, refl = reference(q, k8, v8, cq, ck, causal=True, k_descale=kd, v_descale=vd)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_wide_batch_invariant_mode_is_bitwise_stable(device):
    # num_splits == 1 (vLLM's batch-invariant mode): a request's rows reduce
    # their keys in one fixed order whatever else is in the batch.
    qlens, klens = [200, 70, 333], [260, 70, 500]
    q, k, v = _qkv(device, torch.bfloat16, qlens, klens, 8, 2, 256, 256, seed=15)
    cq, ck = cu(qlens, device), cu(klens, device)
    full = vllm_varlen(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=True, num_splits=1)
    q2 = q[qlens[0]:qlens[0] + qlens[1]]
    k2 = k[klens[0]:klens[0] + klens[1]]
    v2 = v[klens[0]:klens[0] + klens[1]]
    alone = vllm_varlen(q2, k2, v2, qlens[1], cu([qlens[1]], device), klens[1],
                        cu_seqlens_k=cu([klens[1]], device), causal=True, num_splits=1)
    assert torch.equal(full[qlens[0]:qlens[0] + qlens[1]], alone)
    ref, _ = reference(q, k, v, cq, ck, causal=True)
    assert_attention_close(full, ref, torch.bfloat16)


@pytest.mark.parametrize("page", [16, 32, 64, 256])
@pytest.mark.parametrize("dims", [(256, 256), (192, 128)])
def test_wide_paged_cache_against_oracle(device, page, dims):
    # vLLM prefill over a paged cache (permuted pages, K and V as views of one
    # packed allocation): page boxes gathered through the block table, pages
    # past each sequence zero-filled, NaN in the unused tail slots.
    dq, dv = dims
    g = torch.Generator().manual_seed(16 + page)
    qlens, klens = [150, 64, 1], [700, 300, 129]
    cols = max(klens) // page + 1
    packed = torch.randn(3 * cols, page, 2, dq + dv, generator=g).to(torch.bfloat16).to(device)
    kc, vc = packed.split([dq, dv], dim=-1)
    table = torch.randperm(3 * cols, generator=g).int().reshape(3, cols).to(device)
    for b, n in enumerate(klens):
        last = table[b, n // page].item()
        packed[last, n % page:] = float("nan")
    q = torch.randn(sum(qlens), 8, dq, generator=g).to(torch.bfloat16).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    out, lse = vllm_varlen(q, kc, vc, max(qlens), cq, max(klens), seqused_k=used, block_table=table,
                           causal=True, return_softmax_lse=True)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, causal=True)
    assert torch.isfinite(out).all()
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_wide_paged_softcap_window_sinks(device):
    g = torch.Generator().manual_seed(17)
    qlens, klens, page = [200, 77], [520, 900], 16
    cols = max(klens) // page + 1
    kc = torch.randn(2 * cols, page, 4, 256, generator=g).to(torch.float16).to(device)
    vc = torch.randn(2 * cols, page, 4, 256, generator=g).to(torch.float16).to(device)
    table = torch.randperm(2 * cols, generator=g).int().reshape(2, cols).to(device)
    q = (2 * torch.randn(sum(qlens), 8, 256, generator=g)).to(torch.float16).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    sinks = torch.linspace(-1, 1, 8, device=device)
    out, lse = vllm_varlen(q, kc, vc, max(qlens), cq, max(klens), seqused_k=used, block_table=table,
                           causal=True, window_size=[300, 0], softcap=30.0, s_aux=sinks, return_softmax_lse=True)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, causal=True, window=(300, 0),
                          softcap=30.0, sinks=sinks)
    assert_attention_close(out, ref, torch.float16)
    assert_lse_close(lse, refl)
