"""ALiBi prefill on the tcgen05 kernel against the oracle: scores minus
slope * |q_abs - key| (lower-right aligned), bf16/f16, head dims 64/128,
causal and not, per-head [H] and per-request [B, H] slopes, windows and sinks,
ALiBi together with a softcap (the capped score minus the bias, reference
kernels/attention.metal:47-51), a paged vLLM call over an FP8 E4M3 cache, and
single-query ALiBi decode (which keeps the split-KV kernels)."""

import pytest
import torch

from flash_attn_b200 import flash_attn_varlen_func
from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_attention
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dim", [128, 64])
@pytest.mark.parametrize("causal", [True, False])
def test_alibi_prefill(device, dtype, dim, causal):
    g = torch.Generator().manual_seed(91)
    qlens, klens = [300, 1, 129, 520], [300, 70, 400, 520]
    q = torch.randn(sum(qlens), 8, dim, generator=g).to(dtype).to(device)
    k = torch.randn(sum(klens), 2, dim, generator=g).to(dtype).to(device)
    v = torch.randn(sum(klens), 2, dim, generator=g).to(dtype).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    slopes = torch.tensor([2.0 ** (-(i + 1)) for i in range(8)], device=device)
    out, lse = flash_attn_varlen_func(q, k, v, cq, ck, max(qlens), max(klens), causal=causal,
                                      alibi_slopes=slopes, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=causal, alibi=slopes)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


def _kernel_names(fn):
    """Names of the CUDA kernels ``fn`` launches (empty if the profiler sees none)."""
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.key for e in prof.key_averages() if e.device_type == torch.autograd.DeviceType.CUDA}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dim", [128, 64])
@pytest.mark.parametrize("causal", [True, False])
def test_alibi_with_softcap_prefill(device, dtype, dim, causal):
    g = torch.Generator().manual_seed(95)
    qlens, klens = [300, 1, 129, 520], [300, 70, 400, 520]
    q = (3 * torch.randn(sum(qlens), 8, dim, generator=g)).to(dtype).to(device)
    k = torch.randn(sum(klens), 2, dim, generator=g).to(dtype).to(device)
    v = torch.randn(sum(klens), 2, dim, generator=g).to(dtype).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    slopes = torch.tensor([2.0 ** (-(i + 1)) for i in range(8)], device=device)
    sinks = torch.linspace(-1, 1, 8, device=device)
    run = lambda: vllm_attention(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=causal, softcap=6.0,
                                 alibi_slopes=slopes, s_aux=sinks, return_softmax_lse=True)
    out, lse = run()
    ref, refl = reference(q, k, v, cq, ck, causal=causal, softcap=6.0, alibi=slopes, sinks=sinks)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)
    names = _kernel_names(run)
    if names:  # the combination runs on the tensor-core prefill, not the mma.sync fallback
        assert any("prefill_sm100_kernel" in n for n in names), names


def test_alibi_per_request_slopes_window_sinks(device):
    g = torch.Generator().manual_seed(92)
    qlens, klens = [200, 256, 40], [900, 256, 40]
    q = torch.randn(sum(qlens), 16, 128, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(sum(klens), 4, 128, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn(sum(klens), 4, 128, generator=g).to(torch.bfloat16).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    slopes = torch.rand(3, 16, generator=g).to(device) * 0.2
    sinks = torch.linspace(-2, 2, 16, device=device)
    out, lse = vllm_attention(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=True,
                              window_size=[300, 0], alibi_slopes=slopes, s_aux=sinks, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=True, window=(300, 0), alibi=slopes, sinks=sinks)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_alibi_paged_fp8_prefill(device):
    g = torch.Generator().manual_seed(93)
    qlens, klens, page = [150, 64], [700, 300], 16
    cols = max(klens) // page + 1
    raw = torch.randn(2 * cols, page, 2, 256, generator=g)
    packed = raw.to(torch.float8_e4m3fn).to(device)
    kc, vc = packed.split(128, dim=-1)
    table = torch.randperm(2 * cols, generator=g).int().reshape(2, cols).to(device)
    q = torch.randn(sum(qlens), 8, 128, generator=g).to(torch.bfloat16).to(device)
    cq = cu(qlens, device)
    used = torch.tensor(klens, dtype=torch.int32, device=device)
    slopes = torch.tensor([0.05 * (i + 1) for i in range(8)], device=device)
    out, lse = vllm_attention(q, kc, vc, max(qlens), cq, max(klens), seqused_k=used, block_table=table,
                              causal=True, alibi_slopes=slopes, return_softmax_lse=True)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, causal=True, alibi=slopes)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_alibi_single_query_decode(device):
    g = torch.Generator().manual_seed(94)
    B, H, HK, D, page = 3, 8, 2, 128, 16
    lens = [17, 900, 2500]
    cols = max(lens) // page + 1
    kc = torch.randn(B * cols, page, HK, D, generator=g).to(torch.bfloat16).to(device)
    vc = torch.randn_like(kc)
    table = torch.randperm(B * cols, generator=g).int().reshape(B, cols).to(device)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16).to(device)
    cq = torch.arange(B + 1, dtype=torch.int32, device=device)
    used = torch.tensor(lens, dtype=torch.int32, device=device)
    slopes = torch.tensor([0.01 * (i + 1) for i in range(H)], device=device)
    out, lse = vllm_attention(q, kc, vc, 1, cq, max(lens), seqused_k=used, block_table=table, causal=True,
                              alibi_slopes=slopes, return_softmax_lse=True)
    ref, refl = reference(q, kc, vc, cq, used_k=used, block_table=table, causal=True, alibi=slopes)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)
