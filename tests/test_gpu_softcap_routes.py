"""Softcap on the tcgen05 prefill kernels: both tanh routes against the oracle.

The reference applies the softcap as cap * tanh(score / cap) before ALiBi and
the masks (flash_attn_mps/kernels/attention.metal:47-51). The tensor-core
prefill kernels evaluate tanh per key tile and warp in one of two ways: an
FMA-pipe polynomial when every score of the warp's 32 query rows satisfies
|score * scale / cap| <= 3/4, else the identity tanh(y) = 1 - 2/(e^(2y)+1).
These cases make the polynomial route cover its whole range, make both routes
occur within one call (rows with large-magnitude queries force the identity
route on their warps only), and run ALiBi with a softcap and the wide-head-dim
kernel on both routes; every result is checked against the float64 oracle
(reference tests/reference.py:6-90) with the reference's tolerances
(max-abs 1e-2 on 16-bit outputs, LSE 1e-3).
"""

import pytest
import torch

from flash_attn_b200 import flash_attn_varlen_func
from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_varlen
from helpers import assert_attention_close, assert_lse_close, cu, reference

pytestmark = pytest.mark.gpu


def _qkv(device, dtype, qlens, klens, hq, hk, d, seed, q_mul=1.0, k_mul=1.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sum(qlens), hq, d, generator=g) * q_mul
    k = torch.randn(sum(klens), hk, d, generator=g) * k_mul
    v = torch.randn(sum(klens), hk, d, generator=g)
    return q, k, v.to(dtype).to(device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [128, 64])
def test_polynomial_route_over_its_range(device, dtype, d):
    # q, k ~ 3 N(0,1): scaled scores ~ 9 N(0,1), so with cap 60 the warps' largest
    # |score * scale / cap| spread up to the route's 3/4 limit.
    qlens = [200, 700, 1100]
    q, k, v = _qkv(device, dtype, qlens, qlens, 8, 2, d, seed=31, q_mul=3.0, k_mul=3.0)
    q, k = q.to(dtype).to(device), k.to(dtype).to(device)
    c = cu(qlens, device)
    out, lse = flash_attn_varlen_func(q, k, v, c, c, max(qlens), max(qlens), causal=True, softcap=60.0,
                                      return_softmax_lse=True)
    ref, refl = reference(q, k, v, c, c, causal=True, softcap=60.0)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_routes_mixed_within_one_call(device, dtype):
    # Most warps see |y| <= 0.2 (polynomial); query rows 32..63 of every
    # sequence and the last rows of the longest one are scaled by 30, which
    # sends their warps (and only theirs) to the identity route.
    qlens, klens = [300, 129, 1500], [420, 129, 1500]
    q, k, v = _qkv(device, dtype, qlens, klens, 8, 2, 128, seed=32)
    starts = [0, qlens[0], qlens[0] + qlens[1]]
    for s0 in starts:
        q[s0 + 32:s0 + 64] *= 30.0
    q[-100:] *= 30.0
    q, k = q.to(dtype).to(device), k.to(dtype).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    sinks = torch.linspace(-2, 2, 8, device=device)
    out, lse = vllm_varlen(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=True,
                           window_size=[700, 0], softcap=20.0, s_aux=sinks, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=True, window=(700, 0), softcap=20.0, sinks=sinks)
    assert_attention_close(out, ref, dtype)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("causal", [True, False])
def test_alibi_softcap_polynomial_route(device, causal):
    # cap 50 with N(0,1) inputs: every warp takes the polynomial route, then
    # the ALiBi bias is subtracted before the row max.
    qlens, klens = [300, 1, 129, 640], [300, 70, 400, 640]
    q, k, v = _qkv(device, torch.bfloat16, qlens, klens, 8, 2, 128, seed=33)
    q, k = q.to(torch.bfloat16).to(device), k.to(torch.bfloat16).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    slopes = torch.tensor([2.0 ** (-(i + 1)) for i in range(8)], device=device)
    out, lse = vllm_varlen(q, k, v, max(qlens), cq, max(klens), cu_seqlens_k=ck, causal=causal, softcap=50.0,
                           alibi_slopes=slopes, return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=causal, softcap=50.0, alibi=slopes)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


def test_alibi_softcap_mixed_routes(device):
    qlens = [520, 900]
    q, k, v = _qkv(device, torch.bfloat16, qlens, qlens, 8, 2, 128, seed=34)
    q[96:128] *= 40.0
    q[qlens[0] + 600:qlens[0] + 640] *= 40.0
    q, k = q.to(torch.bfloat16).to(device), k.to(torch.bfloat16).to(device)
    c = cu(qlens, device)
    slopes = torch.tensor([2.0 ** (-(i + 1) / 2) for i in range(8)], device=device)
    out, lse = vllm_varlen(q, k, v, max(qlens), c, max(qlens), cu_seqlens_k=c, causal=True, softcap=30.0,
                           alibi_slopes=slopes, return_softmax_lse=True)
    ref, refl = reference(q, k, v, c, c, causal=True, softcap=30.0, alibi=slopes)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)


@pytest.mark.parametrize("dims", [(256, 256), (192, 128)])
@pytest.mark.parametrize("cap", [2.0, 25.0])
def test_wide_kernel_routes(device, dims, cap):
    # cap 2: identity route on (nearly) every warp; cap 25: polynomial route
    # except on the rows scaled by 30.
    dq, dv = dims
    qlens, klens = [77, 300, 640], [300, 300, 900]
    g = torch.Generator().manual_seed(35)
    q = torch.randn(sum(qlens), 8, dq, generator=g)
    k = torch.randn(sum(klens), 2, dq, generator=g)
    v = torch.randn(sum(klens), 2, dv, generator=g).to(torch.bfloat16).to(device)
    q[100:140] *= 30.0
    q, k = q.to(torch.bfloat16).to(device), k.to(torch.bfloat16).to(device)
    cq, ck = cu(qlens, device), cu(klens, device)
    out, lse = flash_attn_varlen_func(q, k, v, cq, ck, max(qlens), max(klens), causal=True, softcap=cap,
                                      return_softmax_lse=True)
    ref, refl = reference(q, k, v, cq, ck, causal=True, softcap=cap)
    assert_attention_close(out, ref, torch.bfloat16)
    assert_lse_close(lse, refl)
