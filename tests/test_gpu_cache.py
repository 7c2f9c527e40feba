"""store_kvcache / FP8 quantisation / append / rotary on the GPU.

Cases follow the reference's tests/test_cache.py; expectations come from the
oracle (oracle/cache.py, oracle/fp8.py) or from torch's float8_e4m3fn cast of
clamp(x/scale, -448, 448), which is the reference's own FP8 expectation
(tests/test_cache.py:52). Every comparison here is bit-exact.
"""

import numpy as np
import pytest
import torch

import oracle
from flash_attn_b200 import store_kvcache
from flash_attn_b200._cache import append_kvcache, rotary

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_store_strides_offsets_and_skipped_slots(device, dtype, index_dtype):
    k = torch.arange(5 * 4 * 12, device=device, dtype=torch.float32).to(dtype).reshape(5, 4, 12)[1:, ::2, 1::2]
    v = (k[..., :4] + 100).transpose(0, 1).contiguous().transpose(0, 1)
    kb = torch.full((4, 8, 4, 14), -3, device=device, dtype=dtype)
    vb = torch.full((4, 8, 4, 10), -5, device=device, dtype=dtype)
    kc, vc = kb[1:3, ::2, ::2, 1:13:2], vb[1:3, ::2, ::2, 1:9:2]
    ke, ve = kb.cpu(), vb.cpu()
    kev, vev = ke[1:3, ::2, ::2, 1:13:2], ve[1:3, ::2, ::2, 1:9:2]
    slots = torch.tensor([99, 6, 99, -1, 99, 0, 99, 3], dtype=index_dtype, device=device)[1::2]
    for t, slot in enumerate([6, -1, 0, 3]):
        if slot >= 0:
            kev[slot // 4, slot % 4] = k[t].cpu()
            vev[slot // 4, slot % 4] = v[t].cpu()
    store_kvcache(k, v, kc, vc, slots)
    assert torch.equal(kb.cpu(), ke)
    assert torch.equal(vb.cpu(), ve)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_store_preserves_float_bits(device, dtype):
    special = torch.tensor([0., -0., float("inf"), -float("inf"), float("nan"), 1e-30, -1e-30], dtype=dtype)
    k = special.reshape(1, 1, -1).to(device)
    cache = torch.empty((1, 1, 1, special.numel()), dtype=dtype, device=device)
    store_kvcache(k, k, cache, cache, torch.tensor([0], device=device))
    assert torch.equal(cache.cpu().view(torch.uint8).flatten(), special.view(torch.uint8))


def test_fp8_rne_saturation_and_scales(device):
    representable = torch.arange(127, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    ties = (representable[:-1] + representable[1:]) / 2
    values = torch.cat((representable, ties, -representable, -ties,
                        torch.tensor([1000., -1000., float("inf"), -float("inf")])))
    values = values[:, None, None].expand(-1, 2, 3).contiguous()
    scale = torch.tensor([.5, 2.])
    k = (values * scale[None, :, None]).to(device)
    v = (values * 4).to(device)
    # Each cache is a view with a nonzero storage offset and a strided dimension.
    kb = torch.empty((2, len(values), 2, 6), dtype=torch.float8_e4m3fn, device=device)
    vb = torch.empty_like(kb)
    kc, vc = kb[1:, :, :, ::2], vb[1:, :, :, ::2]
    store_kvcache(k, v, kc, vc, torch.arange(len(values), device=device),
                  k_scale=scale.to(device), v_scale=4.)
    expected = values.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(kc.view(torch.uint8).cpu()[0], expected)
    assert torch.equal(vc.view(torch.uint8).cpu()[0], expected)


@pytest.mark.parametrize("src_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_fp8_exhaustive_against_torch_cast(device, src_dtype):
    # Every bf16 bit pattern (and its f16/f32 value) under eight per-head scales,
    # vectorised 16-byte path: bit-exact with torch's cast of the clamped quotient.
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float()
    bits = bits[torch.isfinite(bits)]
    x = bits.to(src_dtype)
    x = x[torch.isfinite(x)]
    # Powers of two plus scales whose quotients are inexact (the division must
    # still round exactly like x / scale in float32).
    scale = torch.tensor([1.0, 0.5, 2.0, 3.0 / 448.0, 0.1, 1.0 / 3.0, 1.7 / 448.0, 0.0123],
                         dtype=torch.float32)
    heads = scale.numel()
    rows = x.reshape(-1, 1, 1).expand(-1, heads, 8).contiguous()
    cache = torch.empty((rows.shape[0], 1, heads, 8), dtype=torch.float8_e4m3fn, device=device)
    store_kvcache(rows.to(device), rows.to(device), cache, cache,
                  torch.arange(rows.shape[0], device=device), k_scale=scale.to(device),
                  v_scale=scale.to(device))
    expected = (rows.float() / scale[None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(cache.view(torch.uint8).cpu()[:, 0], expected.view(torch.uint8))
    # The oracle's encoder agrees with both.
    codes = oracle.e4m3_encode((rows.float() / scale[None, :, None]).numpy())
    np.testing.assert_array_equal(codes, expected.view(torch.uint8).numpy())


@pytest.mark.parametrize("src_dtype", [torch.bfloat16, torch.float16])
def test_fp8_row_path_specials_and_extreme_scales(device, src_dtype):
    # 16-bit rows of one token per warp (the row kernel): infinities, NaNs,
    # signed zeros, the largest finite values and subnormals under scales that
    # make the products overflow or underflow, plus zero, negative and
    # non-finite scales (IEEE division per element). Bit-exact with torch's
    # cast of clamp(x / scale, -448, 448).
    info = torch.finfo(src_dtype)
    vals = torch.tensor([0., -0., float("inf"), -float("inf"), float("nan"), info.max, -info.max,
                         info.tiny, -info.tiny, info.tiny / 4, 1.0, -1.0, 447.5, 464., -465., 3e-3],
                        dtype=torch.float32).to(src_dtype)
    scale = torch.tensor([1e-30, 1e30, 0.0, -0.5, -3.0 / 448.0, float("inf"), 2.0 ** -20, 1.0 / 448.0],
                         dtype=torch.float32)
    heads, dim = scale.numel(), 16
    rows = vals.reshape(1, 1, -1).expand(3, heads, dim).contiguous()
    cache = torch.empty((3, 1, heads, dim), dtype=torch.float8_e4m3fn, device=device)
    store_kvcache(rows.to(device), rows.to(device), cache, cache, torch.arange(3, device=device),
                  k_scale=scale.to(device), v_scale=scale.to(device))
    expected = (rows.to(device).float() / scale.to(device)[None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    got, want = cache.view(torch.uint8)[:, 0], expected.view(torch.uint8)
    bad = (got != want).nonzero().tolist()
    assert not bad, [(scale[h].item(), vals[d].item(), int(got[t, h, d]), int(want[t, h, d])) for t, h, d in bad[:8]]


def test_fp8_random_float32_quotients_round_exactly(device):
    # Full-mantissa float32 inputs over a wide exponent range and inexact
    # per-head scales: codes equal torch's cast of the IEEE quotient.
    g = torch.Generator().manual_seed(9)
    tokens, heads, dim = 2048, 8, 64
    x = torch.randn(tokens, heads, dim, generator=g) * torch.exp2(torch.randint(-12, 12, (tokens, heads, dim),
                                                                                  generator=g).float())
    scale = torch.rand(heads, generator=g) * 0.9 + 0.05
    cache = torch.empty((tokens, 1, heads, dim), dtype=torch.float8_e4m3fn, device=device)
    store_kvcache(x.to(device), x.to(device), cache, cache, torch.arange(tokens, device=device),
                  k_scale=scale.to(device), v_scale=scale.to(device))
    expected = (x / scale[None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(cache.view(torch.uint8).cpu()[:, 0], expected.view(torch.uint8))


def test_store_matches_oracle_at_bench_shape_sample(device):
    # Config-4 style: bf16 N(0,1) rows, per-head scales U[1/448, 4/448], permuted slots.
    g = torch.Generator().manual_seed(4)
    tokens, heads, dim, page = 4096, 8, 128, 16
    x = torch.randn(tokens, heads, dim, generator=g).to(torch.bfloat16)
    scale = (1 + 3 * torch.rand(heads, generator=g)) / 448
    slots = torch.randperm(tokens + 64, generator=g)[:tokens].to(torch.int32)
    cache = torch.zeros(((tokens + 64) // page, page, heads, dim), dtype=torch.float8_e4m3fn, device=device)
    store_kvcache(x.to(device), x.to(device), cache, cache, slots.to(device), k_scale=scale.to(device),
                  v_scale=scale.to(device))
    expected = np.zeros(cache.shape, dtype=np.uint8)
    oracle.store_kvcache(x.float().numpy(), expected, slots.numpy(), scale.numpy(), fp8=True)
    np.testing.assert_array_equal(cache.view(torch.uint8).cpu().numpy(), expected)


@pytest.mark.parametrize("paged", [False, True])
def test_append_batch_remapping_and_boundaries(device, paged):
    k = torch.arange(2 * 3 * 2 * 4, device=device, dtype=torch.float32).reshape(2, 3, 2, 4)
    v = k[..., :2] + 70
    kc = torch.full((6 if paged else 3, 4 if paged else 12, 2, 4), -1., device=device)
    vc = torch.full((*kc.shape[:-1], 2), -2., device=device)
    table = torch.tensor([[5, 0, 2], [1, 4, 3], [2, 3, 1]], device=device, dtype=torch.int32) if paged else None
    lengths = torch.tensor([3, 6], device=device, dtype=torch.int32)
    rows = torch.tensor([1, 0], device=device, dtype=torch.int32)
    ke = oracle.append_kvcache(k.cpu().numpy(), kc.cpu().numpy(), [3, 6], cache_batch_idx=[1, 0],
                               block_table=None if table is None else table.cpu().numpy())
    ve = oracle.append_kvcache(v.cpu().numpy(), vc.cpu().numpy(), [3, 6], cache_batch_idx=[1, 0],
                               block_table=None if table is None else table.cpu().numpy())
    append_kvcache(k, v, kc, vc, lengths, cache_batch_idx=rows,
                   cache_leftpad=torch.tensor([2, 1], device=device), block_table=table)
    np.testing.assert_array_equal(kc.cpu().numpy(), ke)
    np.testing.assert_array_equal(vc.cpu().numpy(), ve)
    assert torch.equal(lengths.cpu(), torch.tensor([3, 6], dtype=torch.int32))


def test_append_fp8_scales(device):
    k = torch.randn((2, 2, 3, 5), device=device)
    v = torch.randn((2, 2, 3, 7), device=device)
    kc = torch.empty((2, 4, 3, 5), dtype=torch.float8_e4m3fn, device=device)
    vc = torch.empty((2, 4, 3, 7), dtype=torch.float8_e4m3fn, device=device)
    scale = torch.tensor([.5, 1., 2.], device=device)
    append_kvcache(k, v, kc, vc, 1, k_scale=scale, v_scale=2.)
    ke = (k.cpu() / scale.cpu()[None, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    ve = (v.cpu() / 2).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(kc.cpu()[:, 1:3].contiguous().view(torch.uint8), ke)
    assert torch.equal(vc.cpu()[:, 1:3].contiguous().view(torch.uint8), ve)


def test_fp8_default_scale_with_float16_default_dtype(device):
    old = torch.get_default_dtype()
    try:
        torch.set_default_dtype(torch.float16)
        k = torch.tensor([[[1., 2., 3., 4.]]], device=device)
        cache = torch.empty((1, 1, 1, 4), device=device, dtype=torch.float8_e4m3fn)
        store_kvcache(k, k, cache, cache, torch.tensor([0], device=device))
        expected = k.cpu().to(torch.float8_e4m3fn).view(torch.uint8)
        assert torch.equal(cache.view(torch.uint8).cpu()[0], expected)
    finally:
        torch.set_default_dtype(old)


@pytest.mark.parametrize("interleaved", [True, False])
@pytest.mark.parametrize("mode", ["global", "causal", "local"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_rotary_modes_strides_and_partial_head(device, interleaved, mode, dtype):
    q = torch.randn((2, 3, 4, 16), device=device).to(dtype)[..., 1::2]
    k = torch.randn((2, 2, 2, 16), device=device).to(dtype)[..., 1::2]
    angles = torch.randn((20, 4), device=device)[:, ::2]
    cos, sin = angles.cos(), angles.sin()
    lengths = torch.tensor([2, 7], device=device)
    window = (3, -1) if mode == "local" else [-1, -1]
    qr, kr = rotary(q, k, cos, sin, lengths, rotary_interleaved=interleaved,
                    causal=mode == "causal", window_size=window)
    qe = oracle.rotary(q.cpu().float().numpy(), cos.cpu().numpy(), sin.cpu().numpy(), [2, 7],
                       interleaved, mode != "global")
    ke = oracle.rotary(k.cpu().float().numpy(), cos.cpu().numpy(), sin.cpu().numpy(), [2, 7],
                       interleaved, True)
    tol = dict(rtol=1e-5, atol=5e-7) if dtype == torch.float32 else dict(rtol=8e-3, atol=8e-3)
    torch.testing.assert_close(qr.cpu().double(), torch.from_numpy(qe).to(dtype).double(), **tol)
    torch.testing.assert_close(kr.cpu().double(), torch.from_numpy(ke).to(dtype).double(), **tol)
    assert torch.equal(qr.cpu()[..., 4:], q.cpu()[..., 4:])


@pytest.mark.parametrize("cache_dtype", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("paged", [False, True])
@pytest.mark.parametrize("interleaved", [True, False])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("table_dtype", [torch.float32, torch.bfloat16])
def test_fused_rotary_append_equals_rotary_then_append(device, cache_dtype, paged, interleaved, causal,
                                                       table_dtype):
    from flash_attn_b200._cache import append_kvcache, rotary, rotary_append_kvcache
    g = torch.Generator().manual_seed(61)
    B, S, H, HK, D, rot, cap, page = 3, 5, 8, 2, 128, 96, 64, 16
    q = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(B, S, HK, D, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn(B, S, HK, D, generator=g).to(torch.bfloat16).to(device)
    angles = torch.rand(cap + S, rot // 2, generator=g) * 6
    cos, sin = angles.cos().to(table_dtype).to(device), angles.sin().to(table_dtype).to(device)
    lengths = torch.tensor([0, 17, 40], dtype=torch.int32, device=device)
    scale = torch.tensor([.02, .05], device=device) if cache_dtype == torch.float8_e4m3fn else None
    if paged:
        kc = torch.zeros(B * cap // page, page, HK, D, dtype=cache_dtype, device=device)
        table = torch.randperm(B * cap // page, generator=g).int().reshape(B, cap // page).to(device)
        extra = dict(block_table=table)
    else:
        kc = torch.zeros(B + 1, cap, HK, D, dtype=cache_dtype, device=device)
        extra = dict(cache_batch_idx=torch.tensor([2, 0, 3], dtype=torch.int32, device=device))
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    q_rot, k_rot = rotary(q, k, cos, sin, lengths, rotary_interleaved=interleaved, causal=causal)
    append_kvcache(k_rot, v, kc, vc, lengths, k_scale=scale, v_scale=scale, **extra)
    q_fused = rotary_append_kvcache(q, k, v, kc2, vc2, cos, sin, lengths, rotary_interleaved=interleaved,
                                    causal=causal, k_scale=scale, v_scale=scale, **extra)
    assert torch.equal(q_fused, q_rot)
    assert torch.equal(kc2.view(torch.uint8), kc.view(torch.uint8))
    assert torch.equal(vc2.view(torch.uint8), vc.view(torch.uint8))


def _strided_copy(x):
    """Same values with inner stride 2: the scalar append/RoPE kernels take it."""
    wide = torch.empty(*x.shape[:-1], 2 * x.shape[-1], dtype=x.dtype, device=x.device)
    view = wide[..., ::2]
    view.copy_(x)
    return view


@pytest.mark.parametrize("cache", ["same", "fp8"])
@pytest.mark.parametrize("interleaved", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_vectorized_append_and_rope_match_scalar_kernels(device, cache, interleaved, dtype):
    from flash_attn_b200._cache import append_kvcache, rotary_append_kvcache
    cache_dtype = dtype if cache == "same" else torch.float8_e4m3fn
    g = torch.Generator().manual_seed(62)
    B, S, H, HK, D, page = 4, 300, 16, 8, 128, 16
    cols = (S + 40) // page + 1
    q = torch.randn(B, S, H, D, generator=g).to(dtype).to(device)
    k = (torch.randn(B, S, HK, D, generator=g) * 3).to(dtype).to(device)
    v = (torch.randn(B, S, HK, D, generator=g) * 3).to(dtype).to(device)
    angles = torch.rand(cols * page, D // 2, generator=g) * 6
    cos, sin = angles.cos().to(device), angles.sin().to(device)
    table = torch.randperm(B * cols, generator=g).int().reshape(B, cols).to(device)
    lengths = torch.tensor([0, 3, 40, 17], dtype=torch.int32, device=device)
    scale = torch.tensor([.01 * (i + 1) for i in range(HK)], device=device) \
        if cache_dtype == torch.float8_e4m3fn else None
    caches = [torch.zeros(B * cols, page, HK, D, dtype=cache_dtype, device=device) for _ in range(8)]
    # Plain append: vectorized (contiguous) vs scalar (strided inputs).
    append_kvcache(k, v, caches[0], caches[1], lengths, block_table=table, k_scale=scale, v_scale=scale)
    append_kvcache(_strided_copy(k), _strided_copy(v), caches[2], caches[3], lengths, block_table=table,
                   k_scale=scale, v_scale=scale)
    assert torch.equal(caches[0].view(torch.uint8), caches[2].view(torch.uint8))
    assert torch.equal(caches[1].view(torch.uint8), caches[3].view(torch.uint8))
    # Fused RoPE + append.
    kw = dict(rotary_interleaved=interleaved, causal=True, block_table=table, k_scale=scale, v_scale=scale)
    q_vec = rotary_append_kvcache(q, k, v, caches[4], caches[5], cos, sin, lengths, **kw)
    q_sca = rotary_append_kvcache(_strided_copy(q), _strided_copy(k), _strided_copy(v), caches[6], caches[7],
                                  cos, sin, lengths, **kw)
    assert torch.equal(q_vec, q_sca)
    assert torch.equal(caches[4].view(torch.uint8), caches[6].view(torch.uint8))
    assert torch.equal(caches[5].view(torch.uint8), caches[7].view(torch.uint8))
    assert caches[4].view(torch.uint8).any()
