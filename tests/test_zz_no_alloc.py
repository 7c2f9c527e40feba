"""fa_decode_fwd_noalloc: split-KV decode for callers that cannot allocate.

Some callers cannot hand the library a device workspace: an FFI host that only
holds raw pointers from another framework's allocator, a process whose device
memory is pre-reserved by a pool it does not control, or a decode loop that
must not call cudaMalloc. fa_decode_fwd_noalloc keeps the split-KV partials in
a static device array inside the library. This test calls it through the C ABI
twice in a row and checks each result against the existing entry point
(fa_attention_fwd with a caller workspace), plus the clear rejection of a
request whose partials exceed the static array. It lives in its own file,
collected last, and passes alone in a fresh process or after the other tests.
"""

import ctypes

import pytest
import torch

from flash_attn_b200 import _attention, _capi

pytestmark = pytest.mark.gpu


def _case(device, seed, kv_dtype):
    g = torch.Generator().manual_seed(seed)
    batch, hq, hk, d, page = 4, 16, 4, 128, 16
    lengths = [3000, 1, 2047, 1500]
    columns = (max(lengths) + page - 1) // page
    pages = batch * columns + 3
    k = torch.randn(pages, page, hk, d, generator=g)
    v = torch.randn(pages, page, hk, d, generator=g)
    if kv_dtype == torch.float8_e4m3fn:
        k, v = (k * 40).to(kv_dtype), (v * 40).to(kv_dtype)
    else:
        k, v = k.to(kv_dtype), v.to(kv_dtype)
    table = torch.randperm(pages, generator=g)[:batch * columns].to(torch.int32).reshape(batch, columns)
    q = torch.randn(batch, hq, d, generator=g).to(torch.bfloat16)
    kw = dict(cu_seqlens_q=torch.arange(batch + 1, dtype=torch.int32, device=device),
              cu_seqlens_k=None, seqused_k=torch.tensor(lengths, dtype=torch.int32, device=device),
              max_seqlen_q=1, max_seqlen_k=max(lengths), block_table=table.to(device),
              softmax_scale=None, causal=False, window_size=(-1, -1), alibi_slopes=None, softcap=0.0,
              s_aux=None, q_descale=None,
              k_descale=torch.full((batch, hk), 1 / 40, device=device) if kv_dtype == torch.float8_e4m3fn else None,
              v_descale=torch.full((batch, hk), 1 / 40, device=device) if kv_dtype == torch.float8_e4m3fn else None,
              num_splits=8, mask_mod=None, aux_tensors=None, leftpad_k=None, deterministic=False)
    return q.to(device), k.to(device), v.to(device), kw


def _noalloc(q, k, v, kw):
    out = torch.empty(q.shape[0], q.shape[1], v.shape[-1], dtype=q.dtype, device=q.device)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    args, keep = _attention.build_args(q, k, v, out, lse, **kw)
    lib = _capi.library()
    _capi.check(lib.fa_decode_fwd_noalloc(ctypes.byref(args), _capi.stream_of(q.device)))
    return out, lse


def _existing(q, k, v, kw):
    out = torch.empty(q.shape[0], q.shape[1], v.shape[-1], dtype=q.dtype, device=q.device)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    return _attention.run(q, k, v, out, lse, **kw)


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_noalloc_decode_matches_existing_entry_point_twice(device, kv_dtype):
    for seed in (0, 1):  # two calls in a row share the static scratch
        q, k, v, kw = _case(device, seed, kv_dtype)
        want, want_lse = _existing(q, k, v, kw)
        got, got_lse = _noalloc(q, k, v, kw)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=5e-2)
        torch.testing.assert_close(got_lse, want_lse, atol=1e-3, rtol=0)


def test_noalloc_rejects_partials_beyond_the_static_scratch(device):
    q, k, v, kw = _case(device, 2, torch.bfloat16)
    q = q.repeat(32, 2, 1)[:128]
    kw = dict(kw, cu_seqlens_q=torch.arange(129, dtype=torch.int32, device=device),
              seqused_k=torch.full((128,), 16, dtype=torch.int32, device=device),
              block_table=kw["block_table"][:1].repeat(128, 1), max_seqlen_k=16, num_splits=2048)
    k = k.repeat(1, 1, 2, 1)[:, :, :8]
    v = v.repeat(1, 1, 2, 1)[:, :, :8]
    with pytest.raises(ValueError, match="static scratch"):
        _noalloc(q, k, v, kw)
