"""fa_decode_fwd_noalloc: split-KV decode for callers that cannot allocate.

Some callers cannot hand the library a device workspace: an FFI host that only
holds raw pointers from another framework's allocator, a process whose device
memory is pre-reserved by a pool it does not control, or a decode loop that
must not call cudaMalloc. fa_decode_fwd_noalloc keeps the split-KV partials in
a static device array inside the library. This test calls it through the C ABI
twice in a row and checks each result against the existing entry point
(fa_attention_fwd with a caller workspace). Both run the same plan and the
same kernels, so their results must be bit-identical: a misplaced partial or
LSE offset inside the static array would change them only slightly, and a
tolerance could hide it. It also covers the num_splits == 1 (batch-invariant)
route after a split call has left data in the array, a library-chosen split
count lowered to fit the array, and the clear rejection of an explicit split
count whose partials exceed it. It lives in its own file, collected last, and
passes alone in a fresh process or after the other tests.
"""

import ctypes

import pytest
import torch

from flash_attn_b200 import _attention, _capi

pytestmark = pytest.mark.gpu


def _case(device, seed, kv_dtype, num_splits=8, lengths=(3000, 1, 2047, 1500)):
    g = torch.Generator().manual_seed(seed)
    lengths = list(lengths)
    batch, hq, hk, d, page = len(lengths), 16, 4, 128, 16
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
              num_splits=num_splits, mask_mod=None, aux_tensors=None, leftpad_k=None, deterministic=False)
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


def _assert_identical(got, got_lse, want, want_lse):
    torch.cuda.synchronize()
    assert torch.equal(got, want), f"out differs, max-abs {(got.float() - want.float()).abs().max().item()}"
    assert torch.equal(got_lse, want_lse), "lse differs"


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_noalloc_decode_matches_existing_entry_point_twice(device, kv_dtype):
    for seed in (0, 1):  # two calls in a row share the static scratch
        q, k, v, kw = _case(device, seed, kv_dtype)
        want, want_lse = _existing(q, k, v, kw)
        got, got_lse = _noalloc(q, k, v, kw)
        _assert_identical(got, got_lse, want, want_lse)


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_noalloc_single_split_after_a_split_call(device, kv_dtype):
    # A split call first leaves partials in the static array; num_splits == 1
    # then runs the batch-invariant route, whose work counter lives in the
    # same array and must be cleared by that launch, twice in a row.
    q, k, v, kw = _case(device, 3, kv_dtype, num_splits=8)
    _noalloc(q, k, v, kw)
    for seed in (4, 5):
        q, k, v, kw = _case(device, seed, kv_dtype, num_splits=1)
        want, want_lse = _existing(q, k, v, kw)
        got, got_lse = _noalloc(q, k, v, kw)
        _assert_identical(got, got_lse, want, want_lse)


def test_noalloc_lowers_a_library_chosen_split_count_to_fit(device):
    # 512 requests x 32 query heads: the library's own rule picks 4 splits for
    # FP8 K/V, whose partials (32 MiB + LSEs) exceed the static array; with
    # num_splits == 0 the entry point lowers the count to 3 instead of failing.
    lengths = [1024] * 512
    q, k, v, kw = _case(device, 6, torch.float8_e4m3fn, num_splits=0, lengths=lengths)
    q = q.repeat(1, 2, 1)  # 32 query heads over 4 KV heads
    want, want_lse = _existing(q, k, v, dict(kw, num_splits=3))
    for _ in range(2):
        got, got_lse = _noalloc(q, k, v, kw)
        _assert_identical(got, got_lse, want, want_lse)
    default, default_lse = _existing(q, k, v, kw)  # 4 splits, caller workspace
    torch.cuda.synchronize()
    torch.testing.assert_close(got.float(), default.float(), atol=2e-2, rtol=5e-2)
    torch.testing.assert_close(got_lse, default_lse, atol=1e-3, rtol=0)


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
