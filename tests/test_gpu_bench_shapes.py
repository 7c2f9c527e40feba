"""Parity at the exact shapes bench.py times (configs 3 and 4).

The benchmark lines are only worth their roofline fractions if the work they
time is right. These tests build each configuration with bench.py's own
builders (same seeds, sizes, page permutations and, for config 4, the FP8
cache written by store_kvcache with per-head scales), run the library's
default split plan on the whole batch, and compare a seeded sample of
requests -- the shortest, the longest and four more, all heads -- against the
float64 oracle (reference tests/reference.py:6-90 restated in oracle/). The
same sampled requests then run alone as a small batch, where the split rules
take their other branches: the library's default (more splits to fill the
GPU), an explicit two-split plan, and num_splits == 1 (the batch-invariant
route). Tail slots of each request's last page are NaN-poisoned first, as in
the reference's paged decode test (tests/test_decode.py:23-52).

Gates: the north-star tolerances (max-abs 1e-2 on 16-bit outputs after the
reference's assert_attention_close, 1e-3 on the LSE) plus a scale-aware one
(1 % of the largest reference output), because long-context decode outputs
are averages of many values and a fixed 1e-2 alone would be loose.
"""

import numpy as np
import pytest
import torch

import bench
import oracle
from flash_attn_b200._attention import attention
from helpers import assert_attention_close, assert_lse_close

pytestmark = pytest.mark.gpu


# The oracle's E4M3 decoding of all 256 codes, applied by table lookup (the
# same values as decoding each byte, without 1 GB temporaries per request).
_E4M3 = oracle.e4m3_decode(np.arange(256, dtype=np.uint8))


def _oracle_request(q_row, k_rows, v_rows, k_descale=None, v_descale=None):
    """Float64 oracle for one single-query request over contiguous K/V rows."""
    def host(x):
        if x.dtype == torch.float8_e4m3fn:
            return _E4M3[x.view(torch.uint8).cpu().numpy()]
        return x.cpu().double().numpy()
    length = k_rows.shape[0]
    out, lse = oracle.attention(
        q_row[None].cpu().double().numpy(), host(k_rows), host(v_rows), np.array([0, 1]),
        cu_k=np.array([0, length]),
        k_descale=None if k_descale is None else k_descale[None].cpu().double().numpy(),
        v_descale=None if v_descale is None else v_descale[None].cpu().double().numpy())
    return torch.from_numpy(out[0]), torch.from_numpy(lse[:, 0])


def _check(out_row, lse_row, ref_out, ref_lse, dtype):
    assert_attention_close(out_row, ref_out, dtype)
    assert_lse_close(lse_row, ref_lse)
    err = (out_row.detach().cpu().double() - ref_out).abs().max().item()
    scale = ref_out.abs().max().item()
    assert err <= 1e-2 * scale + 2e-5, f"max-abs {err:.3e} against largest output {scale:.3e}"


def _poison_tails(cache, table, lengths, page):
    """NaN in every slot past each request's length on its last page."""
    for b, length in enumerate(lengths):
        length = int(length)
        if length % page:
            cache[int(table[b, length // page]), length % page:] = float("nan")


def _subset_calls(q, k_cache, v_cache, table, lengths, picks, page, **kw):
    """The sampled requests alone as one batch, under three split plans."""
    dev = q.device
    sel = torch.tensor(picks, device=dev)
    sub_q = q[sel].contiguous()
    sub_table = table[sel].contiguous()
    used = torch.tensor([int(lengths[b]) for b in picks], dtype=torch.int32, device=dev)
    cu_q = torch.arange(len(picks) + 1, dtype=torch.int32, device=dev)
    sub_kw = {k: (v[sel].contiguous() if torch.is_tensor(v) and v.dim() == 2 else v) for k, v in kw.items()}
    results = {}
    for splits in (0, 2, 1):
        out = torch.empty_like(sub_q)
        results[splits] = attention(sub_q, k_cache, v_cache, cu_seqlens_q=cu_q, seqused_k=used, max_seqlen_q=1,
                                    max_seqlen_k=int(max(int(lengths[b]) for b in picks)), block_table=sub_table,
                                    out=out, num_splits=splits, **sub_kw)
    return results


def test_config3_paged_bf16_decode_at_bench_shape():
    cfg = dict(bench.CFG3)
    w = bench.build_cfg3(cfg)
    ctx, page = w["ctx"], cfg["page"]
    for cache in (w["k_cache"], w["v_cache"]):
        _poison_tails(cache, w["table"].cpu(), ctx, page)
    out = torch.empty_like(w["q"])
    out, lse = attention(w["q"], w["k_cache"], w["v_cache"], cu_seqlens_q=w["cu_q"], seqused_k=w["used"],
                         max_seqlen_q=1, max_seqlen_k=int(ctx.max()), block_table=w["table"], out=out)
    picks = bench.sample_requests(ctx)
    assert int(ctx[picks[0]]) == int(ctx.min()) and int(ctx[picks[1]]) == int(ctx.max())
    subset = _subset_calls(w["q"], w["k_cache"], w["v_cache"], w["table"], ctx, picks, page)
    torch.cuda.synchronize()
    for i, b in enumerate(picks):
        length = int(ctx[b])
        k_rows = bench.gather_request(w["k_cache"], w["table"], b, length, page)
        v_rows = bench.gather_request(w["v_cache"], w["table"], b, length, page)
        ref_out, ref_lse = _oracle_request(w["q"][b], k_rows, v_rows)
        _check(out[b], lse[:, b], ref_out, ref_lse, torch.bfloat16)
        for splits, (sub_out, sub_lse) in subset.items():
            _check(sub_out[i], sub_lse[:, i], ref_out, ref_lse, torch.bfloat16)


def test_config4_fp8_split_kv_decode_at_bench_shape():
    cfg = dict(bench.CFG4)
    k_cache, v_cache, table, ks, vs = bench.build_fp8_cache(0, 1, cfg)
    q_host, _ = bench.cfg4_query(cfg)
    dev = k_cache.device
    q = q_host.to(dev)
    B, C, HK = cfg["batch"], cfg["ctx"], cfg["hkv"]
    kd = ks.reshape(1, HK).expand(B, HK)
    vd = vs.reshape(1, HK).expand(B, HK)
    used = torch.full((B,), C, dtype=torch.int32, device=dev)
    cu_q = torch.arange(B + 1, dtype=torch.int32, device=dev)
    out = torch.empty(B, cfg["hq"], cfg["d"], dtype=torch.bfloat16, device=dev)
    out, lse = attention(q, k_cache, v_cache, cu_seqlens_q=cu_q, seqused_k=used, max_seqlen_q=1,
                         max_seqlen_k=C, block_table=table, k_descale=kd, v_descale=vd, out=out)
    picks = bench.sample_requests([C] * B)
    subset = _subset_calls(q, k_cache, v_cache, table, [C] * B, picks, cfg["page"],
                           k_descale=kd.contiguous(), v_descale=vd.contiguous())
    torch.cuda.synchronize()
    for i, b in enumerate(picks):
        k_rows = bench.gather_request(k_cache, table, b, C, cfg["page"])
        v_rows = bench.gather_request(v_cache, table, b, C, cfg["page"])
        ref_out, ref_lse = _oracle_request(q[b], k_rows, v_rows, kd[b], vd[b])
        del k_rows, v_rows
        _check(out[b], lse[:, b], ref_out, ref_lse, torch.bfloat16)
        for splits, (sub_out, sub_lse) in subset.items():
            _check(sub_out[i], sub_lse[:, i], ref_out, ref_lse, torch.bfloat16)


def test_config4_store_kvcache_writes_the_torch_cast():
    # The cache config 4 decodes is itself the product of store_kvcache: a
    # sampled slice of the written codes equals torch's float8_e4m3fn cast of
    # clamp(x / scale, -448, 448) of the same bf16 rows (bit-exact).
    cfg = dict(bench.CFG4, batch=2, ctx=8192)
    k_cache, v_cache, table, ks, vs = bench.build_fp8_cache(0, 1, cfg)
    # Rebuild the first request's bf16 rows from the builder's generator.
    dev = k_cache.device
    g = torch.Generator(device=dev).manual_seed(4 * 1000 + 0 + 7)
    n = cfg["batch"] * cfg["ctx"]
    k = torch.randn(n, cfg["hkv"], cfg["d"], device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn(n, cfg["hkv"], cfg["d"], device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
    for b in range(cfg["batch"]):
        rows = slice(b * cfg["ctx"], (b + 1) * cfg["ctx"])
        for x, cache, scale in ((k, k_cache, ks), (v, v_cache, vs)):
            want = (x[rows].float() / scale.reshape(1, -1, 1)).clamp(-448, 448).to(torch.float8_e4m3fn)
            got = bench.gather_request(cache, table, b, cfg["ctx"], cfg["page"])
            assert torch.equal(got.view(torch.uint8), want.view(torch.uint8))
