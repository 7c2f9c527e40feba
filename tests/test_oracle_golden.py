"""Pin the CPU oracle to golden vectors produced by the reference itself.

``tests/golden/make_golden.py`` ran the reference's ``tests/reference.py``
and its test-file expectations on seeded inputs; these tests check that the
numpy restatement in ``oracle/`` reproduces every stored output.
"""

import glob
import os
from types import SimpleNamespace

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as f:
        return {k: f[k] for k in f.files}


def _float(g, key, fp8_flag):
    x = g[key]
    if bool(g[fp8_flag]):
        return oracle.e4m3_decode(x)
    return x.astype(np.float64)


ATTN = sorted(os.path.basename(p)[5:-4] for p in glob.glob(os.path.join(GOLDEN, "attn_*.npz")))


@pytest.mark.parametrize("name", ATTN)
def test_attention_oracle_matches_reference(name):
    g = load("attn_" + name)
    mask = None
    if "mask" in g:
        kind, win, clamp = (int(x) for x in g["mask"])
        mask = SimpleNamespace(kind=kind, sliding_window_left=win, clamp_prefix_to_window=bool(clamp))
    causal = g["causal"]
    out, lse = oracle.attention(
        _float(g, "q", "q_fp8"), _float(g, "k", "kv_fp8"), _float(g, "v", "kv_fp8"), g["cu_q"],
        cu_k=g.get("cu_k"), used_k=g.get("used_k"), block_table=g.get("block_table"),
        causal=bool(causal) if causal.ndim == 0 else causal, window=tuple(int(w) for w in g["window"]),
        softcap=float(g["softcap"]), alibi=g.get("alibi"), sinks=g.get("sinks"),
        q_descale=g.get("q_descale"), k_descale=g.get("k_descale"), v_descale=g.get("v_descale"),
        mask=mask, aux=None if mask is None else (g["aux0"], g["aux1"]), leftpad=g.get("leftpad"))
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(np.isneginf(lse), np.isneginf(g["lse"]))
    finite = np.isfinite(g["lse"])
    np.testing.assert_allclose(lse[finite], g["lse"][finite], rtol=1e-8, atol=1e-8)


def test_fp8_encoder_matches_torch_saturating_cast():
    g = load("fp8_codec")
    x = g["x"].astype(np.float32) / g["scale"].astype(np.float32)
    codes = oracle.e4m3_encode(x)
    np.testing.assert_array_equal(codes, g["codes"])


def test_fp8_decoder_matches_every_code():
    g = load("fp8_codec")
    decoded = oracle.e4m3_decode(np.arange(256, dtype=np.uint8))
    np.testing.assert_array_equal(np.isnan(decoded), np.isnan(g["decode_table"]))
    finite = ~np.isnan(decoded)
    np.testing.assert_array_equal(decoded[finite], g["decode_table"][finite].astype(np.float64))


def test_merge_pair_matches_reference_formula():
    g = load("merge_pair")
    out, lse = oracle.merge_pair(g["left"], g["la"], g["right"], g["lb"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-12, atol=1e-12)
    np.testing.assert_array_equal(np.isneginf(lse), np.isneginf(g["lse"]))
    finite = np.isfinite(g["lse"])
    np.testing.assert_allclose(lse[finite], g["lse"][finite], rtol=1e-12)


def test_merge_partials_matches_reference_formula():
    g = load("merge_partials")
    out, lse = oracle.merge_partials(g["partial"], g["lse"])
    np.testing.assert_allclose(out, g["out"], rtol=1e-12, atol=1e-12)
    finite = np.isfinite(g["out_lse"])
    np.testing.assert_allclose(lse[finite], g["out_lse"][finite], rtol=1e-12)
    np.testing.assert_array_equal(np.isneginf(lse), ~finite)


@pytest.mark.parametrize("interleaved", [True, False])
@pytest.mark.parametrize("advance", [True, False])
def test_rotary_matches_reference_helper(interleaved, advance):
    g = load("rotary")
    out = oracle.rotary(g["x"], g["cos"], g["sin"], g["lengths"], interleaved, advance)
    np.testing.assert_allclose(out, g[f"out_{int(interleaved)}{int(advance)}"], rtol=1e-6, atol=1e-6)


def test_store_and_append_follow_reference_expectations():
    # test_cache.py:10-27 and 57-75: the expected caches are built by explicit loops.
    x = np.arange(4 * 2 * 6, dtype=np.float64).reshape(4, 2, 6)
    cache = np.full((2, 4, 2, 6), -3.0)
    oracle.store_kvcache(x, cache, np.array([6, -1, 0, 3]))
    expected = np.full((2, 4, 2, 6), -3.0)
    for t, slot in enumerate([6, -1, 0, 3]):
        if slot >= 0:
            expected[slot // 4, slot % 4] = x[t]
    np.testing.assert_array_equal(cache, expected)
    k = np.arange(2 * 3 * 2 * 4, dtype=np.float64).reshape(2, 3, 2, 4)
    for paged in (False, True):
        kc = np.full((6 if paged else 3, 4 if paged else 12, 2, 4), -1.0)
        table = np.array([[5, 0, 2], [1, 4, 3], [2, 3, 1]]) if paged else None
        expected = kc.copy()
        for b, row in enumerate([1, 0]):
            for j in range(3):
                pos = [3, 6][b] + j
                block, offset = (int(table[b, pos // 4]), pos % 4) if paged else (row, pos)
                expected[block, offset] = k[b, j]
        oracle.append_kvcache(k, kc, np.array([3, 6]), cache_batch_idx=np.array([1, 0]),
                              block_table=table)
        np.testing.assert_array_equal(kc, expected)
