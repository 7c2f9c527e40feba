"""KV-cache writes restated in numpy (oracle; test infrastructure only).

* ``store_kvcache`` follows ``flash_attn_mps/kernels/cache.metal:20-39`` and
  ``_cache.py:67-85``: ``cache[slot // P, slot % P, h, :] = x[t, h, :]``,
  or the saturating E4M3 code of ``float32(x) / float32(scale[h])`` for an FP8
  cache; slots < 0 or >= N*P are skipped.
* ``append_kvcache`` follows ``cache.metal:41-56`` and ``_cache.py:99-127``:
  new token j of request b goes to position ``lengths[b] + j`` of cache row
  ``cache_batch_idx[b]`` (continuous) or of page ``block_table[b, pos // P]``
  (paged); out-of-range rows, positions and pages are skipped.
* ``rotary`` follows ``cache.metal:58-76`` and ``_cache.py:130-155``: RoPE at
  ``lengths[b] + j`` (Q advances with j only when causal or local), in
  interleaved or split-half pairing; dims beyond ``2 * rotary_dim/2`` copy.

Arrays are float numpy arrays (caches of an FP8 dtype are uint8 codes).
"""

import numpy as np

from .fp8 import e4m3_encode


def _scales(scale, heads):
    if scale is None:
        return np.ones(heads, dtype=np.float32)
    s = np.asarray(scale, dtype=np.float32).reshape(-1)
    return np.broadcast_to(s, (heads,)) if s.size == 1 else s


def store_kvcache(x, cache, slots, scale=None, fp8=False):
    """Write x [T,H,D] into cache [N,P,H,D] in place and return it."""
    x = np.asarray(x)
    tokens, heads = x.shape[0], x.shape[1]
    blocks, page = cache.shape[0], cache.shape[1]
    s = _scales(scale, heads)
    for t, slot in enumerate(np.asarray(slots).reshape(-1).tolist()):
        if slot < 0 or slot >= blocks * page:
            continue
        if fp8:
            cache[slot // page, slot % page] = e4m3_encode(
                x[t].astype(np.float32) / s[:, None])
        else:
            cache[slot // page, slot % page] = x[t]
    return cache


def append_kvcache(x, cache, lengths, cache_batch_idx=None, block_table=None,
                   scale=None, fp8=False):
    """Append x [B,Snew,H,D] at the old lengths; lengths are not modified."""
    x = np.asarray(x)
    batch, snew, heads = x.shape[:3]
    page = cache.shape[1]
    lengths = np.broadcast_to(np.asarray(lengths).reshape(-1), (batch,))
    paged = block_table is not None
    remap = not paged and cache_batch_idx is not None
    rows = cache.shape[0] if not paged else np.asarray(block_table).shape[0]
    idx = None if not remap else np.broadcast_to(np.asarray(cache_batch_idx).reshape(-1), (batch,))
    table = None if not paged else np.asarray(block_table)
    capacity = table.shape[1] * page if paged else page
    s = _scales(scale, heads)
    for b in range(batch):
        row = int(idx[b]) if remap else b
        for j in range(snew):
            pos = int(lengths[b]) + j
            if row < 0 or row >= rows or pos < 0 or pos >= capacity:
                continue
            block = int(table[row, pos // page]) if paged else row
            offset = pos % page if paged else pos
            if block < 0 or block >= cache.shape[0]:
                continue
            value = x[b, j]
            if fp8:
                value = e4m3_encode(value.astype(np.float32) / s[:, None])
            cache[block, offset] = value
    return cache


def rotary(x, cos, sin, lengths, interleaved=True, advance=True):
    """Rotate x [B,S,H,D] at positions lengths[b] (+ j when advance)."""
    x = np.asarray(x, dtype=np.float64)
    cos = np.asarray(cos, dtype=np.float64)
    sin = np.asarray(sin, dtype=np.float64)
    half = cos.shape[1]
    batch, seq = x.shape[:2]
    lengths = np.broadcast_to(np.asarray(lengths).reshape(-1), (batch,))
    out = x.copy()
    for b in range(batch):
        for j in range(seq):
            pos = int(lengths[b]) + (j if advance else 0)
            c, s = cos[pos], sin[pos]
            if interleaved:
                a, z = x[b, j, :, 0:2 * half:2], x[b, j, :, 1:2 * half:2]
                out[b, j, :, 0:2 * half:2] = a * c - z * s
                out[b, j, :, 1:2 * half:2] = z * c + a * s
            else:
                a, z = x[b, j, :, :half], x[b, j, :, half:2 * half]
                out[b, j, :, :half] = a * c - z * s
                out[b, j, :, half:2 * half] = z * c + a * s
    return out
