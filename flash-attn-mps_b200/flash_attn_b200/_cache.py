"""KV-cache writes over the CUDA library (mirrors flash_attn_mps/_cache.py).

* ``store_kvcache`` (reference ``_cache.py:67-85``): slot scatter of new K/V
  rows, bit-exact copies or saturating FP8 E4M3 codes of ``x / scale[h]``;
  K and V go out in one launch.
* ``append_kvcache`` (``_cache.py:99-127``): append at the old lengths of a
  continuous or paged cache; lengths are not modified.
* ``rotary`` (``_cache.py:130-155``): RoPE of Q and new K at their absolute
  positions, interleaved or split-half.
"""

import torch

from . import _capi

_FLOATS = (torch.float16, torch.bfloat16, torch.float32)


def _cuda(*tensors):
    if any(t.device.type != "cuda" for t in tensors if t is not None):
        raise ValueError("operations require CUDA tensors")


def _scale(scale, heads, device):
    """Scalar or per-head float32 scale (reference _cache.py:55-59)."""
    if scale is None:
        return None
    scale = torch.as_tensor(scale, device=device, dtype=torch.float32)
    if scale.numel() not in (1, heads):
        raise ValueError("scale must be scalar or have one value per KV head")
    return scale.reshape(-1)


def _check_cache_dtype(x, cache):
    if x.dtype not in _FLOATS:
        raise TypeError("input dtype must be float16, bfloat16 or float32")
    if cache.dtype != torch.float8_e4m3fn and cache.dtype != x.dtype:
        raise TypeError("cache dtype must match input or be float8_e4m3fn")


def store_kvcache(k, v, k_cache, v_cache, slot_mapping, *, k_scale=None, v_scale=None):
    """Scatter [tokens, heads, dim] K/V into physical cache slots; -1 skips."""
    _cuda(k, v, k_cache, v_cache, slot_mapping)
    if k.ndim != 3 or v.ndim != 3 or k.shape[:2] != v.shape[:2]:
        raise ValueError("K/V must have matching [tokens, heads, dim] shapes")
    if (slot_mapping.ndim != 1 or slot_mapping.numel() != k.shape[0]
            or slot_mapping.dtype not in (torch.int32, torch.int64)):
        raise ValueError("slot_mapping must be int32/int64 with one slot per token")
    for x, cache in ((k, k_cache), (v, v_cache)):
        if cache.ndim != 4 or cache.shape[2:] != x.shape[1:]:
            raise ValueError("cache must have shape [blocks, block_size, heads, dim]")
        _check_cache_dtype(x, cache)
    ks = _scale(k_scale, k.shape[1], k.device) if k_cache.dtype == torch.float8_e4m3fn else None
    vs = _scale(v_scale, v.shape[1], v.device) if v_cache.dtype == torch.float8_e4m3fn else None
    if not k.numel() and not v.numel():
        return
    t = _capi.tensor
    args = [t(k), t(v), t(k_cache), t(v_cache), t(slot_mapping), t(ks), t(vs)]
    lib = _capi.library()
    _capi.check(lib.fa_store_kvcache(*map(_capi.ref, args), _capi.stream_of(k.device)))


def _integers(value, count, device):
    if value is None:
        value = 0
    value = torch.as_tensor(value, dtype=torch.int32, device=device)
    if value.numel() == 1:
        value = value.reshape(1).expand(count)
    if value.numel() != count:
        raise ValueError(f"expected {count} integer values")
    return value.contiguous()


def append_kvcache(k, v, k_cache, v_cache, cache_seqlens, *, cache_batch_idx=None,
                   cache_leftpad=None, block_table=None, k_scale=None, v_scale=None):
    """Append [batch, new_tokens, heads, dim] K/V without changing lengths.

    FA2 lengths are physical exclusive ends that already include any left
    padding, so new tokens land at length + j (never length + leftpad + j).
    """
    _cuda(k, v, k_cache, v_cache, block_table)
    if k.ndim != 4 or v.ndim != 4 or k.shape[:3] != v.shape[:3]:
        raise ValueError("K/V must have matching [batch, new_tokens, heads, dim] shapes")
    batch = k.shape[0]
    lengths = _integers(cache_seqlens, batch, k.device)
    remap = block_table is None and cache_batch_idx is not None
    indices = _integers(cache_batch_idx, batch, k.device) if remap else None
    if cache_leftpad is not None:
        _integers(cache_leftpad, batch, k.device)
    if block_table is not None:
        if block_table.ndim != 2:
            raise ValueError("block_table must have shape [cache_batch, blocks_per_sequence]")
        block_table = block_table.to(torch.int32)
    for x, cache in ((k, k_cache), (v, v_cache)):
        if cache.ndim != 4 or cache.shape[2:] != x.shape[2:]:
            raise ValueError("cache must have shape [rows, capacity, heads, dim]")
        _check_cache_dtype(x, cache)
    ks = _scale(k_scale, k.shape[2], k.device) if k_cache.dtype == torch.float8_e4m3fn else None
    vs = _scale(v_scale, v.shape[2], v.device) if v_cache.dtype == torch.float8_e4m3fn else None
    if not k.numel() and not v.numel():
        return
    t = _capi.tensor
    args = [t(k), t(v), t(k_cache), t(v_cache), t(lengths), t(indices), t(block_table), t(ks), t(vs)]
    lib = _capi.library()
    _capi.check(lib.fa_append_kvcache(*map(_capi.ref, args), _capi.stream_of(k.device)))


def rotary(q, k, cos, sin, cache_seqlens, *, rotary_interleaved=True, causal=False,
           window_size=(-1, -1)):
    """Rotate new K at old_length + j and Q at its causal/local absolute position."""
    _cuda(q, k, cos, sin)
    if q.ndim != 4 or (k is not None and (k.ndim != 4 or q.shape[0] != k.shape[0])):
        raise ValueError("Q/K must have shape [batch, tokens, heads, dim]")
    if cos.ndim != 2 or sin.shape != cos.shape or cos.shape[1] * 2 > q.shape[-1]:
        raise ValueError("rotary cosine/sine must have shape [positions, rotary_dim/2]")
    cosine, sine = cos.float(), sin.float()
    lengths = _integers(cache_seqlens, q.shape[0], q.device)
    outputs = []
    lib = _capi.library()
    for x, advance in ((q, bool(causal) or tuple(window_size) != (-1, -1)), (k, True)):
        if x is None:
            outputs.append(None)
            continue
        if cos.shape[1] * 2 > x.shape[-1]:
            raise ValueError("rotary dimension exceeds head dimension")
        if x.dtype not in _FLOATS:
            raise TypeError("input dtype must be float16, bfloat16 or float32")
        output = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        if x.numel():
            t = _capi.tensor
            args = [t(x), t(output), t(cosine), t(sine), t(lengths)]
            _capi.check(lib.fa_rotary(*map(_capi.ref, args), int(bool(rotary_interleaved)),
                                      int(advance), _capi.stream_of(x.device)))
        outputs.append(output)
    return tuple(outputs)


def rotary_append_kvcache(q, k, v, k_cache, v_cache, cos, sin, cache_seqlens, *, rotary_interleaved=True,
                          causal=False, window_size=(-1, -1), cache_batch_idx=None, cache_leftpad=None,
                          block_table=None, k_scale=None, v_scale=None):
    """``rotary`` of Q and the new K followed by ``append_kvcache`` of (rotated K, V), in one launch.

    Same validation and the same values as the two calls in sequence (the
    rotated K is rounded to its dtype before it is appended); returns the
    rotated Q. ``flash_attn_with_kvcache`` uses it when it gets rotary tables
    and new K/V.
    """
    _cuda(q, k, v, cos, sin, k_cache, v_cache, block_table)
    if q.ndim != 4 or k.ndim != 4 or q.shape[0] != k.shape[0]:
        raise ValueError("Q/K must have shape [batch, tokens, heads, dim]")
    if cos.ndim != 2 or sin.shape != cos.shape or cos.shape[1] * 2 > q.shape[-1]:
        raise ValueError("rotary cosine/sine must have shape [positions, rotary_dim/2]")
    if cos.shape[1] * 2 > k.shape[-1]:
        raise ValueError("rotary dimension exceeds head dimension")
    for x in (q, k):
        if x.dtype not in _FLOATS:
            raise TypeError("input dtype must be float16, bfloat16 or float32")
    if cos.dtype not in _FLOATS or sin.dtype != cos.dtype:
        cos, sin = cos.float(), sin.float()
    if v.ndim != 4 or k.shape[:3] != v.shape[:3]:
        raise ValueError("K/V must have matching [batch, new_tokens, heads, dim] shapes")
    batch = k.shape[0]
    lengths = _integers(cache_seqlens, batch, k.device)
    remap = block_table is None and cache_batch_idx is not None
    indices = _integers(cache_batch_idx, batch, k.device) if remap else None
    if cache_leftpad is not None:
        _integers(cache_leftpad, batch, k.device)
    if block_table is not None:
        if block_table.ndim != 2:
            raise ValueError("block_table must have shape [cache_batch, blocks_per_sequence]")
        block_table = block_table.to(torch.int32)
    for x, cache in ((k, k_cache), (v, v_cache)):
        if cache.ndim != 4 or cache.shape[2:] != x.shape[2:]:
            raise ValueError("cache must have shape [rows, capacity, heads, dim]")
        _check_cache_dtype(x, cache)
    ks = _scale(k_scale, k.shape[2], k.device) if k_cache.dtype == torch.float8_e4m3fn else None
    vs = _scale(v_scale, v.shape[2], v.device) if v_cache.dtype == torch.float8_e4m3fn else None
    q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    advance_q = bool(causal) or tuple(window_size) != (-1, -1)
    t = _capi.tensor
    args = [t(q), t(q_out), t(k), t(v), t(k_cache), t(v_cache), t(lengths), t(indices), t(block_table),
            t(ks), t(vs), t(cos), t(sin)]
    lib = _capi.library()
    _capi.check(lib.fa_rotary_append_kvcache(*map(_capi.ref, args), int(bool(rotary_interleaved)),
                                             int(advance_q), _capi.stream_of(q.device)))
    return q_out
