"""Inference-only FlashAttention-2 interfaces for CUDA (B200) tensors.

Public names, signatures, tensor layouts and validation errors follow the
reference's ``flash_attn_mps/interface.py`` (FA2 inference contract,
``docs/contracts.md``). All attention math runs in the CUDA library; this
module reshapes dense/packed inputs to the packed varlen form, validates
arguments before anything is launched, and orchestrates RoPE -> append ->
attention for ``flash_attn_with_kvcache``.
"""

from dataclasses import dataclass
from functools import lru_cache

import torch

_INT32 = torch.int32


@lru_cache(maxsize=64)
def _uniform_offsets(batch, length, device):
    """Immutable cu_seqlens shared by layers with the same dense batch shape."""
    offsets = torch.arange(batch + 1, device=device, dtype=_INT32)
    return offsets if length == 1 else offsets * length


@dataclass(frozen=True)
class MaskSpec:
    """A supported vLLM mask semantic (not an executable callback).

    kind 1 = multimodal bidirectional prefix ranges, kind 2 = rolling SWA with
    an always-visible prefix (reference interface.py:49-55).
    """

    kind: int
    sliding_window_left: int = -1
    clamp_prefix_to_window: bool = False


def _reshape(x, *shape):
    # Reshape FP8 through its bytes so a required copy never reinterprets values.
    if x.dtype == torch.float8_e4m3fn:
        return x.view(torch.uint8).reshape(*shape).view(x.dtype)
    return x.reshape(*shape)


def _inference_only(dropout_p, return_attn_probs, *tensors):
    if dropout_p != 0:
        raise NotImplementedError("flash-attn-b200 implements inference; dropout_p must be 0")
    if return_attn_probs:
        raise NotImplementedError(
            "return_attn_probs is a training/debug interface; use return_softmax_lse=True")
    if any(t is not None and t.requires_grad for t in tensors):
        raise NotImplementedError("flash-attn-b200 implements inference without backward")


def _on(tensor, device):
    return tensor is not None and tensor.device == device


def _validate(q, k, v, cu_q, cu_k, used_k, block_table, out=None):
    """Tensor-contract checks of reference interface.py:77-115 (CUDA wording)."""
    for name, tensor in (("q", q), ("k", k), ("v", v)):
        if tensor.device.type != "cuda":
            raise ValueError(f"{name} must be a CUDA tensor")
    if q.ndim != 3 or k.ndim not in (3, 4) or v.ndim != k.ndim:
        raise ValueError("expected q [T,H,D] and matching packed or paged K/V")
    if k.shape[:-1] != v.shape[:-1] or q.shape[-1] != k.shape[-1]:
        raise ValueError("Q/K head dimensions and K/V token/head dimensions must match")
    if k.shape[-2] == 0 or q.shape[-2] % k.shape[-2]:
        raise ValueError("query heads must be divisible by KV heads")
    if not (1 <= q.shape[-1] <= 512 and 1 <= v.shape[-1] <= 512):
        raise ValueError("head dimensions must be between 1 and 512")
    if cu_q.ndim != 1 or cu_q.numel() < 1 or cu_q.dtype != _INT32:
        raise ValueError("cu_seqlens_q must be int32 [batch+1]")
    batch = cu_q.numel() - 1
    if (cu_k is None) == (used_k is None):
        raise ValueError("provide exactly one of cu_seqlens_k and seqused_k")
    for name, tensor, shape in (("cu_seqlens_q", cu_q, (batch + 1,)),
                                ("cu_seqlens_k", cu_k, (batch + 1,)),
                                ("seqused_k", used_k, (batch,))):
        if tensor is not None and (not _on(tensor, q.device) or tensor.dtype != _INT32
                                   or tuple(tensor.shape) != shape):
            raise ValueError(f"{name} must be a CUDA int32 tensor of shape {shape}")
    if block_table is not None:
        if (k.ndim != 4 or block_table.ndim != 2 or block_table.shape[0] != batch
                or block_table.dtype != _INT32 or not _on(block_table, q.device)):
            raise ValueError("paged KV requires a CUDA int32 block_table [B,P]")
    elif k.ndim != 3:
        raise ValueError("4D KV requires block_table")
    if out is not None and (tuple(out.shape) != (q.shape[0], q.shape[1], v.shape[-1])
                            or out.device != q.device):
        raise ValueError("out must have shape [total_q, query_heads, value_head_dim] on CUDA")


def _check_features(q, k, batch, causal, window_size, softcap, num_splits, max_seqlen_q,
                    max_seqlen_k, mask_mod, aux_tensors, alibi_slopes, s_aux, descales):
    """Feature checks of reference interface.py:127-160."""
    heads, kvheads = q.shape[1], k.shape[-2]
    if len(window_size) != 2 or min(window_size) < -1:
        raise ValueError("window_size must contain two bounds >= -1")
    if softcap < 0 or num_splits < 0 or max_seqlen_q < 0 or max_seqlen_k < 0:
        raise ValueError("softcap, lengths, and num_splits must be nonnegative")
    if mask_mod is not None and not isinstance(mask_mod, MaskSpec):
        raise TypeError("mask_mod must be an mm_prefix_mask() or rswa_mask() descriptor")
    if torch.is_tensor(causal) and (tuple(causal.shape) != (batch,) or causal.dtype != torch.bool
                                    or causal.device != q.device):
        raise ValueError("dynamic causal must be a CUDA bool [B] tensor")
    for name, tensor in descales:
        if tensor is not None and (tuple(tensor.shape) != (batch, kvheads)
                                   or tensor.dtype != torch.float32 or tensor.device != q.device):
            raise ValueError(f"{name} must be a CUDA float32 [B,Hkv] tensor")
    if alibi_slopes is not None and (
            tuple(alibi_slopes.shape) not in ((heads,), (batch, heads))
            or alibi_slopes.device != q.device or alibi_slopes.dtype != torch.float32):
        raise ValueError("alibi_slopes must be CUDA float32 [Hq] or [B,Hq]")
    if s_aux is not None and (tuple(s_aux.shape) != (heads,) or s_aux.device != q.device):
        raise ValueError("s_aux must be a CUDA [Hq] tensor")
    if mask_mod is not None:
        if mask_mod.kind not in (1, 2) or aux_tensors is None or len(aux_tensors) != 2:
            raise ValueError("a supported mask requires its two auxiliary tensors")
        shapes = ((q.shape[0], 2), (batch + 1,)) if mask_mod.kind == 1 else ((batch,), (1,))
        for tensor, shape in zip(aux_tensors, shapes):
            if tuple(tensor.shape) != shape or tensor.dtype != _INT32 or tensor.device != q.device:
                raise ValueError(f"mask auxiliary tensor must be CUDA int32 {shape}")
    elif aux_tensors is not None:
        raise ValueError("aux_tensors require a mask descriptor")


def _run(q, k, v, *, cu_seqlens_q, cu_seqlens_k=None, seqused_k=None,
         max_seqlen_q, max_seqlen_k, block_table=None, softmax_scale=None,
         causal=False, window_size=(-1, -1), alibi_slopes=None, softcap=0.0,
         s_aux=None, q_descale=None, k_descale=None, v_descale=None, out=None,
         num_splits=0, mask_mod=None, aux_tensors=None, leftpad_k=None,
         deterministic=False, cp_world_size=1, cp_rank=0, cp_tot_seqused_k=None):
    """Validate everything, then run the packed attention core."""
    _inference_only(0, False, q, k, v, alibi_slopes, s_aux, q_descale, k_descale, v_descale, out)
    _validate(q, k, v, cu_seqlens_q, cu_seqlens_k, seqused_k, block_table, out)
    batch = cu_seqlens_q.numel() - 1
    _check_features(q, k, batch, causal, window_size, softcap, num_splits, max_seqlen_q,
                    max_seqlen_k, mask_mod, aux_tensors, alibi_slopes, s_aux,
                    (("q_descale", q_descale), ("k_descale", k_descale), ("v_descale", v_descale)))
    from ._attention import attention
    return attention(
        q, k, v, cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k, seqused_k=seqused_k,
        max_seqlen_q=max_seqlen_q, max_seqlen_k=max_seqlen_k, block_table=block_table,
        softmax_scale=softmax_scale, causal=causal, window_size=window_size,
        alibi_slopes=alibi_slopes, softcap=softcap, s_aux=s_aux, q_descale=q_descale,
        k_descale=k_descale, v_descale=v_descale, out=out, num_splits=num_splits,
        mask_mod=mask_mod, aux_tensors=aux_tensors, leftpad_k=leftpad_k,
        deterministic=deterministic,
        cp_world_size=cp_world_size, cp_rank=cp_rank, cp_tot_seqused_k=cp_tot_seqused_k)


def flash_attn_varlen_func(
    q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
    dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
    softcap=0.0, alibi_slopes=None, deterministic=False, return_attn_probs=False,
    block_table=None, *, return_softmax_lse=False, out=None,
):
    """Packed or paged variable-length attention with lower-right causality."""
    _inference_only(dropout_p, return_attn_probs, q, k, v)
    if block_table is not None and (k.ndim != 4 or k.shape[1] % 16):
        raise ValueError("paged KV requires a page size divisible by 16")
    result, lse = _run(
        q, k, v, cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k,
        max_seqlen_q=max_seqlen_q, max_seqlen_k=max_seqlen_k, block_table=block_table,
        softmax_scale=softmax_scale, causal=causal, window_size=window_size, softcap=softcap,
        alibi_slopes=alibi_slopes, num_splits=1 if deterministic else 0, out=out,
        deterministic=deterministic)
    return (result, lse) if return_softmax_lse else result


def flash_attn_func(
    q, k, v, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
    softcap=0.0, alibi_slopes=None, deterministic=False, return_attn_probs=False, *,
    return_softmax_lse=False,
):
    """Dense attention: Q [B,Sq,Hq,D], K/V [B,Sk,Hkv,D]; LSE [B,Hq,Sq]."""
    if (q.ndim != 4 or k.ndim != 4 or v.ndim != 4 or q.shape[0] != k.shape[0]
            or k.shape[:3] != v.shape[:3]):
        raise ValueError("dense attention requires matching 4D batches")
    batch, sq, heads = q.shape[:3]
    sk = k.shape[1]
    out, lse = flash_attn_varlen_func(
        _reshape(q, -1, *q.shape[2:]), _reshape(k, -1, *k.shape[2:]),
        _reshape(v, -1, *v.shape[2:]), _uniform_offsets(batch, sq, q.device),
        _uniform_offsets(batch, sk, q.device), sq, sk, dropout_p, softmax_scale, causal,
        window_size, softcap, alibi_slopes, deterministic, return_attn_probs,
        return_softmax_lse=True)
    out = out.reshape(batch, sq, heads, v.shape[-1])
    lse = lse.reshape(heads, batch, sq).transpose(0, 1)
    return (out, lse) if return_softmax_lse else out


def flash_attn_qkvpacked_func(qkv, *args, **kwargs):
    """Dense QKV [B,S,3,H,D]."""
    if qkv.ndim != 5 or qkv.shape[2] != 3:
        raise ValueError("qkv must have shape [B,S,3,H,D]")
    return flash_attn_func(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], *args, **kwargs)


def flash_attn_kvpacked_func(q, kv, *args, **kwargs):
    """Dense Q [B,Sq,Hq,D], KV [B,Sk,2,Hkv,D]."""
    if kv.ndim != 5 or kv.shape[2] != 2:
        raise ValueError("kv must have shape [B,S,2,H,D]")
    return flash_attn_func(q, kv[:, :, 0], kv[:, :, 1], *args, **kwargs)


def flash_attn_varlen_qkvpacked_func(qkv, cu_seqlens, max_seqlen, *args, **kwargs):
    """Packed QKV [T,3,H,D]."""
    if qkv.ndim != 4 or qkv.shape[1] != 3:
        raise ValueError("qkv must have shape [T,3,H,D]")
    return flash_attn_varlen_func(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu_seqlens, cu_seqlens,
                                  max_seqlen, max_seqlen, *args, **kwargs)


def flash_attn_varlen_kvpacked_func(q, kv, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                    max_seqlen_k, *args, **kwargs):
    """Packed KV [T,2,Hkv,D]."""
    if kv.ndim != 4 or kv.shape[1] != 2:
        raise ValueError("kv must have shape [T,2,H,D]")
    return flash_attn_varlen_func(q, kv[:, 0], kv[:, 1], cu_seqlens_q, cu_seqlens_k,
                                  max_seqlen_q, max_seqlen_k, *args, **kwargs)


def flash_attn_with_kvcache(
    q, k_cache, v_cache, k=None, v=None, rotary_cos=None, rotary_sin=None,
    cache_seqlens=None, cache_batch_idx=None, cache_leftpad=None, block_table=None,
    softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0,
    rotary_interleaved=True, alibi_slopes=None, num_splits=0, return_softmax_lse=False,
):
    """Attention over a cache, optionally appending KV at the supplied old lengths.

    Cache lengths are not mutated: they are the physical exclusive end before
    the append. ``cache_leftpad`` excludes a leading portion of a continuous
    cache from attention without moving append positions.
    """
    _inference_only(0, False, q, k, v, k_cache, v_cache)
    if q.ndim != 4 or k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("q and KV caches must be 4D")
    if (k is None) != (v is None):
        raise ValueError("k and v must be provided together")
    if block_table is not None and cache_leftpad is not None:
        raise ValueError("FlashAttention does not combine paged cache with cache_leftpad")
    if block_table is not None and k_cache.shape[1] % 16:
        raise ValueError("paged KV requires a page size divisible by 16")
    batch, sq = q.shape[:2]
    if cache_seqlens is None:
        if k is not None or block_table is not None:
            raise ValueError("cache_seqlens is required for append or paged cache")
        cache_seqlens = k_cache.shape[1]
    if isinstance(cache_seqlens, int):
        lengths = torch.full((batch,), cache_seqlens, device=q.device, dtype=_INT32)
    else:
        lengths = cache_seqlens
    if tuple(lengths.shape) != (batch,) or lengths.dtype != _INT32 or lengths.device != q.device:
        raise ValueError("cache_seqlens must be an int or CUDA int32 [B]")
    if (rotary_cos is None) != (rotary_sin is None):
        raise ValueError("rotary_cos and rotary_sin must be provided together")
    if rotary_cos is not None and k is None:
        raise ValueError("rotary embedding requires new k and v")
    if k is not None:
        if k.ndim != 4 or v.ndim != 4 or k.shape[0] != batch or v.shape[:3] != k.shape[:3]:
            raise ValueError("new k/v must have matching [B,Snew,Hkv,D] dimensions")
        if rotary_cos is not None:
            # RoPE of Q and new K fused with the append (one launch, same values).
            from ._cache import rotary_append_kvcache
            q = rotary_append_kvcache(q, k, v, k_cache, v_cache, rotary_cos, rotary_sin, lengths,
                                      rotary_interleaved=rotary_interleaved, causal=causal,
                                      window_size=window_size, cache_batch_idx=cache_batch_idx,
                                      cache_leftpad=cache_leftpad, block_table=block_table)
        else:
            from ._cache import append_kvcache
            append_kvcache(k, v, k_cache, v_cache, lengths, cache_batch_idx=cache_batch_idx,
                           cache_leftpad=cache_leftpad, block_table=block_table)
        lengths = lengths + k.shape[1]
    if block_table is None:
        rows = cache_batch_idx
        if rows is None:
            rows = torch.arange(batch, device=q.device, dtype=_INT32)
        # A continuous cache is a paged cache with one page per row.
        table = rows.to(_INT32).reshape(batch, 1)
        max_k = k_cache.shape[1]
    else:
        # The page table already selects physical storage for each query row.
        table = block_table
        max_k = table.shape[1] * k_cache.shape[1]
    if cache_leftpad is not None:
        lengths = lengths - cache_leftpad
    out, lse = _run(
        _reshape(q, -1, *q.shape[2:]), k_cache, v_cache,
        cu_seqlens_q=_uniform_offsets(batch, sq, q.device), seqused_k=lengths,
        max_seqlen_q=sq, max_seqlen_k=max_k, block_table=table, softmax_scale=softmax_scale,
        causal=causal, window_size=window_size, alibi_slopes=alibi_slopes, softcap=softcap,
        num_splits=num_splits, leftpad_k=cache_leftpad)
    out = out.reshape(batch, sq, q.shape[2], v_cache.shape[-1])
    lse = lse.reshape(q.shape[2], batch, sq).transpose(0, 1)
    return (out, lse) if return_softmax_lse else out
