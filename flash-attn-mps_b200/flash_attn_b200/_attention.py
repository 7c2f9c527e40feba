"""Attention entry over the CUDA library (mirrors flash_attn_mps/_attention.py).

``attention`` keeps the reference signature and checks
(``flash_attn_mps/_attention.py:88-161``) and returns ``(out, lse)`` with the
natural-log LSE in ``[heads, total_q]`` order. Kernel choice, split-KV and the
partial merge happen inside ``fa_attention_fwd``; this module only validates,
allocates the caller-visible outputs and the split workspace, and passes
pointers, strides and the current stream. No tensor value is read on the host.
"""

import torch

from . import _capi

_SUPPORTED = (torch.float16, torch.bfloat16, torch.float32, torch.float8_e4m3fn)
_OUT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _launch(args, device):
    """Single point where attention work is handed to the GPU."""
    lib = _capi.library()
    _capi.check(lib.fa_attention_fwd(_capi.ref(args), _capi.stream_of(device)))


def _f32(t, device):
    if t is None:
        return None
    return t.to(device=device, dtype=torch.float32)


def _i32(t, device):
    if t is None:
        return None
    return t.to(device=device, dtype=torch.int32)


def build_args(q, k, v, out, lse, *, cu_seqlens_q, cu_seqlens_k, seqused_k, max_seqlen_q,
               max_seqlen_k, block_table, softmax_scale, causal, window_size, alibi_slopes,
               softcap, s_aux, q_descale, k_descale, v_descale, num_splits, mask_mod,
               aux_tensors, leftpad_k, deterministic, cp_world_size=1, cp_rank=0,
               cp_tot_seqused_k=None):
    """Fill the C argument struct; returns it plus the tensors it points into."""
    device = q.device
    keep = []

    def t(x):
        if x is not None:
            keep.append(x)
        return _capi.tensor(x)

    a = _capi.AttentionArgs()
    a.q, a.k, a.v, a.out, a.lse = t(q), t(k), t(v), t(out), t(lse)
    a.cu_seqlens_q = t(cu_seqlens_q)
    a.cu_seqlens_k = t(cu_seqlens_k)
    a.seqused_k = t(seqused_k)
    a.block_table = t(block_table)
    a.leftpad_k = t(_i32(leftpad_k, device))
    if torch.is_tensor(causal):
        a.causal_per_seq = t(causal.to(device=device, dtype=torch.bool))
        a.causal = 0
    else:
        a.causal = int(bool(causal))
    a.alibi_slopes = t(_f32(alibi_slopes, device))
    a.s_aux = t(s_aux if s_aux is None or s_aux.dtype in _OUT_DTYPES else _f32(s_aux, device))
    a.q_descale = t(_f32(q_descale, device))
    a.k_descale = t(_f32(k_descale, device))
    a.v_descale = t(_f32(v_descale, device))
    kind = 0 if mask_mod is None else int(mask_mod.kind)
    a.mask_kind = kind
    a.mask_window = -1 if mask_mod is None else int(mask_mod.sliding_window_left)
    a.mask_clamp = 0 if mask_mod is None else int(bool(mask_mod.clamp_prefix_to_window))
    if kind:
        a.mask_aux0 = t(_i32(aux_tensors[0], device))
        a.mask_aux1 = t(_i32(aux_tensors[1], device))
    a.batch = cu_seqlens_q.numel() - 1
    a.max_seqlen_q = int(max_seqlen_q)
    a.max_seqlen_k = int(max_seqlen_k)
    dq = q.shape[-1]
    a.softmax_scale = float(softmax_scale if softmax_scale is not None else dq ** -0.5)
    a.softcap = float(softcap)
    a.window_left, a.window_right = int(window_size[0]), int(window_size[1])
    a.num_splits = int(num_splits)
    a.deterministic = int(bool(deterministic))
    if cp_world_size > 1:
        a.cp_world_size, a.cp_rank = int(cp_world_size), int(cp_rank)
        a.cp_tot_seqused_k = t(_i32(cp_tot_seqused_k, device))
    return a, keep


def run(q, k, v, out, lse, **kw):
    """Size and attach the split workspace, then launch."""
    args, keep = build_args(q, k, v, out, lse, **kw)
    lib = _capi.library()
    size = _capi.ctypes.c_size_t(0)
    _capi.check(lib.fa_attention_workspace_size(_capi.ref(args), _capi.ref(size)))
    if size.value:
        workspace = torch.empty(size.value, dtype=torch.uint8, device=q.device)
        keep.append(workspace)
        args.workspace = _capi.tensor(workspace)
    _launch(args, q.device)
    return out, lse


def attention(
    q, k, v, *, cu_seqlens_q, cu_seqlens_k=None, seqused_k=None,
    max_seqlen_q, max_seqlen_k, block_table=None, softmax_scale=None,
    causal=False, window_size=(-1, -1), alibi_slopes=None, softcap=0.,
    s_aux=None, q_descale=None, k_descale=None, v_descale=None, out=None,
    num_splits=0, mask_mod=None, aux_tensors=None, leftpad_k=None, deterministic=False,
    cp_world_size=1, cp_rank=0, cp_tot_seqused_k=None, lse=None,
):
    """Return packed output and natural-log LSE in ``[heads, total_q]`` order.

    ``out`` and ``lse`` (fp32 ``[heads, total_q]``, any strides) may be given
    to receive the result in place.

    ``cp_world_size > 1`` (context parallelism): k/v hold this rank's strided
    share of every sequence (local key j = global position
    j * cp_world_size + cp_rank), ``cp_tot_seqused_k`` the global KV lengths;
    the result is this rank's partial state for an LSE merge across ranks.
    """
    if q.device.type != "cuda" or k.device != q.device or v.device != q.device:
        raise ValueError("q, k and v must be on the same CUDA device")
    if q.ndim != 3 or k.ndim not in (3, 4) or v.ndim != k.ndim:
        raise ValueError("q must be packed 3-D; k/v must be packed 3-D or paged 4-D")
    if any(x.dtype not in _SUPPORTED for x in (q, k, v)):
        raise TypeError("attention supports FP16, BF16, FP32 and FP8 E4M3FN")
    tokens, heads, dq = q.shape
    kvheads, dv = k.shape[-2], v.shape[-1]
    if not (1 <= dq <= 512 and 1 <= dv <= 512):
        raise ValueError("query/key and value head dimensions must be in 1..512")
    if k.shape[-1] != dq or v.shape[:-1] != k.shape[:-1]:
        raise ValueError("key/value shapes must agree except for their last dimension")
    if heads < 1 or kvheads < 1 or heads % kvheads:
        raise ValueError("query heads must be a positive multiple of KV heads")
    if (k.ndim == 4) != (block_table is not None):
        raise ValueError("paged 4-D KV requires block_table; packed 3-D KV does not")
    if cu_seqlens_k is None and seqused_k is None:
        raise ValueError("cu_seqlens_k or seqused_k is required")
    if num_splits < 0:
        raise ValueError("num_splits must be nonnegative")
    if cp_world_size > 1:
        if not 0 <= cp_rank < cp_world_size:
            raise ValueError("cp_rank must be in [0, cp_world_size)")
        if (cp_tot_seqused_k is None or cp_tot_seqused_k.dtype != torch.int32 or cp_tot_seqused_k.ndim != 1
                or cp_tot_seqused_k.numel() != cu_seqlens_q.numel() - 1 or cp_tot_seqused_k.device != q.device):
            raise ValueError("context parallelism needs cp_tot_seqused_k as CUDA int32 [num_seqs]")
    out_dtype = torch.float16 if q.dtype == torch.float8_e4m3fn else q.dtype
    if out is None:
        out = torch.empty((tokens, heads, dv), dtype=out_dtype, device=q.device)
    elif tuple(out.shape) != (tokens, heads, dv) or out.device != q.device:
        raise ValueError("out must have shape [total_q, query_heads, value_dim] on CUDA")
    if out.dtype not in _OUT_DTYPES:
        raise TypeError("out must have FP16, BF16 or FP32 dtype")
    if tokens == 0:
        return out, torch.empty((heads, 0), device=q.device, dtype=torch.float32)
    if max_seqlen_q <= 0 or max_seqlen_k < 0:
        raise ValueError("nonempty q requires positive max_seqlen_q and nonnegative max_seqlen_k")
    if cu_seqlens_q.numel() - 1 < 1:
        raise ValueError("cu_seqlens_q must contain at least two offsets")
    if max_seqlen_q == 1 and tokens > cu_seqlens_q.numel() - 1:
        # reference _decode.py:54-55
        raise ValueError("decode accepts at most one query per request")
    if lse is None:
        lse = torch.empty((heads, tokens), device=q.device, dtype=torch.float32)
    elif tuple(lse.shape) != (heads, tokens) or lse.dtype != torch.float32 or lse.device != q.device:
        raise ValueError("lse must be CUDA float32 [query_heads, total_q]")
    return run(q, k, v, out, lse, cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k,
               seqused_k=seqused_k, max_seqlen_q=max_seqlen_q, max_seqlen_k=max_seqlen_k,
               block_table=block_table, softmax_scale=softmax_scale, causal=causal,
               window_size=window_size, alibi_slopes=alibi_slopes, softcap=softcap,
               s_aux=s_aux, q_descale=q_descale, k_descale=k_descale, v_descale=v_descale,
               num_splits=num_splits, mask_mod=mask_mod, aux_tensors=aux_tensors,
               leftpad_k=leftpad_k, deterministic=deterministic, cp_world_size=cp_world_size,
               cp_rank=cp_rank, cp_tot_seqused_k=cp_tot_seqused_k)
