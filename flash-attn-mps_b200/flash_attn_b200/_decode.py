"""Single-query decode entry (mirrors flash_attn_mps/_decode.py:40-99).

``decode_attention`` keeps the reference signature. It requires at most one
query per request (cu_seqlens_q differences in {0, 1}) and hands the call to
the library with ``max_seqlen_q = 1``, which routes it to the tensor-core
paged decode kernel (or the generic kernel outside that kernel's envelope),
with split-KV partials merged on the device.
"""

import torch

from . import _attention


def decode_attention(q, k, v, *, cu_seqlens_q, cu_seqlens_k=None, seqused_k=None,
                     max_seqlen_k, block_table=None, softmax_scale=None, out=None,
                     leftpad_k=None, num_splits=0, s_aux=None, q_descale=None,
                     k_descale=None, v_descale=None, window_size=(-1, -1), softcap=0.):
    """Attend one query per nonempty request; returns output and natural LSE."""
    tokens, heads, dq = q.shape
    dv = v.shape[-1]
    batch = cu_seqlens_q.numel() - 1
    if tokens > batch:
        raise ValueError("decode accepts at most one query per request")
    out_dtype = torch.float16 if q.dtype == torch.float8_e4m3fn else q.dtype
    if out is None:
        out = torch.empty((tokens, heads, dv), dtype=out_dtype, device=q.device)
    lse = torch.empty((heads, tokens), dtype=torch.float32, device=q.device)
    if not tokens:
        return out, lse
    return _attention.run(
        q, k, v, out, lse, cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k,
        seqused_k=seqused_k, max_seqlen_q=1, max_seqlen_k=max_seqlen_k,
        block_table=block_table, softmax_scale=softmax_scale, causal=False,
        window_size=window_size, alibi_slopes=None, softcap=softcap, s_aux=s_aux,
        q_descale=q_descale, k_descale=k_descale, v_descale=v_descale,
        num_splits=num_splits, mask_mod=None, aux_tensors=None, leftpad_k=leftpad_k,
        deterministic=False)
