"""Stable merging of attention states (mirrors flash_attn_mps/_merge.py).

``merge_attn_states`` (reference ``_merge.py:20-41``) merges two states in
place-safe fashion; ``_merge_partials`` (``_merge.py:44-57``) merges N split
partials. Both run the CUDA merge kernels.
"""

import torch

from . import _capi


def _cuda(*tensors):
    if any(t.device.type != "cuda" for t in tensors if t is not None):
        raise ValueError("operations require CUDA tensors")


def merge_attn_states(out, left_out, left_lse, right_out, right_lse, out_lse=None):
    """Write the LSE-weighted merge to ``out``; LSE uses natural logarithms.

    Outputs are [tokens, heads, dim], LSE tensors are FP32 [heads, tokens].
    An empty state has LSE=-inf; merging two empty states yields zero and -inf.
    ``out`` and ``out_lse`` may alias the corresponding left state.
    """
    _cuda(out, left_out, left_lse, right_out, right_lse, out_lse)
    if out.ndim != 3 or left_out.shape != out.shape or right_out.shape != out.shape:
        raise ValueError("output states must have matching [tokens, heads, dim] shapes")
    if left_out.dtype != out.dtype or right_out.dtype != out.dtype:
        raise TypeError("output state dtypes must match")
    expected = (out.shape[1], out.shape[0])
    for lse in (left_lse, right_lse, out_lse):
        if lse is not None and (tuple(lse.shape) != expected or lse.dtype != torch.float32):
            raise ValueError("LSE tensors must be float32 [heads, tokens]")
    if not out.numel():
        return
    t = _capi.tensor
    args = [t(out), t(left_out), t(left_lse), t(right_out), t(right_lse), t(out_lse)]
    lib = _capi.library()
    _capi.check(lib.fa_merge_attn_states(*map(_capi.ref, args), _capi.stream_of(out.device)))


def _merge_partials(partial_out, partial_lse, out=None, out_lse=None):
    """Merge [splits,tokens,heads,dim] and [splits,heads,tokens] states.

    Returns ``(out [tokens, heads, dim], lse [heads, tokens])``; ``out`` and
    ``out_lse`` may be supplied (any strides, ``out`` any float dtype).
    """
    _cuda(partial_out, partial_lse)
    if partial_out.ndim != 4 or tuple(partial_lse.shape) != (
            partial_out.shape[0], partial_out.shape[2], partial_out.shape[1]):
        raise ValueError("partial states require [splits,tokens,heads,dim] and [splits,heads,tokens]")
    if partial_lse.dtype != torch.float32:
        raise TypeError("partial LSE must be float32")
    splits, tokens, heads, dim = partial_out.shape
    if out is None:
        out = torch.empty((tokens, heads, dim), dtype=partial_out.dtype, device=partial_out.device)
    if out_lse is None:
        out_lse = torch.empty((heads, tokens), dtype=torch.float32, device=partial_out.device)
    if tokens and heads:
        t = _capi.tensor
        args = [t(partial_out), t(partial_lse), t(out), t(out_lse)]
        lib = _capi.library()
        _capi.check(lib.fa_merge_partials(*map(_capi.ref, args), _capi.stream_of(out.device)))
    return out, out_lse
