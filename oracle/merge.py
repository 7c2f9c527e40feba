"""Stable LSE merges restated in numpy (oracle; test infrastructure only).

``merge_pair`` follows ``flash_attn_mps/kernels/merge.metal:9-28``
(``merge_attn_states``): an empty state has LSE -inf; two empty states give
zero output and -inf; a +inf LSE takes all the weight; a zero weight never
multiplies its (possibly NaN) payload.

``merge_partials`` follows ``merge.metal:30-58`` (the N-way split merge also
used by ``attention_decode.metal:151-207``): lse* = m + log sum exp(lse_s - m),
out = sum exp(lse_s - lse*) o_s over splits with nonzero weight.
"""

import numpy as np


def _weights(lse, maximum):
    with np.errstate(invalid="ignore", over="ignore"):
        w = np.where(maximum == np.inf, (lse == maximum).astype(np.float64),
                     np.exp(lse - maximum))
    return np.where(maximum == -np.inf, 0.0, w)


def merge_pair(left, left_lse, right, right_lse):
    """left/right [T,H,D], lse [H,T] -> (out [T,H,D], lse [H,T]) in float64."""
    left = np.asarray(left, dtype=np.float64)
    right = np.asarray(right, dtype=np.float64)
    a = np.asarray(left_lse, dtype=np.float64).T        # [T,H]
    b = np.asarray(right_lse, dtype=np.float64).T
    maximum = np.maximum(a, b)
    empty = maximum == -np.inf
    wa, wb = _weights(a, maximum), _weights(b, maximum)
    total = wa + wb
    value = (np.where(wa[..., None] > 0, wa[..., None] * np.nan_to_num(left, nan=0.0), 0.0)
             + np.where(wb[..., None] > 0, wb[..., None] * np.nan_to_num(right, nan=0.0), 0.0))
    # A positive weight keeps its payload, NaN included.
    value = np.where((wa[..., None] > 0) & np.isnan(left), np.nan, value)
    value = np.where((wb[..., None] > 0) & np.isnan(right), np.nan, value)
    with np.errstate(invalid="ignore", divide="ignore"):
        value = np.where(empty[..., None], value, value / np.where(empty, 1.0, total)[..., None])
        out_lse = np.where(empty, -np.inf, maximum + np.log(np.where(empty, 1.0, total)))
    return value, out_lse.T


def merge_partials(partial, partial_lse):
    """partial [S,T,H,D], lse [S,H,T] -> (out [T,H,D], lse [H,T]) in float64."""
    partial = np.asarray(partial, dtype=np.float64)
    lse = np.asarray(partial_lse, dtype=np.float64)
    splits, tokens, heads, dim = partial.shape
    if splits == 0:
        return np.zeros((tokens, heads, dim)), np.full((heads, tokens), -np.inf)
    maximum = lse.max(axis=0)                                   # [H,T]
    empty = maximum == -np.inf
    w = _weights(lse, maximum[None])                            # [S,H,T]
    denominator = w.sum(axis=0)
    wt = w.transpose(0, 2, 1)[..., None]                        # [S,T,H,1]
    value = np.where(wt > 0, wt * np.nan_to_num(partial, nan=0.0), 0.0).sum(axis=0)
    value = np.where(((wt > 0) & np.isnan(partial)).any(axis=0), np.nan, value)
    den = np.where(empty, 1.0, denominator).T[..., None]
    out = np.where(empty.T[..., None], 0.0, value / den)
    with np.errstate(divide="ignore"):
        out_lse = np.where(empty, -np.inf, maximum + np.log(np.where(empty, 1.0, denominator)))
    return out, out_lse
