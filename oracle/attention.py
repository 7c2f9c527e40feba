"""Float64 attention oracle (test infrastructure only).

A vectorised numpy restatement of the reference's CPU oracle
``tests/reference.py:6-90`` (``attention_reference``), covering every feature
of the hot path:

* paged K/V gathered through ``block_table`` with ``leftpad`` (reference.py:43-51)
* GQA/MQA, here by reshaping queries to [Hkv, group, Sq, D] instead of
  expanding keys (reference.py:28, 52)
* q/k/v descales ``[B, Hkv]`` (reference.py:33-36, 42, 52-53)
* scale -> softcap tanh -> ALiBi (reference.py:54-62)
* lower-right causal and window keep masks (reference.py:57-68); query row i of
  a request with Sq queries and Sk keys sits at absolute position i + Sk - Sq
  (``docs/contracts.md:32-37``)
* vLLM mask kinds 1 (mm-prefix) and 2 (rolling SWA) (reference.py:69-80)
* sinks as an extra logit column that only enters the LSE (reference.py:83-88)
* natural-log LSE; fully masked rows give zero output and -inf LSE
  (reference.py:86-89)

Inputs are numpy arrays already decoded to float (use ``oracle.fp8.e4m3_decode``
for FP8 storage). Returns ``out [T, Hq, Dv]`` and ``lse [Hq, T]`` in float64.
"""

import numpy as np


def _as_list(x):
    if x is None:
        return None
    return [int(v) for v in np.asarray(x).reshape(-1)]


def _descale(tensor, b, groups, heads):
    if tensor is None:
        return 1.0
    return np.asarray(tensor, dtype=np.float64)[b][groups].reshape(heads, 1, 1)


def _logsumexp(x):
    m = np.max(x, axis=-1, keepdims=True, initial=-np.inf)
    finite = np.isfinite(m)
    safe = np.where(finite, m, 0.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        s = np.log(np.sum(np.exp(x - safe), axis=-1, keepdims=True)) + safe
    return np.where(finite, s, m)[..., 0]


def attention(q, k, v, cu_q, cu_k=None, used_k=None, block_table=None, scale=None,
              causal=False, window=(-1, -1), softcap=0.0, alibi=None, sinks=None,
              q_descale=None, k_descale=None, v_descale=None, mask=None, aux=None,
              leftpad=None, max_elems=1 << 25):
    """Reference attention semantics of ``tests/reference.py:6-90`` in float64.

    ``mask`` is any object with ``kind``, ``sliding_window_left`` and
    ``clamp_prefix_to_window`` attributes (the reference's ``MaskSpec``,
    ``interface.py:49-55``). ``causal`` may be a bool or a per-request
    sequence of bools (dynamic causal).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    cu_q = _as_list(cu_q)
    cu_k = _as_list(cu_k)
    if cu_k is not None:
        lengths = [b - a for a, b in zip(cu_k, cu_k[1:])]
    else:
        lengths = _as_list(used_k)
    table = None if block_table is None else np.asarray(block_table).astype(np.int64)
    if not isinstance(causal, (bool, int)):
        causal = [bool(c) for c in np.asarray(causal).reshape(-1)]
    leftpad = _as_list(leftpad)
    heads, hkv, dq, dv = q.shape[1], k.shape[-2], q.shape[-1], v.shape[-1]
    group = heads // hkv
    groups = np.arange(heads) // group
    out = np.zeros((q.shape[0], heads, dv), dtype=np.float64)
    lse = np.full((heads, q.shape[0]), -np.inf, dtype=np.float64)
    scale = dq ** -0.5 if scale is None else float(scale)
    slopes_all = None if alibi is None else np.asarray(alibi, dtype=np.float64)
    sink_all = None if sinks is None else np.asarray(sinks, dtype=np.float64).reshape(heads)
    kind = 0 if mask is None else int(mask.kind)

    for b, length in enumerate(lengths):
        start, end = cu_q[b], cu_q[b + 1]
        if start == end:
            continue
        sq = end - start
        offset = 0 if leftpad is None else leftpad[b]
        if table is not None:
            positions = np.arange(offset, offset + length)
            physical = table[b, positions // k.shape[1]]
            key = k[physical, positions % k.shape[1]]
            value = v[physical, positions % v.shape[1]]
        else:
            ks = (0 if cu_k is None else cu_k[b]) + offset
            key, value = k[ks:ks + length], v[ks:ks + length]
        # [Hkv, L, D] with the K/V descale of each KV head.
        kd = _descale(k_descale, b, np.arange(hkv), hkv)
        vd = _descale(v_descale, b, np.arange(hkv), hkv)
        key = key.transpose(1, 0, 2) * kd
        value = value.transpose(1, 0, 2) * vd
        query = q[start:end].transpose(1, 0, 2) * _descale(q_descale, b, groups, heads)
        query = query.reshape(hkv, group, sq, dq)
        causal_b = causal[b] if isinstance(causal, list) else bool(causal)
        slopes = None
        if slopes_all is not None:
            slopes = slopes_all if slopes_all.ndim == 1 else slopes_all[b]
        rows = max(1, max_elems // max(1, heads * max(length, 1)))
        for r0 in range(0, sq, rows):
            r1 = min(sq, r0 + rows)
            qpos = np.arange(length - sq + r0, length - sq + r1)[:, None]
            kpos = np.arange(length)[None, :]
            scores = np.matmul(query[:, :, r0:r1], key.transpose(0, 2, 1)[:, None]) * scale
            scores = scores.reshape(heads, r1 - r0, length)
            if softcap:
                scores = np.tanh(scores / softcap) * softcap
            if slopes is not None:
                scores = scores - slopes[:, None, None] * np.abs(qpos - kpos)
            keep = (kpos <= qpos) if causal_b else np.ones((r1 - r0, length), dtype=bool)
            if window[0] >= 0:
                keep = keep & (kpos >= qpos - window[0])
            if window[1] >= 0:
                keep = keep & (kpos <= qpos + window[1])
            if kind == 1:
                ranges = np.asarray(aux[0]).reshape(-1, 2)[start + r0:start + r1]
                keep = kpos <= qpos
                if mask.sliding_window_left >= 0:
                    keep = keep & (qpos - kpos < mask.sliding_window_left)
                prefix = (kpos >= ranges[:, :1]) & (kpos <= ranges[:, 1:2])
                if mask.clamp_prefix_to_window:
                    prefix = prefix & (qpos - kpos < mask.sliding_window_left)
                keep = keep | prefix
            elif kind == 2:
                prefix_len = int(np.asarray(aux[0]).reshape(-1)[b])
                width = int(np.asarray(aux[1]).reshape(-1)[0])
                keep = (kpos <= qpos) & ((kpos < prefix_len) | (qpos - kpos < width))
            scores = np.where(keep[None], scores, -np.inf)
            all_scores = scores
            if sink_all is not None:
                sink = np.broadcast_to(sink_all[:, None, None], (heads, r1 - r0, 1))
                all_scores = np.concatenate((scores, sink), axis=-1)
            lrow = _logsumexp(all_scores)
            with np.errstate(invalid="ignore"):
                probs = np.nan_to_num(np.exp(scores - lrow[..., None]), nan=0.0)
            probs = probs.reshape(hkv, group, r1 - r0, length)
            o = np.matmul(probs, value[:, None])          # [Hkv, G, rows, Dv]
            out[start + r0:start + r1] = o.reshape(heads, r1 - r0, dv).transpose(1, 0, 2)
            lse[:, start + r0:start + r1] = lrow
    return out, lse


def visible_pairs(q_lens, k_lens, causal=True, window=(-1, -1)):
    """Number of unmasked (query, key) pairs, for FLOP accounting in tests."""
    total = 0
    for sq, sk in zip(q_lens, k_lens):
        qpos = np.arange(sk - sq, sk)[:, None]
        kpos = np.arange(sk)[None, :]
        keep = (kpos <= qpos) if causal else np.ones((sq, sk), dtype=bool)
        if window[0] >= 0:
            keep &= kpos >= qpos - window[0]
        if window[1] >= 0:
            keep &= kpos <= qpos + window[1]
        total += int(keep.sum())
    return total
