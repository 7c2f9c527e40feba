"""Shared test helpers: run the numpy oracle on torch inputs, compare results."""

import numpy as np
import torch

import oracle


def to_np(x):
    """torch tensor -> float64 numpy (FP8 decoded by the oracle's codec)."""
    if x is None:
        return None
    x = x.detach()
    if x.dtype == torch.float8_e4m3fn:
        return oracle.e4m3_decode(x.view(torch.uint8).cpu().numpy())
    if x.dtype in (torch.int32, torch.int64, torch.bool):
        return x.cpu().numpy()
    return x.cpu().double().numpy()


def reference(q, k, v, cu_q, cu_k=None, used_k=None, block_table=None, scale=None,
              causal=False, window=(-1, -1), softcap=0.0, alibi=None, sinks=None,
              q_descale=None, k_descale=None, v_descale=None, mask=None, aux=None,
              leftpad=None):
    """The oracle's float64 attention on torch inputs -> torch float64 (CPU)."""
    out, lse = oracle.attention(
        to_np(q), to_np(k), to_np(v), to_np(cu_q), cu_k=to_np(cu_k), used_k=to_np(used_k),
        block_table=to_np(block_table), scale=scale,
        causal=to_np(causal) if torch.is_tensor(causal) else causal, window=tuple(window),
        softcap=softcap, alibi=to_np(alibi), sinks=to_np(sinks), q_descale=to_np(q_descale),
        k_descale=to_np(k_descale), v_descale=to_np(v_descale), mask=mask,
        aux=None if aux is None else [to_np(a) for a in aux],
        leftpad=to_np(leftpad) if torch.is_tensor(leftpad) else leftpad)
    return torch.from_numpy(out), torch.from_numpy(lse)


def assert_attention_close(actual, expected, dtype=torch.float16):
    """Reference tolerance helper (tests/reference.py:93-96) plus the 1e-2 gate.

    bf16: atol 2e-2 / rtol 5e-2, otherwise atol 2e-3 / rtol 1e-2. For 16-bit
    outputs additionally max |actual - expected| <= 1e-2 once the expectation
    is rounded to the output dtype (one output ulp of slack).
    """
    atol, rtol = (2e-2, 5e-2) if dtype == torch.bfloat16 else (2e-3, 1e-2)
    a = actual.detach().cpu().double()
    torch.testing.assert_close(a, expected, atol=atol, rtol=rtol, check_dtype=False)
    if actual.dtype in (torch.float16, torch.bfloat16):
        rounded = expected.to(actual.dtype).double()
        ulp = (rounded.abs() * (2.0 ** -7 if actual.dtype == torch.bfloat16 else 2.0 ** -10)).clamp_min(1e-6)
        finite = torch.isfinite(rounded)
        err = (a - rounded).abs()[finite]
        assert bool((err <= 1e-2 + ulp[finite]).all()), f"max-abs {err.max().item():.3e} > 1e-2"


def assert_lse_close(actual, expected, atol=1e-3, rtol=0.0):
    """LSE gate: |lse - ref| <= 1e-3 (and identical -inf pattern)."""
    a = actual.detach().cpu().double()
    assert torch.equal(torch.isneginf(a), torch.isneginf(expected)), "-inf pattern differs"
    finite = torch.isfinite(expected)
    torch.testing.assert_close(a[finite], expected[finite], atol=atol, rtol=rtol)


def cu(lengths, device):
    values = [0]
    for n in lengths:
        values.append(values[-1] + int(n))
    return torch.tensor(values, dtype=torch.int32, device=device)


def np_seed(seed):
    return np.random.default_rng(seed)
