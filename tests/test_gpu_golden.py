"""The CUDA path against the golden vectors produced by the reference itself.

tests/golden/attn_*.npz hold seeded inputs and the outputs of the reference's
CPU oracle (tests/reference.py of flash-attn-mps); this runs the library on the
same inputs and compares, independently of oracle/.
"""

import glob
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from flash_attn_b200._attention import attention
from flash_attn_b200.interface import MaskSpec
from helpers import assert_attention_close, assert_lse_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAMES = sorted(os.path.basename(p)[5:-4] for p in glob.glob(os.path.join(GOLDEN, "attn_*.npz")))


def _tensor(g, key, dtype, device, fp8=False):
    if key not in g:
        return None
    x = torch.from_numpy(np.ascontiguousarray(g[key]))
    if fp8:
        return x.view(torch.float8_e4m3fn).to(device)
    return x.to(dtype).to(device) if dtype is not None else x.to(device)


@pytest.mark.parametrize("name", NAMES)
def test_cuda_path_matches_reference_golden(device, name):
    with np.load(os.path.join(GOLDEN, f"attn_{name}.npz")) as f:
        g = {k: f[k] for k in f.files}
    q_fp8, kv_fp8 = bool(g["q_fp8"]), bool(g["kv_fp8"])
    # Golden inputs were float16/bfloat16/float32 tensors stored exactly as f32/f16.
    qdtype = torch.float16 if g["q"].dtype == np.float16 else torch.bfloat16 if name.startswith("softcap") else torch.float32
    q = _tensor(g, "q", None if q_fp8 else qdtype, device, q_fp8)
    kdtype = torch.float16 if g["k"].dtype == np.float16 else torch.bfloat16 if name.startswith("softcap") else torch.float32
    k = _tensor(g, "k", None if kv_fp8 else kdtype, device, kv_fp8)
    v = _tensor(g, "v", None if kv_fp8 else kdtype, device, kv_fp8)
    cu_q = _tensor(g, "cu_q", None, device)
    cu_k = _tensor(g, "cu_k", None, device)
    used = _tensor(g, "used_k", None, device)
    table = _tensor(g, "block_table", None, device)
    causal = g["causal"]
    causal = bool(causal) if causal.ndim == 0 else torch.from_numpy(causal).to(device)
    mask = None
    aux = None
    if "mask" in g:
        kind, win, clamp = (int(x) for x in g["mask"])
        mask = MaskSpec(kind, win, bool(clamp))
        aux = [_tensor(g, "aux0", None, device), _tensor(g, "aux1", None, device)]
    qlens = np.diff(g["cu_q"])
    klens = np.diff(g["cu_k"]) if "cu_k" in g else g["used_k"]
    out, lse = attention(
        q, k, v, cu_seqlens_q=cu_q, cu_seqlens_k=cu_k, seqused_k=used,
        max_seqlen_q=int(qlens.max()), max_seqlen_k=int(max(klens.max(), 0)), block_table=table,
        causal=causal, window_size=tuple(int(w) for w in g["window"]), softcap=float(g["softcap"]),
        alibi_slopes=_tensor(g, "alibi", torch.float32, device),
        s_aux=_tensor(g, "sinks", torch.float32, device),
        q_descale=_tensor(g, "q_descale", torch.float32, device),
        k_descale=_tensor(g, "k_descale", torch.float32, device),
        v_descale=_tensor(g, "v_descale", torch.float32, device),
        mask_mod=mask, aux_tensors=aux, leftpad_k=_tensor(g, "leftpad", None, device))
    expected = torch.from_numpy(g["out"]).double()
    assert_attention_close(out, expected, out.dtype)
    assert_lse_close(lse, torch.from_numpy(g["lse"]).double())
