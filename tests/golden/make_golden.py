"""Generate the golden vectors that pin ``oracle/`` to the reference.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py /path/to/flash-attn-mps

It imports the reference's own CPU float64 oracle ``tests/reference.py``
(``attention_reference``) and the expectation-building code of its tests
(``tests/test_cache.py:106-122`` ``_rotary_reference``; the FP8 expectation
``values.clamp(-448, 448).to(torch.float8_e4m3fn)`` of ``tests/test_cache.py:52``;
the merge formulas of ``tests/test_merge.py:21-24, 56-59``), evaluates them on
seeded CPU inputs, and writes ``tests/golden/*.npz``. Nothing at test time
reads the reference; the tests read only the committed ``.npz`` files.
"""

import math
import os
import sys
from dataclasses import dataclass

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


@dataclass(frozen=True)
class Mask:  # same fields as the reference's interface.MaskSpec (interface.py:49-55)
    kind: int
    sliding_window_left: int = -1
    clamp_prefix_to_window: bool = False


def _np(t):
    if t is None:
        return None
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    if t.dtype == torch.bfloat16:
        return t.float().numpy()          # exact: bf16 -> f32
    return t.numpy()


def _save(name, **arrays):
    clean = {k: v for k, v in arrays.items() if v is not None}
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **clean)


def attention_cases(ref):
    g = torch.Generator().manual_seed(20261201)

    def randn(*shape, dtype=torch.float16, s=1.0):
        return (torch.randn(*shape, generator=g) * s).to(dtype)

    cases = {}

    # Config 1 of the benchmark plan: dense causal GQA fp16 [2,128,16,128].
    q, k, v = randn(2, 128, 16, 128), randn(2, 128, 8, 128), randn(2, 128, 8, 128)
    cu = torch.arange(3, dtype=torch.int32) * 128
    cases["cfg1_dense_causal_gqa"] = dict(
        q=q.flatten(0, 1), k=k.flatten(0, 1), v=v.flatten(0, 1), cu_q=cu, cu_k=cu,
        causal=True)

    # Ragged GQA + DiffKV, causal (test_interface.py:12-24 shapes).
    cases["ragged_diffkv"] = dict(
        q=randn(21, 4, 40), k=randn(25, 2, 40), v=randn(25, 2, 24),
        cu_q=torch.tensor([0, 1, 4, 21], dtype=torch.int32),
        cu_k=torch.tensor([0, 5, 8, 25], dtype=torch.int32), causal=True)

    # Paged K/V with leftpad across requests (test_attention_core.py:31-49).
    parent = randn(12, 2, 32, 160, dtype=torch.float32)
    kp, vp = parent.transpose(1, 2).split((96, 64), dim=-1)
    cases["paged_leftpad"] = dict(
        q=randn(39, 4, 96, dtype=torch.float32), k=kp.contiguous(), v=vp.contiguous(),
        cu_q=torch.tensor([0, 1, 6, 39], dtype=torch.int32),
        used_k=torch.tensor([69, 81, 33], dtype=torch.int32),
        block_table=torch.tensor([[7, 2, 9, 1], [4, 6, 3, 10], [5, 8, 0, 11]], dtype=torch.int32),
        leftpad=torch.tensor([5, 9, 1], dtype=torch.int32), causal=True)

    # Windows + sinks (test_attention_core.py:101-113).
    for i, (window, causal) in enumerate((((0, 0), True), ((15, 2), False),
                                          ((-1, 7), False), ((127, -1), True))):
        cases[f"window_sink_{i}"] = dict(
            q=randn(71, 4, 32), k=randn(307, 2, 32), v=randn(307, 2, 32),
            cu_q=torch.tensor([0, 3, 38, 71], dtype=torch.int32),
            cu_k=torch.tensor([0, 300, 300, 307], dtype=torch.int32),
            window=window, causal=causal, sinks=torch.tensor([-2., 0., 1., 3.]))

    # Softcap with fully masked rows (test_attention_core.py:135-149).
    for cap in (0.25, 1.0, 3.0):
        cases[f"softcap_{cap}"] = dict(
            q=randn(73, 4, 64, dtype=torch.bfloat16, s=3), k=randn(100, 2, 64, dtype=torch.bfloat16, s=3),
            v=randn(100, 2, 64, dtype=torch.bfloat16),
            cu_q=torch.tensor([0, 3, 38, 73], dtype=torch.int32),
            cu_k=torch.tensor([0, 0, 97, 100], dtype=torch.int32), causal=True, softcap=cap)

    # vLLM scores: ALiBi + sinks + window + softcap + dynamic causal (test_vllm.py:18-34).
    cases["vllm_alibi_dynamic"] = dict(
        q=randn(22, 4, 64), k=randn(182, 2, 64), v=randn(182, 2, 32),
        cu_q=torch.tensor([0, 1, 5, 22], dtype=torch.int32),
        cu_k=torch.tensor([0, 65, 165, 182], dtype=torch.int32),
        causal=torch.tensor([True, False, True]), window=(15, 15), softcap=2.0,
        alibi=torch.tensor([.1, .2, .3, .4]), sinks=torch.tensor([-1., 0., 1., 2.]))

    # vLLM masks over a paged cache (test_vllm.py:37-64).
    table = torch.tensor([[5, 1, 7, 3, 0]], dtype=torch.int32)
    kk, vv = randn(257, 2, 64), randn(257, 2, 32)
    paged_k = torch.zeros(8, 64, 2, 64, dtype=torch.float16)
    paged_v = torch.zeros(8, 64, 2, 32, dtype=torch.float16)
    pos = torch.arange(257)
    paged_k[table[0, pos // 64].long(), pos % 64] = kk
    paged_v[table[0, pos // 64].long(), pos % 64] = vv
    ranges = torch.full((96, 2), -1, dtype=torch.int32)
    ranges[31:61] = torch.tensor([192, 221], dtype=torch.int32)
    qm = randn(96, 4, 64)
    cuq = torch.tensor([0, 96], dtype=torch.int32)
    for kind in ("mm", "mm_window", "mm_clamp", "rswa"):
        if kind == "rswa":
            mask, aux = Mask(2), [torch.tensor([64], dtype=torch.int32), torch.tensor([16], dtype=torch.int32)]
        else:
            mask = Mask(1, -1 if kind == "mm" else 16, kind == "mm_clamp")
            aux = [ranges, cuq]
        cases[f"mask_{kind}"] = dict(
            q=qm, k=paged_k, v=paged_v, cu_q=cuq, used_k=torch.tensor([257], dtype=torch.int32),
            block_table=table, mask=mask, aux=aux)

    # FP8 q/k/v with broadcast descales (test_vllm.py:67-80).
    q8 = randn(10, 4, 32, dtype=torch.float32).to(torch.float8_e4m3fn)
    k8 = randn(42, 2, 32, dtype=torch.float32).to(torch.float8_e4m3fn)
    v8 = randn(42, 2, 64, dtype=torch.float32).to(torch.float8_e4m3fn)
    cases["fp8_descales"] = dict(
        q=q8, k=k8, v=v8, cu_q=torch.tensor([0, 3, 10], dtype=torch.int32),
        cu_k=torch.tensor([0, 19, 42], dtype=torch.int32), causal=True,
        q_descale=torch.tensor([[.8, 1.2]]).expand(2, 2).contiguous(),
        k_descale=torch.tensor([[.3], [.7]]).expand(2, 2).contiguous(),
        v_descale=torch.tensor([[.9, 1.1]]).expand(2, 2).contiguous())

    # Paged FP8 decode with sink + window + softcap (test_decode.py:111-137).
    raw = torch.randn(25, 16, 2, 256, generator=g)
    raw[24] = float("nan")
    packed = raw.to(torch.float8_e4m3fn)
    kd8, vd8 = (t.contiguous() for t in packed.split(128, dim=-1))
    cases["decode_fp8_sink_window_softcap"] = dict(
        q=randn(3, 8, 128), k=kd8, v=vd8, cu_q=torch.tensor([0, 1, 2, 3], dtype=torch.int32),
        used_k=torch.tensor([0, 33, 97], dtype=torch.int32),
        leftpad=torch.tensor([0, 3, 1], dtype=torch.int32),
        block_table=torch.tensor([[24] * 8, [3, 8, 11, 24, 24, 24, 24, 24],
                                  [4, 10, 7, 6, 2, 13, 21, 24]], dtype=torch.int32),
        q_descale=torch.tensor([[1., .75]]).expand(3, 2).contiguous(),
        k_descale=torch.tensor([[.5]]).expand(3, 2).contiguous(),
        v_descale=torch.tensor([[.25, 1.]]).expand(3, 2).contiguous(),
        sinks=torch.linspace(-3, 3, 16)[::2].contiguous(), softcap=.7, window=(15, 0))

    # Empty KV with sinks (test_attention_core.py:52-63).
    cases["empty_kv_sinks"] = dict(
        q=randn(13, 4, 32), k=torch.empty(0, 2, 32, dtype=torch.float16),
        v=torch.empty(0, 2, 32, dtype=torch.float16),
        cu_q=torch.tensor([0, 7, 13], dtype=torch.int32),
        cu_k=torch.tensor([0, 0, 0], dtype=torch.int32), sinks=torch.tensor([-10., 0., 1., 10.]))

    for name, c in cases.items():
        kw = dict(cu_k=c.get("cu_k"), used_k=c.get("used_k"), block_table=c.get("block_table"),
                  scale=c.get("scale"), causal=c.get("causal", False), window=c.get("window", (-1, -1)),
                  softcap=c.get("softcap", 0.0), alibi=c.get("alibi"), sinks=c.get("sinks"),
                  q_descale=c.get("q_descale"), k_descale=c.get("k_descale"),
                  v_descale=c.get("v_descale"), mask=c.get("mask"), aux=c.get("aux"),
                  leftpad=c.get("leftpad"))
        out, lse = ref.attention_reference(c["q"], c["k"], c["v"], c["cu_q"], **kw)
        mask = c.get("mask")
        causal = c.get("causal", False)
        _save("attn_" + name,
              q=_np(c["q"]), k=_np(c["k"]), v=_np(c["v"]),
              q_fp8=np.array(c["q"].dtype == torch.float8_e4m3fn),
              kv_fp8=np.array(c["k"].dtype == torch.float8_e4m3fn),
              cu_q=_np(c["cu_q"]), cu_k=_np(c.get("cu_k")), used_k=_np(c.get("used_k")),
              block_table=_np(c.get("block_table")), leftpad=_np(c.get("leftpad")),
              causal=_np(causal) if torch.is_tensor(causal) else np.array(bool(causal)),
              window=np.array(c.get("window", (-1, -1))), softcap=np.array(c.get("softcap", 0.0)),
              alibi=_np(c.get("alibi")), sinks=_np(c.get("sinks")),
              q_descale=_np(c.get("q_descale")), k_descale=_np(c.get("k_descale")),
              v_descale=_np(c.get("v_descale")),
              mask=None if mask is None else np.array([mask.kind, mask.sliding_window_left,
                                                       int(mask.clamp_prefix_to_window)]),
              aux0=None if mask is None else _np(c["aux"][0]),
              aux1=None if mask is None else _np(c["aux"][1]),
              out=out.float().numpy(), lse=lse.numpy())
    return sorted(cases)


def fp8_cases():
    # The known-answer set of test_cache.py:39-54 plus every bf16 bit pattern
    # under four scales; expectation = torch's cast of clamp(x/scale,-448,448).
    representable = torch.arange(127, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    ties = (representable[:-1] + representable[1:]) / 2
    kat = torch.cat((representable, ties, -representable, -ties,
                     torch.tensor([1000., -1000., float("inf"), -float("inf")])))
    bf = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float()
    bf = bf[~torch.isnan(bf)]
    scales = torch.tensor([1.0, 0.5, 2.0, 3.0 / 448.0], dtype=torch.float32)
    x = torch.cat([kat] + [bf] * len(scales))
    s = torch.cat([torch.ones_like(kat)] + [torch.full_like(bf, float(v)) for v in scales])
    codes = (x / s).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    decoded = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float()
    _save("fp8_codec", x=x.numpy(), scale=s.numpy(), codes=codes.numpy(),
          decode_table=decoded.numpy())


def merge_cases():
    g = torch.Generator().manual_seed(7)
    # test_merge.py:10-27 extreme LSEs; expectation from its logaddexp formula.
    left = torch.randn(3, 3, 7, generator=g).double()
    right = torch.randn(3, 3, 7, generator=g).double()
    la = torch.tensor([[1000., -1000., -float("inf")], [-float("inf"), 0., 10.], [-float("inf"), -50., 50.]]).double()
    lb = torch.tensor([[1001., -1001., 0.], [-float("inf"), -float("inf"), 11.], [1., 50., -50.]]).double()
    le = torch.logaddexp(la, lb)
    wa = (la - le).exp().nan_to_num(0).T.unsqueeze(-1)
    wb = (lb - le).exp().nan_to_num(0).T.unsqueeze(-1)
    expected = wa * left + wb * right
    _save("merge_pair", left=left.numpy(), right=right.numpy(), la=la.numpy(), lb=lb.numpy(),
          out=expected.numpy(), lse=le.numpy())
    # test_merge.py:44-61 N-way merge with -inf parts and NaN payloads.
    p = torch.randn(5, 3, 3, 7, generator=g).double()
    lsep = torch.randn(5, 3, 3, generator=g).double()
    lsep[:, 0, 1] = -float("inf")
    p[:, 1, 0] = float("nan")
    expected_lse = torch.logsumexp(lsep, dim=0)
    weights = (lsep - expected_lse).exp().nan_to_num(0).transpose(1, 2).unsqueeze(-1)
    values = torch.where(weights > 0, p, 0.)
    expected = (weights * values).sum(0)
    _save("merge_partials", partial=p.numpy(), lse=lsep.numpy(), out=expected.numpy(),
          out_lse=expected_lse.numpy())


def rotary_cases(test_cache):
    g = torch.Generator().manual_seed(11)
    q = torch.randn(2, 3, 4, 16, generator=g)[..., 1::2].contiguous()
    angles = torch.randn(20, 4, generator=g)[:, ::2].contiguous()
    cos, sin = angles.cos(), angles.sin()
    lengths = torch.tensor([2, 7])
    results = {}
    for interleaved in (True, False):
        for advance in (True, False):
            results[f"out_{int(interleaved)}{int(advance)}"] = test_cache._rotary_reference(
                q, cos, sin, lengths, interleaved, advance).numpy()
    _save("rotary", x=q.numpy(), cos=cos.numpy(), sin=sin.numpy(), lengths=lengths.numpy(),
          **results)


def main(reference_root):
    sys.path.insert(0, reference_root)
    sys.path.insert(0, os.path.join(reference_root, "tests"))
    import reference as ref          # tests/reference.py of the reference checkout
    import test_cache                # for _rotary_reference (tests/test_cache.py:106-122)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    names = attention_cases(ref)
    fp8_cases()
    merge_cases()
    rotary_cases(test_cache)
    print("wrote", len(names), "attention cases +", "fp8_codec merge_pair merge_partials rotary")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLASH_ATTN_MPS_ROOT", "."))
