"""The reference's frozen SDPA engine attention -- TEST INFRASTRUCTURE ONLY.

Restates ``sdpa_baseline`` of the reference (benchmarks/bench_attention.py:24-55,
"frozen behavior of nano-vLLM forward_mps before native integration") as an
attention back-end for the serving loop: the step's K/V are index-copied into
the paged cache at their slots, and every request attends over its pages in
the table with a lower-right causal mask. The reference evaluates SDPA in the
model dtype (or float64, ``fp64_forward`` at validate_nanovllm.py:27-34); this
restatement evaluates in float64 on the tensors' device and rounds the output
to the query dtype, so it is the stricter of the two.

Used only by tests (teacher-forced KL check, validate_nanovllm.py:77-106) and
by the CPU-baseline leg of the serving workload in bench.py.
"""

import math

import torch


class SdpaAttention:
    """Attention back-end with the ``NativeAttention`` calling convention."""

    rotates = False

    def __init__(self, shape, cache, cos, sin):
        self.shape, self.cache = shape, cache

    def __call__(self, layer, q, k, v, step):
        kc, vc = self.cache.k[layer], self.cache.v[layer]
        # bench_attention.py:26-30: scatter the step's K/V into the cache.
        kc.flatten(0, 1).index_copy_(0, step.slots, k)
        vc.flatten(0, 1).index_copy_(0, step.slots, v)
        offsets = step.cu_q.tolist()
        lengths = step.end.tolist()
        page = kc.shape[1]
        group = q.shape[1] // k.shape[1]
        outputs = []
        for i, length in enumerate(lengths):
            start, end = offsets[i], offsets[i + 1]
            blocks = self.cache.table[i, :math.ceil(length / page)].long()
            key = kc[blocks].flatten(0, 1)[:length].double().repeat_interleave(group, dim=1)
            value = vc[blocks].flatten(0, 1)[:length].double().repeat_interleave(group, dim=1)
            query = q[start:end].double()
            scores = torch.einsum("qhd,khd->hqk", query, key) * self.shape.scale
            # Lower-right causal: query row r sits at absolute position length - rows + r.
            rows = end - start
            qpos = torch.arange(rows, device=q.device)[:, None] + (length - rows)
            kpos = torch.arange(length, device=q.device)[None, :]
            scores = scores.masked_fill(kpos > qpos, float("-inf"))
            probs = torch.softmax(scores, dim=-1)
            outputs.append(torch.einsum("hqk,khd->qhd", probs, value).to(q.dtype))
        return torch.cat(outputs)
