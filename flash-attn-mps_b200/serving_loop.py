"""A serving loop around the attention path: a minimal Qwen3-architecture decoder.

Random-init bf16 weights of the Qwen3-0.6B shape (28 layers, hidden 1024,
16 query / 8 KV heads of 128, MLP 3072 with SiLU gating, vocab 151936 with
tied embeddings, per-head q/k RMS norms, half-split RoPE with theta 1e6), a
batch of prompts prefilled into a paged cache of 16-token pages whose page
table is a seeded permutation, then greedy decode steps. Every attention call
goes through flash_attn_b200's public API in one of two ways:

* ``NativeAttention`` -- the reference's nano-vLLM integration
  (benchmarks/bench_attention.py:58-70): the model applies RoPE, then
  ``store_kvcache`` of the step's K/V, ``flash_attn_varlen_func`` over the
  paged cache for prefill and ``flash_attn_with_kvcache`` for decode;
* ``FusedAttention`` -- ``flash_attn_with_kvcache`` with new ``k``/``v`` and
  rotary tables: RoPE of Q and K plus the cache append in one launch, then
  attention. Every request of a step has the same number of new tokens.

The GEMMs, norms and sampling around attention are plain torch: this module is
plumbing that runs the library inside a serving loop (the decode step is
capturable as one CUDA graph) and lets it be checked against the reference's
frozen SDPA engine path with the teacher-forced KL protocol of
benchmarks/validate_nanovllm.py:77-106.
"""

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class Qwen3Shape:
    vocab: int = 151936
    hidden: int = 1024
    layers: int = 28
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 3072
    rope_theta: float = 1e6
    eps: float = 1e-6
    page: int = 16

    @property
    def scale(self):
        return self.head_dim ** -0.5


def init_weights(shape, device, seed=0, std=0.02):
    """Seeded random bf16 weights (linear weights are [out, in])."""
    g = torch.Generator(device=device).manual_seed(seed)

    def normal(*size):
        return (torch.randn(*size, generator=g, device=device) * std).to(torch.bfloat16)

    def norm_weight(n):
        return (1 + 0.1 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)

    H, D = shape.hidden, shape.head_dim
    layers = [dict(ln1=norm_weight(H), wqkv=normal((shape.heads + 2 * shape.kv_heads) * D, H),
                   q_norm=norm_weight(D), k_norm=norm_weight(D), wo=normal(H, shape.heads * D),
                   ln2=norm_weight(H), w_gate_up=normal(2 * shape.intermediate, H),
                   w_down=normal(H, shape.intermediate))
              for _ in range(shape.layers)]
    return dict(embed=normal(shape.vocab, H), layers=layers, norm=norm_weight(H))


def rope_tables(shape, positions, device):
    """fp32 cos/sin [positions, head_dim/2] (computed in float64)."""
    inv = shape.rope_theta ** (-torch.arange(0, shape.head_dim, 2, dtype=torch.float64) / shape.head_dim)
    angle = torch.arange(positions, dtype=torch.float64)[:, None] * inv[None]
    return angle.cos().float().to(device), angle.sin().float().to(device)


def apply_rope(x, cos, sin, positions):
    """Half-split RoPE of [tokens, heads, dim] at ``positions`` in fp32, rounded to x's dtype."""
    c = cos[positions][:, None, :]
    s = sin[positions][:, None, :]
    x1, x2 = x.float().chunk(2, dim=-1)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


class PagedCache:
    """Per-layer K/V caches [pages, page, kv_heads, head_dim] and a permuted page table."""

    def __init__(self, shape, requests, capacity, device, seed=0, dtype=torch.bfloat16):
        P = shape.page
        cols = (capacity + P - 1) // P
        pages = requests * cols
        perm = torch.randperm(pages, generator=torch.Generator().manual_seed(seed)).to(torch.int32)
        self.table = perm.reshape(requests, cols).to(device)
        self.capacity = cols * P
        self.k = [torch.zeros(pages, P, shape.kv_heads, shape.head_dim, dtype=dtype, device=device)
                  for _ in range(shape.layers)]
        self.v = [torch.zeros_like(c) for c in self.k]

    def slots(self, rows, positions, page):
        """Physical slot of (request row, position) pairs, as int64; -1 (skipped by
        every store) for positions past the table, whose column is clamped so the
        gather stays in bounds."""
        cols = self.table.shape[1]
        col = positions // page
        slot = self.table[rows, col.clamp(max=cols - 1)].long() * page + positions % page
        return torch.where(col < cols, slot, torch.full_like(slot, -1))


@dataclass
class Step:
    """Metadata of one model step over a batch of requests (device tensors)."""
    prefill: bool
    cu_q: torch.Tensor       # [B+1] int32 offsets of the new tokens
    cu_k: torch.Tensor       # [B+1] int32 offsets of the cached lengths after the step
    positions: torch.Tensor  # [T] int64 absolute positions of the new tokens
    start: torch.Tensor      # [B] int32 cache length before the step
    end: torch.Tensor        # [B] int32 cache length after the step
    slots: torch.Tensor      # [T] int64 physical cache slots of the new tokens
    max_q: int
    max_k: int
    uniform: int             # new tokens per request (all equal), 0 when ragged
    host: dict = field(default_factory=dict)  # host copies of lengths, when known


def prefill_step(cache, lengths, page, device):
    """Step metadata for prompts of ``lengths`` tokens written from position 0."""
    B = len(lengths)
    lens = torch.tensor(lengths, dtype=torch.int32)
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    rows = torch.repeat_interleave(torch.arange(B), lens).to(device)
    positions = torch.cat([torch.arange(n) for n in lengths]).to(device)
    cu, lens = cu.to(device), lens.to(device)
    return Step(True, cu, cu, positions, torch.zeros_like(lens), lens, cache.slots(rows, positions, page),
                max(lengths), max(lengths), lengths[0] if len(set(lengths)) == 1 else 0,
                {"start": [0] * B, "end": list(lengths)})


def decode_step(cache, start, page):
    """Step metadata for one new token per request at positions ``start`` (device int32 [B]).

    Only device ops: the step can be rebuilt inside a captured CUDA graph.
    """
    B = start.shape[0]
    device = start.device
    positions = start.long()
    end = start + 1
    cu_q = torch.arange(B + 1, dtype=torch.int32, device=device)
    cu_k = torch.cat([torch.zeros(1, dtype=torch.int32, device=device), torch.cumsum(end, 0, dtype=torch.int32)])
    rows = torch.arange(B, device=device)
    return Step(False, cu_q, cu_k, positions, start, end, cache.slots(rows, positions, page),
                1, cache.capacity, 1)


class NativeAttention:
    """store_kvcache + flash_attn_varlen_func / flash_attn_with_kvcache (reference
    benchmarks/bench_attention.py:58-70); the model applies RoPE first."""

    rotates = False

    def __init__(self, shape, cache, cos, sin):
        self.shape, self.cache = shape, cache

    def __call__(self, layer, q, k, v, step):
        from flash_attn_b200 import flash_attn_varlen_func, flash_attn_with_kvcache, store_kvcache
        kc, vc = self.cache.k[layer], self.cache.v[layer]
        store_kvcache(k, v, kc, vc, step.slots)
        if step.prefill:
            return flash_attn_varlen_func(q, kc, vc, step.cu_q, step.cu_k, step.max_q, step.max_k,
                                          softmax_scale=self.shape.scale, causal=True,
                                          block_table=self.cache.table)
        return flash_attn_with_kvcache(q.unsqueeze(1), kc, vc, cache_seqlens=step.end,
                                       block_table=self.cache.table, softmax_scale=self.shape.scale,
                                       causal=True).reshape_as(q)


class FusedAttention:
    """flash_attn_with_kvcache with new K/V and rotary tables: RoPE + append + attention."""

    rotates = True

    def __init__(self, shape, cache, cos, sin):
        self.shape, self.cache, self.cos, self.sin = shape, cache, cos, sin

    def __call__(self, layer, q, k, v, step):
        from flash_attn_b200 import flash_attn_with_kvcache
        if not step.uniform:
            raise ValueError("the fused path needs the same number of new tokens in every request")
        B, S = step.start.shape[0], step.uniform
        out = flash_attn_with_kvcache(
            q.view(B, S, *q.shape[1:]), self.cache.k[layer], self.cache.v[layer],
            k=k.view(B, S, *k.shape[1:]), v=v.view(B, S, *v.shape[1:]), rotary_cos=self.cos,
            rotary_sin=self.sin, cache_seqlens=step.start, block_table=self.cache.table,
            softmax_scale=self.shape.scale, causal=True, rotary_interleaved=False)
        return out.view(q.shape[0], q.shape[1], -1)


class Qwen3Loop:
    """Forward pass of the decoder for one step; attention through ``backend``."""

    def __init__(self, shape, weights, backend, cos, sin):
        self.shape, self.w, self.backend, self.cos, self.sin = shape, weights, backend, cos, sin

    def forward(self, tokens, step):
        """Logits (fp32 [B, vocab]) of the last new token of every request."""
        s, w = self.shape, self.w
        H, D, T = s.hidden, s.head_dim, tokens.shape[0]
        x = F.embedding(tokens, w["embed"])
        for i, lw in enumerate(w["layers"]):
            h = F.rms_norm(x, (H,), lw["ln1"], s.eps)
            q, k, v = F.linear(h, lw["wqkv"]).split([s.heads * D, s.kv_heads * D, s.kv_heads * D], dim=-1)
            q = F.rms_norm(q.reshape(T, s.heads, D), (D,), lw["q_norm"], s.eps)
            k = F.rms_norm(k.reshape(T, s.kv_heads, D), (D,), lw["k_norm"], s.eps)
            v = v.reshape(T, s.kv_heads, D)
            if not self.backend.rotates:
                q = apply_rope(q, self.cos, self.sin, step.positions)
                k = apply_rope(k, self.cos, self.sin, step.positions)
            o = self.backend(i, q, k, v, step)
            x = x + F.linear(o.reshape(T, s.heads * D), lw["wo"])
            h = F.rms_norm(x, (H,), lw["ln2"], s.eps)
            gate, up = F.linear(h, lw["w_gate_up"]).chunk(2, dim=-1)
            x = x + F.linear(F.silu(gate) * up, lw["w_down"])
        if step.prefill:
            x = x[(step.cu_q[1:] - 1).long()]
        return F.linear(F.rms_norm(x, (H,), w["norm"], s.eps), w["embed"]).float()


class Engine:
    """Model + paged cache + attention back-end for a fixed set of requests."""

    def __init__(self, shape, weights, backend_cls, requests, capacity, device, seed=0):
        self.shape = shape
        self.cache = PagedCache(shape, requests, capacity, device, seed)
        self.cos, self.sin = rope_tables(shape, self.cache.capacity, device)
        self.backend = backend_cls(shape, self.cache, self.cos, self.sin)
        self.model = Qwen3Loop(shape, weights, self.backend, self.cos, self.sin)

    def prefill(self, prompts):
        """prompts: list of 1-D int64 device tensors -> (logits [B, vocab], start [B] int32)."""
        step = prefill_step(self.cache, [int(p.shape[0]) for p in prompts], self.shape.page,
                            prompts[0].device)
        return self.model.forward(torch.cat(prompts), step), step.end.clone()

    def decode(self, tokens, start):
        """One token per request at positions ``start``; returns logits [B, vocab]."""
        return self.model.forward(tokens, decode_step(self.cache, start, self.shape.page))


class DecodeGraph:
    """One greedy decode step captured as a CUDA graph over static buffers.

    Each replay reads ``tokens`` and ``start``, writes the next greedy tokens
    into ``tokens`` and column ``col`` of ``history``, and advances ``start``
    and ``col`` by one, so replays chain without host work.
    """

    def __init__(self, engine, tokens, start, history):
        self.engine = engine
        self.tokens, self.start, self.history = tokens, start, history
        self.col = torch.zeros(1, dtype=torch.long, device=tokens.device)
        self.written = 0  # host count of history columns filled, bounds the replays
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            engine.decode(self.tokens, self.start)  # warm-up outside capture
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            logits = engine.decode(self.tokens, self.start)
            self.tokens.copy_(logits.argmax(dim=-1))
            self.history.index_copy_(1, self.col, self.tokens[:, None])
            self.start.add_(1)
            self.col.add_(1)

    def reset(self, tokens, start, col=0):
        self.tokens.copy_(tokens)
        self.start.copy_(start)
        self.col.fill_(col)
        self.written = col

    def replay(self):
        if self.written >= self.history.shape[1]:
            raise IndexError("decode graph replayed past the end of its token history")
        self.graph.replay()
        self.written += 1
