"""Host logic of the serving loop on CPU (no GPU): page slots, positions and the
step metadata, run with the frozen-SDPA back-end (oracle) on a tiny shape.
Decoding tokens one at a time after a prefill must reproduce the logits of a
single longer prefill, and ragged requests must not disturb one another."""

import torch

from oracle.engine_sdpa import SdpaAttention
from serving_loop import Engine, Qwen3Shape, init_weights

SHAPE = Qwen3Shape(vocab=211, hidden=64, layers=2, heads=4, kv_heads=2, head_dim=32, intermediate=96)


def _engine(requests, capacity):
    weights = init_weights(SHAPE, torch.device("cpu"), seed=3, std=0.2)
    return Engine(SHAPE, weights, SdpaAttention, requests, capacity, torch.device("cpu"), seed=4)


def test_incremental_decode_matches_longer_prefill():
    g = torch.Generator().manual_seed(1)
    full = [torch.randint(0, SHAPE.vocab, (n,), generator=g) for n in (21, 40, 17)]
    extra = 5
    engine = _engine(3, 64)
    logits, start = engine.prefill([p[:-extra] for p in full])
    for j in range(extra):
        tokens = torch.stack([p[len(p) - extra + j] for p in full])
        logits = engine.decode(tokens, start)
        start = start + 1
    reference, end = _engine(3, 64).prefill(full)
    assert torch.equal(end, start)
    torch.testing.assert_close(logits, reference, atol=2e-2, rtol=0)


def test_ragged_requests_are_independent():
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, SHAPE.vocab, (n,), generator=g) for n in (9, 33, 1)]
    together, _ = _engine(3, 48).prefill(prompts)
    for i, p in enumerate(prompts):
        alone, _ = _engine(1, 48).prefill([p])
        torch.testing.assert_close(together[i:i + 1], alone, atol=2e-2, rtol=0)


def test_slots_past_the_table_are_skipped():
    from serving_loop import PagedCache
    cache = PagedCache(SHAPE, 2, 32, torch.device("cpu"), seed=1)
    rows = torch.tensor([0, 0, 1, 1])
    positions = torch.tensor([0, 31, 32, 1000])
    slots = cache.slots(rows, positions, SHAPE.page)
    assert slots[0] == cache.table[0, 0] * 16 and slots[1] == cache.table[0, 1] * 16 + 15
    assert slots[2:].tolist() == [-1, -1]
