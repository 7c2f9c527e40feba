"""The library inside a serving loop (Qwen3-0.6B-shaped decoder, random bf16 weights).

Teacher-forced protocol of the reference's engine validation
(benchmarks/validate_nanovllm.py:77-106): the frozen SDPA path (oracle,
float64) records logits and greedy choices at every sampler call; the run whose
attention goes through flash_attn_b200 consumes those choices, and per request
and sampler call KL(ref || ours) at temperature 1 must stay <= 1e-3 nats with
the same greedy choice. With random weights the top two logits can tie within
bf16 noise, so a greedy choice is compared only where the reference's top-1
margin exceeds 0.05. The decode step captured as a CUDA graph must replay the
eager steps.
"""

import pytest
import torch

from oracle.engine_sdpa import SdpaAttention
from serving_loop import DecodeGraph, Engine, FusedAttention, NativeAttention, Qwen3Shape, init_weights

pytestmark = pytest.mark.gpu

KL_LIMIT = 1e-3   # nats, validate_nanovllm.py:19
MARGIN = 0.05     # greedy choices are compared where the reference's top-1 lead exceeds this


@pytest.fixture(scope="module")
def model():
    shape = Qwen3Shape()
    return shape, init_weights(shape, torch.device("cuda"), seed=5)


def _prompts(lengths, vocab, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g).cuda() for n in lengths]


def _generate(backend, shape, weights, prompts, steps, forced=None):
    """(logits per sampler call, chosen tokens per call); ``forced`` replaces the choices."""
    engine = Engine(shape, weights, backend, len(prompts), max(p.shape[0] for p in prompts) + steps + 1,
                    prompts[0].device, seed=9)
    logits, start = engine.prefill(prompts)
    trace, chosen = [logits], []
    for i in range(steps + 1):
        tokens = forced[i] if forced is not None else trace[-1].argmax(dim=-1)
        chosen.append(tokens)
        if i == steps:
            break
        trace.append(engine.decode(tokens, start))
        start = start + 1
    return trace, chosen


def _check_teacher_forced(ref_trace, ref_tokens, trace):
    assert len(trace) == len(ref_trace)
    for index, (ref, act) in enumerate(zip(ref_trace, trace)):
        assert torch.isfinite(act).all(), f"non-finite logits at sampler call {index}"
        ref_logp = ref.double().log_softmax(dim=-1)
        act_logp = act.double().log_softmax(dim=-1)
        kl = (ref_logp.exp() * (ref_logp - act_logp)).sum(dim=-1)
        assert float(kl.max()) <= KL_LIMIT, f"KL {float(kl.max()):.3e} at sampler call {index}"
        top2 = ref.topk(2, dim=-1).values
        decided = (top2[:, 0] - top2[:, 1]) > MARGIN
        assert torch.equal(act.argmax(dim=-1)[decided], ref_tokens[index][decided]), \
            f"greedy choice differs at sampler call {index}"


@pytest.mark.parametrize("backend", [NativeAttention, FusedAttention])
def test_teacher_forced_kl_against_sdpa(model, backend):
    shape, weights = model
    # Ragged prompts for the vLLM-style path; the fused path needs equal lengths.
    lengths = [37, 300, 129, 1] if backend is NativeAttention else [200] * 4
    prompts = _prompts(lengths, shape.vocab, seed=11)
    steps = 12
    ref_trace, ref_tokens = _generate(SdpaAttention, shape, weights, prompts, steps)
    trace, _ = _generate(backend, shape, weights, prompts, steps, forced=ref_tokens)
    _check_teacher_forced(ref_trace, ref_tokens, trace)


def test_decode_graph_replays_eager_steps(model):
    shape, weights = model
    prompts = _prompts([64] * 8, shape.vocab, seed=12)
    steps = 6
    trace, chosen = _generate(FusedAttention, shape, weights, prompts, steps)
    engine = Engine(shape, weights, FusedAttention, len(prompts), 64 + steps + 1, prompts[0].device, seed=9)
    logits, start = engine.prefill(prompts)
    torch.testing.assert_close(logits, trace[0], atol=0, rtol=0)
    history = torch.zeros(len(prompts), steps, dtype=torch.long, device="cuda")
    graph = DecodeGraph(engine, logits.argmax(dim=-1), start.clone(), history)
    graph.reset(chosen[0], start)
    for _ in range(steps):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(history, torch.stack(chosen[1:], dim=1))
    with pytest.raises(IndexError):
        graph.replay()
