"""KV-sharded decode (``ShardedDecoder``): one spawned process per GPU, with the
peer-memory exchange (push + flags + bounded wait) and with the NCCL all-gather.

Each rank holds its ``kv_shard`` slice of every sequence in its own paged cache,
decodes it, and one all-gather of the packed (out, lse) rows plus the N-way
merge must equal decode over the whole KV (oracle), sinks counted once. The
world is 2 ranks on 2 GPUs (ranks never share a GPU); on a 1-GPU box the test
skips, since a single rank would exercise no exchange (the gloo test in
test_distributed_cpu.py covers the host-side logic there).
"""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paged(rows, page, device):
    """Sequences (lists of [n, HK, D] tensors) -> paged cache, block table, lengths."""
    counts = [int(r.shape[0]) for r in rows]
    cols = max((c + page - 1) // page for c in counts) + 1
    cache = torch.zeros(len(rows) * cols, page, *rows[0].shape[1:], dtype=rows[0].dtype)
    for b, r in enumerate(rows):
        for i in range(r.shape[0]):
            cache[b * cols + i // page, i % page] = r[i]
    table = torch.arange(len(rows) * cols, dtype=torch.int32).reshape(len(rows), cols)
    return cache.to(device), table.to(device), torch.tensor(counts, dtype=torch.int32, device=device)


def _worker(rank, world, port, kv, exchange, queue):
    import torch.distributed as dist
    from flash_attn_b200.distributed import ShardedDecoder, kv_shard
    from helpers import assert_attention_close, assert_lse_close, reference
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=device)
    try:
        g = torch.Generator().manual_seed(91)
        B, HQ, HK, D = 4, 16, 2, 128
        lengths = [1, 700, 3000, 0]
        dtype = torch.bfloat16 if kv == "bf16" else torch.float8_e4m3fn
        keys = [torch.randn(n, HK, D, generator=g).to(dtype) for n in lengths]
        vals = [torch.randn(n, HK, D, generator=g).to(dtype) for n in lengths]
        q = torch.randn(B, HQ, D, generator=g).to(torch.bfloat16).to(device)
        sinks = torch.linspace(-1, 1, HQ).to(device)
        spans = [kv_shard(n, rank, world) for n in lengths]
        kc, table, used = _paged([k[s:e] for k, (s, e) in zip(keys, spans)], 16, device)
        vc, _, _ = _paged([v[s:e] for v, (s, e) in zip(vals, spans)], 16, device)
        cq = torch.arange(B + 1, dtype=torch.int32, device=device)
        decoder = ShardedDecoder(B, HQ, D, torch.bfloat16, device, exchange=exchange)
        assert decoder.exchange == exchange
        results = []
        for _ in range(3):  # buffers (both parities of the peer-memory exchange) are reused across steps
            out, lse = decoder.step(q, kc, vc, cu_seqlens_q=cq, seqused_k=used,
                                    max_seqlen_k=max(int(used.max()), 1), block_table=table, s_aux=sinks)
            results.append((out.clone(), lse.clone()))
        torch.cuda.synchronize()
        from flash_attn_b200 import _capi
        assert _capi.library().fa_pipeline_timeouts(1) == 0, "an exchange wait timed out"
        for o, l in results[1:]:
            assert torch.equal(o, results[0][0]) and torch.equal(l, results[0][1])
        kf, tf, uf = _paged(keys, 16, "cpu")
        vf, _, _ = _paged(vals, 16, "cpu")
        ref, refl = reference(q, kf, vf, cq, used_k=uf, block_table=tf, sinks=sinks)
        assert_attention_close(out, ref, torch.bfloat16)
        assert_lse_close(lse, refl)
        queue.put((rank, "ok"))
    except Exception as exc:  # report to the parent
        queue.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_sharded_decoder_matches_full_decode(kv, exchange):
    if torch.cuda.device_count() < 2:
        pytest.skip("the exchange needs 2 GPUs (one rank per GPU); a single rank would exercise no exchange")
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kv, exchange, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert sorted(results) == [(r, "ok") for r in range(world)], results
