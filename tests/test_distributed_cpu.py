"""KV-sharded decode plumbing on 2 gloo ranks (CPU, no GPU).

Each rank computes its slice's partial attention with the oracle, the product's
``gather_partials`` all-gathers the states over gloo, and the oracle's N-way
merge must reproduce full attention (sinks only on rank 0, empty slices
contribute nothing). This exercises the shard ranges and the gather layout
that the GPU path uses with NCCL.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_queue):
    import oracle
    from flash_attn_b200.distributed import gather_partials, kv_shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        B, HQ, HK, D = 3, 4, 2, 16
        lengths = [37, 1, 64]
        q = rng.standard_normal((B, HQ, D))
        keys = [rng.standard_normal((L, HK, D)) for L in lengths]
        vals = [rng.standard_normal((L, HK, D)) for L in lengths]
        sinks = np.array([0.5, -1.0, 2.0, 0.0])
        outs, lses = [], []
        for b in range(B):
            s, e = kv_shard(lengths[b], rank, world)
            k = keys[b][s:e]
            v = vals[b][s:e]
            o, l = oracle.attention(q[b:b + 1], k, v, [0, 1], cu_k=[0, e - s],
                                    sinks=sinks if rank == 0 else None)
            outs.append(o[0])
            lses.append(l[:, 0])
        partial = torch.from_numpy(np.stack(outs)).float()            # [B,HQ,D]
        partial_lse = torch.from_numpy(np.stack(lses, axis=1)).float()  # [HQ,B]
        gathered, gathered_lse = gather_partials(partial, partial_lse)
        merged, merged_lse = oracle.merge_partials(gathered.double().numpy(), gathered_lse.double().numpy())
        full_o, full_l = [], []
        for b in range(B):
            o, l = oracle.attention(q[b:b + 1], keys[b], vals[b], [0, 1], cu_k=[0, lengths[b]], sinks=sinks)
            full_o.append(o[0])
            full_l.append(l[:, 0])
        np.testing.assert_allclose(merged, np.stack(full_o), rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(merged_lse, np.stack(full_l, axis=1), rtol=1e-5, atol=1e-6)
        assert tuple(gathered.shape) == (world, B, HQ, D)
        result_queue.put((rank, "ok"))
    except Exception as exc:  # report to the parent
        result_queue.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_decode_gather_and_merge_on_gloo(world):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert sorted(results) == [(r, "ok") for r in range(world)], results


def test_kv_shard_ranges_cover_every_token():
    from flash_attn_b200.distributed import kv_shard
    for length in (0, 1, 7, 131072):
        for world in (1, 2, 4, 8):
            spans = [kv_shard(length, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == length
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
