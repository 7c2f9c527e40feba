"""Benchmark: paged-decode HBM TB/s (and prefill TFLOP/s) vs the B200 roofline.

Default workload (the one quoted at 1/2/4/8 GPUs):
long-context FP8 E4M3 paged decode with split-KV. 64 requests x 131072 cached
tokens, page 16, 32 query / 8 KV heads, head_dim 128. The cache is built by
store_kvcache from seeded N(0,1) bf16 rows with per-head scales U[1/448,4/448]
through a seeded slot_mapping over randomly permuted pages. With N GPUs the KV
sequence is sharded: rank r owns tokens [r*C/N, (r+1)*C/N) of every request in
its own page pool; each rank decodes its shard to an fp32 partial (out, LSE),
the partials are all-gathered with NCCL and merged by the merge kernel.

`value` = algorithmic bytes of one decode step (every cached K/V byte read once
plus tables, q and out) / max-over-ranks device time per step (strong scaling).
`e2e` = the same bytes / the time of a full serving step through the public API
with host buffers: H2D of q and of the step's new K/V token, store_kvcache of
that token, attention, D2H of the output.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload fp8_decode|prefill|prefill_softcap_window|prefill_fp8kv|prefill_alibi|prefill_alibi_softcap|bf16_decode|serving]
                    [--attention-path fused|native] [--small]
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "flash-attn-mps_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "paged-decode HBM TB/s & prefill TFLOP/s vs B200 roofline at 1/2/4/8 GPUs"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# --------------------------------------------------------------------- clocks
# Host-time windows (time.monotonic() before the first timed launch, after the
# synchronize that ends the timed region) of every timed region so far; the
# clock record of a measurement keeps the samples taken inside its windows.
TIMED_WINDOWS = []


class ClockSampler:
    """SM clocks and throttle reasons sampled while a measurement runs
    (read-only). In-process NVML reads every 5 ms, timestamped, so that a timed
    region of tens of milliseconds still gets several samples and the record
    can be limited to the timed windows; `nvidia-smi -lms 200` when NVML is
    unavailable. The device is the torch device `index`, matched to NVML by
    PCI bus id."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits (nvml.h): HW slowdown 0x8 (and HW power
    # brake 0x80), HW thermal 0x40, SW thermal 0x20, SW power cap 0x4.
    REASONS = (("hw_slowdown", 0x8 | 0x80), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index, period_s=0.005):
        self.index = index
        self.period = period_s
        self.proc = None
        self.thread = None
        self.lines = []
        self.samples = []  # (host time, sm_mhz, reasons bitmask)
        self.smax = None
        self.stop_flag = threading.Event()
        self.source = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(self.index)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def start(self):
        try:
            import pynvml
            handle = self._nvml_handle()
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))

            def poll():
                while not self.stop_flag.is_set():
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                        self.samples.append((time.monotonic(), float(sm), int(rs)))
                    except Exception:
                        pass
                    self.stop_flag.wait(self.period)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            self.source = "nvml 5 ms"
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            self.source = "nvidia-smi 200 ms"
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    @staticmethod
    def in_windows(samples, windows):
        """The samples taken inside any of the host-time windows."""
        return [x for x in samples if any(t0 <= x[0] <= t1 for t0, t1 in windows)]

    def stop(self, windows=None):
        """Median SM clock and the throttle reasons seen. With ``windows``
        (host-time spans of the timed regions) only samples inside them count;
        if none fell inside, all samples of the run are reported and
        ``timed_windows_only`` is false."""
        if self.source is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"], "samples": 0}
        if self.proc is None:
            self.stop_flag.set()
            self.thread.join(timeout=2)
            inside = self.in_windows(self.samples, windows) if windows else []
            use = inside or self.samples
            sm = [x for _, x, _ in use]
            reasons = sorted({name for _, _, mask in use for name, bit in self.REASONS if mask & bit})
            out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.smax,
                   "reasons": reasons, "samples": len(sm), "source": self.source}
            if windows:
                out["timed_windows_only"] = bool(inside)
                out["timed_s"] = round(sum(t1 - t0 for t0, t1 in windows), 4)
            return out
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = [n for n, _ in self.REASONS]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "source": self.source}


# ------------------------------------------------------------------ helpers
def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(value, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------ config 4 setup
CFG4 = dict(batch=64, ctx=131072, page=16, hq=32, hkv=8, d=128)


def build_fp8_cache(rank, world, cfg, seed=4):
    """This rank's shard of the config-4 FP8 paged cache, built by store_kvcache."""
    import torch
    from flash_attn_b200 import store_kvcache
    B, C, P, HK, D = cfg["batch"], cfg["ctx"], cfg["page"], cfg["hkv"], cfg["d"]
    shard = C // world
    pages_per_req = shard // P
    n_pages = B * pages_per_req
    dev = torch.device("cuda")
    gen = torch.Generator(device="cpu").manual_seed(seed * 1000 + rank)
    perm = torch.randperm(n_pages, generator=gen).to(torch.int32)
    table = perm.reshape(B, pages_per_req).to(dev)
    ks = ((1 + 3 * torch.rand(HK, generator=gen)) / 448).to(dev)
    vs = ((1 + 3 * torch.rand(HK, generator=gen)) / 448).to(dev)
    k_cache = torch.empty(n_pages, P, HK, D, dtype=torch.float8_e4m3fn, device=dev)
    v_cache = torch.empty_like(k_cache)
    g = torch.Generator(device=dev).manual_seed(seed * 1000 + rank + 7)
    chunk_req = max(1, (1 << 20) // shard)
    pos = torch.arange(shard, device=dev)
    for b0 in range(0, B, chunk_req):
        b1 = min(B, b0 + chunk_req)
        n = (b1 - b0) * shard
        k = torch.randn(n, HK, D, device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
        v = torch.randn(n, HK, D, device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
        slots = (table[b0:b1, pos // P].long() * P + (pos % P)).reshape(-1)
        store_kvcache(k, v, k_cache, v_cache, slots, k_scale=ks, v_scale=vs)
        del k, v
    torch.cuda.synchronize()
    return k_cache, v_cache, table, ks, vs


def cfg4_query(cfg, seed=99):
    """Config-4 queries [B, Hq, D] bf16 on the host (seeded)."""
    import torch
    gq = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(cfg["batch"], cfg["hq"], cfg["d"], generator=gq).to(torch.bfloat16), gq


def build_cfg3(cfg):
    """Config 3 exactly as timed: B requests with contexts ~U[cmin, cmax]
    (seeded), a bf16 paged cache of N(0,1) rows whose pages come from a seeded
    random permutation, and N(0,1) queries. Returns a dict of device tensors
    plus the host-side contexts and pages per request."""
    import numpy as np
    import torch
    rng = np.random.default_rng(cfg["seed"])
    ctx = rng.integers(cfg["cmin"], cfg["cmax"] + 1, size=cfg["batch"])
    P = cfg["page"]
    pages_per = (ctx + P - 1) // P
    n_pages = int(pages_per.sum())
    max_pages = int(pages_per.max())
    perm = torch.from_numpy(rng.permutation(n_pages).astype(np.int32))
    table = torch.zeros(cfg["batch"], max_pages, dtype=torch.int32)
    off = 0
    for b in range(cfg["batch"]):
        table[b, :pages_per[b]] = perm[off:off + pages_per[b]]
        off += pages_per[b]
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(cfg["seed"])
    kc = torch.randn(n_pages, P, cfg["hkv"], cfg["d"], device=dev, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(n_pages, P, cfg["hkv"], cfg["d"], device=dev, generator=g, dtype=torch.bfloat16)
    q = torch.randn(cfg["batch"], cfg["hq"], cfg["d"], device=dev, generator=g, dtype=torch.bfloat16)
    return {"q": q, "k_cache": kc, "v_cache": vc, "table": table.to(dev),
            "used": torch.from_numpy(ctx.astype(np.int32)).to(dev),
            "cu_q": torch.arange(cfg["batch"] + 1, dtype=torch.int32, device=dev),
            "ctx": ctx, "pages_per": pages_per}


def gather_request(cache, table, b, length, page):
    """Rows [length, Hkv, D] of request b of a paged cache (device gather)."""
    n = (length + page - 1) // page
    return cache[table[b, :n].long()].reshape(-1, *cache.shape[2:])[:length]


def torch_decode_reference(q, k_rows, v_rows, k_descale=None, v_descale=None, scale=None):
    """fp32 single-query attention of one request on the GPU: q [Hq, D],
    K/V rows [L, Hkv, D] (any float or FP8 dtype), per-KV-head descales.
    Returns out [Hq, Dv] and natural-log LSE [Hq] in fp32."""
    import torch
    hq, d = q.shape
    hkv = k_rows.shape[1]
    scale = d ** -0.5 if scale is None else scale
    k = k_rows.float().permute(1, 0, 2)  # [Hkv, L, D]
    v = v_rows.float().permute(1, 0, 2)
    if k_descale is not None:
        k = k * k_descale.float().reshape(hkv, 1, 1)
    if v_descale is not None:
        v = v * v_descale.float().reshape(hkv, 1, 1)
    qg = q.float().reshape(hkv, hq // hkv, d)
    s = torch.matmul(qg, k.transpose(1, 2)) * scale  # [Hkv, G, L]
    lse = torch.logsumexp(s, dim=-1)
    o = torch.matmul(torch.exp(s - lse[..., None]), v)
    return o.reshape(hq, -1), lse.reshape(hq)


def sample_requests(lengths, count=6, seed=0):
    """Shortest, longest and count-2 further seeded distinct request indices."""
    import numpy as np
    lengths = np.asarray(lengths)
    picked = [int(np.argmin(lengths)), int(np.argmax(lengths))]
    if picked[0] == picked[1]:
        picked = [0, len(lengths) - 1]
    rng = np.random.default_rng(seed)
    rest = [i for i in rng.permutation(len(lengths)).tolist() if i not in picked]
    return picked + rest[:max(0, count - 2)]


def check_close(out, lse, ref_out, ref_lse, what):
    """The north-star gate (max-abs 1e-2 on outputs, 1e-3 on LSE) plus a
    scale-aware one (1 % of the reference's largest output), since long-context
    decode outputs are small averages."""
    err = (out.float() - ref_out).abs().max().item()
    scale = ref_out.abs().max().item()
    lerr = (lse.float() - ref_lse).abs().max().item()
    if not (err <= 1e-2 and err <= 1e-2 * scale + 2e-5 and lerr <= 1e-3):
        raise AssertionError(f"{what}: max-abs {err:.3e} (largest output {scale:.3e}), LSE max-abs {lerr:.3e}")
    return err, lerr


def cfg4_bytes(cfg):
    B, C, HK, D, HQ = cfg["batch"], cfg["ctx"], cfg["hkv"], cfg["d"], cfg["hq"]
    kv = B * C * HK * 2 * D * 1
    table = B * (C // cfg["page"]) * 4
    qo = 2 * B * HQ * D * 2
    return kv + table + qo


def profiled_traffic(name, key="traffic_bytes_per_full_launch"):
    """DRAM bytes per launch recorded from an ncu capture in profiles/ (or None)."""
    path = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith(key + ":"):
            return float(line.split(":", 1)[1])
    return None


def run_fp8_decode(args, rank, world, peaks, peak_kind):
    import torch
    import torch.distributed as dist
    from flash_attn_b200 import store_kvcache
    from flash_attn_b200._attention import attention

    cfg = dict(CFG4)
    if args.small:
        cfg["ctx"] = 8192  # profiling case: 1.07 GB of FP8 cache, still far larger than L2
    B, C, HQ, HK, D = cfg["batch"], cfg["ctx"], cfg["hq"], cfg["hkv"], cfg["d"]
    shard = C // world
    dev = torch.device("cuda")
    k_cache, v_cache, table, ks, vs = build_fp8_cache(rank, world, cfg)
    q_host, gq = cfg4_query(cfg)
    q_host = q_host.pin_memory()
    q = q_host.to(dev)
    kd = ks.reshape(1, HK).expand(B, HK)
    vd = vs.reshape(1, HK).expand(B, HK)
    cu_q = torch.arange(B + 1, dtype=torch.int32, device=dev)
    used = torch.full((B,), shard, dtype=torch.int32, device=dev)
    sinks = None
    out = torch.empty(B, HQ, D, dtype=torch.bfloat16, device=dev)
    partial = torch.empty(B, HQ, D, dtype=torch.float32, device=dev)
    decoder = None
    if world > 1:
        from flash_attn_b200.distributed import ShardedDecoder
        decoder = ShardedDecoder(B, HQ, D, torch.bfloat16, dev)

    def step(q_in):
        if world == 1:
            return attention(q_in, k_cache, v_cache, cu_seqlens_q=cu_q, seqused_k=used, max_seqlen_q=1,
                             max_seqlen_k=shard, block_table=table, k_descale=kd, v_descale=vd,
                             s_aux=sinks, out=out)
        return decoder.step(q_in, k_cache, v_cache, cu_seqlens_q=cu_q, seqused_k=used,
                            max_seqlen_k=shard, block_table=table, k_descale=kd, v_descale=vd,
                            s_aux=sinks)

    # ---- device-resident timing --------------------------------------------
    for _ in range(args.warmup):
        step(q)
    barrier(world)
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    from flash_attn_b200._capi import kernel_launches
    launches_before = kernel_launches()
    t0 = time.monotonic()
    start.record(stream)
    for _ in range(args.steps):
        step(q)
    end.record(stream)
    barrier(world)
    windows = [(t0, time.monotonic())]
    launches = kernel_launches() - launches_before
    ms = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms, world)

    # ---- dominant kernel alone: the local decode operation (decode + split merge)
    k_start, k_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    t0 = time.monotonic()
    k_start.record(stream)
    for _ in range(args.steps):
        attention(q, k_cache, v_cache, cu_seqlens_q=cu_q, seqused_k=used, max_seqlen_q=1,
                  max_seqlen_k=shard, block_table=table, k_descale=kd, v_descale=vd,
                  out=partial if world > 1 else out)
    k_end.record(stream)
    barrier(world)
    windows.append((t0, time.monotonic()))
    kernel_ms = max_over_ranks(k_start.elapsed_time(k_end) / args.steps, world)
    clocks = sampler.stop(windows) if sampler else None

    # ---- end to end through the public API with host buffers ----------------
    new_k_host = torch.randn(B, HK, D, generator=gq).to(torch.bfloat16).pin_memory()
    new_v_host = torch.randn(B, HK, D, generator=gq).to(torch.bfloat16).pin_memory()
    out_host = torch.empty(B, HQ, D, dtype=torch.bfloat16).pin_memory()
    # The new token replaces the last cached position, keeping the context fixed.
    last = shard - 1
    slots = (table[:, last // cfg["page"]].long() * cfg["page"] + last % cfg["page"]).contiguous()
    is_last_rank = rank == world - 1

    def e2e_step():
        qd = q_host.to(dev, non_blocking=True)
        if is_last_rank:
            nk = new_k_host.to(dev, non_blocking=True)
            nv = new_v_host.to(dev, non_blocking=True)
            store_kvcache(nk, nv, k_cache, v_cache, slots, k_scale=ks, v_scale=vs)
        o = step(qd)
        result = o[0] if isinstance(o, tuple) else o
        out_host.copy_(result, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier(world)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e_end.record(stream)
    barrier(world)
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end) / args.steps, world)

    parity = cfg4_parity(q, k_cache, v_cache, table, kd, vd, used, cu_q, shard, cfg, world, step, partial)

    total_bytes = cfg4_bytes(cfg)
    rank_bytes = total_bytes / world
    value = total_bytes / (ms * 1e-3) / 1e12
    achieved_gbs = rank_bytes / (kernel_ms * 1e-3) / 1e9
    result = {
        "value": value, "unit": "TB/s", "ms_per_step": ms,
        "e2e": {"value": total_bytes / (e2e_ms * 1e-3) / 1e12, "unit": "TB/s",
                "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": q_host.numel() * 2 + (new_k_host.numel() + new_v_host.numel()) * 2,
                "d2h_bytes_per_step": out_host.numel() * 2},
        "roofline": {"bound": "hbm", "kernel": "decode_mma_kernel (+ its split merge)",
                     "achieved": achieved_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved_gbs / peaks["hbm_gbs"], "peak_kind": f"{peak_kind} (hbm_gbs)",
                     "traffic": (profiled_traffic("decode_mma_fp8_cfg4.md") / world
                                 if profiled_traffic("decode_mma_fp8_cfg4.md") and not args.small else None),
                     "traffic_source": "profiles/decode_mma_fp8_cfg4.md (ncu, small case scaled)",
                     "algorithmic_bytes_per_launch": rank_bytes,
                     "kernel_ms": kernel_ms},
        "dtype": "fp8_e4m3 KV / bf16 q, fp32 softmax",
        "config": {"workload": "cfg4 long-context FP8 E4M3 paged decode, split-KV"
                               + (" (small profiling case)" if args.small else ""),
                   "batch": B, "context": C, "block_size": cfg["page"], "q_heads": HQ, "kv_heads": HK,
                   "head_dim": D, "l2": "17.2 GB cache > L2, no flush",
                   "parallelism": (f"kv-seq sharded x{world}, {decoder.exchange} exchange + merge" if decoder
                                   else "single GPU")},
        "gpu_launches": launches,
        "clocks": clocks,
        "parity": parity,
    }
    return result


def cfg4_parity(q, k_cache, v_cache, table, kd, vd, used, cu_q, shard, cfg, world, step, partial):
    """Sampled self-check of the timed configuration (outside every timed
    region): for the first, the last and 4 seeded requests, this rank's fp32
    partial over its KV shard and the merged bf16 output of a step against a
    torch fp32 reference computed on the GPU from the same cache bytes."""
    import torch
    import torch.distributed as dist
    from flash_attn_b200._attention import attention
    B, P = cfg["batch"], cfg["page"]
    picks = sample_requests([shard] * B)
    _, part_lse = attention(q, k_cache, v_cache, cu_seqlens_q=cu_q, seqused_k=used, max_seqlen_q=1,
                            max_seqlen_k=shard, block_table=table, k_descale=kd, v_descale=vd, out=partial)
    merged = step(q)
    merged_out, merged_lse = merged if isinstance(merged, tuple) else (merged, None)
    refs_o, refs_l = [], []
    worst = 0.0
    for b in picks:
        k_rows = gather_request(k_cache, table, b, shard, P)
        v_rows = gather_request(v_cache, table, b, shard, P)
        ro, rl = torch_decode_reference(q[b], k_rows, v_rows, kd[b], vd[b])
        err, _ = check_close(partial[b], part_lse[:, b], ro, rl, f"cfg4 request {b} partial")
        worst = max(worst, err)
        refs_o.append(ro)
        refs_l.append(rl)
    ro = torch.stack(refs_o)  # [S, Hq, D]
    rl = torch.stack(refs_l)  # [S, Hq]
    if world > 1:
        go = [torch.empty_like(ro) for _ in range(world)]
        gl = [torch.empty_like(rl) for _ in range(world)]
        dist.all_gather(go, ro)
        dist.all_gather(gl, rl)
        gl_t = torch.stack(gl)
        rl = torch.logsumexp(gl_t, dim=0)
        ro = sum(torch.exp(gl_t[r] - rl)[..., None] * go[r] for r in range(world))
    for i, b in enumerate(picks):
        check_close(merged_out[b], rl[i] if merged_lse is None else merged_lse[:, b], ro[i], rl[i],
                    f"cfg4 request {b} merged output")
    return {"status": "ok", "requests": picks, "max_abs": worst,
            "against": "torch fp32 on the same cache bytes"}


# ------------------------------------------------- config 2 / config 3 (N=1)
CFG2 = dict(seqs=32, lmin=64, lmax=4096, hq=32, hkv=8, d=128, seed=2)
CFG3 = dict(batch=256, cmin=512, cmax=32768, page=16, hq=32, hkv=8, d=128, seed=3)


def cfg2_lengths(cfg):
    import numpy as np
    rng = np.random.default_rng(cfg["seed"])
    return rng.integers(cfg["lmin"], cfg["lmax"] + 1, size=cfg["seqs"]).tolist()


def cfg2_flops(lengths, cfg, window=-1, dims=None):
    pairs = 0
    for L in lengths:
        if window < 0:
            pairs += L * (L + 1) // 2
        else:
            w = window + 1
            pairs += sum(min(i + 1, w) for i in range(L))
    dq, dv = dims if dims else (cfg["d"], cfg["d"])
    return cfg["hq"] * (2 * dq + 2 * dv) * pairs


BURST_WINDOW_S = 0.04  # timed window of a secondary held against the burst peak


def rested(measure, pause=2.0):
    """Run a secondary measurement after a short idle pause (the headline run
    leaves the GPU at its power cap with lowered SM clocks) and attach the SM
    clocks sampled while it ran."""
    import torch
    time.sleep(pause)
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    first = len(TIMED_WINDOWS)
    result = measure()
    result["clocks"] = sampler.stop(TIMED_WINDOWS[first:])
    return result


def time_loop(fn, steps, warmup, min_seconds=0.0):
    """Device time per call of ``fn`` over ``steps`` calls after ``warmup``
    (CUDA events on the current stream). With ``min_seconds`` the step count is
    raised so that the timed region lasts at least that long (estimated from
    three calls), which gives the clock sampler several samples; returns
    (ms, steps) then, else ms."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if min_seconds > 0:
        s.record(stream)
        for _ in range(3):
            fn()
        e.record(stream)
        torch.cuda.synchronize()
        est = max(s.elapsed_time(e) / 3, 1e-3)
        steps = max(steps, int(min_seconds * 1e3 / est) + 1)
    t0 = time.monotonic()
    s.record(stream)
    for _ in range(steps):
        fn()
    e.record(stream)
    torch.cuda.synchronize()
    TIMED_WINDOWS.append((t0, time.monotonic()))
    ms = s.elapsed_time(e) / steps
    return (ms, steps) if min_seconds > 0 else ms


def run_prefill(peaks, peak_kind, steps=20, warmup=5, softcap=0.0, window=(-1, -1), small=False, fp8_kv=False,
                kv_slice=None, alibi=False, min_seconds=0.0, sustained=False, dims=None):
    """Config 2: varlen causal prefill bf16 through flash_attn_varlen_func.

    ``fp8_kv``: the same lengths over FP8 E4M3 K/V with per-(request, KV head)
    descales through the vLLM entry (vLLM's FP8 KV-cache prefill): an exact
    16-bit copy of the K/V rows, then the tcgen05 prefill.
    ``kv_slice=(h0, h1)``: only KV heads [h0, h1) and their query heads (one
    GPU's share when the prefill is sharded by head groups).
    ``alibi``: the standard geometric ALiBi slopes 2^(-8(h+1)/H) per query head.
    ``dims=(dq, dv)``: other QK / V head dims (256/256, DiffKV 192/128).
    """
    import torch
    from flash_attn_b200 import flash_attn_varlen_func
    from flash_attn_b200.vllm import flash_attn_varlen_func as vllm_varlen
    cfg = dict(CFG2)
    if small:
        cfg["seqs"] = 4  # profiling case
    lens = cfg2_lengths(cfg)
    total = sum(lens)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(cfg["seed"])
    dq, dv = dims if dims else (cfg["d"], cfg["d"])
    q = torch.randn(total, cfg["hq"], dq, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(total, cfg["hkv"], dq, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(total, cfg["hkv"], dv, device=dev, generator=g).to(torch.bfloat16)
    if kv_slice is not None:
        group = cfg["hq"] // cfg["hkv"]
        h0, h1 = kv_slice
        q = q[:, h0 * group:h1 * group].contiguous()
        k, v = k[:, h0:h1].contiguous(), v[:, h0:h1].contiguous()
        cfg["hq"], cfg["hkv"] = (h1 - h0) * group, h1 - h0
    cu = torch.tensor([0] + list(__import__("itertools").accumulate(lens)), dtype=torch.int32, device=dev)
    out = torch.empty(total, cfg["hq"], dv, dtype=q.dtype, device=dev)
    if fp8_kv:
        k, v = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
        kd = torch.full((len(lens), cfg["hkv"]), 0.5, device=dev)
        vd = torch.full((len(lens), cfg["hkv"]), 2.0, device=dev)
        timed = time_loop(lambda: vllm_varlen(q, k, v, max(lens), cu, max(lens), cu_seqlens_k=cu, causal=True,
                                              k_descale=kd, v_descale=vd, out=out), steps, warmup, min_seconds)
    else:
        slopes = (torch.tensor([2.0 ** (-8.0 * (h + 1) / cfg["hq"]) for h in range(cfg["hq"])], device=dev)
                  if alibi else None)
        timed = time_loop(lambda: flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), causal=True,
                                                         softcap=softcap, window_size=window, alibi_slopes=slopes,
                                                         out=out),
                          steps, warmup, min_seconds)
    ms, steps = timed if isinstance(timed, tuple) else (timed, steps)
    flops = cfg2_flops(lens, cfg, window[0], dims)
    tflops = flops / (ms * 1e-3) / 1e12
    return {"workload": "cfg2 varlen causal prefill bf16, 32 seqs L~U[64,4096], 32q/8kv, D=128"
                        + (f", softcap={softcap}, window={tuple(window)}" if softcap or window[0] >= 0 else "")
                        + (", FP8 E4M3 K/V + descales" if fp8_kv else "")
                        + (f", KV heads {kv_slice[0]}..{kv_slice[1] - 1} only" if kv_slice else "")
                        + (", ALiBi slopes" if alibi else "")
                        + (f", head dims {dq}/{dv}" if dims else "")
                        + (" (small profiling case)" if small else ""),
            "total_tokens": total, "tflop_per_step": flops / 1e12, "ms_per_step": ms, "steps": steps,
            "TFLOP/s": tflops,
            "roofline": dict(roofline_tensor(tflops, peaks, peak_kind, sustained), **prefill_traffic(
                plain=not (softcap or window[0] >= 0 or fp8_kv or kv_slice or alibi or dims or small),
                tokens=total, cfg=cfg, dims=(dq, dv)))}


def prefill_traffic(plain, tokens, cfg, dims):
    """DRAM bytes of one config-2 prefill launch from the ncu capture in
    profiles/ (plain config-2 workload only), beside the algorithmic bytes:
    Q, K and V read once, the output and the LSE written once."""
    dq, dv = dims
    alg = tokens * (cfg["hq"] * dq * 2 + cfg["hkv"] * (dq + dv) * 2 + cfg["hq"] * dv * 2 + cfg["hq"] * 4)
    traffic = profiled_traffic("prefill_sm100_cfg2_traffic.md") if plain else None
    return {"traffic": traffic, "algorithmic_bytes": alg,
            "traffic_source": "profiles/prefill_sm100_cfg2_traffic.md (ncu, full launch)" if traffic else None}


def roofline_tensor(tflops, peaks, peak_kind, sustained=False):
    """Tensor-bound roofline: the burst cuBLAS bf16 peak for a kernel timed in a
    short window at full clocks, the sustained one (seconds-long loop under the
    power cap) for a window long enough to reach the power cap."""
    burst = peaks["bf16_tflops"]
    sus = peaks.get("bf16_tflops_sustained", burst)
    peak = sus if sustained else burst
    return {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s", "frac": tflops / peak,
            "peak_kind": f"{peak_kind} bf16_tflops{'_sustained' if sustained else ' burst'}",
            "frac_of_burst": tflops / burst, "frac_of_sustained": tflops / sus}


def run_bf16_decode(peaks, peak_kind, steps=50, warmup=5, small=False, min_seconds=0.0, d=128):
    """Config 3: paged bf16 decode, B=256, ctx ~U[512, 32768], page 16, plus a
    sampled check of the timed output against a torch fp32 reference. With
    d=256: the same layout at head dim 256 over 64 requests (8.8 GB of cache)."""
    import torch
    from flash_attn_b200._attention import attention
    cfg = dict(CFG3, d=d)
    if d != 128:
        cfg["batch"] = 64
    if small:
        cfg["batch"] = 16  # profiling case
    w = build_cfg3(cfg)
    ctx, pages_per = w["ctx"], w["pages_per"]
    out = torch.empty_like(w["q"])
    lse_box = []

    def call():
        lse_box[:] = [attention(w["q"], w["k_cache"], w["v_cache"], cu_seqlens_q=w["cu_q"], seqused_k=w["used"],
                                max_seqlen_q=1, max_seqlen_k=int(ctx.max()), block_table=w["table"], out=out)[1]]

    timed = time_loop(call, steps, warmup, min_seconds=min_seconds)
    ms, steps = timed if isinstance(timed, tuple) else (timed, steps)
    worst = 0.0
    picks = sample_requests(ctx)
    for b in picks:
        ro, rl = torch_decode_reference(w["q"][b], gather_request(w["k_cache"], w["table"], b, int(ctx[b]), cfg["page"]),
                                        gather_request(w["v_cache"], w["table"], b, int(ctx[b]), cfg["page"]))
        worst = max(worst, check_close(out[b], lse_box[0][:, b], ro, rl, f"cfg3 request {b}")[0])
    nbytes = int(ctx.sum()) * cfg["hkv"] * 2 * cfg["d"] * 2 + int(pages_per.sum()) * 4 + 2 * w["q"].numel() * 2
    gbs = nbytes / (ms * 1e-3) / 1e9
    del w
    return {"workload": f"cfg3 paged bf16 decode, B={cfg['batch']}, ctx~U[512,32768], page 16, 32q/8kv, D={d}",
            "bytes_per_step": nbytes, "ms_per_step": ms, "steps": steps, "TB/s": gbs / 1e3,
            "parity": {"status": "ok", "requests": len(picks), "max_abs": worst},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "peak_kind": f"{peak_kind} hbm_gbs"}}


# ------------------------------------------------------- config 5 (N=1)
CFG5 = dict(requests=64, prompt=1024, decode_steps=256, seed=5)


def _graph_ms(fn, reps, warmup=2):
    """Device time of ``fn`` captured as one CUDA graph, per replay."""
    import torch
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    ms = time_loop(graph.replay, reps, warmup)
    del graph
    return ms


def cpu_serving_sample(prompt=256, decode_steps=16, seed=5):
    """The reference's frozen SDPA engine path (oracle) on host cores: 1 request."""
    import torch
    from oracle.engine_sdpa import SdpaAttention
    from serving_loop import Engine, Qwen3Shape, init_weights
    shape = Qwen3Shape()
    cpu = torch.device("cpu")
    weights = init_weights(shape, cpu, seed=seed)
    engine = Engine(shape, weights, SdpaAttention, 1, prompt + decode_steps + 1, cpu, seed=seed)
    tokens = torch.randint(0, shape.vocab, (prompt,), generator=torch.Generator().manual_seed(seed))
    t0 = time.perf_counter()
    logits, start = engine.prefill([tokens])
    for _ in range(decode_steps):
        logits = engine.decode(logits.argmax(dim=-1), start)
        start = start + 1
    dt = time.perf_counter() - t0
    return {"value": (decode_steps + 1) / dt, "unit": "output tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "seconds": dt,
            "sample": f"1 request: {prompt}-token prompt + {decode_steps} greedy decode steps, full 28-layer "
                      f"model, torch CPU GEMMs + float64 SDPA attention (the reference's frozen SDPA path)"}


def run_store(peaks, peak_kind, steps=20, warmup=3, fp8=True, tokens=524288, min_seconds=0.0):
    """store_kvcache bandwidth on config 4's cache-build shape: `tokens` new
    bf16 K and V rows [T, 8, 128] scattered into a page-16 cache through a
    seeded permutation of slots, quantised to FP8 E4M3 with per-head scales
    U[1/448, 4/448] (or copied as bf16). Algorithmic bytes per call: inputs read
    + cache written + slots. Checks a sample of the written codes against
    torch's float8_e4m3fn cast of clamp(x / scale) (or the bf16 bits)."""
    import torch
    from flash_attn_b200 import store_kvcache
    dev = torch.device("cuda")
    H, D, P = 8, 128, 16
    gen = torch.Generator(device="cpu").manual_seed(11)
    slots = torch.randperm(tokens, generator=gen).to(torch.int64).to(dev)
    ks = ((1 + 3 * torch.rand(H, generator=gen)) / 448).to(dev)
    vs = ((1 + 3 * torch.rand(H, generator=gen)) / 448).to(dev)
    g = torch.Generator(device=dev).manual_seed(12)
    k = torch.randn(tokens, H, D, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(tokens, H, D, device=dev, generator=g).to(torch.bfloat16)
    cdt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kc = torch.empty(tokens // P, P, H, D, dtype=cdt, device=dev)
    vc = torch.empty_like(kc)
    sc = dict(k_scale=ks, v_scale=vs) if fp8 else {}
    timed = time_loop(lambda: store_kvcache(k, v, kc, vc, slots, **sc), steps, warmup, min_seconds)
    ms, steps = timed if isinstance(timed, tuple) else (timed, steps)
    # Sampled check: the rows of 4096 seeded tokens.
    pick = torch.randperm(tokens, generator=gen)[:4096].to(dev)
    sl = slots[pick]
    for x, cache, scale in ((k, kc, ks), (v, vc, vs)):
        got = cache.view(-1, H, D)[sl]
        want = ((x[pick].float() / scale.reshape(1, -1, 1)).clamp(-448, 448).to(torch.float8_e4m3fn)
                if fp8 else x[pick])
        if not torch.equal(got.view(torch.uint8), want.view(torch.uint8)):
            raise AssertionError("store_kvcache wrote other bytes than the reference cast")
    elems = 2 * tokens * H * D
    nbytes = elems * (2 + (1 if fp8 else 2)) + tokens * 8
    gbs = nbytes / (ms * 1e-3) / 1e9
    del k, v, kc, vc
    return {"workload": f"store_kvcache bf16 -> {'FP8 E4M3 (per-head scales)' if fp8 else 'bf16'}, "
                        f"{tokens} tokens x 8 heads x 128 (K and V), random slots, page 16",
            "bytes_per_step": nbytes, "ms_per_step": ms, "steps": steps, "TB/s": gbs / 1e3,
            "parity": {"status": "ok", "against": "torch cast of clamp(x / scale) (bit-exact), 4096 rows"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "peak_kind": f"{peak_kind} hbm_gbs"}}


def run_rope_append(peaks, peak_kind, steps=20, warmup=3, requests=16, tokens=1024, min_seconds=0.0):
    """Fused RoPE + paged append (what flash_attn_with_kvcache does before
    attention in config 5's prefill): Q [B, S, 16, 128] rotated into a new
    tensor, K rotated and V appended at positions 0..S-1 of a page-16 bf16
    cache through a seeded page permutation, split-half pairs, fp32 cos/sin.
    Algorithmic bytes: Q, K, V read once, rotated Q and the K/V cache rows
    written once, the cos/sin rows of the S positions read once. Checks a
    sample of tokens bit for bit against torch's fp32 rotation."""
    import torch
    from flash_attn_b200._cache import rotary_append_kvcache
    dev = torch.device("cuda")
    B, S, HQ, HK, D, P = requests, tokens, 16, 8, 128, 16
    g = torch.Generator(device=dev).manual_seed(13)
    q = torch.randn(B, S, HQ, D, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(B, S, HK, D, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(B, S, HK, D, device=dev, generator=g).to(torch.bfloat16)
    pages = S // P
    gen = torch.Generator(device="cpu").manual_seed(14)
    table = torch.randperm(B * pages, generator=gen).to(torch.int32).reshape(B, pages).to(dev)
    kc = torch.zeros(B * pages, P, HK, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=dev).float() / D))
    ang = torch.arange(S, device=dev).float()[:, None] * inv[None, :]
    cos, sin = ang.cos(), ang.sin()
    lengths = torch.zeros(B, dtype=torch.int32, device=dev)
    box = []

    def call():
        box[:] = [rotary_append_kvcache(q, k, v, kc, vc, cos, sin, lengths, rotary_interleaved=False,
                                        causal=True, block_table=table)]

    timed = time_loop(call, steps, warmup, min_seconds)
    ms, steps = timed if isinstance(timed, tuple) else (timed, steps)
    torch.cuda.synchronize()

    def rope(x, pos):
        xf = x.float()
        h = D // 2
        c, s_ = cos[pos][:, None, :], sin[pos][:, None, :]
        x1, x2 = xf[..., :h], xf[..., h:]
        return torch.cat((x1 * c - x2 * s_, x2 * c + x1 * s_), dim=-1).to(torch.bfloat16)

    pos = torch.arange(0, S, 97, device=dev)
    for b in (0, B - 1):
        want_q = rope(q[b, pos], pos)
        if not torch.equal(box[0][b, pos], want_q):
            raise AssertionError("rotated q differs from torch's fp32 rotation")
        slots = table[b, pos // P].long() * P + pos % P
        if not torch.equal(kc.view(-1, HK, D)[slots], rope(k[b, pos], pos)):
            raise AssertionError("appended rotated K differs from torch's fp32 rotation")
        if not torch.equal(vc.view(-1, HK, D)[slots], v[b, pos]):
            raise AssertionError("appended V differs")
    nbytes = 2 * (q.numel() + k.numel() + v.numel()) * 2 + 2 * cos.numel() * 4
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": f"fused RoPE + paged append, {B} x {S} new tokens, 16q/8kv heads, D=128, page 16, bf16",
            "bytes_per_step": nbytes, "ms_per_step": ms, "steps": steps, "TB/s": gbs / 1e3,
            "parity": {"status": "ok", "against": "torch fp32 rotation (bit-exact), sampled tokens"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "peak_kind": f"{peak_kind} hbm_gbs"}}


def run_serving(peaks, peak_kind, steps=2, warmup=3, small=False, path="fused", cpu_baseline=False):
    """Config 5: Qwen3-0.6B-shaped serving loop, attention through the library.

    One step = prefill of every prompt (eager) + ``decode_steps`` greedy decode
    steps (one CUDA graph replay each). value = output tokens / s (the first
    token comes from the prefill); attention's share is measured by timing the
    28 layers' attention calls alone, captured in graphs, for the prefill step
    and for a decode step at the mid-loop position.
    """
    import torch
    from flash_attn_b200._capi import kernel_launches
    from serving_loop import (DecodeGraph, Engine, FusedAttention, NativeAttention, Qwen3Shape,
                              decode_step, init_weights, prefill_step)
    cfg = dict(CFG5)
    if small:
        # Profiling case: the prefill's RoPE/append inputs (134 MB) exceed L2,
        # about 2 GB of caches on the device.
        cfg.update(requests=16, prompt=1024, decode_steps=16)
    B, S, N = cfg["requests"], cfg["prompt"], cfg["decode_steps"]
    shape = Qwen3Shape()
    dev = torch.device("cuda")
    weights = init_weights(shape, dev, seed=cfg["seed"])
    backend = FusedAttention if path == "fused" else NativeAttention
    engine = Engine(shape, weights, backend, B, S + N + 1, dev, seed=cfg["seed"])
    prompts_host = torch.randint(0, shape.vocab, (B, S),
                                 generator=torch.Generator().manual_seed(cfg["seed"])).pin_memory()
    prompts = prompts_host.to(dev)
    history = torch.zeros(B, N + 1, dtype=torch.long, device=dev)
    history_host = torch.empty(B, N + 1, dtype=torch.long).pin_memory()

    c0 = kernel_launches()
    logits, start = engine.prefill(list(prompts.unbind(0)))
    prefill_launches = kernel_launches() - c0
    c0 = kernel_launches()
    graph = DecodeGraph(engine, logits.argmax(dim=-1), start.clone(), history)
    decode_launches = (kernel_launches() - c0) // 2  # one eager warm-up + one capture

    def loop(src):
        logits, start = engine.prefill(list(src.unbind(0)))
        first = logits.argmax(dim=-1)
        history[:, 0].copy_(first)
        graph.reset(first, start, col=1)
        for _ in range(N):
            graph.replay()

    for _ in range(warmup):
        loop(prompts)
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    time.sleep(0.3)
    first = len(TIMED_WINDOWS)
    ms = time_loop(lambda: loop(prompts), steps, 0)
    prefill_ms = time_loop(lambda: engine.prefill(list(prompts.unbind(0))), steps, 1)
    clocks = sampler.stop(TIMED_WINDOWS[first:])

    def e2e_loop():
        prompts.copy_(prompts_host, non_blocking=True)
        loop(prompts)
        history_host.copy_(history, non_blocking=True)

    e2e_ms = time_loop(e2e_loop, steps, 1)

    # Attention alone: the 28 layers' calls on the prefill step and on one decode step.
    g = torch.Generator(device=dev).manual_seed(7)
    T = B * S
    q = torch.randn(T, shape.heads, shape.head_dim, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(T, shape.kv_heads, shape.head_dim, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn_like(k)
    pstep = prefill_step(engine.cache, [S] * B, shape.page, dev)
    dstart = torch.full((B,), S + N // 2, dtype=torch.int32, device=dev)
    dstep = decode_step(engine.cache, dstart, shape.page)

    def layers_attention(step, rows):
        for i in range(shape.layers):  # outputs die each iteration: the graph pool reuses them
            engine.backend(i, q[:rows], k[:rows], v[:rows], step)

    attn_prefill_ms = _graph_ms(lambda: layers_attention(pstep, T), 3)
    attn_decode_ms = _graph_ms(lambda: layers_attention(dstep, B), 20)
    decode_step_ms = (ms - prefill_ms) / N
    del q, k, v

    out_tokens = B * (N + 1)
    flops = shape.layers * shape.heads * 4 * shape.head_dim * B * S * (S + 1) // 2
    tflops = flops / (attn_prefill_ms * 1e-3) / 1e12
    line = {
        "value": out_tokens / (ms * 1e-3), "unit": "output tokens/s", "ms_per_step": ms,
        "workload": f"cfg5: Qwen3-0.6B-shaped serving loop, random bf16 weights, {B} requests x {S}-token "
                    f"prompts (prefill) + {N} greedy decode steps (CUDA graph), page 16, "
                    f"attention path '{path}'" + (" (small profiling case)" if small else ""),
        "prefill_ms": prefill_ms, "decode_step_ms": decode_step_ms,
        "attention": {"prefill_ms": attn_prefill_ms, "prefill_share": attn_prefill_ms / prefill_ms,
                      "decode_step_ms": attn_decode_ms, "decode_share": attn_decode_ms / decode_step_ms,
                      "prefill_attention_tflop": flops / 1e12},
        "e2e": {"value": out_tokens / (e2e_ms * 1e-3), "unit": "output tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": prompts_host.numel() * 8, "d2h_bytes_per_step": history_host.numel() * 8},
        "roofline": {"bound": "tensor", "kernel": "prefill_sm100_kernel (28 layers' prefill attention"
                     + (", with the fused RoPE+append launches)" if path == "fused" else ", with store_kvcache)"),
                     "achieved": tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / peaks["bf16_tflops"], "peak_kind": f"{peak_kind} (bf16_tflops, burst)",
                     "traffic": None},
        "gpu_launches": steps * (prefill_launches + N * decode_launches),
        "clocks": clocks,
    }
    del graph, engine, weights
    torch.cuda.empty_cache()
    if cpu_baseline:
        line["cpu_baseline"] = cpu_serving_sample()
    return line


def multi_gpu_secondary(rank, world, peaks, peak_kind):
    """Configs 2 and 3 at N > 1, where they shard with no communication:
    config-2 prefill split by KV-head groups (each rank takes HKV/N KV heads
    and their query heads) and config-3 decode as one full replica per GPU.
    Whole-job aggregates over the max-over-ranks device time."""
    out = {}
    hkv = CFG2["hkv"]
    if hkv % world == 0:
        per = hkv // world
        barrier(world)
        r = run_prefill(peaks, peak_kind, kv_slice=(rank * per, (rank + 1) * per))
        ms = max_over_ranks(r["ms_per_step"], world)
        flops = r["tflop_per_step"] * world * 1e12  # equal head shares
        out["prefill_cfg2_head_sharded"] = {
            "workload": f"cfg2 prefill, {per} KV head(s) + {per * CFG2['hq'] // hkv} query heads per GPU, no communication",
            "ms_per_step": ms, "TFLOP/s": flops / (ms * 1e-3) / 1e12,
            "per_gpu_TFLOP/s": flops / world / (ms * 1e-3) / 1e12}
    barrier(world)
    r = run_bf16_decode(peaks, peak_kind)
    ms = max_over_ranks(r["ms_per_step"], world)
    out["decode_cfg3_replicas"] = {
        "workload": "cfg3 paged bf16 decode, one full replica per GPU, no communication",
        "ms_per_step": ms, "TB/s": world * r["bytes_per_step"] / (ms * 1e-3) / 1e12,
        "per_gpu_TB/s": r["bytes_per_step"] / (ms * 1e-3) / 1e12}
    barrier(world)
    return out


# ------------------------------------------------------------------ CPU legs
def cpu_fp8_decode_sample(cfg, requests=1, seed=4):
    """The oracle (reference CPU math, float64) on a bounded sample of config 4."""
    import numpy as np
    import oracle
    rng = np.random.default_rng(seed)
    C, HQ, HK, D = cfg["ctx"], cfg["hq"], cfg["hkv"], cfg["d"]
    codes_k = rng.integers(0, 256, size=(requests * C, HK, D), dtype=np.uint8)
    codes_v = rng.integers(0, 256, size=(requests * C, HK, D), dtype=np.uint8)
    codes_k[(codes_k & 0x7F) == 0x7F] = 0  # no NaN codes
    codes_v[(codes_v & 0x7F) == 0x7F] = 0
    q = rng.standard_normal((requests, HQ, D))
    cu_q = np.arange(requests + 1)
    cu_k = np.arange(requests + 1) * C
    desc = np.full((requests, HK), 1 / 112.0)
    t0 = time.perf_counter()
    k = oracle.e4m3_decode(codes_k)
    v = oracle.e4m3_decode(codes_v)
    oracle.attention(q, k, v, cu_q, cu_k=cu_k, k_descale=desc, v_descale=desc)
    dt = time.perf_counter() - t0
    nbytes = requests * C * HK * 2 * D
    return nbytes / dt / 1e12, dt, f"{requests} request x {C} tokens of cfg4 (FP8 decode + float64 attention)"


def blas_threads():
    """Threads numpy's BLAS uses for the oracle's matrix products (the oracle's
    element-wise numpy work runs on one thread)."""
    try:
        import threadpoolctl
        counts = [d["num_threads"] for d in threadpoolctl.threadpool_info() if d.get("user_api") == "blas"]
        if counts:
            return max(counts)
    except Exception:
        pass
    return os.cpu_count()


def cpu_baseline_block(cfg):
    import numpy as np  # noqa: F401
    value, dt, sample = cpu_fp8_decode_sample(cfg)
    return {"value": value, "unit": "TB/s", "cores": blas_threads(), "host_cpus": os.cpu_count(),
            "kind": "port", "sample": sample, "seconds": round(dt, 3)}


def rounded(x, digits=6):
    """Floats rounded to ``digits`` significant digits, recursively (short lines)."""
    if isinstance(x, float):
        return float(f"{x:.{digits}g}")
    if isinstance(x, dict):
        return {k: rounded(v, digits) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [rounded(v, digits) for v in x]
    return x


def run_reference(args):
    """--impl reference: the reference's CPU math path (oracle port) on host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    cfg = dict(CFG4)
    times = []
    for _ in range(args.warmup):
        cpu_fp8_decode_sample(cfg)
    for _ in range(args.steps):
        value, dt, sample = cpu_fp8_decode_sample(cfg)
        times.append(dt)
    ms = statistics.median(times) * 1e3
    nbytes = cfg["ctx"] * cfg["hkv"] * 2 * cfg["d"]
    value = nbytes / (ms * 1e-3) / 1e12
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp8_e4m3 KV decoded to float64", "data": "synthetic",
        "config": {"workload": "cfg4: long-context FP8 E4M3 paged decode (bounded CPU sample per step)",
                   "batch": cfg["batch"], "context": cfg["ctx"], "q_heads": cfg["hq"],
                   "kv_heads": cfg["hkv"], "head_dim": cfg["d"]},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": blas_threads(), "host_cpus": os.cpu_count(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def check_build_id():
    """The loaded library's build id; refuses to measure a library built from
    other sources than the ones checked out beside this file."""
    from flash_attn_b200 import _capi
    sys.path.insert(0, os.path.join(ROOT, "flash-attn-mps_b200"))
    import build
    have, want = _capi.build_id(), build.source_hash()
    if have != want:
        raise SystemExit(f"libflash_attn_b200.so was built from other sources (build id {have}, sources {want}); "
                         "run `python flash-attn-mps_b200/build.py`")
    return have


def secondary_line(name, r):
    """One short JSON line for a secondary measurement."""
    roof = r.get("roofline", {})
    if "TFLOP/s" in r:
        value, unit = r["TFLOP/s"], "TFLOP/s"
    elif "TB/s" in r:
        value, unit = r["TB/s"], "TB/s"
    else:
        value, unit = r["value"], r["unit"]
    line = {"secondary": name, "value": round(value, 2), "unit": unit,
            "ms_per_step": round(r["ms_per_step"], 4), "steps": r.get("steps"),
            "roofline": {k: (round(v, 4) if isinstance(v, float) else v) for k, v in roof.items()
                         if k in ("bound", "achieved", "peak", "unit", "frac", "peak_kind", "frac_of_burst", "traffic",
                                  "algorithmic_bytes") and v is not None},
            "clocks": r.get("clocks"), "workload": r.get("workload")}
    for key in ("parity", "attention", "e2e"):
        if key in r:
            line[key] = r[key]
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["fp8_decode", "prefill", "prefill_softcap_window", "prefill_fp8kv",
                                           "prefill_alibi", "prefill_alibi_softcap", "bf16_decode", "serving", "store_fp8", "store_bf16",
                                           "rope_append", "prefill_d256", "prefill_diffkv", "decode_d256"],
                    default="fp8_decode", help="headline is fp8_decode (config 4); the others run on rank 0 only")
    ap.add_argument("--attention-path", choices=["fused", "native"], default="fused",
                    help="serving workload: fused RoPE+append with_kvcache calls, or store_kvcache + varlen")
    ap.add_argument("--small", action="store_true", help="shrunken workload for ncu captures")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the config-2/3 measurements")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        line = run_reference(args)
        if line is not None:
            print(json.dumps(line))
        return
    import torch
    rank, world, local = dist_setup(args.gpus)
    peaks, peak_kind = load_peaks()
    if args.workload != "fp8_decode":
        # Single-workload runs (profiling and secondary measurements), rank 0 only.
        if rank == 0:
            if args.workload == "prefill":
                r = run_prefill(peaks, peak_kind, steps=args.steps, warmup=args.warmup, small=args.small)
                value, unit = r["TFLOP/s"], "TFLOP/s"
            elif args.workload == "serving":
                # One step is a whole serving loop (~0.5 s): at most 5 timed loops.
                steps = min(args.steps, 5)
                r = run_serving(peaks, peak_kind, steps=steps, warmup=args.warmup, small=args.small,
                                path=args.attention_path, cpu_baseline=not args.no_cpu_baseline and not args.small)
                r["config"] = {"workload": r.pop("workload"),
                               "l2": "weights (1.2 GB) and paged caches (9.5 GB) larger than L2; no flush"}
                r.update({"metric": METRIC, "n_gpus": 1, "steps": steps, "warmup": args.warmup,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "bf16", "data": "synthetic (seeded random weights and prompts)"})
                print(json.dumps(r))
                return
            elif args.workload == "prefill_alibi":
                r = run_prefill(peaks, peak_kind, steps=args.steps, warmup=args.warmup, small=args.small, alibi=True)
                value, unit = r["TFLOP/s"], "TFLOP/s"
            elif args.workload == "prefill_alibi_softcap":
                r = run_prefill(peaks, peak_kind, steps=args.steps, warmup=args.warmup, small=args.small, alibi=True,
                                softcap=50.0)
                value, unit = r["TFLOP/s"], "TFLOP/s"
            elif args.workload == "prefill_fp8kv":
                r = run_prefill(peaks, peak_kind, steps=args.steps, warmup=args.warmup, small=args.small, fp8_kv=True)
                value, unit = r["TFLOP/s"], "TFLOP/s"
            elif args.workload in ("prefill_d256", "prefill_diffkv"):
                r = run_prefill(peaks, peak_kind, steps=args.steps, warmup=args.warmup, small=args.small,
                                dims=(256, 256) if args.workload == "prefill_d256" else (192, 128))
                value, unit = r["TFLOP/s"], "TFLOP/s"
            elif args.workload == "decode_d256":
                r = run_bf16_decode(peaks, peak_kind, steps=args.steps, warmup=args.warmup, small=args.small, d=256)
                value, unit = r["TB/s"], "TB/s"
            elif args.workload == "rope_append":
                r = run_rope_append(peaks, peak_kind, steps=args.steps, warmup=args.warmup,
                                    requests=4 if args.small else 16)
                value, unit = r["TB/s"], "TB/s"
            elif args.workload in ("store_fp8", "store_bf16"):
                r = run_store(peaks, peak_kind, steps=args.steps, warmup=args.warmup,
                              fp8=args.workload == "store_fp8", tokens=65536 if args.small else 524288)
                value, unit = r["TB/s"], "TB/s"
            elif args.workload == "prefill_softcap_window":
                r = run_prefill(peaks, peak_kind, steps=args.steps, warmup=args.warmup, softcap=50.0,
                                window=(1024, 0), small=args.small)
                value, unit = r["TFLOP/s"], "TFLOP/s"
            else:
                r = run_bf16_decode(peaks, peak_kind, steps=args.steps, warmup=args.warmup, small=args.small)
                value, unit = r["TB/s"], "TB/s"
            print(json.dumps({"metric": METRIC, "value": value, "unit": unit, "n_gpus": 1,
                              "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                              "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                              "dtype": "bf16 q, fp8_e4m3 K/V" if args.workload == "prefill_fp8kv" else "bf16",
                              "data": "synthetic (seeded)",
                              "config": {"workload": r["workload"]}, "roofline": r["roofline"]}))
        return
    build_id = check_build_id()
    res = run_fp8_decode(args, rank, world, peaks, peak_kind)
    multi = (multi_gpu_secondary(rank, world, peaks, peak_kind)
             if world > 1 and not args.no_secondary and not args.small else None)
    if rank == 0:
        line = {"metric": METRIC, "value": res["value"], "unit": res["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": res["dtype"], "data": "synthetic (seeded)", "config": res["config"],
                "e2e": res["e2e"], "roofline": res["roofline"], "gpu_launches": res["gpu_launches"],
                "clocks": res["clocks"], "parity": res["parity"], "build_id": build_id}
        # Secondary workloads: one short JSON line each, printed before the
        # headline line (the last line), the most important one last.
        if world == 1 and not args.no_secondary and not args.small:
            secondaries = [
                ("serving_cfg5", lambda: run_serving(peaks, peak_kind)),
                ("store_kvcache_fp8", lambda: rested(lambda: run_store(peaks, peak_kind, min_seconds=0.3), 0.5)),
                ("rope_append", lambda: rested(lambda: run_rope_append(peaks, peak_kind, min_seconds=0.3), 0.5)),
                ("decode_cfg3", lambda: rested(lambda: run_bf16_decode(peaks, peak_kind, min_seconds=1.2))),
                ("decode_d256", lambda: rested(lambda: run_bf16_decode(peaks, peak_kind, min_seconds=0.3, d=256))),
                # Prefill held against the burst peak (a cuBLAS GEMM timed in a
                # short window at full clocks) is timed the same way: a window
                # of ~40 ms after an idle pause. At full clocks the prefill
                # draws more than the 1 kW cap allows; within ~100 ms the cap
                # lowers the clocks (config 2: ~975 TFLOP/s over 20-35 launches,
                # ~885 over 100, 836 over 300).
                ("prefill_cfg2_fp8kv", lambda: rested(lambda: run_prefill(peaks, peak_kind, fp8_kv=True,
                                                                          min_seconds=BURST_WINDOW_S))),
                ("prefill_cfg2_d256", lambda: rested(lambda: run_prefill(peaks, peak_kind, dims=(256, 256),
                                                                         min_seconds=BURST_WINDOW_S))),
                ("prefill_cfg2_diffkv", lambda: rested(lambda: run_prefill(peaks, peak_kind, dims=(192, 128),
                                                                           min_seconds=BURST_WINDOW_S))),
                ("prefill_cfg2_softcap_window", lambda: rested(lambda: run_prefill(
                    peaks, peak_kind, softcap=50.0, window=(1024, 0), min_seconds=BURST_WINDOW_S))),
                # Over a window of seconds the GPU sits at its power cap with
                # lowered clocks: that run is held against the sustained peak.
                ("prefill_cfg2_sustained", lambda: rested(lambda: run_prefill(peaks, peak_kind, min_seconds=2.0,
                                                                              sustained=True))),
                ("prefill_cfg2", lambda: rested(lambda: run_prefill(peaks, peak_kind, min_seconds=BURST_WINDOW_S))),
            ]
            for name, measure in secondaries:
                print(json.dumps(rounded(secondary_line(name, measure()))), flush=True)
        if multi:
            for name, r in multi.items():
                print(json.dumps(rounded(dict({"secondary": name}, **r))), flush=True)
        if world == 1 and not args.no_cpu_baseline and not args.small:
            line["cpu_baseline"] = cpu_baseline_block(CFG4)
        print(json.dumps(rounded(line)))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
