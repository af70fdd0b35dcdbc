#!/usr/bin/env python
"""Benchmark of the FlexKV transfer data plane on B200 (one JSON line).

Workload (Llama-3-8B KV shape): 32 layers, 8 KV heads,
head_dim 128, 16 tokens per block, bf16 (32 KiB chunks, 2 MiB per block over
all layers).  GPU pool 16384 blocks (32 one-GiB layer tensors), pinned CPU
pool up to 32768 blocks (64 GiB; scaled to the box's RAM and recorded).  A
step moves one 2048-block batch host->device and one device->host (4 GiB
each way); block ids are a seeded permutation with 50% of the blocks in joint
contiguous runs of length U[1,64] and 50% scattered singletons; four batches
rotate so consecutive steps touch different blocks.  Every batch is far
larger than L2 (no flush needed).

  value  — device-timed GB/s (CUDA events on the launch stream) with plans
           (ids validated, coalesced and resident on the device) prepared
           before the timed region.
  e2e    — GB/s through the reference-facing call
           flexkv_b200.c_ext.transfer_kv_blocks with host id tensors, wall
           clock, synchronous per call like the reference.
  --impl reference — the reference's own transfer.cu built from its source
           (oracle/_ref) driven the way its worker drives it
           (transfer_sms=8, pinned id tensors, synchronous).

Multi-GPU (torchrun): every rank runs the same per-GPU workload on its own
GPU and pools (data parallel, no collective on the data path); value is the
bytes of all ranks over the max-over-ranks time (weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PCIE_GEN5_X16_GBS = 63.0  # 32 GT/s * 16 lanes * 128/130 / 8, per direction

CONFIGS = {
    "cfg2_llama3_8b": dict(layers=32, heads=8, head_dim=128, tpb=16, gpu_blocks=16384,
                           cpu_blocks=32768, batch=2048, run_frac=0.5, max_run=64),
    "cfg5_dsv3_mla": dict(layers=61, heads=1, head_dim=576, tpb=64, gpu_blocks=8192,
                          cpu_blocks=16384, batch=1024, run_frac=0.5, max_run=128, mla=True),
    "cfg4_qwen2_7b": dict(layers=28, heads=4, head_dim=128, tpb=16, gpu_blocks=8192,
                          cpu_blocks=16384, batch=4224, run_frac=0.0, max_run=1),
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def make_batch(n, gpu_pool, cpu_pool, seed, run_frac, max_run):
    """Joint runs (both ids advance by one) covering run_frac of the blocks,
    lengths U[1,max_run]; the rest scattered singletons; shuffled run order."""
    rng = np.random.default_rng(seed)
    n_run = int(round(n * run_frac))
    lens, left = [], n_run
    while left > 0:
        r = int(min(left, rng.integers(1, max_run + 1)))
        lens.append(r)
        left -= r
    lens += [1] * (n - n_run)

    def starts(pool):
        # Segments in a random order, separated by random gaps sharing the
        # pool's free space: disjoint, and spread over the whole pool.
        assert n <= pool, "pool smaller than the batch"
        cuts = np.sort(rng.integers(0, pool - n + 1, len(lens)))
        gaps = np.diff(np.concatenate([[0], cuts]))
        st = [0] * len(lens)
        pos = 0
        for j, idx in enumerate(rng.permutation(len(lens))):
            pos += int(gaps[j])
            st[idx] = pos
            pos += lens[idx]
        return st

    gs, cs = starts(gpu_pool), starts(cpu_pool)
    g, c = [], []
    for i in rng.permutation(len(lens)):
        g += range(gs[i], gs[i] + lens[i])
        c += range(cs[i], cs[i] + lens[i])
    return np.array(g, dtype=np.int64), np.array(c, dtype=np.int64)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self._stop = threading.Event()
        self._th = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.rows.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._th = threading.Thread(target=self._run, daemon=True)
        self._th.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._th.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local}"))
    else:
        torch.cuda.set_device(local)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def _reduce(ws, x: float, op: str) -> float:
    """All-reduce one float over the ranks (timing plumbing only, never data)."""
    if ws == 1:
        return x
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(ws, x: float) -> float:
    return _reduce(ws, x, "max")


def sum_over_ranks(ws, x: float) -> float:
    return _reduce(ws, x, "sum")


def rank_batches(cfg: dict, cpu_blocks: int, local: int, nbatches: int = 4):
    """The block-id batches of one data-parallel rank: its own seeds, its
    own pools, no id shared with another rank's work."""
    return [make_batch(cfg["batch"], cfg["gpu_blocks"], cpu_blocks, 1000 * local + s,
                       cfg["run_frac"], cfg["max_run"]) for s in range(nbatches)]


def mem_available_bytes() -> int:
    with open("/proc/meminfo") as f:
        for line in f:
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    return 0


class Setup:
    """Pools, layouts and id batches of one rank."""

    def __init__(self, cfg: dict, layout: str, ws: int, local: int, cpu_blocks_override: int = 0,
                 nbatches: int = 4):
        from flexkv_b200 import c_ext
        from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
        self.cfg = cfg
        mla = cfg.get("mla", False)
        self.kv = 1 if mla else 2
        L, H, D, tpb = cfg["layers"], cfg["heads"], cfg["head_dim"], cfg["tpb"]
        self.chunk = tpb * H * D * 2
        self.block_bytes = L * self.kv * self.chunk
        cpu_blocks = cfg["cpu_blocks"]
        avail = mem_available_bytes()
        fit = int(0.55 * avail / max(ws, 1) / self.block_bytes)
        if cpu_blocks_override:
            cpu_blocks = cpu_blocks_override
        elif fit < cpu_blocks:
            cpu_blocks = max(fit, cfg["batch"] * 2)
        self.cpu_blocks = cpu_blocks
        self.gpu_layout = KVCacheLayout(KVCacheLayoutType.LAYERWISE, L, cfg["gpu_blocks"], tpb, H, D, mla)
        self.cpu_layout = KVCacheLayout(KVCacheLayoutType[layout], L, cpu_blocks, tpb, H, D, mla)
        per = self.gpu_layout.div_layer(L)
        e = 2
        self.g_kv, self.g_blk = per.get_kv_stride() * e, per.get_block_stride() * e
        self.c_kv = self.cpu_layout.get_kv_stride() * e
        self.c_layer = self.cpu_layout.get_layer_stride() * e
        self.c_blk = self.cpu_layout.get_block_stride() * e
        self.gpu_layer_bytes = per.get_total_elements() * e
        dev = torch.device(f"cuda:{local}")
        t0 = time.time()
        self.layers = []
        for _ in range(L):
            t = torch.empty(per.kv_shape, dtype=torch.bfloat16, device=dev)
            t.normal_()
            self.layers.append(t)
        self.ptrs = torch.tensor([t.data_ptr() for t in self.layers], dtype=torch.int64)
        t1 = time.time()
        cpu_bytes = self.cpu_layout.get_total_elements() * e
        self.cpu = torch.empty(cpu_bytes // 2, dtype=torch.bfloat16)
        c_ext.cudaHostRegister(self.cpu, advise_hugepages=True)
        t2 = time.time()
        log(f"[rank{local}] gpu pool {L}x{self.gpu_layer_bytes / 2**30:.2f} GiB in {t1 - t0:.1f}s, "
            f"cpu pool {cpu_bytes / 2**30:.1f} GiB registered in {t2 - t1:.1f}s")
        self.batches = rank_batches(cfg, cpu_blocks, local, nbatches)
        self.batch_bytes = cfg["batch"] * self.block_bytes

    def close(self):
        from flexkv_b200 import c_ext
        c_ext.cudaHostUnregister(self.cpu)


def measure_extras(S, plans, stream, K):
    """Two extra figures on the same pools: the host link's copy-engine peak
    (one large contiguous cudaMemcpyAsync each way from the pinned pool, the
    measured roofline of the link) and the duplex rate (the H2D of batch k
    and the D2H of batch k+1 in flight together on two streams)."""
    n = min(S.batch_bytes, 2 << 30)
    gbuf = torch.empty(n, dtype=torch.uint8, device="cuda")
    hbuf = S.cpu.view(torch.uint8)[:n]
    peak = {}
    for name, fn in (("h2d", lambda: gbuf.copy_(hbuf, non_blocking=True)),
                     ("d2h", lambda: hbuf.copy_(gbuf, non_blocking=True))):
        fn()
        ts = []
        for _ in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        peak[name] = round(n / (statistics.median(ts) / 1e3) / 1e9, 2)
    del gbuf
    side = torch.cuda.Stream()
    ts = []
    for k in range(max(K, 3)):
        h = plans[k % len(plans)][0]
        d = plans[(k + 1) % len(plans)][1]
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record(stream)
        side.wait_event(a)
        h.execute(stream=stream)
        d.execute(stream=side)
        c.record(side)
        stream.wait_event(c)
        b.record(stream)
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    duplex = 2 * S.batch_bytes / (statistics.median(ts) / 1e3) / 1e9
    return {"link_peak_measured": dict(peak, unit="GB/s", bytes=n,
                                       how="one contiguous cudaMemcpyAsync each way from the pinned pool, median of 3"),
            "duplex": {"value": round(duplex, 2), "unit": "GB/s",
                       "how": "H2D of batch k and D2H of batch k+1 at once on two streams (median step)"}}


def run_ours(args, ws, rank, local, cfg):
    from flexkv_b200 import c_ext
    S = Setup(cfg, args.layout, ws, local, args.cpu_blocks)
    mode_kw = {}
    use_ce = False
    if args.mode == "sm":
        mode_kw["ce_min_run_bytes"] = 0
    elif args.mode == "ce":
        use_ce = True
    elif args.mode == "hybrid":
        mode_kw["ce_min_run_bytes"] = args.ce_min_run_bytes
    plans = []
    for g, c in S.batches:
        pair = []
        for h2d in (True, False):
            pair.append(c_ext.TransferPlan(
                torch.from_numpy(g), S.ptrs, S.g_kv, S.g_blk, torch.from_numpy(c), S.cpu, S.c_kv,
                S.c_layer, S.c_blk, S.chunk, 0, args.transfer_sms, h2d, use_ce,
                cfg.get("mla", False), gpu_layer_bytes=S.gpu_layer_bytes, **mode_kw))
        plans.append(pair)
    stats = [p.stats() for p in plans[0]]
    stream = torch.cuda.current_stream()
    K, W = args.steps, args.warmup

    def step(k, evs=None):
        h, d = plans[k % len(plans)]
        if evs is None:
            h.execute()
            d.execute()
        else:
            evs[0].record(stream)
            h.execute(kernel_events=(evs[1], evs[2]))
            evs[3].record(stream)
            d.execute(kernel_events=(evs[4], evs[5]))
            evs[6].record(stream)

    for k in range(W):
        step(k)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(K)]
    for row in evs:  # torch creates the CUDA event on first record
        for e in row:
            e.record(stream)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    with sampler:
        barrier(ws)
        launches0 = c_ext.kernel_launch_count()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for k in range(K):
            step(W + k, evs[k])
        t_end.record(stream)
        torch.cuda.synchronize()
        launches = c_ext.kernel_launch_count() - launches0
        barrier(ws)
        elapsed_ms = t_start.elapsed_time(t_end)
        # e2e through the reference-facing call, host id tensors, synchronous
        host_ids = [(torch.from_numpy(g).pin_memory(), torch.from_numpy(c).pin_memory())
                    for g, c in S.batches]

        def call(k, h2d):
            g, c = host_ids[k % len(host_ids)]
            c_ext.transfer_kv_blocks(g, S.ptrs, S.g_kv, S.g_blk, c, S.cpu, S.c_kv, S.c_layer,
                                     S.c_blk, S.chunk, 0, args.transfer_sms, h2d, use_ce,
                                     cfg.get("mla", False), **mode_kw)

        for k in range(W):
            call(k, True)
            call(k, False)
        barrier(ws)
        w0 = time.perf_counter()
        for k in range(K):
            call(W + k, True)
            call(W + k, False)
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - w0
        barrier(ws)
    clocks = sampler.summary()
    extras = {} if args.no_extras else measure_extras(S, plans, stream, K)

    h2d_ms = [evs[k][0].elapsed_time(evs[k][3]) for k in range(K)]
    d2h_ms = [evs[k][3].elapsed_time(evs[k][6]) for k in range(K)]
    kh_ms = [evs[k][1].elapsed_time(evs[k][2]) for k in range(K)]
    kd_ms = [evs[k][4].elapsed_time(evs[k][5]) for k in range(K)]
    max_elapsed = max_over_ranks(ws, elapsed_ms)
    max_e2e = max_over_ranks(ws, e2e_s)
    total_bytes = sum_over_ranks(ws, 2.0 * K * S.batch_bytes)
    value = total_bytes / (max_elapsed / 1e3) / 1e9
    e2e = total_bytes / max_e2e / 1e9
    bb = S.batch_bytes
    h2d_gbs = bb / (statistics.mean(h2d_ms) / 1e3) / 1e9
    d2h_gbs = bb / (statistics.mean(d2h_ms) / 1e3) / 1e9
    # Roofline of the transfer op (the SM kernel plus the copy-engine runs it
    # overlaps with share one host link, so the op is the unit that meets the
    # link's bound).  Headline: the slower direction.  Peak: the link's
    # copy-engine rate measured live on the same pool (MEASURED_PEAKS.json
    # has no host-link figure), with the nominal PCIe Gen5 x16 rate beside it.
    # DRAM traffic per op: the algorithmic bytes times the (read+write)/payload
    # ratio of the kernel's ncu capture (profiles/kv_copy_kernel_cfg2_small_full.md).
    TRAFFIC_RATIO = {"h2d": 0.781, "d2h": 1.016}
    out = None
    if rank == 0:
        lp = extras.get("link_peak_measured")
        dirs = {"h2d": (h2d_gbs, kh_ms, stats[0]), "d2h": (d2h_gbs, kd_ms, stats[1])}
        head = min(dirs, key=lambda d: dirs[d][0])
        ach, kms, st = dirs[head]
        peak = lp[head] if lp else PCIE_GEN5_X16_GBS
        roof = {"bound": "pcie", "kernel": f"transfer op {head.upper()} (kv_copy_kernel + copy-engine runs)",
                "achieved": round(ach, 2), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": int(bb * TRAFFIC_RATIO[head]),
                "peak_source": ("measured live: one contiguous cudaMemcpyAsync of 2 GiB on the same "
                                "pinned pool (MEASURED_PEAKS.json has no host-link figure)") if lp else
                               "nominal PCIe Gen5 x16 (no live measurement in this run)",
                "nominal_peak": PCIE_GEN5_X16_GBS, "frac_of_nominal": round(ach / PCIE_GEN5_X16_GBS, 4),
                "per_direction": {d: {"achieved": round(v[0], 2),
                                      "peak": (lp[d] if lp else PCIE_GEN5_X16_GBS),
                                      "frac": round(v[0] / (lp[d] if lp else PCIE_GEN5_X16_GBS), 4)}
                                  for d, v in dirs.items()}}
        if st["sm_chunks"] > 0 and statistics.mean(kms) > 0:
            kmean = statistics.mean(kms)
            roof["sm_kernel"] = {"name": f"kv_copy_kernel<{head.upper()}>",
                                 "bytes_per_launch": st["sm_bytes"], "avg_launch_ms": round(kmean, 3),
                                 "achieved_alongside_copy_engines": round(st["sm_bytes"] / kmean / 1e6, 2),
                                 "copy_engine_bytes_per_op": st["ce_bytes"]}
        out = {
            "metric": "KV GB/s per GPU and box (H2D/D2H, 1/2/4/8 B200), % of PCIe Gen5 x16 peak",
            "value": round(value, 3), "unit": "GB/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": round(max_elapsed / K, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 (byte copy)", "data": "synthetic",
            "config": {"workload": args.config + (" (reduced: profiling case)" if (args.batch or args.gpu_blocks) else ""),
                       "layout": args.layout, "mode": args.mode,
                       "layers": cfg["layers"], "kv_heads": cfg["heads"], "head_dim": cfg["head_dim"],
                       "tokens_per_block": cfg["tpb"], "batch_blocks": cfg["batch"],
                       "batch_bytes_per_direction": bb, "gpu_pool_blocks": cfg["gpu_blocks"],
                       "cpu_pool_blocks": S.cpu_blocks, "cpu_pool_blocks_requested": cfg["cpu_blocks"],
                       "run_frac": cfg["run_frac"], "max_run": cfg["max_run"],
                       "transfer_sms": args.transfer_sms, "parallelism": f"dp{ws} (independent)",
                       "l2": "inputs larger than L2 (4 GiB per batch), no flush"},
            "per_direction_gbs": {"h2d": round(h2d_gbs, 2), "d2h": round(d2h_gbs, 2)},
            "blocks_per_s": round(value * 1e9 / S.block_bytes, 1),
            "box_roofline_frac": round(value / (PCIE_GEN5_X16_GBS * ws), 4),
            "roofline": roof,
            "plan": {"h2d": stats[0], "d2h": stats[1]},
            "e2e": {"value": round(e2e, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": int(bb + 16 * cfg["batch"] + 8 * cfg["layers"]),
                    "d2h_bytes_per_step": int(bb),
                    "how": "flexkv_b200.c_ext.transfer_kv_blocks, pinned host id tensors, synchronous calls, wall clock"},
            "gpu_launches": int(launches), "clocks": clocks,
        }
        out.update(extras)
    for p in plans:
        for x in p:
            x.close()
    return out, S


def cpu_baseline(S, seconds: float = 8.0):
    """The oracle (oracle/oracle.c, the CPU restatement of the reference copy)
    gathering/scattering a 256-block sample of the same workload on host
    memory with every host core."""
    from oracle import oracle as O
    cfg = S.cfg
    n = 256
    g, c = make_batch(n, 512, S.cpu_blocks, 77, cfg["run_frac"], cfg["max_run"])
    layer_bytes = S.gpu_layer_bytes * 512 // cfg["gpu_blocks"]
    imgs = [np.empty(layer_bytes, dtype=np.uint8) for _ in range(cfg["layers"])]
    cpu = S.cpu.view(torch.uint8).numpy()
    threads = len(os.sched_getaffinity(0))
    g_kv = S.g_kv * 512 // cfg["gpu_blocks"]
    moved, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for h2d in (True, False):
            O.transfer(n, 0, g, imgs, g_kv, S.g_blk, c, cpu, S.c_kv, S.c_layer, S.c_blk, 0,
                       S.chunk, h2d, cfg.get("mla", False), num_threads=threads)
            moved += n * S.block_bytes
    dt = time.perf_counter() - t0
    return {"value": round(moved / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n}-block {S.cpu_layout.type.value} gather+scatter between the host pool and "
                      f"host images of the GPU layers, repeated for {dt:.1f}s"}


def run_reference(args, ws, rank, local, cfg):
    """The reference's transfer.cu (oracle/_ref) the way its worker calls it."""
    from oracle import oracle as O
    if rank != 0:
        return None, None
    if not O.reference_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libref_transfer.so not built "
                "(needs the reference tree at build time)"}, None
    S = Setup(cfg, args.layout, 1, local, args.cpu_blocks)
    ref = O.ref_lib()
    ptrs = S.ptrs.pin_memory()
    ids = [(torch.from_numpy(g).pin_memory(), torch.from_numpy(c).pin_memory()) for g, c in S.batches]
    stream = torch.cuda.current_stream().cuda_stream
    sms = 8  # flexkv/common/config.py:50-51 worker default

    def call(k, h2d, use_ce=False):
        g, c = ids[k % len(ids)]
        rc = ref.ref_transfer_kv_blocks(len(g), 0, len(S.layers), g.data_ptr(), ptrs.data_ptr(),
                                        S.g_kv, S.g_blk, c.data_ptr(), S.cpu.data_ptr(), S.c_kv,
                                        S.c_layer, S.c_blk, 0, S.chunk, stream, sms, int(h2d),
                                        int(use_ce), int(cfg.get("mla", False)))
        if rc != 0:
            raise RuntimeError(f"reference transfer_kv_blocks CUDA error {rc}")

    K, W = args.steps, args.warmup
    for k in range(W):
        call(k, True)
        call(k, False)
    sampler = ClockSampler(local)
    with sampler:
        torch.cuda.synchronize()
        per = {"h2d": [], "d2h": []}
        t0 = time.perf_counter()
        for k in range(K):
            a = time.perf_counter()
            call(W + k, True)
            b = time.perf_counter()
            call(W + k, False)
            per["h2d"].append(b - a)
            per["d2h"].append(time.perf_counter() - b)
        dt = time.perf_counter() - t0
        # CE mode (one cudaMemcpyAsync per chunk), one step
        a = time.perf_counter()
        call(W + K, True, use_ce=True)
        b = time.perf_counter()
        call(W + K, False, use_ce=True)
        ce = (time.perf_counter() - a, b - a, time.perf_counter() - b)
    bb = S.batch_bytes
    value = 2 * K * bb / dt / 1e9
    out = {
        "impl": "reference",
        "metric": "KV GB/s per GPU and box (H2D/D2H, 1/2/4/8 B200), % of PCIe Gen5 x16 peak",
        "value": round(value, 3), "unit": "GB/s", "n_gpus": ws, "steps": K, "warmup": W,
        "ms_per_step": round(dt / K * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (byte copy)", "data": "synthetic",
        "config": {"workload": args.config, "layout": args.layout, "transfer_sms": sms,
                   "batch_blocks": cfg["batch"], "cpu_pool_blocks": S.cpu_blocks,
                   "parallelism": "rank 0 only"},
        "per_direction_gbs": {"h2d": round(bb / statistics.mean(per["h2d"]) / 1e9, 2),
                              "d2h": round(bb / statistics.mean(per["d2h"]) / 1e9, 2)},
        "ce_mode": {"value": round(2 * bb / ce[0] / 1e9, 3), "h2d": round(bb / ce[1] / 1e9, 2),
                    "d2h": round(bb / ce[2] / 1e9, 2), "unit": "GB/s",
                    "how": "use_ce_transfer=True: one cudaMemcpyAsync per (layer,kv,block) chunk, one step"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": 1, "kind": "reference",
                         "sample": "the reference's transfer.cu kernel (transfer_sms=8) driven from one "
                                   "host thread with pinned ids, synchronous per call, full batches"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "clocks": sampler.summary(),
    }
    return out, S


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2_llama3_8b")
    ap.add_argument("--layout", choices=["LAYERWISE", "BLOCKWISE"], default="LAYERWISE")
    ap.add_argument("--mode", choices=["auto", "sm", "ce", "hybrid"], default="auto")
    ap.add_argument("--ce-min-run-bytes", type=int, default=1 << 20)
    ap.add_argument("--transfer-sms", type=int, default=-1)
    ap.add_argument("--cpu-blocks", type=int, default=0, help="override the CPU pool size")
    ap.add_argument("--cpu-baseline-seconds", type=float, default=8.0)
    ap.add_argument("--batch", type=int, default=0, help="override blocks per batch (profiling case)")
    ap.add_argument("--gpu-blocks", type=int, default=0, help="override the GPU pool size")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the link-peak and duplex measurements (profiling runs)")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3
    if args.impl == "reference" and int(os.environ.get("RANK", "0")) != 0:
        return  # the reference arm runs on rank 0 only
    if args.impl == "reference":
        os.environ["WORLD_SIZE"] = "1"  # no process group: rank 0 alone
    ws, rank, local = dist_setup()
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["batch"] = args.batch
    if args.gpu_blocks:
        cfg["gpu_blocks"] = args.gpu_blocks
    if args.impl == "reference":
        out, S = run_reference(args, ws, rank, local, cfg)
    else:
        out, S = run_ours(args, ws, rank, local, cfg)
        if rank == 0 and ws == 1:
            out["cpu_baseline"] = cpu_baseline(S, args.cpu_baseline_seconds)
        elif rank == 0:
            out["cpu_baseline"] = None
    if S is not None:
        S.close()
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
