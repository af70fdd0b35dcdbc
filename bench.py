#!/usr/bin/env python
"""Benchmark of the FlexKV transfer data plane on B200 (one JSON line).

Default workload (Llama-3-8B KV shape): 32 layers, 8 KV
heads, head_dim 128, 16 tokens per block, bf16 (32 KiB chunks, 2 MiB per
block over all layers).  GPU pool 16384 blocks (32 one-GiB layer tensors),
pinned CPU pool up to 32768 blocks (64 GiB; scaled to the box's RAM and
recorded).  A step moves one 2048-block batch host->device and another
device->host (4 GiB each way), one after the other as FlexKV's worker does;
block ids are seeded permutations with 50% of the blocks in joint contiguous
runs of length U[1,64] and 50% scattered singletons; four steps rotate so
consecutive steps touch different blocks.  Every batch is far larger than L2
(no flush needed).

Other configurations (--config): cfg5_dsv3_mla (DeepSeek-V3 MLA latent KV,
1024-block batches, runs of 128 : singletons 1:1, both directions at once),
cfg4_qwen2_7b (Qwen2-7B shape, 256 requests of U[1,32] scattered blocks per
step, mixed get/put, directions overlapped), cfg3_llama3_70b_tp (Llama-3-70B,
one TP group of --tp ranks driven from one process).

  value  — device-timed GB/s (CUDA events on the call streams) of every op
           made through the reference-facing call,
           c_ext.transfer_kv_blocks, with pinned host id tensors: one
           synchronous call per op as FlexKV's worker makes it (per-direction
           streams when the workload overlaps directions), so id validation,
           coalescing and the id-table upload are inside the timed region.
           plan_replay beside it runs the same ops from TransferPlans built
           beforehand, and brackets the SM kernel for the roofline.
  e2e    — GB/s through the public API that replaces FlexKV's
           TransferEngine (flexkv_b200.engine.TransferEngine: one graph per
           op, host id tensors, wall clock; H2D and D2H ops in flight
           together); per_op_calls beside it is the wall clock of the value
           leg.
  extras — link peaks measured live (each rank alone, and all ranks at
           once when N > 1), the duplex rate, and at N = 1 on cfg2 the
           XXH64 hashing, small-op latency, CPU-tier put path (device index
           + fused put against the reference's per-request path) and
           SSD-tier measurements.
  --impl reference — the reference's own transfer.cu built from its source
           (oracle/_ref) driven the way its worker drives it: one op at a
           time, transfer_sms=8, pinned id tensors, synchronous, on pools
           built the stock way (one flat host tensor, Portable
           cudaHostRegister); nothing of flexkv_b200 is loaded.
  --hash-only / --ssd-only / --put-only — only that measurement, one JSON
           line (--put-only on the --config shape).

Multi-GPU (torchrun): every rank runs the same per-GPU workload on its own
GPU and pools (data parallel, no collective on the data path); value is the
bytes of all ranks over the max-over-ranks time (weak scaling).  The line
adds each rank's H2D and D2H rates (per_rank) and the box's per-direction
sums against N x the single-GPU link peak and against the peak measured
with every rank copying at once (box).
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
METRIC = "KV GB/s per GPU and box (H2D/D2H, 1/2/4/8 B200), % of PCIe Gen5 x16 peak"

CONFIGS = {
    "cfg2_llama3_8b": dict(layers=32, heads=8, head_dim=128, tpb=16, gpu_blocks=16384,
                           cpu_blocks=32768, batch=2048, run_frac=0.5, max_run=64,
                           kind="batch", concurrent=False, layout="LAYERWISE"),
    "cfg5_dsv3_mla": dict(layers=61, heads=1, head_dim=576, tpb=64, gpu_blocks=8192,
                          cpu_blocks=16384, batch=1024, run_frac=0.5, max_run=128, fixed_run=True,
                          mla=True, kind="batch", concurrent=True, layout="BLOCKWISE"),
    "cfg3_llama3_70b_tp": dict(layers=80, heads=8, head_dim=128, tpb=64, gpu_blocks=4096,
                               cpu_blocks=8192, batch=512, run_frac=0.0, max_run=1, kind="tp",
                               concurrent=False, layout="BLOCKWISE"),
    "cfg4_qwen2_7b": dict(layers=28, heads=4, head_dim=128, tpb=16, gpu_blocks=8192,
                          cpu_blocks=16384, requests=256, max_req_blocks=32, run_frac=0.0,
                          max_run=1, kind="requests", concurrent=True, layout="LAYERWISE"),
}
# DRAM traffic per payload byte of the SM copy kernel, from its ncu capture
# (profiles/kv_copy_kernel_cfg2_small_full.md): H2D writes, D2H reads.
TRAFFIC_RATIO = {"h2d": 0.787, "d2h": 1.010}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def make_batch(n, gpu_pool, cpu_pool, seed, run_frac, max_run, fixed_run=False):
    """Joint runs (both ids advance by one) covering run_frac of the blocks,
    lengths U[1,max_run] (or exactly max_run); the rest scattered singletons;
    runs and singletons in a shuffled order, spread over both pools."""
    rng = np.random.default_rng(seed)
    n_run = int(round(n * run_frac))
    lens, left = [], n_run
    while left > 0:
        r = max_run if fixed_run else int(rng.integers(1, max_run + 1))
        r = min(left, r)
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


def rank_steps(cfg: dict, cpu_blocks: int, local: int, nsteps: int = 4):
    """The ops of each step of one data-parallel rank: its own seeds, its own
    pools, no id shared with another rank's work.  An op is (gpu_ids,
    cpu_ids, is_host_to_device)."""
    steps = []
    for s in range(nsteps):
        seed = 1000 * local + 10 * s
        if cfg["kind"] == "batch":
            ops = []
            for j, h2d in enumerate((True, False)):
                g, c = make_batch(cfg["batch"], cfg["gpu_blocks"], cpu_blocks, seed + j,
                                  cfg["run_frac"], cfg["max_run"], cfg.get("fixed_run", False))
                ops.append((g, c, h2d))
        else:
            rng = np.random.default_rng(seed)
            sizes = rng.integers(1, cfg["max_req_blocks"] + 1, cfg["requests"])
            g, c = make_batch(int(sizes.sum()), cfg["gpu_blocks"], cpu_blocks, seed + 1, 0.0, 1)
            dirs = rng.integers(0, 2, cfg["requests"]).astype(bool)
            ops, o = [], 0
            for n, h2d in zip(sizes.tolist(), dirs.tolist()):
                ops.append((g[o:o + n], c[o:o + n], bool(h2d)))
                o += n
        steps.append(ops)
    return steps


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


def mem_available_bytes() -> int:
    with open("/proc/meminfo") as f:
        for line in f:
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    return 0


def kv_strides(kind: str, L: int, N: int, tpb: int, H: int, D: int, mla: bool) -> dict:
    """Element strides of FlexKV's KVCacheLayout (flexkv/common/storage.py:
    59-149) for a pool of N blocks: LAYERWISE [L, kv, N, tpb, H, D] or
    BLOCKWISE [N, L, kv, tpb, H, D].  Plain arithmetic, so the reference arm
    needs nothing of flexkv_b200."""
    kv = 1 if mla else 2
    chunk = tpb * H * D
    if kind == "LAYERWISE":
        st = {"layer": kv * N * chunk, "kv": N * chunk, "block": chunk}
    else:
        st = {"layer": kv * chunk, "kv": chunk, "block": L * kv * chunk}
    st.update(chunk=chunk, total=L * kv * N * chunk, kv_dim=kv)
    return st


def stock_host_register(t: torch.Tensor) -> None:
    """Page-lock a host tensor the way FlexKV's worker does: one plain
    cudaHostRegister with flag 1 (Portable), no huge-page advice
    (flexkv/transfer/worker.py:35-41)."""
    rc = torch.cuda.cudart().cudaHostRegister(t.data_ptr(), t.numel() * t.element_size(), 1)
    if int(getattr(rc, "value", rc)) != 0:
        raise RuntimeError(f"cudaHostRegister failed with error code {rc}")


def stock_host_unregister(t: torch.Tensor) -> None:
    torch.cuda.cudart().cudaHostUnregister(t.data_ptr())


def fit_cpu_blocks(cfg: dict, ws: int, block_bytes: int, override: int = 0) -> int:
    """The configuration's host pool, scaled down to 55 % of the box's
    available RAM shared by the ws ranks (and never below two batches)."""
    if override:
        return override
    fit = int(0.55 * mem_available_bytes() / max(ws, 1) / block_bytes)
    min_blocks = 2 * cfg.get("batch", cfg.get("requests", 1) * cfg.get("max_req_blocks", 1))
    return cfg["cpu_blocks"] if fit >= cfg["cpu_blocks"] else max(fit, min_blocks)


class Setup:
    """Pools, strides and per-step ops of one rank.

    stock=False: the host pool is page-locked by flexkv_b200
    (c_ext.cudaHostRegister with huge-page advice).  stock=True (the
    reference arm): the pool is one flat torch tensor, as FlexKV's
    CPUAllocator.allocate makes it (flexkv/storage/allocator.py:93-113),
    registered with the worker's plain Portable cudaHostRegister; nothing of
    flexkv_b200 is imported."""

    def __init__(self, cfg: dict, layout: str, ws: int, local: int, cpu_blocks_override: int = 0,
                 gpu_alloc: str = "per-layer", stock: bool = False):
        self.cfg = cfg
        self.stock = stock
        self.mla = cfg.get("mla", False)
        self.kv = 1 if self.mla else 2
        L, H, D, tpb = cfg["layers"], cfg["heads"], cfg["head_dim"], cfg["tpb"]
        e = 2
        self.chunk = tpb * H * D * e
        self.block_bytes = L * self.kv * self.chunk
        self.cpu_blocks = cpu_blocks = fit_cpu_blocks(cfg, ws, self.block_bytes, cpu_blocks_override)
        self.layout = layout
        g = kv_strides("LAYERWISE", 1, cfg["gpu_blocks"], tpb, H, D, self.mla)  # one layer
        c = kv_strides(layout, L, cpu_blocks, tpb, H, D, self.mla)
        self.g_kv, self.g_blk = g["kv"] * e, g["block"] * e
        self.c_kv, self.c_layer, self.c_blk = c["kv"] * e, c["layer"] * e, c["block"] * e
        self.gpu_layer_bytes = g["total"] * e
        layer_shape = (self.kv, cfg["gpu_blocks"], tpb, H, D)
        dev = torch.device(f"cuda:{local}")
        t0 = time.time()
        self.layers = []
        self.gpu_alloc = gpu_alloc
        if gpu_alloc == "contiguous":
            # One allocation viewed as per-layer [kv, N, tpb, H, D] tensors.
            self._gpu_base = torch.empty((L,) + layer_shape, dtype=torch.bfloat16, device=dev)
            self._gpu_base.normal_()
            self.layers = [self._gpu_base[l] for l in range(L)]
        else:
            for _ in range(L):
                t = torch.empty(layer_shape, dtype=torch.bfloat16, device=dev)
                t.normal_()
                self.layers.append(t)
        self.ptrs = torch.tensor([t.data_ptr() for t in self.layers], dtype=torch.int64)
        t1 = time.time()
        cpu_bytes = c["total"] * e
        self.cpu = torch.empty(cpu_bytes // 2, dtype=torch.bfloat16)
        if stock:
            stock_host_register(self.cpu)
        else:
            from flexkv_b200 import c_ext
            c_ext.cudaHostRegister(self.cpu, advise_hugepages=True)
        t2 = time.time()
        log(f"[rank{local}] gpu pool {L}x{self.gpu_layer_bytes / 2**30:.2f} GiB in {t1 - t0:.1f}s, "
            f"cpu pool {cpu_bytes / 2**30:.1f} GiB registered in {t2 - t1:.1f}s"
            + (" (stock: flat tensor, Portable cudaHostRegister)" if stock else ""))
        self.steps = rank_steps(cfg, cpu_blocks, local)
        self.step_bytes = {d: sum(len(g) for g, c, h in self.steps[0] if h == (d == "h2d")) * self.block_bytes
                           for d in ("h2d", "d2h")}

    @property
    def gpu_layout(self):
        """flexkv_b200's KVCacheLayout of the GPU pool (our arm only)."""
        from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
        c = self.cfg
        return KVCacheLayout(KVCacheLayoutType.LAYERWISE, c["layers"], c["gpu_blocks"], c["tpb"], c["heads"],
                             c["head_dim"], self.mla)

    @property
    def cpu_layout(self):
        """flexkv_b200's KVCacheLayout of the host pool (our arm only)."""
        from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
        c = self.cfg
        return KVCacheLayout(KVCacheLayoutType[self.layout], c["layers"], self.cpu_blocks, c["tpb"], c["heads"],
                             c["head_dim"], self.mla)

    def close(self):
        if self.stock:
            stock_host_unregister(self.cpu)
        else:
            from flexkv_b200 import c_ext
            c_ext.cudaHostUnregister(self.cpu)


def mode_kwargs(args):
    if args.mode == "sm":
        return {"ce_min_run_bytes": 0}, False
    if args.mode == "ce":
        return {}, True
    if args.mode == "hybrid":
        return {"ce_min_run_bytes": args.ce_min_run_bytes}, False
    return {}, False


def measure_link_peaks(S, stream, sync=None):
    """The host link's copy-engine rate on the same pinned pool: one large
    contiguous cudaMemcpyAsync each way, and both ways at once (the measured
    roofline of the path).  sync, when given, runs before each timed phase
    (a barrier: every rank copies at once)."""
    n = min(max(S.step_bytes.values()), 2 << 30)
    g1 = torch.empty(n, dtype=torch.uint8, device="cuda")
    g2 = torch.empty(n, dtype=torch.uint8, device="cuda")
    h1 = S.cpu.view(torch.uint8)[:n]
    h2 = S.cpu.view(torch.uint8)[n:2 * n]
    side = torch.cuda.Stream()
    peak = {}

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        if sync is not None:
            sync()
        ts = []
        for _ in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    peak["h2d"] = round(n / timed(lambda: g1.copy_(h1, non_blocking=True)) / 1e6, 2)
    peak["d2h"] = round(n / timed(lambda: h1.copy_(g1, non_blocking=True)) / 1e6, 2)

    def both():
        ev = torch.cuda.Event()
        ev.record(stream)
        side.wait_event(ev)
        g1.copy_(h1, non_blocking=True)
        with torch.cuda.stream(side):
            h2.copy_(g2, non_blocking=True)
        done = torch.cuda.Event()
        done.record(side)
        stream.wait_event(done)

    peak["duplex_total"] = round(2 * n / timed(both) / 1e6, 2)
    del g1, g2
    return dict(peak, unit="GB/s", bytes=n,
                how="contiguous cudaMemcpyAsync from the pinned pool (each way, and both at once), median of 3")


def _fs_type(path: str) -> str:
    """Filesystem type of the mount holding path (longest mount prefix)."""
    best, typ = "", "unknown"
    path = os.path.realpath(path)
    with open("/proc/mounts") as f:
        for line in f:
            parts = line.split()
            if len(parts) >= 3 and path.startswith(parts[1]) and len(parts[1]) > len(best):
                best, typ = parts[1], parts[2]
    return typ


def measure_ssd(steps: int = 3):
    """SSD tier: cfg2's Llama-3-8B block (32 layers x K,V x 32 KiB = 2 MiB),
    BLOCKWISE on both sides (the reference requires one layout type), one
    SSD device (a directory on the box's own disk, FLEXKV_SSD_BENCH_DIR or
    ./_ssd_bench), 512-block batches (1 GiB) of 50 % joint runs.  Writes
    (H2DISK), then reads (DISK2H, O_DIRECT where the filesystem allows) after
    a sync, for our SSD tier and for the C restatement of the reference's
    per-chunk loop (32 threads per device, as CPUSSDDiskTransferWorker
    passes).  Wall clock around each synchronous call, median of `steps`."""
    import shutil
    from flexkv_b200 import c_ext
    from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
    from flexkv_b200.ssd import SsdStrides, allocate_ssd_files
    from oracle import oracle as O
    L, H, D, tpb, nblk, batch = 32, 8, 128, 16, 4096, 512
    def pin(t):  # page-aligned (O_DIRECT) either way: pinned memory, or an aligned view
        if torch.cuda.is_available():
            return t.pin_memory()
        raw = np.empty(t.numel() + 4096, np.uint8)
        off = (-raw.ctypes.data) % 4096
        a = torch.from_numpy(raw[off:off + t.numel()])
        a.copy_(t)
        return a
    lay = KVCacheLayout(KVCacheLayoutType.BLOCKWISE, L, nblk, tpb, H, D)
    root = os.environ.get("FLEXKV_SSD_BENCH_DIR") or os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                                   "_ssd_bench")
    os.makedirs(root, exist_ok=True)
    try:
        files, per_file = allocate_ssd_files(lay, 2, root, max_blocks_per_file=nblk)
        st = SsdStrides.of(lay, lay, 1, 2)
        nbytes_pool = lay.get_total_elements() * 2
        pool = pin(torch.empty(nbytes_pool, dtype=torch.uint8))
        pool.view(torch.int64).copy_(torch.arange(nbytes_pool // 8, dtype=torch.int64) * 0x9E3779B97F4A7C15)
        back = pin(torch.zeros(nbytes_pool, dtype=torch.uint8))
        batches = [make_batch(batch, nblk, nblk, 70 + j, 0.5, 64) for j in range(steps + 1)]
        ours = c_ext.SSDIOCTX(files, 1)
        ours_ring = c_ext.SSDIOCTX(files, 1, 128, 0)  # io_uring, 128 requests in flight
        ref = O.SsdRefContext(files, 1)
        layers = torch.arange(0, L, dtype=torch.int32)

        def run_ours(pool_t, s_ids, c_ids, is_read):
            c_ext.transfer_kv_blocks_ssd(ours, layers, pool_t.data_ptr(), torch.from_numpy(s_ids),
                                         torch.from_numpy(c_ids), st.cpu_layer_stride_in_bytes,
                                         st.cpu_kv_stride_in_bytes, st.ssd_layer_stride_in_bytes,
                                         st.ssd_kv_stride_in_bytes, st.chunk_size_in_bytes,
                                         st.block_stride_in_bytes, is_read, per_file, 1, 32, False)

        def run_ring(pool_t, s_ids, c_ids, is_read):
            c_ext.transfer_kv_blocks_ssd(ours_ring, layers, pool_t.data_ptr(), torch.from_numpy(s_ids),
                                         torch.from_numpy(c_ids), st.cpu_layer_stride_in_bytes,
                                         st.cpu_kv_stride_in_bytes, st.ssd_layer_stride_in_bytes,
                                         st.ssd_kv_stride_in_bytes, st.chunk_size_in_bytes,
                                         st.block_stride_in_bytes, is_read, per_file, 1, 32, False)

        def run_ref(pool_t, s_ids, c_ids, is_read):
            ref.transfer(0, L, pool_t.data_ptr(), s_ids, c_ids, st, is_read, 1, 32, False)

        arms = [("reference_style", run_ref), ("ours", run_ours)]
        if ours_ring.uses_io_uring:
            arms.append(("ours_io_uring", run_ring))
        res = {}
        for name, fn in arms:
            tw, tr = [], []
            for j, (g, c) in enumerate(batches):  # ssd ids = g, cpu ids = c
                t0 = time.perf_counter()
                fn(pool, g, c, False)
                t1 = time.perf_counter()
                os.sync()
                t2 = time.perf_counter()
                fn(back, g, c, True)
                t3 = time.perf_counter()
                if j:  # the first batch warms up
                    tw.append(t1 - t0)
                    tr.append(t3 - t2)
            nbytes = batch * L * 2 * st.chunk_size_in_bytes
            res[name] = {"write_gbs": round(nbytes / statistics.median(tw) / 1e9, 2),
                         "read_gbs": round(nbytes / statistics.median(tr) / 1e9, 2)}
        g, c = batches[-1]
        run_ours(back, g, c, True)
        n_ios, _ = ours.last_stats()
        got = back.numpy()
        want_t = pin(torch.zeros(nbytes_pool, dtype=torch.uint8))
        ref.transfer(0, L, want_t.data_ptr(), g, c, st, True, 1, 32, False)
        want = want_t.numpy()
        if not np.array_equal(got.reshape(nblk, -1)[c], want.reshape(nblk, -1)[c]):
            raise RuntimeError("SSD tier read different bytes than the reference-style loop")
        ours.close()
        ours_ring.close()
        ref.close()
        return {"config": {"workload": "cfg2 Llama-3-8B blocks, BLOCKWISE CPU and SSD", "block_bytes": 2 << 20,
                           "batch_blocks": batch, "batch_bytes": batch * (2 << 20), "ssd_devices": 1,
                           "filesystem": _fs_type(root), "threads_per_device": 32,
                           "reads": "after os.sync(); O_DIRECT where the filesystem allows it"},
                "ours": res["ours"], "ours_io_uring": res.get("ours_io_uring"),
                "reference_style": res["reference_style"],
                "requests_per_batch": {"ours": int(n_ios), "reference_style": batch * L * 2},
                "how": "wall clock around each synchronous call, median of %d batches" % steps}
    finally:
        shutil.rmtree(root, ignore_errors=True)


def measure_hash():
    """XXH64 block hashing: one 1M-token sequence (65536 blocks of 16) and a
    batch of 256 requests of U[1,32] blocks, on the GPU (device buffers, and
    host buffers end to end) against the CPU restatement of hash.cpp's loop
    (oracle, one thread, update+digest per block like the reference)."""
    from flexkv_b200 import c_ext
    from oracle import oracle as O
    rng = np.random.default_rng(4)
    toks = rng.integers(0, 152064, 1 << 20).astype(np.int32).astype(np.int64)
    tpb = 16
    nb = toks.size // tpb
    out = {}
    h = c_ext.Hasher()
    dev_t = torch.from_numpy(toks).cuda()
    dev_o = torch.zeros(nb, dtype=torch.uint64, device="cuda")
    host_t = torch.from_numpy(toks).pin_memory()
    host_o = torch.zeros(nb, dtype=torch.uint64)

    def gpu_dev():
        h.reset()
        c_ext.gen_hashes(h, dev_t, tpb, dev_o)
        torch.cuda.synchronize()

    def gpu_host():
        h.reset()
        c_ext.gen_hashes(h, host_t, tpb, host_o)

    def best(fn, n=5):
        fn()
        ts = []
        for _ in range(n):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts)

    t_dev, t_host = best(gpu_dev), best(gpu_host)
    t_cpu = best(lambda: O.gen_hashes(toks, tpb), 3)
    if not np.array_equal(host_o.numpy(), O.gen_hashes(toks, tpb)):
        raise RuntimeError("GPU block hashes differ from the oracle")
    nbytes = toks.nbytes
    out["single_sequence_1M_tokens"] = {
        "blocks": nb, "gpu_device_ms": round(t_dev * 1e3, 3), "gpu_host_buffers_ms": round(t_host * 1e3, 3),
        "cpu_port_1thread_ms": round(t_cpu * 1e3, 3),
        "gpu_device_gbs": round(nbytes / t_dev / 1e9, 2), "cpu_port_gbs": round(nbytes / t_cpu / 1e9, 2)}
    sizes = rng.integers(1, 33, 256) * tpb
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    rt = rng.integers(0, 152064, int(sizes.sum())).astype(np.int64)
    rt_dev = torch.from_numpy(rt).cuda()
    rt_host = torch.from_numpy(rt).pin_memory()

    def b_dev():
        c_ext.gen_hashes_batched(rt_dev, offs, tpb)
        torch.cuda.synchronize()

    t_bd = best(b_dev)
    t_bh = best(lambda: c_ext.gen_hashes_batched(rt_host, offs, tpb))
    t_bc = best(lambda: O.gen_hashes_batched(rt, offs, tpb), 3)
    out["batched_256_requests"] = {
        "tokens": int(sizes.sum()), "gpu_device_ms": round(t_bd * 1e3, 3),
        "gpu_host_buffers_ms": round(t_bh * 1e3, 3), "cpu_port_1thread_ms": round(t_bc * 1e3, 3),
        "gpu_device_mtokens_s": round(sizes.sum() / t_bd / 1e6, 1),
        "cpu_port_mtokens_s": round(sizes.sum() / t_bc / 1e6, 1)}
    # A scheduling step's worth of requests: 4096 of U[1,32] blocks (~1 M tokens).
    sizes = rng.integers(1, 33, 4096) * tpb
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    rt = rng.integers(0, 152064, int(sizes.sum())).astype(np.int64)
    rt_dev = torch.from_numpy(rt).cuda()
    rt_host = torch.from_numpy(rt).pin_memory()
    t_bd = best(lambda: (c_ext.gen_hashes_batched(rt_dev, offs, tpb), torch.cuda.synchronize()))
    t_bh = best(lambda: c_ext.gen_hashes_batched(rt_host, offs, tpb))
    t_bc = best(lambda: O.gen_hashes_batched(rt, offs, tpb), 3)
    ncores = len(os.sched_getaffinity(0))
    t_bm = best(lambda: O.gen_hashes_batched(rt, offs, tpb, ncores), 3)
    if not np.array_equal(c_ext.gen_hashes_batched(rt_host, offs, tpb).numpy(), O.gen_hashes_batched(rt, offs, tpb)):
        raise RuntimeError("batched GPU block hashes differ from the oracle")
    out["batched_4096_requests"] = {
        "tokens": int(sizes.sum()), "gpu_device_ms": round(t_bd * 1e3, 3),
        "gpu_host_buffers_ms": round(t_bh * 1e3, 3), "cpu_port_1thread_ms": round(t_bc * 1e3, 3),
        "gpu_device_mtokens_s": round(sizes.sum() / t_bd / 1e6, 1),
        "gpu_host_buffers_mtokens_s": round(sizes.sum() / t_bh / 1e6, 1),
        "cpu_port_mtokens_s": round(sizes.sum() / t_bc / 1e6, 1),
        "cpu_port_ncores_ms": round(t_bm * 1e3, 3), "cpu_port_ncores": ncores,
        "cpu_port_ncores_mtokens_s": round(sizes.sum() / t_bm / 1e6, 1)}
    h.close()
    return out


def measure_host_torch_path(S, n_blocks: int = 512, reps: int = 3):
    """The reference's host-side torch path on the box's own cores (a
    baseline beside the kernels): H2D gathers the blocks' chunks from the
    pinned pool's view with index_select into pinned staging, copies the
    staging to the GPU in one cudaMemcpyAsync and scatters it into every
    layer with index_copy_; D2H is the mirror image.  A bounded sample of
    n_blocks blocks of the workload's first H2D and D2H batches; torch uses
    every core of this process's affinity."""
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    L = len(S.layers)
    if S.cpu_layout.type.name == "LAYERWISE":
        view = S.cpu.view(L, S.kv, S.cpu_blocks, -1)  # [layer, kv, block, chunk]
        bdim = 2
    else:
        view = S.cpu.view(S.cpu_blocks, L, S.kv, -1)  # [block, layer, kv, chunk]
        bdim = 0
    gpu_views = [t.view(S.kv, S.gpu_layout.num_block, -1) for t in S.layers]  # [kv, block, chunk]
    ops = {h: (g[:n_blocks], c[:n_blocks]) for g, c, h in S.steps[0]}
    out = {}
    for h2d in (True, False):
        g, c = ops[h2d]
        gi, ci = torch.from_numpy(g).cuda(), torch.from_numpy(c)
        ts = []
        for _ in range(reps + 1):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if h2d:
                stage = torch.index_select(view, bdim, ci).pin_memory()
                dev = stage.cuda(non_blocking=True)
                for l in range(L):
                    part = dev[:, l] if bdim == 0 else dev[l]  # [block, kv, chunk] or [kv, block, chunk]
                    if bdim == 0:
                        part = part.transpose(0, 1)
                    gpu_views[l].index_copy_(1, gi, part)
            else:
                stage = torch.stack([gpu_views[l].index_select(1, gi) for l in range(L)], 0)  # [L, kv, n, chunk]
                host = stage.cpu()
                if bdim == 2:
                    view.index_copy_(2, ci, host)
                else:
                    view.index_copy_(0, ci, host.permute(2, 0, 1, 3).contiguous())
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t0)
        out["h2d" if h2d else "d2h"] = round(n_blocks * S.block_bytes / statistics.median(ts[1:]) / 1e9, 2)
    return {"per_direction_gbs": out, "unit": "GB/s", "cores": n, "blocks": n_blocks,
            "how": "index_select gather / index_copy_ scatter on the pool view, one staged copy, "
                   "median of %d" % reps}


def measure_layerwise_read(S, groups: int = 8, reps: int = 3):
    """A layer-wise read graph (convert_read_graph_to_layer_wise_graph,
    transfer_pattern.py:370-428): the workload's first H2D batch split into
    `groups` ops of L/groups layers, each depending on the previous, as a
    prefill that starts on layer group 0 while later groups load
    (wait_at_layer_group, kvmanager.py:480).  Reports when each group's
    completion reaches the caller, in ms from submission (median of reps)."""
    from flexkv_b200.engine import TransferDescriptor, TransferEngine, TransferOp, TransferOpGraph, TransferType
    g, c = next((g, c) for g, c, h in S.steps[0] if h)
    L = len(S.layers)
    per = L // groups
    eng = TransferEngine([S.layers], S.cpu, S.gpu_layout, S.cpu_layout)
    runs = []
    try:
        for _ in range(reps + 1):
            gr = TransferOpGraph()
            ops = []
            for k in range(groups):
                op = TransferOp(graph_id=gr.graph_id, transfer_type=TransferType.H2D, layer_id=k * per,
                                layer_granularity=per,
                                src_descriptor=TransferDescriptor(torch.from_numpy(c)),
                                dst_descriptor=TransferDescriptor(torch.from_numpy(g)))
                gr.add_transfer_op(op)
                if ops:
                    gr.add_dependency(op.op_id, ops[-1].op_id)
                ops.append(op)
            order = {op.op_id: k for k, op in enumerate(ops)}
            t0 = time.perf_counter()
            eng.submit_transfer_graph(gr)
            seen = [None] * groups
            while any(x is None for x in seen):
                for gid, oid in eng.get_completed_graphs_and_ops(timeout=0.001):
                    if gid == gr.graph_id and oid in order:
                        seen[order[oid]] = (time.perf_counter() - t0) * 1e3
            runs.append(seen)
    finally:
        eng.shutdown()
    med = [round(statistics.median(r[k] for r in runs[1:]), 2) for k in range(groups)]
    return {"groups": groups, "layers_per_group": per, "blocks": len(g), "group_done_ms": med,
            "how": "one graph of chained layer-group H2D ops through the TransferEngine; wall clock"}


def put_batches(S, n_batches: int, n_req: int = 256, seed: int = 77, vocab: int = 128256):
    """Put batches: n_req requests of U[1,32] full blocks each; half of
    them extend a prefix (1..all of its blocks) of an earlier request of the
    same or an earlier batch by U[0,16] new blocks.  Token ids int64."""
    tpb = S.cfg["tpb"]
    rng = np.random.default_rng(seed)
    seen, out = [], []
    for _ in range(n_batches):
        toks, gids = [], []
        for _ in range(n_req):
            if seen and rng.random() < 0.5:
                base = seen[rng.integers(len(seen))]
                cut = int(rng.integers(1, len(base) // tpb + 1))
                tok = np.concatenate([base[:cut * tpb], rng.integers(0, vocab, int(rng.integers(0, 17)) * tpb)])
            else:
                tok = rng.integers(0, vocab, int(rng.integers(1, 33)) * tpb)
            tok = tok.astype(np.int64)
            seen.append(tok)
            toks.append(tok)
            gids.append(rng.choice(S.gpu_layout.num_block, len(tok) // tpb, replace=False).astype(np.int64))
        out.append((toks, gids))
    return out


def measure_put_path(S, reps: int = 3):
    """The CPU tier's put and get for batches of requests
    (cache_engine.py:150-219, 412-615, 787-902): per repetition, on a fresh
    index, two consecutive 256-request put batches, then a 256-request get
    batch of sequences the puts cached (all blocks, into new GPU blocks).

    ours: one flexkv_b200.cache_index.CpuCacheIndex call per batch -- put:
      hash, match, allocate, insert, D2H copy of the new blocks, mark ready;
      get: hash, match, H2D copy of the ready prefix -- all on the device,
      from host token buffers (wall clock, synchronous).
    reference-style: per request, the CPU restatement of the reference's
      tree and pool (oracle/cache_index.py: Python control flow like the
      reference's, with the C XXH64) to decide, the reference's own
      transfer.cu (oracle/_ref, transfer_sms=8, ids pinned per op,
      synchronous) to copy, then the put's completion callback.
    control only: the second put batch again -- every block cached, nothing
      copied -- so the time is hashing, matching and deciding.
    layer-wise get: the same get in layer groups (layer_granularity), timed
      to the first group's event (when a prefill could start) and the last."""
    from oracle import cache_index as CI
    from oracle import oracle as O
    from flexkv_b200.cache_index import CpuCacheIndex, KVLayout
    tpb = S.cfg["tpb"]
    layout = KVLayout(S.ptrs, S.g_kv, S.g_blk, S.cpu, S.c_kv, S.c_layer, S.c_blk, S.chunk, S.mla, -1,
                      S.gpu_layer_bytes)
    batches = put_batches(S, 2)
    n_req = len(batches[0][0])
    rng = np.random.default_rng(91)
    every = [t for toks, _ in batches for t in toks]
    gtoks = [every[i] for i in rng.choice(len(every), n_req, replace=False)]
    # distinct GPU destinations across the get batch
    perm = rng.permutation(S.gpu_layout.num_block).astype(np.int64)
    cuts = np.cumsum([0] + [len(t) // tpb for t in gtoks])
    if cuts[-1] > len(perm):
        raise RuntimeError("get batch larger than the GPU pool")
    ggids = [perm[cuts[i]:cuts[i + 1]] for i in range(len(gtoks))]
    ours, ctl, ours_get, ref, ref_ctl, ref_get, moved, got_blocks = [], [], [], [], [], [], [], []
    L = len(S.layers)
    G = next(g for g in range(max(1, L // 8), L + 1) if L % g == 0)  # layer groups of the layer-wise get
    lw_first, lw_all = [], []
    ref_lib = O.ref_lib() if O.reference_available() else None
    ptrs = S.ptrs.pin_memory()
    stream = torch.cuda.current_stream().cuda_stream

    def ref_copy(g, c, h2d):
        gp = torch.from_numpy(g).pin_memory()
        cp = torch.from_numpy(c).pin_memory()
        rc = ref_lib.ref_transfer_kv_blocks(len(gp), 0, len(S.layers), gp.data_ptr(), ptrs.data_ptr(),
                                            S.g_kv, S.g_blk, cp.data_ptr(), S.cpu.data_ptr(), S.c_kv,
                                            S.c_layer, S.c_blk, 0, S.chunk, stream, 8, int(h2d), 0, int(S.mla))
        if rc != 0:
            raise RuntimeError(f"reference transfer_kv_blocks CUDA error {rc}")

    for rep in range(reps + 1):
        ci = CpuCacheIndex(S.cpu_blocks, tpb)
        try:
            ts, blocks = [], 0
            for toks, gids in batches:
                t0 = time.perf_counter()
                res = ci.put(toks, gids, layout)
                ts.append(time.perf_counter() - t0)
                blocks += int(res.num_transferred.sum())
            t0 = time.perf_counter()
            again = ci.put(*batches[1], layout)
            tc = time.perf_counter() - t0
            assert int(again.num_transferred.sum()) == 0
            t0 = time.perf_counter()
            gres = ci.get(gtoks, ggids, layout)
            tg = time.perf_counter() - t0
            evs = [torch.cuda.Event() for _ in range(L // G)]
            for e in evs:
                e.record()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ci.get(gtoks, ggids, layout, synchronous=False, layer_granularity=G, group_events=evs)
            evs[0].synchronize()
            t_first = time.perf_counter() - t0
            evs[-1].synchronize()
            t_lw = time.perf_counter() - t0
        finally:
            ci.close()
        if rep:
            ours.append(sum(ts))
            ctl.append(tc)
            ours_get.append(tg)
            lw_first.append(t_first)
            lw_all.append(t_lw)
            moved.append(blocks)
            got_blocks.append(int(gres.num_transferred.sum()))
        if ref_lib is None:
            continue
        tier = CI.CpuTier(S.cpu_blocks, tpb)
        t_all = t_dec = 0.0
        ref_blocks = 0
        for toks, gids in batches:
            for tok, g in zip(toks, gids):
                t0 = time.perf_counter()
                r = tier.put(tok, g)
                t1 = time.perf_counter()
                if r.num_transferred:
                    ref_copy(r.gpu_blocks, r.cpu_blocks, False)
                t2 = time.perf_counter()
                tier.complete(r)
                t3 = time.perf_counter()
                t_all += t3 - t0
                t_dec += (t1 - t0) + (t3 - t2)
                ref_blocks += r.num_transferred
        t0 = time.perf_counter()
        ref_got = 0
        for tok, g in zip(gtoks, ggids):
            r = tier.get(tok, g)
            if r.num_transferred:
                ref_copy(r.gpu_blocks, r.cpu_blocks, True)
            ref_got += r.num_transferred
        tg_ref = time.perf_counter() - t0
        if rep:
            ref.append(t_all)
            ref_ctl.append(t_dec)
            ref_get.append(tg_ref)
            assert ref_blocks == moved[-1], (ref_blocks, moved[-1])
            assert ref_got == got_blocks[-1], (ref_got, got_blocks[-1])
    bb = S.block_bytes
    med = statistics.median
    out = {
        "requests_per_batch": n_req, "put_batches": len(batches), "blocks_copied": moved[-1],
        "bytes_copied": moved[-1] * bb, "get_blocks_read": got_blocks[-1],
        "ours": {"ms": round(med(ours) * 1e3, 2), "GBps": round(moved[-1] * bb / med(ours) / 1e9, 2),
                 "requests_per_s": round(len(batches) * n_req / med(ours)),
                 "control_us_per_request": round(med(ctl) / n_req * 1e6, 2)},
        "ours_get": {"ms": round(med(ours_get) * 1e3, 2),
                     "GBps": round(got_blocks[-1] * bb / med(ours_get) / 1e9, 2)},
        "ours_get_layerwise": {"layer_granularity": G, "groups": L // G,
                               "first_group_ms": round(med(lw_first) * 1e3, 2),
                               "all_groups_ms": round(med(lw_all) * 1e3, 2)},
        "how": "wall clock, median of %d repetitions on a fresh index" % reps,
    }
    if ref:
        out["reference_style"] = {
            "ms": round(med(ref) * 1e3, 2), "GBps": round(moved[-1] * bb / med(ref) / 1e9, 2),
            "requests_per_s": round(len(batches) * n_req / med(ref)),
            "control_us_per_request": round(med(ref_ctl) / (len(batches) * n_req) * 1e6, 2)}
        out["reference_style_get"] = {"ms": round(med(ref_get) * 1e3, 2),
                                      "GBps": round(got_blocks[-1] * bb / med(ref_get) / 1e9, 2)}
        out["speedup"] = round(med(ref) / med(ours), 2)
        out["speedup_get"] = round(med(ref_get) / med(ours_get), 2)
    return out


def measure_op_latency(S, args, n: int = 200):
    """Latency of one small op, each submitted after the previous finished:
    a 1-block H2D (every layer: 64 chunks of the workload's chunk size)
    through the TransferEngine (submit_transfer_graph, then
    get_completed_graphs_and_ops until it reports the graph) and through
    one synchronous c_ext.transfer_kv_blocks call.  Medians in microseconds."""
    from flexkv_b200 import c_ext
    from flexkv_b200.engine import TransferDescriptor, TransferEngine, TransferOp, TransferOpGraph, TransferType
    rng = np.random.default_rng(5)
    pairs = [(int(g), int(c)) for g, c in zip(rng.integers(0, S.gpu_layout.num_block, n),
                                             rng.integers(0, S.cpu_layout.num_block, n))]
    eng = TransferEngine([S.layers], S.cpu, S.gpu_layout, S.cpu_layout)
    t_eng = []
    try:
        for k, (g, c) in enumerate(pairs):
            gr = TransferOpGraph()
            gr.add_transfer_op(TransferOp(graph_id=gr.graph_id, transfer_type=TransferType.H2D,
                                          src_descriptor=TransferDescriptor(torch.tensor([c])),
                                          dst_descriptor=TransferDescriptor(torch.tensor([g]))))
            t0 = time.perf_counter()
            eng.submit_transfer_graph(gr)
            done = False
            while not done:
                done = any(gid == gr.graph_id and oid == -1
                           for gid, oid in eng.get_completed_graphs_and_ops(timeout=0.001))
            t_eng.append(time.perf_counter() - t0)
    finally:
        eng.shutdown()
    t_call = []
    for g, c in pairs:
        gi, ci = torch.tensor([g]), torch.tensor([c])
        t0 = time.perf_counter()
        c_ext.transfer_kv_blocks(gi, S.ptrs, S.g_kv, S.g_blk, ci, S.cpu, S.c_kv, S.c_layer, S.c_blk, S.chunk, 0,
                                 -1, True, False, S.mla)
        t_call.append(time.perf_counter() - t0)
    med = lambda v: round(statistics.median(v[10:]) * 1e6, 1)
    return {"engine_us": med(t_eng), "direct_call_us": med(t_call), "unit": "us",
            "op": f"1 block H2D ({S.chunk * S.gpu_layout.num_layer * (1 if S.mla else 2)} bytes)",
            "how": "median of %d ops, each after the previous finished; wall clock" % (n - 10)}


def measure_engine(S, args, K, W, ws):
    """Wall-clock seconds for K steps through flexkv_b200.engine.TransferEngine
    (public API: submit_transfer_graph / get_completed_graphs_and_ops) on the
    same pools; H2D and D2H ops run on the engine's two streams."""
    from flexkv_b200.engine import TransferDescriptor, TransferEngine, TransferOp, TransferOpGraph, TransferType
    eng = TransferEngine([S.layers], S.cpu, S.gpu_layout, S.cpu_layout,
                         transfer_sms_h2d=args.transfer_sms, transfer_sms_d2h=args.transfer_sms)
    host_ops = [[(torch.from_numpy(g), torch.from_numpy(c), h) for g, c, h in ops] for ops in S.steps]

    def step(k):
        ids = []
        for g, c, h2d in host_ops[k % len(host_ops)]:
            gr = TransferOpGraph()
            src, dst = (c, g) if h2d else (g, c)
            gr.add_transfer_op(TransferOp(graph_id=gr.graph_id,
                                          transfer_type=TransferType.H2D if h2d else TransferType.D2H,
                                          src_descriptor=TransferDescriptor(src),
                                          dst_descriptor=TransferDescriptor(dst)))
            eng.submit_transfer_graph(gr)
            ids.append(gr.graph_id)
        left = set(ids)
        while left:
            for gid, oid in eng.get_completed_graphs_and_ops(timeout=0.01):
                if oid == -1:
                    left.discard(gid)

    try:
        for k in range(W):
            step(k)
        barrier(ws)
        t0 = time.perf_counter()
        for k in range(K):
            step(W + k)
        dt = time.perf_counter() - t0
        barrier(ws)
        if eng.failed_ops:
            raise RuntimeError(f"engine ops failed: {eng.failed_ops}")
    finally:
        eng.shutdown()
    return dt


def gather_over_ranks(ws, xs):
    """Every rank's list of floats (same length on all ranks), rank-major;
    timing plumbing only, never data."""
    if ws == 1:
        return [list(xs)]
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor(list(xs), dtype=torch.float64, device=dev)
    out = [torch.empty_like(t) for _ in range(ws)]
    dist.all_gather(out, t)
    return [o.cpu().tolist() for o in out]


def run_ours(args, ws, rank, local, cfg, layout, with_hash):
    """value: every op through the reference-facing call
    (c_ext.transfer_kv_blocks with host id tensors, one synchronous call per
    op as FlexKV's worker makes it; per-direction streams when the workload
    overlaps directions), device-timed with CUDA events on the call's
    stream.  plan_replay: the same ops as TransferPlans built before the
    timed region (it also brackets the SM kernel alone for the roofline).
    e2e: the same steps through flexkv_b200.engine.TransferEngine."""
    from flexkv_b200 import c_ext
    S = Setup(cfg, layout, ws, local, args.cpu_blocks, args.gpu_alloc)
    kw, use_ce = mode_kwargs(args)
    conc = cfg["concurrent"]
    plans = [[c_ext.TransferPlan(torch.from_numpy(g), S.ptrs, S.g_kv, S.g_blk, torch.from_numpy(c),
                                 S.cpu, S.c_kv, S.c_layer, S.c_blk, S.chunk, 0, args.transfer_sms,
                                 h2d, use_ce, S.mla, gpu_layer_bytes=S.gpu_layer_bytes, **kw)
              for g, c, h2d in ops] for ops in S.steps]
    host_ops = [[(torch.from_numpy(g).pin_memory(), torch.from_numpy(c).pin_memory(), h)
                 for g, c, h in ops] for ops in S.steps]
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    # Concurrent workloads: each direction alternates over two streams (as
    # the engine's per-direction stream pool does), so one small op's tail
    # overlaps the next op's start.
    pool_h, pool_d = [stream, torch.cuda.Stream()], [side, torch.cuda.Stream()]
    K, W = args.steps, args.warmup
    track_kernels = cfg["kind"] == "batch"

    def new_events(n):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        for e in evs:  # torch creates the CUDA event on its first record
            e.record(stream)
        return evs

    def new_rec(k, kernels):
        nops = len(S.steps[(W + k) % len(S.steps)])
        e = new_events(4 + 2 * nops + (2 * nops if kernels else 0))
        rec = {"start": e[0], "end": e[1], "end_main": e[2], "end_side": e[3],
               "op": [(e[4 + 2 * i], e[5 + 2 * i]) for i in range(nops)]}
        if kernels:
            b = 4 + 2 * nops
            rec["k"] = [(e[b + 2 * i], e[b + 2 * i + 1]) for i in range(nops)]
        return rec

    def run_step(k, rec=None, via_plans=False):
        """Enqueue step k through the per-op call (or the prebuilt plans);
        rec collects events for timing (None = untimed)."""
        ops, ps, hops = S.steps[k % len(S.steps)], plans[k % len(plans)], host_ops[k % len(host_ops)]
        start = rec["start"] if rec is not None else torch.cuda.Event()
        start.record(stream)
        if conc:
            for q in pool_h[1:] + pool_d:
                q.wait_event(start)
        nh = nd = 0
        for i, (g, c, h2d) in enumerate(hops):
            if not conc:
                st = stream
            elif h2d:
                st, nh = pool_h[nh % 2], nh + 1
            else:
                st, nd = pool_d[nd % 2], nd + 1
            if rec is not None and not conc:
                rec["op"][i][0].record(st)
            if via_plans:
                if rec is not None and "k" in rec:
                    ps[i].execute(stream=st, kernel_events=(rec["k"][i][0], rec["k"][i][1]))
                else:
                    ps[i].execute(stream=st)
            else:
                with torch.cuda.stream(st):
                    c_ext.transfer_kv_blocks(g, S.ptrs, S.g_kv, S.g_blk, c, S.cpu, S.c_kv, S.c_layer, S.c_blk,
                                             S.chunk, 0, args.transfer_sms, h2d, use_ce, S.mla,
                                             synchronous=not conc, gpu_layer_bytes=S.gpu_layer_bytes, **kw)
            if rec is not None and not conc:
                rec["op"][i][1].record(st)
        if conc:
            for a, b in ((stream, pool_h[1]), (side, pool_d[1])):
                j = torch.cuda.Event()
                j.record(b)
                a.wait_event(j)
            if rec is not None:
                rec["end_side"].record(side)
                rec["end_main"].record(stream)
            done = torch.cuda.Event()
            done.record(side)
            stream.wait_event(done)
        if rec is not None:
            rec["end"].record(stream)

    def dir_times(recs):
        """Per-direction device ms of each timed step."""
        out = {"h2d": [], "d2h": []}
        for k, rec in enumerate(recs):
            ops = S.steps[(W + k) % len(S.steps)]
            if conc:
                out["h2d"].append(rec["start"].elapsed_time(rec["end_main"]))
                out["d2h"].append(rec["start"].elapsed_time(rec["end_side"]))
            else:
                for d in ("h2d", "d2h"):
                    out[d].append(sum(rec["op"][i][0].elapsed_time(rec["op"][i][1])
                                      for i, op in enumerate(ops) if op[2] == (d == "h2d")))
        return out

    sb = S.step_bytes
    step_total = sb["h2d"] + sb["d2h"]

    def rates(dms):
        return {d: (sb[d] / (statistics.mean(dms[d]) / 1e3) / 1e9 if sb[d] and statistics.mean(dms[d]) > 0
                    else 0.0) for d in ("h2d", "d2h")}

    for k in range(W):
        run_step(k)
        run_step(k, via_plans=True)
    torch.cuda.synchronize()
    recs = [new_rec(k, False) for k in range(K)]
    precs = [new_rec(k, track_kernels) for k in range(K)]
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    with sampler:
        # value: the per-op call path, host id tensors, device-timed
        barrier(ws)
        launches0 = c_ext.kernel_launch_count()
        w0 = time.perf_counter()
        for k in range(K):
            run_step(W + k, recs[k])
        torch.cuda.synchronize()
        calls_wall_s = time.perf_counter() - w0
        launches = c_ext.kernel_launch_count() - launches0
        barrier(ws)
        elapsed_ms = recs[0]["start"].elapsed_time(recs[-1]["end"])
        # plan replay: the same ops from TransferPlans built before timing
        barrier(ws)
        for k in range(K):
            run_step(W + k, precs[k], via_plans=True)
        torch.cuda.synchronize()
        barrier(ws)
        plan_ms = precs[0]["start"].elapsed_time(precs[-1]["end"])
        # e2e: the same steps through the TransferEngine, one single-op
        # graph per op, all submitted, then polled until every graph ended.
        e2e_engine_s = measure_engine(S, args, K, W, ws)
    clocks = sampler.summary()
    dir_ms = dir_times(recs)
    rate = rates(dir_ms)
    plan_rate = rates(dir_times(precs))
    kern_ms = {"h2d": [], "d2h": []}
    if track_kernels:
        for k, rec in enumerate(precs):
            for i, op in enumerate(S.steps[(W + k) % len(S.steps)]):
                kern_ms["h2d" if op[2] else "d2h"].append(rec["k"][i][0].elapsed_time(rec["k"][i][1]))

    extras = {}
    lp_alone = lp_conc = None
    if not args.no_extras:
        for r in range(ws):  # one rank at a time: each GPU's own link
            if r == rank:
                lp_alone = measure_link_peaks(S, stream)
            barrier(ws)
        if ws > 1:  # every rank at once: the host side shared by all links
            lp_conc = measure_link_peaks(S, stream, sync=lambda: barrier(ws))
        extras["link_peak_measured"] = dict(lp_alone)
        if lp_conc is not None:
            extras["link_peak_concurrent"] = dict(
                lp_conc, how="contiguous cudaMemcpyAsync from each rank's pinned pool with every rank "
                             "copying at once (rank 0's rates), median of 3")
        if not conc and cfg["kind"] == "batch":
            ts = []  # the same steps with both directions in flight together
            for k in range(max(K, 3)):
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                side.wait_event(a)
                hp, dp = plans[k % len(plans)]
                hp.execute(stream=stream)
                dp.execute(stream=side)
                c = torch.cuda.Event()
                c.record(side)
                stream.wait_event(c)
                b.record(stream)
                torch.cuda.synchronize()
                ts.append(a.elapsed_time(b))
            extras["duplex"] = {"value": round(step_total / statistics.median(ts) / 1e6, 2), "unit": "GB/s",
                                "how": "the same steps with the H2D and the D2H batch in flight together on two streams"}
        if with_hash and rank == 0 and ws == 1:
            extras["hash"] = measure_hash()
            extras["op_latency"] = measure_op_latency(S, args)
            extras["layerwise_read"] = measure_layerwise_read(S)
            try:
                extras["put_path"] = measure_put_path(S)
            except Exception as e:  # reported, never fatal to the main line
                extras["put_path"] = {"error": f"{type(e).__name__}: {e}"}
            try:  # a reported baseline; a failure is recorded, not fatal
                extras["host_torch_path"] = measure_host_torch_path(S)
            except Exception as e:  # noqa: BLE001
                extras["host_torch_path"] = {"error": f"{type(e).__name__}: {e}"}
            try:  # the SSD tier on the box's own disk; a failure is recorded, not fatal
                extras["ssd"] = measure_ssd()
            except Exception as e:  # noqa: BLE001
                extras["ssd"] = {"error": f"{type(e).__name__}: {e}"}

    # Every rank's figures, for the per-GPU and box-level lines.
    keys = ("h2d", "d2h", "duplex_total")
    mine = [rate["h2d"], rate["d2h"]]
    mine += [float(lp_alone[k]) if lp_alone else 0.0 for k in keys]
    mine += [float(lp_conc[k]) if lp_conc else 0.0 for k in keys]
    allr = gather_over_ranks(ws, mine)
    max_elapsed = max_over_ranks(ws, elapsed_ms)
    max_plan = max_over_ranks(ws, plan_ms)
    max_calls_wall = max_over_ranks(ws, calls_wall_s)
    max_e2e_engine = max_over_ranks(ws, e2e_engine_s)
    total_bytes = sum_over_ranks(ws, float(K * step_total))
    value = total_bytes / (max_elapsed / 1e3) / 1e9
    e2e_engine = total_bytes / max_e2e_engine / 1e9
    out = None
    if rank == 0:
        per_rank = [{"rank": r, "h2d": round(x[0], 2), "d2h": round(x[1], 2),
                     "link_alone": {k: x[2 + i] for i, k in enumerate(keys)} if lp_alone else None,
                     "link_concurrent": {k: x[5 + i] for i, k in enumerate(keys)} if lp_conc else None}
                    for r, x in enumerate(allr)]
        box_dir = {d: round(sum(x[i] for x in allr), 2) for i, d in enumerate(("h2d", "d2h"))}
        sum_alone = {k: round(sum(x[2 + i] for x in allr), 2) for i, k in enumerate(keys)} if lp_alone else None
        sum_conc = {k: round(sum(x[5 + i] for x in allr), 2) for i, k in enumerate(keys)} if lp_conc else None
        # The roofline denominator: each GPU's link measured alone (the
        # single-GPU peak), summed over the ranks; at N > 1 the peak with
        # every rank copying at once is reported beside it.
        lp = lp_alone
        if conc:
            ach = step_total / (elapsed_ms / K / 1e3) / 1e9
            peak = lp["duplex_total"] if lp else 2 * PCIE_GEN5_X16_GBS
            roof = {"bound": "pcie", "kernel": "transfer step, both directions in flight "
                    "(kv_copy_kernel + copy-engine runs), rank 0", "achieved": round(ach, 2), "peak": peak,
                    "unit": "GB/s", "frac": round(ach / peak, 4),
                    "traffic": int(sb["h2d"] * TRAFFIC_RATIO["h2d"] + sb["d2h"] * TRAFFIC_RATIO["d2h"]),
                    "traffic_unit": "DRAM bytes per step",
                    "peak_source": ("measured live: contiguous cudaMemcpyAsync both ways at once on the same "
                                    "pinned pool, this GPU alone (MEASURED_PEAKS.json has no host-link figure)"
                                    if lp else "nominal 2 x PCIe Gen5 x16"),
                    "nominal_peak": 2 * PCIE_GEN5_X16_GBS,
                    "frac_of_nominal": round(ach / (2 * PCIE_GEN5_X16_GBS), 4)}
        else:
            head = min(rate, key=rate.get)
            peak = lp[head] if lp else PCIE_GEN5_X16_GBS
            nops_head = len([o for o in S.steps[0] if o[2] == (head == "h2d")])
            roof = {"bound": "pcie", "kernel": f"transfer op {head.upper()} (kv_copy_kernel + copy-engine runs), "
                    "rank 0", "achieved": round(rate[head], 2), "peak": peak, "unit": "GB/s",
                    "frac": round(rate[head] / peak, 4),
                    "traffic": int(sb[head] * TRAFFIC_RATIO[head] / max(nops_head, 1)),
                    "traffic_unit": "DRAM bytes per op",
                    "peak_source": ("measured live: one contiguous cudaMemcpyAsync of up to 2 GiB on the same "
                                    "pinned pool, this GPU alone (MEASURED_PEAKS.json has no host-link figure)"
                                    if lp else "nominal PCIe Gen5 x16 (no live measurement in this run)"),
                    "nominal_peak": PCIE_GEN5_X16_GBS,
                    "frac_of_nominal": round(rate[head] / PCIE_GEN5_X16_GBS, 4),
                    "per_direction": {d: {"achieved": round(rate[d], 2),
                                          "peak": (lp[d] if lp else PCIE_GEN5_X16_GBS),
                                          "frac": round(rate[d] / (lp[d] if lp else PCIE_GEN5_X16_GBS), 4),
                                          "frac_of_nominal": round(rate[d] / PCIE_GEN5_X16_GBS, 4)}
                                      for d in rate if rate[d] > 0}}
        if track_kernels:
            st0 = {("h2d" if op[2] else "d2h"): p.stats() for op, p in zip(S.steps[0], plans[0])}
            roof["sm_kernel"] = {
                d: {"bytes_per_launch": st0[d]["sm_bytes"], "copy_engine_bytes_per_op": st0[d]["ce_bytes"],
                    "avg_launch_ms": round(statistics.mean(kern_ms[d]), 3),
                    "achieved_alongside_copy_engines": round(st0[d]["sm_bytes"] / statistics.mean(kern_ms[d]) / 1e6, 2)}
                for d in st0 if kern_ms[d] and statistics.mean(kern_ms[d]) > 0}
        box = {"per_direction_gbs": box_dir, "gpus": ws,
               "how": "sum over ranks of each rank's per-direction rate (device-timed, every rank running)"}
        if sum_alone:
            if conc:
                box["frac_of_n_x_single_gpu_peak"] = round(value / sum_alone["duplex_total"], 4)
            else:
                box["frac_of_n_x_single_gpu_peak"] = {d: round(box_dir[d] / sum_alone[d], 4) for d in box_dir
                                                      if sum_alone[d] > 0}
            box["n_x_single_gpu_peak"] = sum_alone
        if sum_conc:
            if conc:
                box["frac_of_concurrent_peak"] = round(value / sum_conc["duplex_total"], 4)
            else:
                box["frac_of_concurrent_peak"] = {d: round(box_dir[d] / sum_conc[d], 4) for d in box_dir
                                                  if sum_conc[d] > 0}
            box["concurrent_peak"] = sum_conc
        box["frac_of_n_x_nominal"] = ({d: round(box_dir[d] / (PCIE_GEN5_X16_GBS * ws), 4) for d in box_dir}
                                      if not conc else round(value / (2 * PCIE_GEN5_X16_GBS * ws), 4))
        nids = sum(len(g) for g, c, h in S.steps[0])
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": ws, "steps": K,
            "warmup": W, "ms_per_step": round(max_elapsed / K, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (byte copy)", "data": "synthetic",
            "config": {"workload": args.config + (" (reduced: profiling case)" if (args.batch or args.gpu_blocks) else ""),
                       "layout": layout, "mode": args.mode, "gpu_alloc": args.gpu_alloc,
                       "directions": "concurrent" if conc else "sequential",
                       "layers": cfg["layers"], "kv_heads": cfg["heads"], "head_dim": cfg["head_dim"],
                       "tokens_per_block": cfg["tpb"], "mla": S.mla, "chunk_bytes": S.chunk,
                       "ops_per_step": len(S.steps[0]), "step_bytes": sb,
                       "gpu_pool_blocks": cfg["gpu_blocks"], "cpu_pool_blocks": S.cpu_blocks,
                       "cpu_pool_blocks_requested": cfg["cpu_blocks"],
                       "cpu_pool_note": ("full size" if S.cpu_blocks >= cfg["cpu_blocks"] else
                                         "scaled to 55% of the box's available RAM over the ranks"),
                       "transfer_sms": args.transfer_sms, "parallelism": f"dp{ws} (independent)",
                       "l2": "inputs larger than L2, no flush",
                       "value_path": "c_ext.transfer_kv_blocks per op, pinned host id tensors, device-timed"},
            "per_direction_gbs": {d: round(v, 2) for d, v in rate.items() if v > 0},
            "blocks_per_s": round(value * 1e9 / S.block_bytes, 1),
            "box_roofline_frac": round(value / (PCIE_GEN5_X16_GBS * ws * (2 if conc else 1)), 4),
            "box": box,
            "per_rank": per_rank,
            "roofline": roof,
            "plan_replay": {"value": round(total_bytes / (max_plan / 1e3) / 1e9, 3), "unit": "GB/s",
                            "per_direction_gbs": {d: round(v, 2) for d, v in plan_rate.items() if v > 0},
                            "how": "the same ops from c_ext.TransferPlan objects built before the timed region"},
            "e2e": {"value": round(e2e_engine, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": int(sb["h2d"] + 16 * nids + 8 * cfg["layers"] * len(S.steps[0])),
                    "d2h_bytes_per_step": int(sb["d2h"]),
                    "how": "flexkv_b200.engine.TransferEngine: one graph per op, submit + poll, host id "
                           "tensors, wall clock (H2D and D2H ops on their own streams)",
                    "per_op_calls": round(total_bytes / max_calls_wall / 1e9, 3),
                    "per_op_calls_how": "wall clock of the value leg: flexkv_b200.c_ext.transfer_kv_blocks, one "
                                        "synchronous call per op (async per direction when the workload "
                                        "overlaps directions)"},
            "gpu_launches": int(launches), "clocks": clocks,
        }
        out.update(extras)
    for ps in plans:
        for p in ps:
            p.close()
    return out, S


class TPSetup:
    """A tensor-parallel group of R GPUs in one process:
    rank r holds heads/R of every layer on cuda:r, and moves its slice to
    byte offset r*gpu_chunk of every chunk of one shared BLOCKWISE host pool
    that holds all heads.  stock=True registers the pool as FlexKV's worker
    does (Setup's docstring) and imports nothing of flexkv_b200."""

    def __init__(self, cfg: dict, R: int, cpu_blocks_override: int = 0, stock: bool = False):
        self.cfg, self.R, self.stock = cfg, R, stock
        L, H, D, tpb = cfg["layers"], cfg["heads"], cfg["head_dim"], cfg["tpb"]
        if H % R:
            raise ValueError(f"{H} KV heads do not divide over {R} ranks")
        e = 2
        g = kv_strides("LAYERWISE", 1, cfg["gpu_blocks"], tpb, H // R, D, False)  # one layer, H/R heads
        self.g_kv, self.g_blk = g["kv"] * e, g["block"] * e
        self.g_chunk = g["chunk"] * e
        self.gpu_layer_bytes = g["total"] * e
        self.block_bytes = L * 2 * tpb * H * D * e  # all heads: the host chunk
        fit = int(0.55 * mem_available_bytes() / self.block_bytes)
        cpu_blocks = cpu_blocks_override or min(cfg["cpu_blocks"], max(fit, 2 * cfg["batch"]))
        self.cpu_blocks = cpu_blocks
        c = kv_strides("BLOCKWISE", L, cpu_blocks, tpb, H, D, False)
        self.c_kv, self.c_layer, self.c_blk = c["kv"] * e, c["layer"] * e, c["block"] * e
        self.c_chunk = c["chunk"] * e
        self.layers = []
        for r in range(R):
            dev = torch.device(f"cuda:{r}")
            base = torch.empty((L, 2, cfg["gpu_blocks"], tpb, H // R, D), dtype=torch.bfloat16, device=dev)
            base.normal_()
            self.layers.append([base[l] for l in range(L)])
        self.cpu = torch.empty(c["total"], dtype=torch.bfloat16)
        if stock:
            stock_host_register(self.cpu)
        else:
            from flexkv_b200 import c_ext
            c_ext.cudaHostRegister(self.cpu, advise_hugepages=True)
        log(f"[tp{R}] gpu pool {L} layers x {R} ranks, cpu pool {self.cpu.numel() * 2 / 2**30:.1f} GiB"
            + (" (stock registration)" if stock else ""))
        self.steps = []
        for s_ in range(4):
            ops = []
            for j, h2d in enumerate((True, False)):
                g_, c_ = make_batch(cfg["batch"], cfg["gpu_blocks"], cpu_blocks, 10 * s_ + j, 0.0, 1)
                ops.append((g_, c_, h2d))
            self.steps.append(ops)
        self.step_bytes = {"h2d": cfg["batch"] * self.block_bytes, "d2h": cfg["batch"] * self.block_bytes}

    @property
    def gpu_layout(self):
        """flexkv_b200's KVCacheLayout of one rank's GPU pool (our arm only)."""
        from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
        c = self.cfg
        return KVCacheLayout(KVCacheLayoutType.LAYERWISE, c["layers"], c["gpu_blocks"], c["tpb"], c["heads"],
                             c["head_dim"]).div_head(self.R)

    @property
    def cpu_layout(self):
        from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
        c = self.cfg
        return KVCacheLayout(KVCacheLayoutType.BLOCKWISE, c["layers"], self.cpu_blocks, c["tpb"], c["heads"],
                             c["head_dim"])

    def close(self):
        if self.stock:
            stock_host_unregister(self.cpu)
        else:
            from flexkv_b200 import c_ext
            c_ext.cudaHostUnregister(self.cpu)


def run_tp(args, cfg, R):
    """cfg3: one op = every rank moving its head slice of a 512-block batch;
    value = device time (CUDA events on each rank's stream, max over ranks),
    e2e = the same steps through the engine (one TP group of R GPUs)."""
    from flexkv_b200 import c_ext
    from flexkv_b200.engine import TransferDescriptor, TransferEngine, TransferOp, TransferOpGraph, TransferType
    S = TPSetup(cfg, R, args.cpu_blocks)
    K, W = args.steps, args.warmup
    streams = [torch.cuda.Stream(device=r) for r in range(R)]
    plans = [[[c_ext.TransferPlan(torch.from_numpy(g), torch.tensor([t.data_ptr() for t in S.layers[r]]),
                                  S.g_kv, S.g_blk, torch.from_numpy(c), S.cpu, S.c_kv, S.c_layer, S.c_blk,
                                  S.g_chunk, 0, args.transfer_sms, h2d, False, False,
                                  cpu_startoff_inside_chunks=r * S.g_chunk, device=r)
               for r in range(R)] for g, c, h2d in ops] for ops in S.steps]

    def step(k, evs=None):
        for oi, per_rank in enumerate(plans[k % 4]):
            for r, p in enumerate(per_rank):
                with torch.cuda.device(r):
                    if evs is not None:
                        evs[r][2 * oi].record(streams[r])
                    p.execute(stream=streams[r])
                    if evs is not None:
                        evs[r][2 * oi + 1].record(streams[r])
            for r in range(R):
                streams[r].synchronize()  # the reference's group joins every op

    for k in range(W):
        step(k)
    rec = []
    for k in range(K):
        evs = []
        for r in range(R):
            with torch.cuda.device(r):
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
                for e_ in ev:
                    e_.record(streams[r])
                evs.append(ev)
        rec.append(evs)
    for r in range(R):
        torch.cuda.synchronize(r)
    sampler = ClockSampler(0)
    with sampler:
        for k in range(K):
            step(W + k, rec[k])
        for r in range(R):
            torch.cuda.synchronize(r)
        eng = TransferEngine(S.layers, S.cpu, S.gpu_layout, S.cpu_layout, tp_size=R)
        try:
            def estep(k):
                ids = []
                for g, c, h2d in S.steps[k % 4]:
                    gr = TransferOpGraph()
                    src, dst = (c, g) if h2d else (g, c)
                    gr.add_transfer_op(TransferOp(graph_id=gr.graph_id,
                                                  transfer_type=TransferType.H2D if h2d else TransferType.D2H,
                                                  src_descriptor=TransferDescriptor(torch.from_numpy(src)),
                                                  dst_descriptor=TransferDescriptor(torch.from_numpy(dst))))
                    eng.submit_transfer_graph(gr)
                    ids.append(gr.graph_id)
                left = set(ids)
                while left:
                    for gid, oid in eng.get_completed_graphs_and_ops(timeout=0.01):
                        if oid == -1:
                            left.discard(gid)
            for k in range(W):
                estep(k)
            t0 = time.perf_counter()
            for k in range(K):
                estep(W + k)
            e2e_s = time.perf_counter() - t0
            failed = dict(eng.failed_ops)
        finally:
            eng.shutdown()
    if failed:
        raise RuntimeError(f"engine ops failed: {failed}")
    per = {"h2d": [], "d2h": []}
    for k in range(K):
        for oi, d in enumerate(("h2d", "d2h")):
            per[d].append(max(rec[k][r][2 * oi].elapsed_time(rec[k][r][2 * oi + 1]) for r in range(R)))
    sb = S.step_bytes
    rate = {d: sb[d] / (statistics.mean(per[d]) / 1e3) / 1e9 for d in per}
    step_ms = statistics.mean([per["h2d"][k] + per["d2h"][k] for k in range(K)])
    value = (sb["h2d"] + sb["d2h"]) / (step_ms / 1e3) / 1e9
    e2e = K * (sb["h2d"] + sb["d2h"]) / e2e_s / 1e9
    head = min(rate, key=rate.get)
    out = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": R, "steps": K, "warmup": W,
        "ms_per_step": round(step_ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (byte copy)", "data": "synthetic",
        "config": {"workload": args.config, "tp": R, "layout": "BLOCKWISE", "layers": cfg["layers"],
                   "kv_heads_total": cfg["heads"], "heads_per_rank": cfg["heads"] // R,
                   "head_dim": cfg["head_dim"], "tokens_per_block": cfg["tpb"],
                   "gpu_chunk_bytes": S.g_chunk, "cpu_chunk_bytes": S.c_chunk, "batch_blocks": cfg["batch"],
                   "gpu_pool_blocks": cfg["gpu_blocks"], "cpu_pool_blocks": S.cpu_blocks,
                   "cpu_pool_blocks_requested": cfg["cpu_blocks"], "parallelism": f"tp{R} (one process)",
                   "directions": "sequential per op (each op joins all ranks, as the reference group)"},
        "per_direction_gbs": {d: round(v, 2) for d, v in rate.items()},
        "box_roofline_frac": round(value / (PCIE_GEN5_X16_GBS * R), 4),
        "roofline": {"bound": "pcie", "kernel": f"tp transfer op {head.upper()} (all ranks)",
                     "achieved": round(rate[head], 2), "peak": PCIE_GEN5_X16_GBS * R, "unit": "GB/s",
                     "frac": round(rate[head] / (PCIE_GEN5_X16_GBS * R), 4), "traffic": None,
                     "peak_source": "nominal PCIe Gen5 x16 per GPU x ranks"},
        "e2e": {"value": round(e2e, 3), "unit": "GB/s", "h2d_bytes_per_step": int(sb["h2d"]),
                "d2h_bytes_per_step": int(sb["d2h"]),
                "how": "flexkv_b200.engine.TransferEngine over the TP group, one graph per op"},
        "clocks": sampler.summary(),
    }
    for ops in plans:
        for per_rank in ops:
            for p in per_rank:
                p.close()
    return out, S


def run_tp_reference(args, cfg, R):
    """The reference's group transfer: one host thread per rank, each running
    its transfer.cu on the rank's device and stream with the rank's byte
    offset inside the host chunk, then a join (tp_transfer_thread_group.cpp
    :48-109), driven one op at a time."""
    from oracle import oracle as O
    if not O.reference_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libref_transfer.so not built"}, None
    S = TPSetup(cfg, R, args.cpu_blocks, stock=True)
    ref = O.ref_lib()
    ptrs = [torch.tensor([t.data_ptr() for t in S.layers[r]], dtype=torch.int64).pin_memory() for r in range(R)]
    host_ops = [[(torch.from_numpy(g).pin_memory(), torch.from_numpy(c).pin_memory(), h)
                 for g, c, h in ops] for ops in S.steps]
    streams = [torch.cuda.Stream(device=r) for r in range(R)]
    errors = []

    def rank_call(r, g, c, h2d):
        torch.cuda.set_device(r)
        rc = ref.ref_transfer_kv_blocks(len(g), 0, cfg["layers"], g.data_ptr(), ptrs[r].data_ptr(), S.g_kv,
                                        S.g_blk, c.data_ptr(), S.cpu.data_ptr(), S.c_kv, S.c_layer, S.c_blk,
                                        r * S.g_chunk, S.g_chunk, streams[r].cuda_stream, 8, int(h2d), 0, 0)
        if rc != 0:
            errors.append(rc)

    def group(g, c, h2d):
        ths = [threading.Thread(target=rank_call, args=(r, g, c, h2d)) for r in range(R)]
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        if errors:
            raise RuntimeError(f"reference transfer CUDA error {errors[0]}")

    K, W = args.steps, args.warmup
    for k in range(W):
        for g, c, h in host_ops[k % 4]:
            group(g, c, h)
    per = {"h2d": 0.0, "d2h": 0.0}
    t0 = time.perf_counter()
    for k in range(K):
        for g, c, h in host_ops[(W + k) % 4]:
            a = time.perf_counter()
            group(g, c, h)
            per["h2d" if h else "d2h"] += time.perf_counter() - a
    dt = time.perf_counter() - t0
    sb = S.step_bytes
    value = K * (sb["h2d"] + sb["d2h"]) / dt / 1e9
    out = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": R,
           "steps": K, "warmup": W, "ms_per_step": round(dt / K * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (byte copy)", "data": "synthetic",
           "config": {"workload": args.config, "tp": R, "transfer_sms": 8, "cpu_pool_blocks": S.cpu_blocks},
           "per_direction_gbs": {d: round(K * sb[d] / per[d] / 1e9, 2) for d in per},
           "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": R, "kind": "reference",
                            "sample": "the reference's transfer.cu per rank from one host thread per rank "
                                      "(its TP thread group's structure), full steps"},
           "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return out, S


def cpu_baseline(S, seconds: float = 8.0):
    """The oracle (oracle/oracle.c, the CPU restatement of the reference copy)
    gathering/scattering a 256-block sample of the same workload on host
    memory with every host core."""
    from oracle import oracle as O
    cfg = S.cfg
    n = 256
    g, c = make_batch(n, 512, S.cpu_blocks, 77, cfg["run_frac"], cfg["max_run"], cfg.get("fixed_run", False))
    layer_bytes = S.gpu_layer_bytes * 512 // cfg["gpu_blocks"]
    imgs = [np.empty(layer_bytes, dtype=np.uint8) for _ in range(cfg["layers"])]
    cpu = S.cpu.view(torch.uint8).numpy()
    threads = len(os.sched_getaffinity(0))
    g_kv = S.g_kv * 512 // cfg["gpu_blocks"]
    moved, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for h2d in (True, False):
            O.transfer(n, 0, g, imgs, g_kv, S.g_blk, c, cpu, S.c_kv, S.c_layer, S.c_blk, 0,
                       S.chunk, h2d, S.mla, num_threads=threads)
            moved += n * S.block_bytes
    dt = max(time.perf_counter() - t0, 1e-9)
    return {"value": round(moved / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n}-block {S.cpu_layout.type.value} gather+scatter between the host pool and "
                      f"host images of the GPU layers, repeated for {dt:.1f}s"}


def run_reference(args, ws, rank, local, cfg, layout):
    """The reference's transfer.cu (oracle/_ref) the way its worker calls it:
    one op at a time, synchronous, transfer_sms=8, pinned ids."""
    from oracle import oracle as O
    if not O.reference_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libref_transfer.so not built "
                "(needs the reference tree at build time)"}, None
    S = Setup(cfg, layout, 1, local, args.cpu_blocks, args.gpu_alloc, stock=True)
    ref = O.ref_lib()
    ptrs = S.ptrs.pin_memory()
    host_ops = [[(torch.from_numpy(g).pin_memory(), torch.from_numpy(c).pin_memory(), h)
                 for g, c, h in ops] for ops in S.steps]
    stream = torch.cuda.current_stream().cuda_stream
    sms = 8  # flexkv/common/config.py:50-51 worker default

    def call(g, c, h2d, use_ce=False):
        rc = ref.ref_transfer_kv_blocks(len(g), 0, len(S.layers), g.data_ptr(), ptrs.data_ptr(),
                                        S.g_kv, S.g_blk, c.data_ptr(), S.cpu.data_ptr(), S.c_kv,
                                        S.c_layer, S.c_blk, 0, S.chunk, stream, sms, int(h2d),
                                        int(use_ce), int(S.mla))
        if rc != 0:
            raise RuntimeError(f"reference transfer_kv_blocks CUDA error {rc}")

    K, W = args.steps, args.warmup
    for k in range(W):
        for g, c, h in host_ops[k % len(host_ops)]:
            call(g, c, h)
    sampler = ClockSampler(local)
    per = {"h2d": 0.0, "d2h": 0.0}
    with sampler:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for k in range(K):
            for g, c, h in host_ops[(W + k) % len(host_ops)]:
                a = time.perf_counter()
                call(g, c, h)
                per["h2d" if h else "d2h"] += time.perf_counter() - a
        dt = time.perf_counter() - t0
        # CE mode (one cudaMemcpyAsync per chunk), one step
        a = time.perf_counter()
        for g, c, h in host_ops[0]:
            call(g, c, h, use_ce=True)
        ce_dt = time.perf_counter() - a
    sb = S.step_bytes
    step_total = sb["h2d"] + sb["d2h"]
    value = K * step_total / dt / 1e9
    out = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": ws,
        "steps": K, "warmup": W, "ms_per_step": round(dt / K * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (byte copy)", "data": "synthetic",
        "config": {"workload": args.config, "layout": layout, "transfer_sms": sms,
                   "gpu_alloc": args.gpu_alloc,
                   "directions": "sequential (one op at a time, as the reference worker)",
                   "ops_per_step": len(S.steps[0]), "step_bytes": sb, "cpu_pool_blocks": S.cpu_blocks,
                   "parallelism": "rank 0 only"},
        "per_direction_gbs": {d: round(K * sb[d] / per[d] / 1e9, 2) for d in per if per[d] > 0},
        "ce_mode": {"value": round(step_total / ce_dt / 1e9, 3), "unit": "GB/s",
                    "how": "use_ce_transfer=True: one cudaMemcpyAsync per (layer,kv,block) chunk, one step"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": 1, "kind": "reference",
                         "sample": "the reference's transfer.cu kernel (transfer_sms=8) driven from one "
                                   "host thread with pinned ids, synchronous per op, full steps"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "clocks": sampler.summary(),
    }
    return out, S


SPLIT_VARIANTS = [
    # (label, SM budget, copy-engine threshold per (layer,kv) row or None = default, loads in flight, ce-only)
    ("sm_only_2sms", 2, 0, 16, False),
    ("sm_only_8sms", 8, 0, 16, False),
    ("sm_only_16sms", 16, 0, 16, False),
    ("hybrid_4sms_256k", 4, 256 << 10, 16, False),
    ("hybrid_4sms_1m", 4, 1 << 20, 16, False),
    ("hybrid_8sms_1m", 8, 1 << 20, 16, False),
    ("hybrid_16sms_1m", 16, 1 << 20, 16, False),
    ("hybrid_16sms_1m_unroll8", 16, 1 << 20, 8, False),
    ("copy_engines_only", -1, None, 16, True),
]


def split_sweep(args, ws, rank, local, cfg, layout):
    """The split between copy-engine runs and the SM kernel, measured: each
    variant's plans are built once, then every variant is timed in turn for
    three rounds (interleaved, so box drift hits all alike); each direction
    alone and both in flight together; with N ranks every rank runs each
    timing at once (barrier before each).  Also the host link's contiguous
    cudaMemcpyAsync peak and the bound the batch pattern allows: its joint
    runs at that peak and the rest at the best measured rate for single
    blocks.  One JSON line (rank 0); per-rank figures at N > 1."""
    from flexkv_b200 import c_ext
    if cfg["kind"] != "batch":
        raise SystemExit("--split-sweep runs on the batch workloads (cfg2_llama3_8b, cfg5_dsv3_mla)")
    S = Setup(cfg, layout, ws, local, args.cpu_blocks, args.gpu_alloc)
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    variants = SPLIT_VARIANTS
    plans = {}
    for label, sms, thr, unroll, ce_only in variants:
        os.environ["FKV_UNROLL"] = str(unroll)
        try:
            kw = {} if thr is None else {"ce_min_run_bytes": thr}
            plans[label] = [[c_ext.TransferPlan(torch.from_numpy(g), S.ptrs, S.g_kv, S.g_blk, torch.from_numpy(c),
                                                S.cpu, S.c_kv, S.c_layer, S.c_blk, S.chunk, 0, sms, h2d, ce_only,
                                                S.mla, gpu_layer_bytes=S.gpu_layer_bytes, **kw)
                             for g, c, h2d in ops] for ops in S.steps]
        finally:
            os.environ.pop("FKV_UNROLL", None)
    stats = {label: plans[label][0][0].stats() for label, *_ in variants}

    def timed(fn):
        barrier(ws)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    res = {label: {"h2d": [], "d2h": [], "duplex": []} for label, *_ in variants}
    for label in plans:  # warm-up
        for ops in plans[label]:
            for p in ops:
                p.execute(stream=stream)
    torch.cuda.synchronize()
    for _ in range(3):
        for label in plans:
            for s, ops in enumerate(plans[label]):
                for (g, c, h2d), p in zip(S.steps[s], ops):
                    ms = timed(lambda: p.execute(stream=stream))
                    res[label]["h2d" if h2d else "d2h"].append(len(g) * S.block_bytes / ms / 1e6)

                def both():
                    e = torch.cuda.Event()
                    e.record(stream)
                    side.wait_event(e)
                    ops[0].execute(stream=stream)
                    ops[1].execute(stream=side)
                    j = torch.cuda.Event()
                    j.record(side)
                    stream.wait_event(j)
                res[label]["duplex"].append(sum(S.step_bytes.values()) / timed(both) / 1e6)
    for label in plans:
        for ops in plans[label]:
            for p in ops:
                p.close()
    lp = measure_link_peaks(S, stream, sync=lambda: barrier(ws))
    mine = [statistics.median(res[label][d]) for label, *_ in variants for d in ("h2d", "d2h", "duplex")]
    mine += [lp["h2d"], lp["d2h"], lp["duplex_total"]]
    allr = gather_over_ranks(ws, mine)
    out = None
    if rank == 0:
        keys = [(label, d) for label, *_ in variants for d in ("h2d", "d2h", "duplex")]
        table = {}
        for i, (label, d) in enumerate(keys):
            vals = [round(x[i], 2) for x in allr]
            table.setdefault(label, {})[d] = vals[0] if ws == 1 else {"per_rank": vals, "box": round(sum(vals), 2)}
        for label, sms, thr, unroll, ce_only in variants:
            table[label].update(sm_budget=sms, ce_min_run_bytes=thr, unroll=unroll, copy_engines_only=ce_only,
                                ce_fraction_h2d=round(stats[label]["ce_bytes"] /
                                                      max(1, stats[label]["ce_bytes"] + stats[label]["sm_bytes"]), 3),
                                ce_copies_h2d=stats[label]["ce_copies"])
        lk = [[round(x[-3], 2), round(x[-2], 2), round(x[-1], 2)] for x in allr]
        run_frac = max(stats[label]["ce_bytes"] / max(1, stats[label]["ce_bytes"] + stats[label]["sm_bytes"])
                       for label, *_ in variants if not label.startswith("copy"))
        r0 = lambda label, d: table[label][d] if ws == 1 else table[label][d]["per_rank"][0]  # noqa: E731
        single = {d: max(r0(label, d) for label, *_ in variants if label.startswith("sm_only"))
                  for d in ("h2d", "d2h")}
        bound = {d: round(1.0 / (run_frac / lk[0][i] + (1 - run_frac) / single[d]), 2)
                 for i, d in enumerate(("h2d", "d2h"))}
        best = {d: max(r0(label, d) for label, *_ in variants) for d in ("h2d", "d2h", "duplex")}
        out = {"split_sweep": table, "workload": args.config, "layout": layout, "gpu_alloc": args.gpu_alloc,
               "n_gpus": ws, "cpu_pool_blocks": S.cpu_blocks,
               "link_contiguous_copy": {"per_rank": lk, "how": "one contiguous cudaMemcpyAsync of up to 2 GiB "
                                        "each way and both at once, every rank at once, median of 3"},
               "pattern_bound": {"gbs": bound, "run_fraction_of_bytes": round(run_frac, 3),
                                 "single_block_rate": single,
                                 "how": "the batch's joint runs at the contiguous-copy peak and the rest at the "
                                        "best SM-only rate, rank 0"},
               "best_measured": best, "best_over_bound": {d: round(best[d] / bound[d], 4) for d in bound},
               "how": "plans built once per variant, three interleaved rounds over the four steps, median; "
                      "device time (CUDA events); duplex = the step's H2D and D2H batch in flight together"}
    S.close()
    return out


def claim_stdout():
    """Keep stdout for the one JSON line: everything else written to file
    descriptor 1 from here on (NCCL's version banner, library notices) goes
    to stderr.  Returns the stream the JSON line is printed on."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    return os.fdopen(saved, "w")


def main():
    out_stream = claim_stdout()
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2_llama3_8b")
    ap.add_argument("--layout", choices=["LAYERWISE", "BLOCKWISE"], default=None,
                    help="host pool layout (default: the configuration's)")
    ap.add_argument("--mode", choices=["auto", "sm", "ce", "hybrid"], default="auto")
    ap.add_argument("--ce-min-run-bytes", type=int, default=1 << 20)
    ap.add_argument("--transfer-sms", type=int, default=-1)
    ap.add_argument("--gpu-alloc", choices=["per-layer", "contiguous"], default="per-layer",
                    help="GPU KV pool as one tensor per layer, or one allocation viewed per layer")
    ap.add_argument("--cpu-blocks", type=int, default=0, help="override the CPU pool size")
    ap.add_argument("--cpu-baseline-seconds", type=float, default=8.0)
    ap.add_argument("--batch", type=int, default=0, help="override blocks per batch (profiling case)")
    ap.add_argument("--gpu-blocks", type=int, default=0, help="override the GPU pool size")
    ap.add_argument("--hash-only", action="store_true",
                    help="only the XXH64 block-hash measurement (one JSON line)")
    ap.add_argument("--ssd-only", action="store_true",
                    help="only the SSD-tier measurement (one JSON line)")
    ap.add_argument("--put-only", action="store_true",
                    help="only the CPU-tier put-path measurement (one JSON line; --config picks the shape)")
    ap.add_argument("--tp", type=int, default=0,
                    help="TP ranks for cfg3 (one process drives them; default: all visible GPUs)")
    ap.add_argument("--split-sweep", action="store_true",
                    help="time the copy-engine/SM split variants on the --config batch workload (one JSON line; "
                         "under torchrun every rank at once)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the link-peak, duplex and hash measurements (profiling runs)")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3
    if args.hash_only:
        torch.cuda.set_device(0)
        print(json.dumps({"hash": measure_hash()}), file=out_stream, flush=True)
        return
    if args.ssd_only:
        print(json.dumps({"ssd": measure_ssd()}), file=out_stream, flush=True)
        return
    if args.put_only:
        torch.cuda.set_device(0)
        cfg = dict(CONFIGS[args.config])
        S = Setup(cfg, args.layout or cfg["layout"], 1, 0, args.cpu_blocks, args.gpu_alloc)
        try:
            print(json.dumps({"put_path": dict(measure_put_path(S), workload=args.config)}), file=out_stream, flush=True)
        finally:
            S.close()
        return
    if args.split_sweep:
        ws, rank, local = dist_setup()
        cfg = dict(CONFIGS[args.config])
        out = split_sweep(args, ws, rank, local, cfg, args.layout or cfg["layout"])
        if rank == 0:
            print(json.dumps(out), file=out_stream, flush=True)
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
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
    layout = args.layout or cfg["layout"]
    with_hash = args.config == "cfg2_llama3_8b" and not (args.batch or args.gpu_blocks)
    if cfg["kind"] == "tp":
        R = args.tp or torch.cuda.device_count()
        out, S = (run_tp_reference if args.impl == "reference" else run_tp)(args, cfg, R)
        if out is not None and args.impl != "reference":
            out["cpu_baseline"] = None
    elif args.impl == "reference":
        out, S = run_reference(args, ws, rank, local, cfg, layout)
    else:
        out, S = run_ours(args, ws, rank, local, cfg, layout, with_hash)
        if rank == 0 and ws == 1:
            out["cpu_baseline"] = cpu_baseline(S, args.cpu_baseline_seconds)
        elif rank == 0:
            out["cpu_baseline"] = None
    if S is not None:
        S.close()
    if rank == 0 and out is not None:
        print(json.dumps(out), file=out_stream, flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
