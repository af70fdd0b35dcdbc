"""CPU: the benchmark's own host logic.

* The reference arm builds its pools without flexkv_b200, from the bench's
  own stride arithmetic (bench.kv_strides); those strides must equal the
  reference's KVCacheLayout for every benchmark configuration, host layout
  and TP degree (tests/golden/layouts.json, made from the reference's class).
* Batches: the joint-run share, distinct ids on both sides, and per-rank
  seeds that give every data-parallel rank its own blocks.
* The host-pool fit: the configured pool when RAM allows, scaled over the
  ranks otherwise, never below two batches.
"""
import json
import os

import numpy as np
import pytest

import bench

LAYOUTS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "layouts.json")))


@pytest.mark.parametrize("key", sorted(LAYOUTS))
def test_stock_strides_equal_the_reference_layout(key):
    g = LAYOUTS[key]
    if "/cpu/" in key:
        kind, L, N, tpb, H, D, mla = g["args"]
        st = bench.kv_strides(kind, L, N, tpb, H, D, mla)
        assert (st["layer"], st["kv"], st["block"], st["chunk"], st["total"]) == \
            (g["layer_stride"], g["kv_stride"], g["block_stride"], g["chunk"], g["total"])
    else:
        kind, L, N, tpb, H, D, mla, tp = g["args"]
        heads = H if mla else H // tp
        st = bench.kv_strides("LAYERWISE", 1, N, tpb, heads, D, mla)  # one layer of one rank
        assert (st["kv"], st["block"], st["chunk"], st["total"]) == \
            (g["kv_stride"], g["block_stride"], g["chunk"], g["total_per_layer"])


@pytest.mark.parametrize("run_frac,max_run,fixed", [(0.5, 64, False), (0.5, 128, True), (0.0, 1, False)])
def test_batches_have_the_run_share_and_distinct_ids(run_frac, max_run, fixed):
    n, gpool, cpool = 2048, 16384, 32768
    g, c = bench.make_batch(n, gpool, cpool, 7, run_frac, max_run, fixed)
    assert len(g) == len(c) == n
    assert len(set(g.tolist())) == n and len(set(c.tolist())) == n
    assert g.min() >= 0 and g.max() < gpool and c.min() >= 0 and c.max() < cpool
    joint = np.flatnonzero((np.diff(g) == 1) & (np.diff(c) == 1))
    in_runs = len(set(joint.tolist()) | set((joint + 1).tolist()))
    assert in_runs <= int(round(n * run_frac)) + 1
    if run_frac == 0:
        assert in_runs <= n // 100  # scattered singletons only touch by chance


def test_every_rank_draws_its_own_blocks():
    cfg = dict(bench.CONFIGS["cfg2_llama3_8b"])
    a = bench.rank_steps(cfg, cfg["cpu_blocks"], 0, nsteps=2)
    b = bench.rank_steps(cfg, cfg["cpu_blocks"], 1, nsteps=2)
    for sa, sb in zip(a, b):
        for (ga, ca, ha), (gb, cb, hb) in zip(sa, sb):
            assert ha == hb and not np.array_equal(ga, gb)
    assert [h for _, _, h in a[0]] == [True, False]  # one H2D and one D2H batch per step


def test_host_pool_fit(monkeypatch):
    cfg = dict(bench.CONFIGS["cfg2_llama3_8b"])
    block = 2 << 20
    monkeypatch.setattr(bench, "mem_available_bytes", lambda: 1 << 40)
    assert bench.fit_cpu_blocks(cfg, 1, block) == cfg["cpu_blocks"]
    assert bench.fit_cpu_blocks(cfg, 32, block) == int(0.55 * (1 << 40) / 32 / block)  # scaled over the ranks
    monkeypatch.setattr(bench, "mem_available_bytes", lambda: 1 << 30)
    assert bench.fit_cpu_blocks(cfg, 8, block) == 2 * cfg["batch"]  # never below two batches
    assert bench.fit_cpu_blocks(cfg, 8, block, override=1234) == 1234
