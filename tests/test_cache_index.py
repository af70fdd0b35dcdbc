"""The CPU restatement of the CPU-tier index, put and get decisions
(oracle/cache_index.py) against the reference's own GlobalCacheEngine,
through the fixture tests/golden/put_path.json (made by
tests/golden/make_put_golden.py)."""
import json
import os

import numpy as np
import pytest

from oracle import cache_index as CI

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "put_path.json")


def scenarios():
    with open(GOLDEN) as f:
        return json.load(f)["scenarios"]


def replay(sc):
    """Run a golden scenario through the oracle; yield (kind, got, want)."""
    if sc.get("num_ssd_blocks", 0):
        yield from replay_two_tier(sc)
        return
    tier = CI.CpuTier(sc["num_cpu_blocks"], sc["tpb"])
    for b, batch in enumerate(sc["batches"]):
        results = []
        for req, want in zip(batch, sc["results"][b]):
            r = tier.put(np.array(req["tokens"], dtype=np.int64), np.array(req["gpu_blocks"], dtype=np.int64))
            results.append(r)
            yield "put", (r.num_skipped, r.num_transferred, r.gpu_blocks.tolist(), r.cpu_blocks.tolist()), \
                (want["skipped"], want["transferred"], want["gpu_blocks"], want["cpu_blocks"])
        if sc["complete_each_batch"]:
            for r in results:
                tier.complete(r)
        for p in sc["probes"][b]:
            m = tier.match(np.array(p["tokens"], dtype=np.int64))
            yield "probe", (m.num_matched, m.num_ready, m.blocks[:m.num_matched]), \
                (p["num_matched"], p["num_ready"], p["blocks"])
        for g in sc["gets"][b]:
            r = tier.get(np.array(g["tokens"], dtype=np.int64), np.array(g["gpu_blocks"], dtype=np.int64),
                         g["block_start"])
            start = r.num_skipped if r.num_transferred else 0
            yield "get", (start, r.num_transferred, r.gpu_blocks.tolist(), r.cpu_blocks.tolist()), \
                (g["mask_start"], g["transferred"], g["copied_gpu_blocks"], g["copied_cpu_blocks"])
        yield "totals", (tier.pool.num_free, tier.tree.total_blocks(), tier.tree.total_ready()), \
            (sc["num_free"][b], sc["total_cached"][b], sc["total_ready"][b])


def replay_two_tier(sc):
    """The scenarios with the SSD tier on: each put's D2H and H2DISK ops,
    each get's ops, and both tiers' totals."""
    tt = CI.TwoTier(sc["num_cpu_blocks"], sc["num_ssd_blocks"], sc["tpb"])
    for b, batch in enumerate(sc["batches"]):
        results = []
        for req, want in zip(batch, sc["results"][b]):
            r = tt.put(np.array(req["tokens"], dtype=np.int64), np.array(req["gpu_blocks"], dtype=np.int64))
            results.append(r)
            ops = []
            if r.num_transferred:
                ops.append(["D2H", r.gpu_blocks.tolist(), r.cpu_blocks.tolist()])
                if len(r.ssd_blocks):
                    ops.append(["H2DISK", r.h2disk_cpu.tolist(), r.ssd_blocks.tolist()])
            yield "put", (r.num_skipped, r.num_transferred, ops), (want["skipped"], want["transferred"], want["ops"])
        if sc["complete_each_batch"]:
            for r in results:
                tt.complete(r)
        for p in sc["probes"][b]:
            m = tt.cpu.match(np.array(p["tokens"], dtype=np.int64))
            yield "probe", (m.num_matched, m.num_ready, m.blocks[:m.num_matched]), \
                (p["num_matched"], p["num_ready"], p["blocks"])
        for g in sc["gets"][b]:
            n, ops = tt.get(np.array(g["tokens"], dtype=np.int64), np.array(g["gpu_blocks"], dtype=np.int64),
                            g["block_start"])
            got = [[k, src.tolist(), dst.tolist() if dst is not None else None] for k, src, dst in ops]
            want_ops = [[k, src, dst] for k, src, dst in g["ops"]]
            yield "get", (n, got), (g["transferred"], want_ops)
        yield "totals", (tt.cpu.pool.num_free, tt.cpu.tree.total_blocks(), tt.cpu.tree.total_ready(),
                         tt.ssd.pool.num_free, tt.ssd.tree.total_blocks()), \
            (sc["num_free"][b], sc["total_cached"][b], sc["total_ready"][b], sc["ssd_num_free"][b],
             sc["ssd_total_cached"][b])


@pytest.mark.parametrize("name", [s["name"] for s in scenarios()])
def test_oracle_matches_reference_put_path(name):
    sc = next(s for s in scenarios() if s["name"] == name)
    n = 0
    for kind, got, want in replay(sc):
        assert got == tuple(want), f"{name}: {kind} #{n}: got {got}, want {want}"
        n += 1
    assert n > 0


def test_golden_covers_the_edge_cases():
    scs = {s["name"]: s for s in scenarios()}
    res = [r for s in scs.values() for b in s["results"] for r in b]
    assert any(r["transferred"] == 0 for r in res)                       # empty puts
    assert any(r["skipped"] > 0 and r["transferred"] > 0 for r in res)   # partial prefix hits
    full = [r for b in scs["pool_full"]["results"] for r in b]
    assert scs["pool_full"]["num_free"][-1] == 0 and sum(r["transferred"] == 0 for r in full) > 5
    assert all(t == 0 for t in scs["callbacks_deferred"]["total_ready"])
    gets = [g for s in scs.values() for b in s["gets"] for g in b]
    assert any(g["transferred"] > 0 and g["block_start"] > 0 for g in gets)  # mid-sequence reads
    assert any(g["transferred"] == 0 for g in gets)                          # nothing ready
    tokens = [len(q["tokens"]) for s in scs.values() for b in s["batches"] for q in b]
    assert min(tokens) < 4  # a request shorter than one block


def test_pool_refreshes_its_snapshot_only_when_short():
    """mempool.py:28-55: recycled ids wait until the snapshot runs out."""
    p = CI.BlockPool(8)
    a = p.allocate(3)
    assert a.tolist() == [0, 1, 2]
    p.recycle(np.array([1]))
    assert p.allocate(4).tolist() == [3, 4, 5, 6]
    assert p.allocate(2).tolist() == [1, 7]  # 2 > 1 left in the snapshot: refresh
    p.recycle(np.array([0]))
    with pytest.raises(ValueError):
        p.recycle(np.array([0]))  # already free
