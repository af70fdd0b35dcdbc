"""GPU tests of the CPU tier's device index and fused put / get paths
(flexkv_b200.cache_index over csrc/block_index.cu):

* the reference's own put and get results (tests/golden/put_path.json, made
  by running its GlobalCacheEngine): per-put outcomes and D2H block lists,
  per-get H2D block lists and return masks, match results of probe
  sequences, pool and index totals;
* the CPU restatement (oracle/cache_index.py) on large random batches;
* the bytes the put copied (oracle transfer);
* the pool's id order under take / recycle (Mempool restatement);
* the caller's eviction (remove + recycle) and the error paths.
"""
import json
import os

import numpy as np
import pytest
import torch

from flexkv_b200 import c_ext
from flexkv_b200._lib import FKV_ERR_INVALID_ARG, FKV_ERR_OUT_OF_RANGE, FlexKVError
from flexkv_b200.cache_index import CpuCacheIndex, KVLayout
from gpu_util import oracle_transfer
from kvcase import Case, fill_bytes
from oracle import cache_index as CI

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "put_path.json")


def golden():
    with open(GOLDEN) as f:
        return {s["name"]: s for s in json.load(f)["scenarios"]}


class Pools:
    """GPU layers and the pinned CPU pool of a case, with host images that
    the oracle transfer updates alongside."""

    def __init__(self, case: Case, seed: int = 7):
        st = case.strides()
        self.case, self.st = case, st
        self.gpu_imgs = [fill_bytes(st["gpu_layer_bytes"], seed + l) for l in range(case.num_layers)]
        self.cpu_img = fill_bytes(st["cpu_pool_bytes"], seed + 99)
        self.layers = [torch.from_numpy(x.copy()).cuda() for x in self.gpu_imgs]
        self.cpu = torch.from_numpy(self.cpu_img.copy()).pin_memory()
        self.layout = KVLayout(torch.tensor([t.data_ptr() for t in self.layers], dtype=torch.int64),
                               st["gpu_kv"], st["gpu_block"], self.cpu, st["cpu_kv"], st["cpu_layer"],
                               st["cpu_block"], st["gpu_chunk"], case.is_mla, -1, st["gpu_layer_bytes"])

    def expect_d2h(self, gids, cids):
        if len(gids):
            oracle_transfer(self.case, self.gpu_imgs, self.cpu_img, np.asarray(gids, dtype=np.int64),
                            np.asarray(cids, dtype=np.int64), False)

    def expect_h2d(self, gids, cids):
        if len(gids):
            oracle_transfer(self.case, self.gpu_imgs, self.cpu_img, np.asarray(gids, dtype=np.int64),
                            np.asarray(cids, dtype=np.int64), True)

    def pool_matches(self) -> bool:
        return np.array_equal(self.cpu.numpy(), self.cpu_img)

    def layers_match(self) -> bool:
        return all(np.array_equal(t.cpu().numpy(), w) for t, w in zip(self.layers, self.gpu_imgs))


@pytest.mark.parametrize("name", [n for n, sc in golden().items() if not sc.get("num_ssd_blocks")])
def test_device_put_path_matches_the_reference(name):
    sc = golden()[name]
    tpb = sc["tpb"]
    pools = Pools(Case("golden", 2, 1, 8, tpb, 256, sc["num_cpu_blocks"]))
    ci = CpuCacheIndex(sc["num_cpu_blocks"], tpb)
    launches0 = c_ext.kernel_launch_count()
    for b, batch in enumerate(sc["batches"]):
        toks = [np.array(q["tokens"], dtype=np.int64) for q in batch]
        gids = [np.array(q["gpu_blocks"], dtype=np.int64) for q in batch]
        res = ci.put(toks, gids, pools.layout, mark_ready=sc["complete_each_batch"])
        for r, want in enumerate(sc["results"][b]):
            got = (int(res.num_skipped[r]), int(res.num_transferred[r]), res.gpu_blocks[r].tolist(),
                   res.cpu_blocks[r].tolist())
            assert got == (want["skipped"], want["transferred"], want["gpu_blocks"], want["cpu_blocks"]), \
                f"batch {b} request {r}"
            pools.expect_d2h(want["gpu_blocks"], want["cpu_blocks"])
        assert pools.pool_matches(), f"batch {b}: pool bytes"
        probes = sc["probes"][b]
        m = ci.match([np.array(p["tokens"], dtype=np.int64) for p in probes])
        for i, p in enumerate(probes):
            assert (int(m.num_matched[i]), int(m.num_ready[i]), m.physical_blocks[i].tolist()) == \
                (p["num_matched"], p["num_ready"], p["blocks"]), f"batch {b} probe {i}"
        for i, gq in enumerate(sc["gets"][b]):
            got = ci.get([np.array(gq["tokens"], dtype=np.int64)], [np.array(gq["gpu_blocks"], dtype=np.int64)],
                         pools.layout, [gq["block_start"]])
            t = int(got.num_transferred[0])
            assert (int(got.block_starts[0]) if t else 0, t, got.gpu_blocks[0].tolist(), got.cpu_blocks[0].tolist()) \
                == (gq["mask_start"], gq["transferred"], gq["copied_gpu_blocks"], gq["copied_cpu_blocks"]), \
                f"batch {b} get {i}"
            pools.expect_h2d(gq["copied_gpu_blocks"], gq["copied_cpu_blocks"])
        assert pools.layers_match(), f"batch {b}: GPU bytes after the gets"
        s = ci.stats()
        assert (s["num_free_blocks"], s["total_cached_blocks"], s["total_ready_blocks"]) == \
            (sc["num_free"][b], sc["total_cached"][b], sc["total_ready"][b])
    assert c_ext.kernel_launch_count() > launches0
    ci.close()


def test_put_requests_gives_the_reference_return_masks():
    """The reference-facing form: (token_ids, token_mask, slot_mapping) per
    request, partial last blocks ignored, return masks as the reference's."""
    sc = golden()["shared_prefixes"]
    tpb = sc["tpb"]
    pools = Pools(Case("golden", 2, 1, 8, tpb, 256, sc["num_cpu_blocks"]))
    ci = CpuCacheIndex(sc["num_cpu_blocks"], tpb)
    for b, batch in enumerate(sc["batches"]):
        reqs = []
        for q in batch:
            tok = torch.tensor(q["tokens"], dtype=torch.int64)
            g = np.array(q["gpu_blocks"], dtype=np.int64)
            slots = np.zeros(len(tok), dtype=np.int64)
            slots[:len(g) * tpb] = np.repeat(g, tpb) * tpb + np.tile(np.arange(tpb), len(g))
            slots[len(g) * tpb:] = 255 * tpb + np.arange(len(tok) - len(g) * tpb)
            reqs.append((tok, torch.ones(len(tok), dtype=torch.bool), torch.from_numpy(slots)))
        masks, _ = ci.put_requests(reqs, pools.layout)
        for r, want in enumerate(sc["results"][b]):
            m = masks[r]
            idx = torch.nonzero(m).flatten()
            assert (int(idx[0]) // tpb if len(idx) else 0, len(idx) // tpb) == (want["skipped"], want["transferred"])
    ci.close()


def test_get_requests_gives_the_reference_return_masks():
    """The reference-facing form of get: a mask from the request's first
    block to read through its last full block, slot mapping of the masked
    tokens; return masks as the reference's."""
    sc = golden()["shared_prefixes"]
    tpb = sc["tpb"]
    pools = Pools(Case("golden", 2, 1, 8, tpb, 256, sc["num_cpu_blocks"]))
    ci = CpuCacheIndex(sc["num_cpu_blocks"], tpb)
    for b, batch in enumerate(sc["batches"]):
        ci.put([np.array(q["tokens"], dtype=np.int64) for q in batch],
               [np.array(q["gpu_blocks"], dtype=np.int64) for q in batch], pools.layout)
        reqs = []
        for gq in sc["gets"][b]:
            tok = torch.tensor(gq["tokens"], dtype=torch.int64)
            bs, g = gq["block_start"], np.array(gq["gpu_blocks"], dtype=np.int64)
            mask = torch.zeros(len(tok), dtype=torch.bool)
            mask[bs * tpb:] = True
            slots = np.zeros(int(mask.sum()), dtype=np.int64)
            slots[:len(g) * tpb] = np.repeat(g, tpb) * tpb + np.tile(np.arange(tpb), len(g))
            slots[len(g) * tpb:] = 255 * tpb + np.arange(len(slots) - len(g) * tpb)
            reqs.append((tok, mask, torch.from_numpy(slots)))
        masks, _ = ci.get_requests(reqs, pools.layout)
        for m, gq in zip(masks, sc["gets"][b]):
            idx = torch.nonzero(m).flatten()
            assert (int(idx[0]) // tpb if len(idx) else 0, len(idx) // tpb) == (gq["mask_start"], gq["transferred"])
    ci.close()


def _requests(rng, n, tpb, max_blocks, vocab, seen, share, gpu_pool):
    toks, gids = [], []
    for _ in range(n):
        if seen and rng.random() < share:
            base = seen[rng.integers(len(seen))]
            cut = int(rng.integers(0, len(base) + 1))
            tok = np.concatenate([base[:cut], rng.integers(0, vocab, int(rng.integers(0, max_blocks * tpb // 2 + 1)))])
        else:
            tok = rng.integers(0, vocab, int(rng.integers(0, max_blocks * tpb + tpb)))
        tok = tok[:max_blocks * tpb + tpb - 1].astype(np.int64)
        seen.append(tok)
        toks.append(tok)
        gids.append(rng.choice(gpu_pool, size=len(tok) // tpb, replace=False).astype(np.int64))
    return toks, gids


@pytest.mark.parametrize("pool_blocks", [20000, 1500])
def test_large_batches_match_the_oracle(pool_blocks):
    """Batches of 256 requests of up to 32 blocks with shared prefixes, in
    the Qwen2-7B token shape (tpb 16); the small pool runs out and its
    puts come back empty from then on, as the reference's would."""
    tpb = 16
    rng = np.random.default_rng(pool_blocks)
    pools = Pools(Case("big", 2, 1, 64, tpb, 8192, pool_blocks), seed=31)
    tier = CI.CpuTier(pool_blocks, tpb)
    ci = CpuCacheIndex(pool_blocks, tpb)
    seen = []
    for b in range(4):
        toks, gids = _requests(rng, 256, tpb, 32, 2000, seen, 0.5, 8192)
        res = ci.put(toks, gids, pools.layout)
        want = [tier.put(t, g) for t, g in zip(toks, gids)]
        for r, w in enumerate(want):
            assert (int(res.num_skipped[r]), int(res.num_transferred[r])) == (w.num_skipped, w.num_transferred), r
            assert res.cpu_blocks[r].tolist() == w.cpu_blocks.tolist(), r
            assert res.gpu_blocks[r].tolist() == w.gpu_blocks.tolist(), r
            pools.expect_d2h(w.gpu_blocks, w.cpu_blocks)
        for w in want:
            tier.complete(w)
        assert pools.pool_matches()
        probes = [seen[i] for i in rng.choice(len(seen), 64, replace=False)]
        m = ci.match(probes)
        for i, p in enumerate(probes):
            w = tier.match(p)
            assert (int(m.num_matched[i]), int(m.num_ready[i]), m.physical_blocks[i].tolist()) == \
                (w.num_matched, w.num_ready, [int(x) for x in w.blocks])
        s = ci.stats()
        assert (s["num_free_blocks"], s["total_cached_blocks"], s["total_ready_blocks"]) == \
            (tier.pool.num_free, tier.tree.total_blocks(), tier.tree.total_ready())
        # gets of earlier sequences from random first blocks
        gtoks = [t for t in (seen[i] for i in rng.choice(len(seen), 256, replace=False)) if len(t) >= tpb]
        starts = [int(rng.integers(0, len(t) // tpb)) for t in gtoks]
        # distinct destinations across the batch (duplicate GPU destinations race, as in the reference)
        perm = rng.permutation(8192).astype(np.int64)
        cuts = np.cumsum([0] + [len(t) // tpb - bs for t, bs in zip(gtoks, starts)])
        ggids = [perm[cuts[i]:cuts[i + 1]] for i in range(len(gtoks))]
        got = ci.get(gtoks, ggids, pools.layout, starts)
        for r, (t, g, bs) in enumerate(zip(gtoks, ggids, starts)):
            w = tier.get(t, g, bs)
            assert (int(got.num_transferred[r]), got.gpu_blocks[r].tolist(), got.cpu_blocks[r].tolist()) == \
                (w.num_transferred, w.gpu_blocks.tolist(), w.cpu_blocks.tolist()), r
            pools.expect_h2d(w.gpu_blocks, w.cpu_blocks)
        assert pools.layers_match()
    ci.close()


def test_match_accepts_device_tokens_and_empty_sequences():
    tpb = 16
    pools = Pools(Case("dev", 2, 1, 64, tpb, 256, 512))
    ci = CpuCacheIndex(512, tpb)
    rng = np.random.default_rng(5)
    toks = [rng.integers(0, 500, n).astype(np.int64) for n in (0, 7, 16, 100, 333)]
    gids = [np.arange(len(t) // tpb, dtype=np.int64) + 10 * i for i, t in enumerate(toks)]
    ci.put(toks, gids, pools.layout)
    m_host = ci.match(toks)
    m_dev = ci.match([torch.from_numpy(t).cuda() for t in toks])
    assert m_host.num_matched.tolist() == m_dev.num_matched.tolist() == [len(t) // tpb for t in toks]
    assert [x.tolist() for x in m_host.physical_blocks] == [x.tolist() for x in m_dev.physical_blocks]
    assert ci.match([]).num_matched.tolist() == []
    ci.close()


def test_pool_order_under_take_and_recycle_matches_mempool():
    """Ids come in the reference Mempool's order: a snapshot of the free
    ids, refreshed only when a request does not fit in what is left."""
    ci = CpuCacheIndex(700, 16)
    pool = CI.BlockPool(700)
    rng = np.random.default_rng(17)
    live = []
    for _ in range(80):
        if rng.random() < 0.55 or not live:
            n = int(rng.integers(0, 90))
            got = ci.take(n)
            want = pool.allocate(min(n, pool.num_free))
            assert got.tolist() == want.tolist()
            live.extend(got.tolist())
        else:
            k = int(rng.integers(1, min(len(live), 70) + 1))
            pick = set(rng.choice(len(live), k, replace=False).tolist())
            ids = np.array([live[i] for i in sorted(pick)], dtype=np.int64)
            ci.recycle(ids)
            pool.recycle(ids)
            live = [x for j, x in enumerate(live) if j not in pick]
        s = ci.stats()
        assert (s["num_free_blocks"], s["pool_snapshot_len"], s["pool_snapshot_offset"]) == \
            (pool.num_free, len(pool.ids), pool.offset)
    ci.close()


def test_caller_eviction_then_put():
    """Eviction is the caller's: remove a request's own blocks, recycle them;
    its match falls back to the shared prefix and later puts reuse the ids
    in Mempool order."""
    tpb = 16
    pools = Pools(Case("evict", 2, 1, 64, tpb, 512, 256))
    ci = CpuCacheIndex(256, tpb)
    pool = CI.BlockPool(256)
    rng = np.random.default_rng(23)
    prefix = rng.integers(0, 1000, 4 * tpb).astype(np.int64)
    a = np.concatenate([prefix, rng.integers(0, 1000, 6 * tpb)]).astype(np.int64)
    b = np.concatenate([prefix, rng.integers(0, 1000, 3 * tpb)]).astype(np.int64)
    res = ci.put([a, b], [np.arange(10), np.arange(100, 107)], pools.layout)
    assert res.num_transferred.tolist() == [10, 3] and res.num_skipped.tolist() == [0, 4]
    pool.allocate(10)
    pool.allocate(3)
    # evict b's own suffix (3 blocks, a leaf)
    removed = ci.remove(res.block_hashes[1][4:])
    assert removed.tolist() == res.cpu_blocks[1].tolist()
    assert ci.remove(res.block_hashes[1][4:]).tolist() == [-1, -1, -1]  # already gone
    ci.recycle(removed)
    pool.recycle(removed)
    m = ci.match([b, a])
    assert m.num_matched.tolist() == [4, 10]
    s = ci.stats()
    assert (s["total_cached_blocks"], s["num_free_blocks"], s["deleted_slots"]) == (10, 246, 3)
    fresh = [rng.integers(1000, 2000, n * tpb).astype(np.int64) for n in (30, 200, 20)]
    res2 = ci.put(fresh, [np.arange(200, 200 + len(f) // tpb) % 512 for f in fresh], pools.layout)
    want = [pool.allocate(min(len(f) // tpb, pool.num_free)) for f in fresh[:2]]
    assert res2.cpu_blocks[0].tolist() == want[0].tolist()
    assert res2.cpu_blocks[1].tolist() == want[1].tolist()
    assert res2.num_transferred.tolist() == [30, 200, 0]  # 16 blocks left: the last put is empty
    ci.close()


def test_errors_leave_the_index_unchanged():
    tpb = 16
    pools = Pools(Case("err", 2, 1, 64, tpb, 64, 128))
    ci = CpuCacheIndex(128, tpb)
    tok = np.arange(5 * tpb, dtype=np.int64)
    ci.put([tok], [np.arange(5)], pools.layout)
    before = ci.stats()
    with pytest.raises(FlexKVError) as e:
        ci.recycle([100])  # never allocated: already free
    assert e.value.code == FKV_ERR_INVALID_ARG
    with pytest.raises(FlexKVError) as e:
        ci.recycle([1, 1])
    assert e.value.code == FKV_ERR_INVALID_ARG
    with pytest.raises(FlexKVError) as e:
        ci.recycle([128])
    assert e.value.code == FKV_ERR_OUT_OF_RANGE
    with pytest.raises(FlexKVError) as e:  # GPU block 64 is past the 64-block layer
        ci.put([np.arange(100, 100 + 2 * tpb, dtype=np.int64)], [np.array([3, 64])], pools.layout)
    assert e.value.code == FKV_ERR_OUT_OF_RANGE
    with pytest.raises(ValueError):
        ci.put([tok], [np.arange(4)], pools.layout)  # one GPU block per full block
    # layouts the copy cannot use are refused before anything changes
    import dataclasses
    pageable = dataclasses.replace(pools.layout, cpu_tensor=torch.zeros_like(pools.cpu, device="cpu").clone())
    with pytest.raises(FlexKVError) as e:
        ci.put([np.arange(200, 200 + 3 * tpb, dtype=np.int64)], [np.arange(3)], pageable)
    assert e.value.code == FKV_ERR_INVALID_ARG
    small = dataclasses.replace(pools.layout, cpu_tensor=pools.cpu[: pools.cpu.numel() // 2])
    with pytest.raises(FlexKVError) as e:  # the index hands out ids the half pool does not hold
        ci.put([np.arange(300, 300 + 3 * tpb, dtype=np.int64)], [np.arange(3)], small)
    assert e.value.code == FKV_ERR_OUT_OF_RANGE
    with pytest.raises(FlexKVError) as e:
        ci.get([tok], [np.arange(5)], small)
    assert e.value.code == FKV_ERR_OUT_OF_RANGE
    assert ci.stats() == before
    assert ci.match([tok]).num_matched.tolist() == [5]
    ci.close()


def test_edge_batches_match_the_oracle():
    """Identical requests in one batch (the second is fully cached by the
    first), a 3000-block sequence beside short ones, requests with no full
    block, and gets that read only the last block."""
    tpb = 16
    rng = np.random.default_rng(41)
    pools = Pools(Case("edge", 2, 1, 64, tpb, 4096, 4096), seed=53)
    tier = CI.CpuTier(4096, tpb)
    ci = CpuCacheIndex(4096, tpb)
    a = rng.integers(0, 5000, 7 * tpb).astype(np.int64)
    long_seq = rng.integers(0, 5000, 3000 * tpb + 5).astype(np.int64)
    toks = [a, a.copy(), np.zeros(0, np.int64), long_seq, rng.integers(0, 5000, tpb - 1).astype(np.int64),
            np.concatenate([a[:3 * tpb], rng.integers(0, 5000, 2 * tpb)]).astype(np.int64)]
    perm = rng.permutation(4096).astype(np.int64)
    cuts = np.cumsum([0] + [len(t) // tpb for t in toks])
    gids = [perm[cuts[i]:cuts[i + 1]] for i in range(len(toks))]
    res = ci.put(toks, gids, pools.layout)
    for r, (t, g) in enumerate(zip(toks, gids)):
        w = tier.put(t, g)
        tier.complete(w)
        assert (int(res.num_skipped[r]), int(res.num_transferred[r]), res.cpu_blocks[r].tolist()) == \
            (w.num_skipped, w.num_transferred, w.cpu_blocks.tolist()), r
        pools.expect_d2h(w.gpu_blocks, w.cpu_blocks)
    assert res.num_transferred.tolist()[:3] == [7, 0, 0]
    assert pools.pool_matches()
    gt = [a, long_seq, toks[5]]
    starts = [len(t) // tpb - 1 for t in gt]
    dst = [np.array([4095 - i], dtype=np.int64) for i in range(len(gt))]
    got = ci.get(gt, dst, pools.layout, starts)
    for r, (t, g, bs) in enumerate(zip(gt, dst, starts)):
        w = tier.get(t, g, bs)
        assert (int(got.num_transferred[r]), got.cpu_blocks[r].tolist()) == (w.num_transferred, w.cpu_blocks.tolist())
        pools.expect_h2d(w.gpu_blocks, w.cpu_blocks)
    assert got.num_transferred.tolist() == [1, 1, 1]
    assert pools.layers_match()
    ci.close()


def test_asynchronous_put_and_get_return_the_decisions_first():
    """synchronous=False returns once the decisions are known (the
    reference's put/get return before their transfers run); the copies and
    the ready marks finish on the stream, and the bytes equal the oracle's
    once the stream has drained."""
    tpb = 16
    rng = np.random.default_rng(61)
    pools = Pools(Case("async", 2, 1, 64, tpb, 2048, 2048), seed=67)
    tier = CI.CpuTier(2048, tpb)
    ci = CpuCacheIndex(2048, tpb)
    seen = []
    toks, gids = _requests(rng, 128, tpb, 24, 3000, seen, 0.5, 2048)
    res = ci.put(toks, gids, pools.layout, synchronous=False)
    want = [tier.put(t, g) for t, g in zip(toks, gids)]
    for r, w in enumerate(want):
        assert (int(res.num_skipped[r]), res.cpu_blocks[r].tolist()) == (w.num_skipped, w.cpu_blocks.tolist())
        pools.expect_d2h(w.gpu_blocks, w.cpu_blocks)
        tier.complete(w)
    torch.cuda.current_stream().synchronize()
    assert pools.pool_matches()
    assert ci.stats()["total_ready_blocks"] == tier.tree.total_ready()
    gt = [t for t in seen if len(t) >= tpb][:64]
    perm = rng.permutation(2048).astype(np.int64)
    cuts = np.cumsum([0] + [len(t) // tpb for t in gt])
    dst = [perm[cuts[i]:cuts[i + 1]] for i in range(len(gt))]
    got = ci.get(gt, dst, pools.layout, synchronous=False)
    for r, (t, g) in enumerate(zip(gt, dst)):
        w = tier.get(t, g)
        assert got.cpu_blocks[r].tolist() == w.cpu_blocks.tolist()
        pools.expect_h2d(w.gpu_blocks, w.cpu_blocks)
    torch.cuda.current_stream().synchronize()
    assert pools.layers_match()
    ci.close()


def test_layerwise_get_completes_group_by_group():
    """layer_granularity: the layers are read in groups, in order, and the
    event of group i marks those layers as loaded (the reference's layer-wise
    read graph, transfer_pattern.py:370-428, waited on by
    wait_at_layer_group); a granularity that does not divide the layers is
    refused as the reference asserts."""
    tpb = 16
    rng = np.random.default_rng(71)
    case = Case("layers", 8, 1, 64, tpb, 1024, 1024)
    pools = Pools(case, seed=73)
    tier = CI.CpuTier(1024, tpb)
    ci = CpuCacheIndex(1024, tpb)
    seen = []
    toks, gids = _requests(rng, 64, tpb, 16, 3000, seen, 0.5, 1024)
    ci.put(toks, gids, pools.layout)
    for t, g in zip(toks, gids):
        tier.complete(tier.put(t, g))
    gt = [t for t in toks if len(t) >= tpb][:32]
    perm = rng.permutation(1024).astype(np.int64)
    cuts = np.cumsum([0] + [len(t) // tpb for t in gt])
    dst = [perm[cuts[i]:cuts[i + 1]] for i in range(len(gt))]
    # expected GPU images: the puts copied D2H (host images of the pool follow the device pool)
    pools.cpu_img[:] = pools.cpu.numpy()
    for t, g in zip(gt, dst):
        w = tier.get(t, g)
        pools.expect_h2d(w.gpu_blocks, w.cpu_blocks)
    events = [torch.cuda.Event() for _ in range(4)]
    got = ci.get(gt, dst, pools.layout, synchronous=False, layer_granularity=2, group_events=events)
    assert int(got.num_transferred.sum()) == int(sum(len(t) // tpb for t in gt))
    for gi, ev in enumerate(events):
        ev.synchronize()
        for l in (2 * gi, 2 * gi + 1):
            assert np.array_equal(pools.layers[l].cpu().numpy(), pools.gpu_imgs[l]), f"layer {l} after group {gi}"
    torch.cuda.current_stream().synchronize()
    assert pools.layers_match()
    with pytest.raises(FlexKVError) as e:
        ci.get(gt[:1], dst[:1], pools.layout, layer_granularity=3)
    assert e.value.code == FKV_ERR_INVALID_ARG
    ci.close()


@pytest.mark.parametrize("name", [n for n, sc in golden().items() if sc.get("num_ssd_blocks")])
def test_two_tier_put_matches_the_reference(tmp_path, name):
    """Puts with the SSD tier on (cache_engine.py:787-902), from the
    reference's own GlobalCacheEngine run with its SSD tier: each put's D2H
    and H2DISK block lists, the gets' H2D lists, both tiers' totals, and the
    bytes on the SSD (read back from the files, compared with the CPU blocks
    they were written from)."""
    from flexkv_b200.cache_index import SsdTier
    from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
    from flexkv_b200.ssd import SsdStrides, allocate_ssd_files
    sc = golden()[name]
    tpb, n_cpu, n_ssd = sc["tpb"], sc["num_cpu_blocks"], sc["num_ssd_blocks"]
    case = Case("golden", 2, 1, 8, tpb, 256, n_cpu)
    pools = Pools(case)
    cpu_layout = case.cpu_layout_obj()
    ssd_layout = KVCacheLayout(KVCacheLayoutType.LAYERWISE, 2, n_ssd, tpb, 1, 8, False)
    files, per_file = allocate_ssd_files(ssd_layout, 2, str(tmp_path / "ssd"), max_blocks_per_file=n_ssd)
    ioctx = c_ext.SSDIOCTX(files, len(files), 0, 0)
    strides = SsdStrides.of(cpu_layout, ssd_layout, sum(len(v) for v in files.values()), 2)
    ci, si = CpuCacheIndex(n_cpu, tpb), CpuCacheIndex(n_ssd, tpb)
    ssd = SsdTier(si, ioctx, strides, 2, per_file)
    written = []
    for b, batch in enumerate(sc["batches"]):
        toks = [np.array(q["tokens"], dtype=np.int64) for q in batch]
        gids = [np.array(q["gpu_blocks"], dtype=np.int64) for q in batch]
        res = ci.put_two_tier(ssd, toks, gids, pools.layout, mark_ready=sc["complete_each_batch"])
        for r, want in enumerate(sc["results"][b]):
            ops = []
            if int(res.num_transferred[r]):
                ops.append(["D2H", res.gpu_blocks[r].tolist(), res.cpu_blocks[r].tolist()])
                if int(res.num_to_ssd[r]):
                    ops.append(["H2DISK", res.h2disk_cpu_blocks[r].tolist(), res.ssd_blocks[r].tolist()])
                    written += list(zip(res.h2disk_cpu_blocks[r].tolist(), res.ssd_blocks[r].tolist()))
            assert (int(res.num_skipped[r]), int(res.num_transferred[r]), ops) == \
                (want["skipped"], want["transferred"], want["ops"]), f"batch {b} put {r}"
        for i, gq in enumerate(sc["gets"][b]):
            got = ci.get([np.array(gq["tokens"], dtype=np.int64)], [np.array(gq["gpu_blocks"], dtype=np.int64)],
                         pools.layout, [gq["block_start"]])
            ops = [["H2D", got.cpu_blocks[0].tolist(), got.gpu_blocks[0].tolist()]] if int(got.num_transferred[0]) else []
            assert ops == gq["ops"], f"batch {b} get {i}"
        sc_c, sc_s = ci.stats(), si.stats()
        assert (sc_c["num_free_blocks"], sc_c["total_cached_blocks"], sc_c["total_ready_blocks"],
                sc_s["num_free_blocks"], sc_s["total_cached_blocks"]) == \
            (sc["num_free"][b], sc["total_cached"][b], sc["total_ready"][b], sc["ssd_num_free"][b],
             sc["ssd_total_cached"][b])
    assert written
    # the SSD holds what the CPU blocks held: read it back into a second pool at the same CPU blocks
    back = torch.zeros_like(pools.cpu).pin_memory()
    cids = np.array([c for c, _ in written], dtype=np.int64)
    sids = np.array([s_ for _, s_ in written], dtype=np.int64)
    c_ext.transfer_kv_blocks_ssd(ioctx, [0, 1], back.data_ptr(), sids, cids, strides.cpu_layer_stride_in_bytes,
                                 strides.cpu_kv_stride_in_bytes, strides.ssd_layer_stride_in_bytes,
                                 strides.ssd_kv_stride_in_bytes, strides.chunk_size_in_bytes,
                                 strides.block_stride_in_bytes, True, per_file,
                                 cpu_pool_bytes=back.numel() * back.element_size())
    st = case.strides()
    a, w = pools.cpu.numpy(), back.numpy()
    for c in cids.tolist():
        for l in range(2):
            for k in range(2):
                o = l * st["cpu_layer"] + k * st["cpu_kv"] + c * st["cpu_block"]
                assert np.array_equal(a[o:o + st["cpu_chunk"]], w[o:o + st["cpu_chunk"]]), (c, l, k)
    ioctx.close()
    ci.close()
    si.close()


def _two_tier(tmp_path, tpb=4, n_cpu=64, n_ssd=64):
    """A two-layer case with a CPU-tier index and an SSD-tier index over
    files under tmp_path."""
    from flexkv_b200.cache_index import SsdTier
    from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
    from flexkv_b200.ssd import SsdStrides, allocate_ssd_files
    case = Case("two_tier", 2, 1, 8, tpb, 256, n_cpu)
    pools = Pools(case)
    ssd_layout = KVCacheLayout(KVCacheLayoutType.LAYERWISE, 2, n_ssd, tpb, 1, 8, False)
    files, per_file = allocate_ssd_files(ssd_layout, 2, str(tmp_path / "ssd"), max_blocks_per_file=n_ssd)
    ioctx = c_ext.SSDIOCTX(files, len(files), 0, 0)
    strides = SsdStrides.of(case.cpu_layout_obj(), ssd_layout, sum(len(v) for v in files.values()), 2)
    ci, si = CpuCacheIndex(n_cpu, tpb), CpuCacheIndex(n_ssd, tpb)
    return case, pools, ci, si, SsdTier(si, ioctx, strides, 2, per_file)


def _ssd_holds_cpu_blocks(case, pools, ssd, pairs):
    """Read the SSD blocks back into a zeroed pool at their CPU blocks and
    compare every chunk with the CPU pool."""
    st, s = case.strides(), ssd.strides
    back = torch.zeros_like(pools.cpu).pin_memory()
    cids = np.array([c for c, _ in pairs], dtype=np.int64)
    sids = np.array([x for _, x in pairs], dtype=np.int64)
    c_ext.transfer_kv_blocks_ssd(ssd.ioctx, [0, 1], back.data_ptr(), sids, cids, s.cpu_layer_stride_in_bytes,
                                 s.cpu_kv_stride_in_bytes, s.ssd_layer_stride_in_bytes, s.ssd_kv_stride_in_bytes,
                                 s.chunk_size_in_bytes, s.block_stride_in_bytes, True, ssd.num_blocks_per_file,
                                 cpu_pool_bytes=back.numel() * back.element_size())
    a, w = pools.cpu.numpy(), back.numpy()
    for c in cids.tolist():
        for l in range(2):
            for k in range(2):
                o = l * st["cpu_layer"] + k * st["cpu_kv"] + c * st["cpu_block"]
                if not np.array_equal(a[o:o + st["cpu_chunk"]], w[o:o + st["cpu_chunk"]]):
                    return False
    return True


def test_two_tier_put_rolls_the_ssd_tier_back_when_its_writes_fail(tmp_path, monkeypatch):
    """An SSD write that fails (a fake of the SSD call raising, on the host)
    leaves no SSD-tier entry pointing at an unwritten block and no SSD block
    leaked; the CPU tier keeps its copy; the same put then succeeds."""
    case, pools, ci, si, ssd = _two_tier(tmp_path)
    rng = np.random.default_rng(5)
    toks = [rng.integers(0, 32000, 4 * n).astype(np.int64) for n in (3, 5)]
    gids = [np.arange(3, dtype=np.int64), np.arange(5, dtype=np.int64) + 10]
    before = si.stats()

    def failing(*a, **k):
        raise OSError("injected SSD write failure")

    monkeypatch.setattr(c_ext, "transfer_kv_blocks_ssd", failing)
    with pytest.raises(OSError):
        ci.put_two_tier(ssd, toks, gids, pools.layout)
    monkeypatch.undo()
    after = si.stats()
    assert (after["num_free_blocks"], after["total_cached_blocks"]) == \
        (before["num_free_blocks"], before["total_cached_blocks"])
    assert si.match(toks).num_matched.tolist() == [0, 0]
    assert ci.match(toks).num_ready.tolist() == [3, 5]  # the CPU tier's part stands
    res = ci.put_two_tier(ssd, toks, gids, pools.layout)
    assert res.num_transferred.tolist() == [0, 0] and res.num_to_ssd.tolist() == [0, 0]  # CPU holds them
    assert si.match(toks).num_matched.tolist() == [0, 0]  # the reference moves nothing when CPU has all
    toks2 = [np.concatenate([t, rng.integers(0, 32000, 4).astype(np.int64)]) for t in toks]
    gids2 = [np.arange(4, dtype=np.int64) + 20, np.arange(6, dtype=np.int64) + 30]
    res = ci.put_two_tier(ssd, toks2, gids2, pools.layout)
    assert res.num_transferred.tolist() == [1, 1] and res.num_to_ssd.tolist() == [4, 6]
    pairs = [(c, x) for r in range(2) for c, x in zip(res.h2disk_cpu_blocks[r].tolist(), res.ssd_blocks[r].tolist())]
    assert _ssd_holds_cpu_blocks(case, pools, ssd, pairs)
    assert si.match(toks2).num_ready.tolist() == [4, 6]
    ssd.ioctx.close()
    ci.close()
    si.close()


def test_two_tier_put_after_ssd_only_eviction(tmp_path):
    """The SSD tier evicted alone (m_s < m_c): the SSD copy of a block below
    m_c comes from its cached CPU block.  While that block is not ready the
    put is refused and allocates nothing; once it is ready the put writes
    the SSD tier, whose bytes then equal the CPU blocks."""
    case, pools, ci, si, ssd = _two_tier(tmp_path)
    rng = np.random.default_rng(9)
    a = rng.integers(0, 32000, 4 * 3).astype(np.int64)
    res = ci.put_two_tier(ssd, [a], [np.arange(3, dtype=np.int64)], pools.layout, mark_ready=False)
    assert res.num_transferred.tolist() == [3] and res.num_to_ssd.tolist() == [3]
    pools.expect_d2h(res.gpu_blocks[0], res.cpu_blocks[0])
    held = si.remove(res.block_hashes[0])
    si.recycle(held[held >= 0])
    ab = np.concatenate([a, rng.integers(0, 32000, 4 * 2).astype(np.int64)])
    c_before, s_before = ci.stats(), si.stats()
    res = ci.put_two_tier(ssd, [ab], [np.arange(5, dtype=np.int64) + 8], pools.layout)
    assert (int(res.num_skipped[0]), int(res.num_transferred[0]), int(res.num_to_ssd[0])) == (0, 0, 0)
    c_after, s_after = ci.stats(), si.stats()
    for k in ("num_free_blocks", "total_cached_blocks"):
        assert (c_after[k], s_after[k]) == (c_before[k], s_before[k]), k
    ci.set_ready(res.block_hashes[0][:3])
    res = ci.put_two_tier(ssd, [ab], [np.arange(5, dtype=np.int64) + 8], pools.layout)
    assert (int(res.num_skipped[0]), int(res.num_transferred[0]), int(res.num_to_ssd[0])) == (3, 2, 5)
    pools.expect_d2h(res.gpu_blocks[0], res.cpu_blocks[0])
    assert pools.pool_matches()
    pairs = list(zip(res.h2disk_cpu_blocks[0].tolist(), res.ssd_blocks[0].tolist()))
    assert len(pairs) == 5
    assert _ssd_holds_cpu_blocks(case, pools, ssd, pairs)
    assert si.match([ab]).num_ready.tolist() == [5]
    ssd.ioctx.close()
    ci.close()
    si.close()
