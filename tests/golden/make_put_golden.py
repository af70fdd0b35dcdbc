"""Regenerate tests/golden/put_path.json by running the reference's own CPU
tier (run in a container that has the reference tree; the fixture travels
without it):

    python tests/golden/make_put_golden.py --reference /path/to/FlexKV

The reference's GlobalCacheEngine (flexkv/cache/cache_engine.py) is imported
from its tree with the SSD and remote tiers off.  Its compiled extension is
not built here, so `flexkv.c_ext` is replaced by a module that computes
gen_hashes with the python `xxhash` package, the library the reference's
hash.cpp links, in the same prefix-chained semantics (hash.cpp:47-66).

Each scenario is a sequence of batches of puts (token ids + one GPU block per
full block).  For every put the fixture records the reference's D2H op (GPU
and CPU block ids) and its return mask as (skipped, transferred) block
counts; after each batch it optionally runs the put callbacks (unlock +
set ready), then records match results of probe sequences, gets of earlier
sequences from a random first block (the H2D op's block lists and the return
mask as (start, transferred) block counts; each get's callback runs at
once), and the pool and tree totals.  The "pool_full" scenario never runs
callbacks, so no cached block is evictable and take() hands out fewer
blocks than asked once the pool is short: those puts come back empty, as
with no eviction.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def install_hash_stub(torch):
    import xxhash
    stub = types.ModuleType("flexkv.c_ext")

    class Hasher:
        def __init__(self):
            self.h = xxhash.xxh64(seed=0)

        def reset(self):
            self.h = xxhash.xxh64(seed=0)

        def update(self, t):
            self.h.update(t.contiguous().numpy().tobytes())

        def digest(self):
            return self.h.intdigest()

    def gen_hashes(hasher, token_ids, tpb, out):
        a = token_ids.to(torch.int64).numpy()
        w = out.view(torch.int64)
        for b in range(a.size // tpb):
            hasher.h.update(a[b * tpb:(b + 1) * tpb].tobytes())
            v = hasher.h.intdigest()
            w[b] = v - (1 << 64) if v >= (1 << 63) else v

    stub.Hasher = Hasher
    stub.gen_hashes = gen_hashes
    stub.get_hash_size = lambda: 8
    return stub


def make_requests(rng, n_batches, per_batch, tpb, max_blocks, vocab, gpu_blocks, share):
    """Batches of (tokens, gpu block ids).  A request reuses a prefix of an
    earlier request (same batch or before) with probability `share`."""
    seen = []
    batches = []
    for _ in range(n_batches):
        batch = []
        for _ in range(per_batch):
            if seen and rng.random() < share:
                base = seen[rng.integers(len(seen))]
                cut = int(rng.integers(0, len(base) + 1))
                extra = int(rng.integers(0, max_blocks * tpb // 2 + 1))
                tok = np.concatenate([base[:cut], rng.integers(0, vocab, extra)])
            else:
                tok = rng.integers(0, vocab, int(rng.integers(0, max_blocks * tpb + tpb)))
            tok = tok[:max_blocks * tpb + tpb - 1].astype(np.int64)
            n = len(tok) // tpb
            g = rng.choice(gpu_blocks, size=n, replace=False).astype(np.int64)
            seen.append(tok)
            batch.append((tok, g))
        batches.append(batch)
    return batches, seen


def ops_of(graph, TransferType):
    """The graph's transfer ops as (type, src ids, dst ids), in op order."""
    out = []
    for op in graph._op_map.values():
        if op.transfer_type == TransferType.VIRTUAL:
            continue
        out.append([op.transfer_type.name, op.src_descriptor.physical_block_ids.tolist(),
                    op.dst_descriptor.physical_block_ids.tolist()])
    return out


def run_scenario(torch, refmods, name, seed, tpb, num_cpu_blocks, n_batches, per_batch,
                 max_blocks, complete_each_batch, share=0.6, vocab=40, num_ssd_blocks=0):
    GlobalCacheEngine, CacheConfig, ModelConfig, SequenceMeta, DeviceType, TransferType = refmods
    rng = np.random.default_rng(seed)
    batches, seen = make_requests(rng, n_batches, per_batch, tpb, max_blocks, vocab, 256, share)
    cc = CacheConfig(tokens_per_block=tpb, enable_cpu=True, enable_ssd=num_ssd_blocks > 0,
                     enable_remote=False, num_cpu_blocks=num_cpu_blocks,
                     num_ssd_blocks=max(num_ssd_blocks, 1))
    mc = ModelConfig(num_layers=2, num_kv_heads=1, head_size=8)
    eng = GlobalCacheEngine(cc, mc)
    out = {"name": name, "tpb": tpb, "num_cpu_blocks": num_cpu_blocks, "num_ssd_blocks": num_ssd_blocks,
           "complete_each_batch": complete_each_batch, "batches": [], "results": [],
           "probes": [], "gets": [], "num_free": [], "total_cached": [], "total_ready": []}
    rid = 0
    for batch in batches:
        res, callbacks = [], []
        out["batches"].append([{"tokens": t.tolist(), "gpu_blocks": g.tolist()} for t, g in batch])
        for tok, g in batch:
            n_tok = len(tok)
            slots = np.zeros(n_tok, dtype=np.int64)
            full = len(g) * tpb
            slots[:full] = (np.repeat(g, tpb) * tpb + np.tile(np.arange(tpb), len(g)))
            slots[full:] = 255 * tpb + np.arange(n_tok - full)
            graph, mask, cb, _ = eng.put(rid, torch.from_numpy(tok), torch.ones(n_tok, dtype=torch.bool),
                                         torch.from_numpy(slots))
            rid += 1
            callbacks.append(cb)
            idx = torch.nonzero(mask).flatten()
            skipped = int(idx[0]) // tpb if len(idx) else 0
            transferred = len(idx) // tpb
            gpu_ids, cpu_ids = [], []
            for op in graph._op_map.values():
                if op.transfer_type == TransferType.D2H:
                    gpu_ids = op.src_descriptor.physical_block_ids.tolist()
                    cpu_ids = op.dst_descriptor.physical_block_ids.tolist()
            res.append({"skipped": skipped, "transferred": transferred,
                        "gpu_blocks": gpu_ids, "cpu_blocks": cpu_ids, "ops": ops_of(graph, TransferType)})
        if complete_each_batch:
            for cb in callbacks:
                cb()
        out["results"].append(res)
        probes = []
        picks = [seen[i] for i in rng.choice(len(seen), size=min(6, len(seen)), replace=False)]
        picks.append(np.concatenate([picks[0], rng.integers(0, vocab, 3 * tpb)]).astype(np.int64))
        picks.append(rng.integers(0, vocab, 5 * tpb).astype(np.int64))
        for tok in picks:
            m = eng.cpu_cache_engine.match(SequenceMeta(token_ids=torch.from_numpy(tok), tokens_per_block=tpb))
            probes.append({"tokens": tok.tolist(), "num_matched": int(m.num_matched_blocks),
                           "num_ready": int(m.num_ready_matched_blocks),
                           "blocks": m.physical_blocks[:m.num_matched_blocks].tolist()})
        out["probes"].append(probes)
        gets = []
        full = [t for t in seen if len(t) >= tpb]
        for i in rng.choice(len(full), size=min(6, len(full)), replace=False):
            tok = full[i]
            n = len(tok) // tpb
            bs = int(rng.integers(0, n))
            g = rng.choice(256, size=n - bs, replace=False).astype(np.int64)
            mask = np.zeros(len(tok), dtype=bool)
            mask[bs * tpb:] = True
            slots = np.zeros(int(mask.sum()), dtype=np.int64)
            slots[:len(g) * tpb] = np.repeat(g, tpb) * tpb + np.tile(np.arange(tpb), len(g))
            slots[len(g) * tpb:] = 255 * tpb + np.arange(len(slots) - len(g) * tpb)
            graph, rmask, cb, _ = eng.get(rid, torch.from_numpy(tok), torch.from_numpy(mask),
                                          torch.from_numpy(slots))
            rid += 1
            idx = torch.nonzero(rmask).flatten()
            gpu_ids, cpu_ids = [], []
            for op in graph._op_map.values():
                if op.transfer_type == TransferType.H2D:
                    gpu_ids = op.dst_descriptor.physical_block_ids.tolist()
                    cpu_ids = op.src_descriptor.physical_block_ids.tolist()
            cb()
            gets.append({"tokens": tok.tolist(), "block_start": bs, "gpu_blocks": g.tolist(),
                         "mask_start": int(idx[0]) // tpb if len(idx) else 0, "transferred": len(idx) // tpb,
                         "copied_gpu_blocks": gpu_ids, "copied_cpu_blocks": cpu_ids,
                         "ops": ops_of(graph, TransferType)})
        out["gets"].append(gets)
        if num_ssd_blocks:
            out.setdefault("ssd_num_free", []).append(int(eng.ssd_cache_engine.mempool.num_free_blocks))
            out.setdefault("ssd_total_cached", []).append(int(eng.ssd_cache_engine.index.total_cached_blocks()))
        out["num_free"].append(int(eng.cpu_cache_engine.mempool.num_free_blocks))
        out["total_cached"].append(int(eng.cpu_cache_engine.index.total_cached_blocks()))
        out["total_ready"].append(int(eng.cpu_cache_engine.index.total_ready_blocks()))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    import torch
    sys.path.insert(0, args.reference)
    import flexkv  # reference package
    stub = install_hash_stub(torch)
    sys.modules["flexkv.c_ext"] = stub
    flexkv.c_ext = stub
    from flexkv.cache.cache_engine import GlobalCacheEngine  # reference code
    from flexkv.common.block import SequenceMeta
    from flexkv.common.config import CacheConfig, ModelConfig
    from flexkv.common.transfer import DeviceType, TransferType
    mods = (GlobalCacheEngine, CacheConfig, ModelConfig, SequenceMeta, DeviceType, TransferType)
    scenarios = [
        run_scenario(torch, mods, "shared_prefixes", 11, 4, 1024, 4, 12, 10, True),
        run_scenario(torch, mods, "in_batch_sharing_tpb2", 12, 2, 512, 3, 16, 12, True, share=0.8),
        run_scenario(torch, mods, "pool_full", 13, 4, 48, 4, 10, 8, False),
        run_scenario(torch, mods, "callbacks_deferred", 14, 8, 256, 3, 10, 6, False, share=0.7),
        # the SSD tier on: puts copy D2H into new CPU blocks and H2DISK the blocks the SSD tier lacks
        run_scenario(torch, mods, "ssd_two_tier", 15, 4, 1024, 3, 12, 10, True, num_ssd_blocks=2048),
        # an SSD pool that runs out (callbacks deferred: nothing evictable): puts come back empty
        # and give their CPU blocks back
        run_scenario(torch, mods, "ssd_pool_full", 16, 4, 512, 3, 10, 8, False, num_ssd_blocks=40),
    ]
    with open(os.path.join(HERE, "put_path.json"), "w") as f:
        json.dump({"source": "reference GlobalCacheEngine.put / CacheEngine.match, CPU tier only",
                   "scenarios": scenarios}, f, separators=(",", ":"))
    print("wrote", os.path.join(HERE, "put_path.json"),
          os.path.getsize(os.path.join(HERE, "put_path.json")), "bytes")


if __name__ == "__main__":
    main()
