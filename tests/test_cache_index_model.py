"""The claim the device index rests on, checked on the CPU: for
prefix-chained block hashes, the reference's tree walk (RadixTreeIndex.
match_prefix with node splits, restated in oracle/cache_index.py) equals
"the leading blocks whose hash is present" over a flat hash -> block map,
for the matched count, the ready count and the physical blocks; and the
CPU-tier put decisions follow from it with the Mempool's id order.  Random
histories of puts (with and without their callbacks), branching prefixes
and repeated requests."""
import numpy as np
import pytest

from oracle import cache_index as CI


class FlatModel:
    """Hash -> (pool block, ready) with the consecutive-puts rule: what the
    device index keeps."""

    def __init__(self, num_blocks, tpb):
        self.tpb = tpb
        self.map = {}
        self.pool = CI.BlockPool(num_blocks)

    def hashes(self, tok):
        return CI.CpuTier(1, self.tpb).hashes(tok)

    def match(self, h):
        m = 0
        while m < len(h) and h[m] in self.map:
            m += 1
        blocks = [self.map[x][0] for x in h[:m]]
        ready = sum(1 for x in h[:m] if self.map[x][1])
        return m, ready, blocks

    def put(self, tok):
        h = self.hashes(tok)
        m, _, _ = self.match(h)
        k = len(h) - m
        if k == 0:
            return (0, 0, []), []
        got = self.pool.allocate(min(k, self.pool.num_free))
        if len(got) < k:
            self.pool.recycle(got)
            return (0, 0, []), []
        for x, c in zip(h[m:], got.tolist()):
            self.map[x] = [c, False]
        return (m, k, got.tolist()), h[m:]

    def complete(self, inserted):
        for x in inserted:
            self.map[x][1] = True


def random_history(seed, n_ops, tpb, pool_blocks):
    rng = np.random.default_rng(seed)
    tier = CI.CpuTier(pool_blocks, tpb)
    flat = FlatModel(pool_blocks, tpb)
    seen, pending = [], []
    for step in range(n_ops):
        # a new request: a fresh sequence, a prefix of an earlier one extended, or an exact repeat
        u = rng.random()
        if seen and u < 0.15:
            tok = seen[rng.integers(len(seen))].copy()
        elif seen and u < 0.7:
            base = seen[rng.integers(len(seen))]
            cut = int(rng.integers(0, len(base) + 1))
            tok = np.concatenate([base[:cut], rng.integers(0, 30, int(rng.integers(0, 6 * tpb)))]).astype(np.int64)
        else:
            tok = rng.integers(0, 30, int(rng.integers(0, 10 * tpb))).astype(np.int64)
        seen.append(tok)
        w = tier.put(tok, np.arange(len(tok) // tpb))
        got, inserted = flat.put(tok)
        assert (w.num_skipped, w.num_transferred, w.cpu_blocks.tolist()) == got, f"step {step}: put"
        pending.append((w, inserted))
        # callbacks run late and out of order
        while pending and rng.random() < 0.5:
            j = int(rng.integers(len(pending)))
            w2, ins2 = pending.pop(j)
            tier.complete(w2)
            flat.complete(ins2)
        # probes
        for _ in range(2):
            p = seen[rng.integers(len(seen))]
            if rng.random() < 0.5:
                p = np.concatenate([p[:int(rng.integers(0, len(p) + 1))], rng.integers(0, 30, 2 * tpb)]).astype(np.int64)
            m = tier.match(p)
            want = flat.match(flat.hashes(p))
            assert (m.num_matched, m.num_ready, [int(x) for x in m.blocks]) == want, f"step {step}: match"
    assert tier.pool.num_free == flat.pool.num_free
    assert tier.tree.total_blocks() == len(flat.map)


@pytest.mark.parametrize("seed,tpb,pool", [(1, 2, 4000), (2, 4, 4000), (3, 1, 4000), (4, 4, 120), (5, 2, 60)])
def test_tree_walk_equals_leading_present_blocks(seed, tpb, pool):
    random_history(seed, 300, tpb, pool)


class FlatTwoTier:
    """Both tiers as flat maps, with the two-tier put rule: D2H the blocks
    the CPU tier lacks, H2DISK the ones the SSD tier lacks, both takes or
    neither."""

    def __init__(self, n_cpu, n_ssd, tpb):
        self.c = FlatModel(n_cpu, tpb)
        self.s = FlatModel(n_ssd, tpb)

    def put(self, tok):
        h = self.c.hashes(tok)
        n = len(h)
        m_c = self.c.match(h)[0]
        m_s = self.s.match(h)[0]
        k, f2 = n - m_c, n - m_s
        if k == 0:
            return (0, 0, [], []), [], []
        got_c = self.c.pool.allocate(min(k, self.c.pool.num_free))
        got_s = self.s.pool.allocate(min(f2, self.s.pool.num_free))
        if len(got_c) < k or len(got_s) < f2:
            self.c.pool.recycle(got_c)
            self.s.pool.recycle(got_s)
            return (0, 0, [], []), [], []
        for x, c in zip(h[m_c:], got_c.tolist()):
            self.c.map[x] = [c, False]
        for x, c in zip(h[m_s:], got_s.tolist()):
            self.s.map[x] = [c, False]
        return (m_c, k, got_c.tolist(), got_s.tolist()), h[m_c:], h[m_s:]


@pytest.mark.parametrize("seed,n_cpu,n_ssd", [(7, 3000, 5000), (8, 200, 5000), (9, 3000, 150)])
def test_two_tier_tree_walks_equal_flat_maps(seed, n_cpu, n_ssd):
    tpb = 2
    rng = np.random.default_rng(seed)
    tt = CI.TwoTier(n_cpu, n_ssd, tpb)
    flat = FlatTwoTier(n_cpu, n_ssd, tpb)
    seen, pending = [], []
    for step in range(300):
        if seen and rng.random() < 0.6:
            base = seen[rng.integers(len(seen))]
            tok = np.concatenate([base[:int(rng.integers(0, len(base) + 1))],
                                  rng.integers(0, 20, int(rng.integers(0, 8 * tpb)))]).astype(np.int64)
        else:
            tok = rng.integers(0, 20, int(rng.integers(0, 12 * tpb))).astype(np.int64)
        seen.append(tok)
        r = tt.put(tok, np.arange(len(tok) // tpb))
        got, ins_c, ins_s = flat.put(tok)
        assert (r.num_skipped, r.num_transferred, r.cpu_blocks.tolist(), r.ssd_blocks.tolist()) == got, step
        pending.append((r, ins_c, ins_s))
        while pending and rng.random() < 0.5:
            r2, c2, s2 = pending.pop(int(rng.integers(len(pending))))
            tt.complete(r2)
            flat.c.complete(c2)
            flat.s.complete(s2)
    assert (tt.cpu.pool.num_free, tt.ssd.pool.num_free) == (flat.c.pool.num_free, flat.s.pool.num_free)
    assert (tt.cpu.tree.total_blocks(), tt.ssd.tree.total_blocks()) == (len(flat.c.map), len(flat.s.map))
