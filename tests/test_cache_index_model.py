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
