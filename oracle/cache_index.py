"""TEST INFRASTRUCTURE ONLY — CPU restatement of FlexKV's CPU-tier cache
index and put decision, the checker for flexkv_b200/csrc/block_index.cu.

Only tests/ and bench.py's CPU-baseline leg use this module.

Restates, in this module's own structure:
  * the prefix tree of block hashes: RadixTreeIndex.match_prefix
    (flexkv/cache/radixtree.py:143-195), insert (:202-256), RadixNode.split
    (:78-98), set_ready (:302-316), lock / unlock (:288-300);
  * the block pool: Mempool.allocate_blocks / recycle_blocks /
    _update_free_ids (flexkv/cache/mempool.py:28-55);
  * the CPU-tier put: GlobalCacheEngine.put (flexkv/cache/cache_engine.py:
    550-615) and _put_impl_local (:787-902) with the SSD and remote tiers
    off, and CacheEngine.take (:87-104) when eviction finds nothing to
    evict (every cached block still locked or not ready, or the caller has
    already made room);
  * the put callback: _transfer_callback -> CacheEngine.cleanup (:904-925,
    :83-85), which unlocks the inserted node and marks it ready;
  * the CPU-tier get: GlobalCacheEngine.get (:150-219) and _get_impl_local
    (:412-548) with the SSD tier off;
  * both with the SSD tier on (TwoTier): the put's D2H into new CPU blocks
    and H2DISK of the blocks the SSD tier lacks, and the get's legs, when
    neither tier's take() evicts.

Pinned by tests/golden/put_path.json, which tests/golden/make_put_golden.py
produced by running the reference's own GlobalCacheEngine.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import oracle as O


class Node:
    """One run of block hashes with their pool block ids (radixtree.py:41-126)."""

    __slots__ = ("hashes", "blocks", "ready", "locks", "parent", "children")

    def __init__(self, hashes: List[int], blocks: List[int], ready: bool, parent=None):
        self.hashes = hashes
        self.blocks = blocks
        self.ready = ready
        self.locks = 0
        self.parent = parent
        self.children: Dict[int, "Node"] = {}

    @property
    def size(self) -> int:
        return len(self.hashes)

    def is_root(self) -> bool:
        return self.parent is None

    def head(self) -> int:
        return self.hashes[0] if self.hashes else 0

    def split_at(self, length: int) -> "Node":
        """Cut this node after `length` blocks; the first part becomes a new
        parent in its place (radixtree.py:78-98)."""
        assert 0 < length < self.size and self.parent is not None
        top = Node(self.hashes[:length], self.blocks[:length], self.ready, self.parent)
        self.hashes = self.hashes[length:]
        self.blocks = self.blocks[length:]
        self.parent.children[top.head()] = top
        top.children[self.head()] = self
        self.parent = top
        return top


@dataclass
class Match:
    num_matched: int = 0
    num_ready: int = 0
    blocks: List[int] = field(default_factory=list)
    last: Optional[Node] = None
    last_len: int = 0


class PrefixTree:
    """Restatement of RadixTreeIndex without the eviction policy."""

    def __init__(self):
        self.root = Node([], [], True)

    def match(self, hashes: Sequence[int]) -> Match:
        """radixtree.py:143-195: walk children by the hash that follows each
        node; in the node where the walk stops, binary-search the matched
        length (block hashes are prefix-chained, so matches form a prefix)."""
        n = len(hashes)
        node, pos, ready, blocks = self.root, 0, 0, []
        last_len = 0
        while pos < n:
            nxt = pos + node.size
            child = node.children.get(hashes[nxt]) if nxt < n else None
            if child is not None:
                if node.ready:
                    ready += node.size
                pos = nxt
                blocks.extend(node.blocks)
                node = child
                continue
            matched = 0
            if not node.is_root():
                lo, hi = 0, min(node.size, n - pos)
                while lo < hi:
                    mid = (lo + hi) // 2
                    if node.hashes[mid] == hashes[pos + mid]:
                        lo = mid + 1
                    else:
                        hi = mid
                matched = lo
                blocks.extend(node.blocks[:matched])
            if node.ready:
                ready += matched
            last_len = matched
            pos += matched
            break
        return Match(pos, ready, blocks, node, last_len)

    def insert(self, hashes: Sequence[int], new_blocks: Sequence[int], ready: bool,
               m: Optional[Match] = None) -> Optional[Node]:
        """radixtree.py:202-256 with num_insert_blocks = all blocks."""
        if m is None:
            m = self.match(hashes)
        if m.num_matched >= len(hashes):
            return None
        assert len(new_blocks) == len(hashes) - m.num_matched
        parent = m.last
        assert m.last_len != 0 or parent.is_root()
        if m.last_len < parent.size:
            parent = parent.split_at(m.last_len)  # the matched part, now the attach point
        node = Node(list(hashes[m.num_matched:]), list(new_blocks), ready, parent)
        parent.children[node.head()] = node
        return node

    def set_ready(self, node: Node, length: int) -> None:
        """radixtree.py:302-316: mark `node` ready and, while `length` is not
        yet covered, its ancestors."""
        node.ready = True
        length -= node.size
        while length > 0:
            node = node.parent
            assert node is not None
            length -= node.size
            node.ready = True
        assert length <= 0

    def total_blocks(self) -> int:
        total, stack = 0, [self.root]
        while stack:
            x = stack.pop()
            total += x.size
            stack.extend(x.children.values())
        return total

    def total_ready(self) -> int:
        total, stack = 0, [self.root]
        while stack:
            x = stack.pop()
            total += x.size if x.ready else 0
            stack.extend(x.children.values())
        return total


class BlockPool:
    """Restatement of Mempool (mempool.py:9-63): ids are handed out in
    ascending order from a snapshot of the free set, refreshed only when a
    request does not fit in what is left of the snapshot."""

    def __init__(self, num_blocks: int):
        self.free = np.ones(num_blocks, dtype=bool)
        self.num_free = num_blocks
        self.ids = np.arange(num_blocks, dtype=np.int64)
        self.offset = 0

    def allocate(self, num: int) -> np.ndarray:
        if num < 0 or num > self.num_free:
            raise ValueError(f"cannot allocate {num} of {self.num_free} free blocks")
        if num > len(self.ids) - self.offset:
            self.ids = np.flatnonzero(self.free).astype(np.int64)
            self.offset = 0
        out = self.ids[self.offset:self.offset + num].copy()
        self.offset += num
        self.free[out] = False
        self.num_free -= num
        return out

    def recycle(self, ids: np.ndarray) -> None:
        ids = np.asarray(ids, dtype=np.int64)
        if self.free[ids].any():
            raise ValueError("recycling a free block")
        self.free[ids] = True
        self.num_free += len(ids)


@dataclass
class PutResult:
    num_skipped: int      # leading blocks already cached (GPU blocks not copied)
    num_transferred: int  # blocks copied GPU -> CPU (0 for an empty put)
    gpu_blocks: np.ndarray
    cpu_blocks: np.ndarray
    node: Optional[Node] = None
    node_size: int = 0


class CpuTier:
    """The CPU tier of GlobalCacheEngine: index + pool + put decision."""

    def __init__(self, num_blocks: int, tokens_per_block: int):
        self.tpb = tokens_per_block
        self.tree = PrefixTree()
        self.pool = BlockPool(num_blocks)

    def hashes(self, token_ids: np.ndarray) -> List[int]:
        aligned = (len(token_ids) // self.tpb) * self.tpb
        if aligned == 0:
            return []
        return [int(x) for x in O.gen_hashes(np.asarray(token_ids[:aligned], dtype=np.int64), self.tpb)]

    def match(self, token_ids: np.ndarray) -> Match:
        return self.tree.match(self.hashes(token_ids))

    def put(self, token_ids: np.ndarray, gpu_blocks: np.ndarray) -> PutResult:
        """cache_engine.py:550-615 and 787-902 (CPU tier): gpu_blocks has one
        GPU block per full block of token_ids (the reference derives it from
        the slot mapping, slot_mapping[::tpb] // tpb)."""
        h = self.hashes(token_ids)
        n = len(h)
        gpu_blocks = np.asarray(gpu_blocks, dtype=np.int64)[:n]
        empty = PutResult(0, 0, np.zeros(0, np.int64), np.zeros(0, np.int64))
        m = self.tree.match(h)
        skipped = min(m.num_matched, n)
        k = n - skipped
        if k == 0:
            return empty
        got = self.pool.allocate(min(k, self.pool.num_free))  # take(strict=False), nothing evicted
        if len(got) < k:
            self.pool.recycle(got)
            return empty
        node = self.tree.insert(h, got, ready=False, m=m)
        node.locks += 1
        return PutResult(skipped, k, gpu_blocks[skipped:].copy(), got, node, node.size)

    def complete(self, r: PutResult) -> None:
        """The put callback: unlock and mark the inserted blocks ready."""
        if r.node is None:
            return
        r.node.locks -= 1
        self.tree.set_ready(r.node, r.node_size)

    def get(self, token_ids: np.ndarray, gpu_blocks: np.ndarray, block_start: int = 0) -> PutResult:
        """cache_engine.py:150-219 and 412-548 (CPU tier, SSD off): the mask
        selects full blocks [block_start, n); gpu_blocks holds one GPU block
        per selected block.  The reference takes the first num_ready matched
        blocks (physical_blocks[:num_ready_matched_blocks]), keeps those in
        the selected range, and reads them into the leading GPU blocks.  A
        get changes neither the tree nor the pool (its lock and callback only
        bracket the copy)."""
        h = self.hashes(token_ids)
        n = len(h)
        gpu_blocks = np.asarray(gpu_blocks, dtype=np.int64)
        empty = PutResult(0, 0, np.zeros(0, np.int64), np.zeros(0, np.int64))
        if n == 0:
            return empty
        assert 0 <= block_start < n and len(gpu_blocks) >= n - block_start
        m = self.tree.match(h)
        ready = m.blocks[:m.num_ready][block_start:n]
        f = len(ready)
        if f == 0:
            return empty
        return PutResult(block_start, f, gpu_blocks[:f].copy(), np.asarray(ready, dtype=np.int64))


@dataclass
class TwoTierPut:
    num_skipped: int
    num_transferred: int
    gpu_blocks: np.ndarray        # D2H sources
    cpu_blocks: np.ndarray        # D2H destinations (new CPU blocks)
    h2disk_cpu: np.ndarray        # H2DISK sources (the reference's cpu_new[-frag2:])
    ssd_blocks: np.ndarray        # H2DISK destinations (new SSD blocks)
    cpu_node: Optional[Node] = None
    cpu_size: int = 0
    ssd_node: Optional[Node] = None
    ssd_size: int = 0


class TwoTier:
    """GlobalCacheEngine with the CPU and SSD tiers (cache_engine.py:787-902
    for puts, :412-548 for gets), when neither tier's take() evicts: every
    block still locked or not ready, or pools large enough."""

    def __init__(self, cpu_blocks: int, ssd_blocks: int, tokens_per_block: int):
        self.cpu = CpuTier(cpu_blocks, tokens_per_block)
        self.ssd = CpuTier(ssd_blocks, tokens_per_block)
        self.tpb = tokens_per_block

    def put(self, token_ids: np.ndarray, gpu_blocks: np.ndarray) -> TwoTierPut:
        h = self.cpu.hashes(token_ids)
        n = len(h)
        gpu_blocks = np.asarray(gpu_blocks, dtype=np.int64)[:n]
        z = np.zeros(0, np.int64)
        empty = TwoTierPut(0, 0, z, z, z, z)
        cm, sm = self.cpu.tree.match(h), self.ssd.tree.match(h)
        skipped = min(cm.num_matched, n)
        frag12 = n - skipped
        if frag12 == 0:
            return empty
        frag2 = n - min(sm.num_matched, n)
        cpu_new = self.cpu.pool.allocate(min(frag12, self.cpu.pool.num_free))
        ssd_new = self.ssd.pool.allocate(min(frag2, self.ssd.pool.num_free))
        if len(cpu_new) < frag12 or len(ssd_new) < frag2:
            self.cpu.pool.recycle(cpu_new)
            self.ssd.pool.recycle(ssd_new)
            return empty
        h2disk_cpu = cpu_new[-frag2:] if frag2 > 0 else z
        cnode = self.cpu.tree.insert(h, cpu_new, ready=False, m=cm)
        cnode.locks += 1
        snode = None
        if len(ssd_new):
            snode = self.ssd.tree.insert(h, ssd_new, ready=False, m=sm)
            snode.locks += 1
        return TwoTierPut(skipped, frag12, gpu_blocks[skipped:].copy(), cpu_new, h2disk_cpu.copy(), ssd_new,
                          cnode, cnode.size, snode, snode.size if snode else 0)

    def complete(self, r: TwoTierPut) -> None:
        """The put callback (cache_engine.py:904-916): both tiers' nodes."""
        for tier, node, size in ((self.cpu, r.cpu_node, r.cpu_size), (self.ssd, r.ssd_node, r.ssd_size)):
            if node is not None:
                node.locks -= 1
                tier.tree.set_ready(node, size)

    def get(self, token_ids: np.ndarray, gpu_blocks: np.ndarray, block_start: int = 0):
        """(num_transferred, [(kind, src_blocks, dst_blocks)...]) as the
        reference's _get_impl_local builds them; with nothing evicted the SSD
        tier never holds a ready block the CPU tier lacks, so the DISK2H leg
        stays empty and this equals CpuTier.get."""
        h = self.cpu.hashes(token_ids)
        n = len(h)
        if n == 0:
            return 0, []
        cm, sm = self.cpu.tree.match(h), self.ssd.tree.match(h)
        cpu_ready = cm.blocks[:cm.num_ready][block_start:n]
        ssd_ready = sm.blocks[:sm.num_ready][block_start:n]
        frag12 = max(len(cpu_ready), len(ssd_ready))
        frag1 = len(cpu_ready)
        frag2 = max(len(ssd_ready) - len(cpu_ready), 0)
        if frag12 == 0:
            return 0, []
        gpu_blocks = np.asarray(gpu_blocks, dtype=np.int64)
        ops = []
        if frag2 > 0:
            ops.append(("DISK2H", np.asarray(ssd_ready[-frag2:], np.int64), None))
        ops.append(("H2D", np.asarray(cpu_ready[:frag1], np.int64), gpu_blocks[:frag1].copy()))
        return frag12, ops
