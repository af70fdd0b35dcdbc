"""Shared helpers for the transfer tests: deterministic data, cases, and the
view-based restatement of the reference semantics used for golden vectors.

Data is a splitmix64 stream of the byte index (stable across numpy/torch
versions, so committed digests stay valid): word k of pool `seed` is
splitmix64(seed << 40 | k).
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (x + np.uint64(0x9E3779B97F4A7C15)) & M64
        z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & M64
        z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & M64
        return z ^ (z >> np.uint64(31))


def fill_bytes(nbytes: int, seed: int) -> np.ndarray:
    """Deterministic uint8 array of nbytes."""
    words = (nbytes + 7) // 8
    k = np.arange(words, dtype=np.uint64) | (np.uint64(seed) << np.uint64(40))
    return splitmix64(k).view(np.uint8)[:nbytes].copy()


def tokens(n: int, vocab: int, seed: int) -> np.ndarray:
    """Stable synthetic token ids in [0, vocab) as int64 (int32 ids widened,
    as the reference hashes int64 token tensors, hash.cpp:53)."""
    k = np.arange(n, dtype=np.uint64) | (np.uint64(seed) << np.uint64(40))
    return (splitmix64(k) % np.uint64(vocab)).astype(np.int32).astype(np.int64)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()


@dataclass
class Case:
    """One transfer configuration in reference terms (bf16 elements)."""
    name: str
    num_layers: int
    heads: int            # heads per rank on the GPU side
    head_dim: int
    tpb: int
    gpu_blocks: int
    cpu_blocks: int
    cpu_layout: str = "LAYERWISE"
    is_mla: bool = False
    tp: int = 1           # ranks sharing a CPU chunk
    layer_id: int = 0     # first layer of the op
    layer_gran: int = -1  # layers in the op (-1 = all)
    chunk_override: int = 0  # pass this chunk size instead of the layout's
    itemsize: int = 2

    @property
    def kv(self) -> int:
        return 1 if self.is_mla else 2

    @property
    def gran(self) -> int:
        return self.num_layers if self.layer_gran < 0 else self.layer_gran

    def gpu_layout(self) -> KVCacheLayout:
        return KVCacheLayout(KVCacheLayoutType.LAYERWISE, self.num_layers, self.gpu_blocks,
                             self.tpb, self.heads, self.head_dim, self.is_mla)

    def cpu_layout_obj(self) -> KVCacheLayout:
        heads_total = self.heads if self.is_mla else self.heads * self.tp
        return KVCacheLayout(KVCacheLayoutType[self.cpu_layout], self.num_layers, self.cpu_blocks,
                             self.tpb, heads_total, self.head_dim, self.is_mla)

    def strides(self) -> dict:
        """Byte strides as the reference workers derive them (worker.py:236-246,
        383-390)."""
        gl = self.gpu_layout().div_layer(self.num_layers)
        cl = self.cpu_layout_obj()
        e = self.itemsize
        gchunk = gl.get_chunk_size() * e
        return {
            "gpu_chunk": self.chunk_override or gchunk,
            "gpu_kv": gl.get_kv_stride() * e,
            "gpu_block": gl.get_block_stride() * e,
            "cpu_chunk": cl.get_chunk_size() * e,
            "cpu_layer": cl.get_layer_stride() * e,
            "cpu_kv": cl.get_kv_stride() * e,
            "cpu_block": cl.get_block_stride() * e,
            "gpu_layer_bytes": gl.get_total_elements() * e,
            "cpu_pool_bytes": cl.get_total_elements() * e,
        }


def view_transfer(case: Case, gpu_layers: List[np.ndarray], cpu_pool: np.ndarray,
                  gpu_ids: np.ndarray, cpu_ids: np.ndarray, h2d: bool, rank: int = 0) -> None:
    """Independent restatement of the reference copy through array views of
    the layouts (the host-side torch gather/scatter path): for each op layer
    l, kv half k and pair i, move the first 16*floor(chunk/16) bytes of GPU
    chunk [k, gpu_ids[i]] of layer l to the CPU chunk at layer
    layer_id + l, byte offset rank*gpu_chunk (0 for MLA)."""
    st = case.strides()
    copy = (st["gpu_chunk"] // 16) * 16
    off = 0 if case.is_mla else rank * st["gpu_chunk"]
    for l in range(case.gran):
        gl = gpu_layers[l]
        cl = case.layer_id + l
        for k in range(case.kv):
            for g, c in zip(gpu_ids.tolist(), cpu_ids.tolist()):
                gs = k * st["gpu_kv"] + g * st["gpu_block"]
                cs = cl * st["cpu_layer"] + k * st["cpu_kv"] + c * st["cpu_block"] + off
                if h2d:
                    gl[gs:gs + copy] = cpu_pool[cs:cs + copy]
                else:
                    cpu_pool[cs:cs + copy] = gl[gs:gs + copy]


def place_segments(rng, lens: List[int], pool: int) -> List[int]:
    """Start ids for segments of the given lengths, disjoint inside
    [0, pool): segments are laid out in a random order separated by random
    gaps that share the pool's free space."""
    n = sum(lens)
    assert n <= pool, "pool smaller than the requested blocks"
    k = len(lens)
    cuts = np.sort(rng.integers(0, pool - n + 1, k))
    gaps = np.diff(np.concatenate([[0], cuts]))
    starts = [0] * k
    pos = 0
    for j, idx in enumerate(rng.permutation(k)):
        pos += int(gaps[j])
        starts[idx] = pos
        pos += lens[idx]
    return starts


def make_ids(n: int, gpu_pool: int, cpu_pool: int, seed: int, run_frac: float = 0.0,
             max_run: int = 64, distinct: bool = True):
    """Block-id pairs: with run_frac > 0, that fraction of the n blocks sits
    in joint runs (both ids advance by one) of length U[1, max_run]; the
    rest are scattered singletons; run order is shuffled, runs stay intact.
    Ids are distinct on both sides when `distinct`."""
    rng = np.random.default_rng(seed)
    if not distinct:
        return (rng.integers(0, gpu_pool, n).astype(np.int64),
                rng.integers(0, cpu_pool, n).astype(np.int64))
    n_run = int(round(n * run_frac))
    lens = []
    left = n_run
    while left > 0:
        r = int(min(left, rng.integers(1, max_run + 1)))
        lens.append(r)
        left -= r
    lens += [1] * (n - n_run)

    def segments(pool: int) -> List[int]:
        return place_segments(rng, lens, pool)

    gs, cs = segments(gpu_pool), segments(cpu_pool)
    order = rng.permutation(len(lens))
    gids, cids = [], []
    for idx in order:
        r = lens[idx]
        gids += list(range(gs[idx], gs[idx] + r))
        cids += list(range(cs[idx], cs[idx] + r))
    return np.array(gids, dtype=np.int64), np.array(cids, dtype=np.int64)
