"""The CPU tier's block index, block pool and fused put path on the device,
over the C ABI ``fkv_cache_index_*`` (csrc/block_index.cu).

Replaces, for the CPU tier of FlexKV's cache engine:
  * ``GlobalCacheEngine.put`` / ``_put_impl_local`` (flexkv/cache/cache_engine.py:
    550-615, 787-902, SSD and remote tiers off): ``CpuCacheIndex.put_requests``
    takes the same (token_ids, token_mask, slot_mapping) per request and gives
    the same return mask, and performs the D2H copy itself;
  * ``CacheEngine.match / insert / take / recycle / cleanup``
    (cache_engine.py:63-107) over ``RadixTreeIndex`` (flexkv/cache/radixtree.py)
    and ``Mempool`` (flexkv/cache/mempool.py): ``match``, ``put``, ``take``,
    ``recycle``, ``set_ready``.

Requests are batched: a list takes effect in order, exactly as consecutive
calls of the reference would, but runs as one stream of kernels (hash ->
match -> allocate -> insert -> copy -> ready) with no host round trip.
Eviction stays with the caller (``remove`` + ``recycle``); a put that the
pool cannot hold comes back empty, as the reference's does when nothing is
evictable.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import TransferDesc, check


@dataclass
class KVLayout:
    """Layout of the D2H copy, in the terms of ``transfer_kv_blocks``:
    per-layer GPU pointers (int64, already sliced to the copied layers),
    byte strides, the page-locked host pool and the chunk size."""

    gpu_layer_ptrs: torch.Tensor
    gpu_kv_stride_in_bytes: int
    gpu_block_stride_in_bytes: int
    cpu_tensor: torch.Tensor
    cpu_kv_stride_in_bytes: int
    cpu_layer_stride_in_bytes: int
    cpu_block_stride_in_bytes: int
    chunk_size_in_bytes: int
    is_mla: bool = False
    transfer_sms: int = -1
    gpu_layer_bytes: int = 0

    def desc(self, host_to_device: bool = False) -> TransferDesc:
        ptrs = self.gpu_layer_ptrs
        if ptrs.dtype != torch.int64 or ptrs.is_cuda:
            raise RuntimeError("gpu_layer_ptrs must be an int64 CPU tensor")
        ptrs = ptrs.contiguous()
        self._ptrs = ptrs  # keep alive for the call
        d = TransferDesc()
        _lib.load().fkv_transfer_desc_init(ctypes.byref(d))
        d.num_layers = ptrs.numel()
        d.is_host_to_device = int(bool(host_to_device))
        d.is_mla = int(bool(self.is_mla))
        d.transfer_sms = int(self.transfer_sms)
        d.gpu_layer_ptrs = ptrs.data_ptr()
        d.cpu_ptr = self.cpu_tensor.data_ptr()
        d.gpu_kv_stride_in_bytes = int(self.gpu_kv_stride_in_bytes)
        d.gpu_block_stride_in_bytes = int(self.gpu_block_stride_in_bytes)
        d.cpu_kv_stride_in_bytes = int(self.cpu_kv_stride_in_bytes)
        d.cpu_layer_stride_in_bytes = int(self.cpu_layer_stride_in_bytes)
        d.cpu_block_stride_in_bytes = int(self.cpu_block_stride_in_bytes)
        d.chunk_size_in_bytes = int(self.chunk_size_in_bytes)
        d.cpu_pool_bytes = self.cpu_tensor.numel() * self.cpu_tensor.element_size()
        d.gpu_layer_bytes = int(self.gpu_layer_bytes)
        return d


class MatchBatch:
    """Results of a batched match: per-request counts, and the pool blocks of
    every matched block in one flat array (block offsets blk_off)."""

    def __init__(self, num_matched: np.ndarray, num_ready: np.ndarray, phys_flat: np.ndarray,
                 blk_off: np.ndarray):
        self.num_matched = num_matched   # [R] leading blocks cached (num_matched_blocks)
        self.num_ready = num_ready       # [R] of them ready (num_ready_matched_blocks)
        self.phys_flat = phys_flat       # per block: its pool block, -1 past the match
        self.blk_off = blk_off

    @property
    def physical_blocks(self) -> List[np.ndarray]:
        """Per request: pool blocks of the matched prefix."""
        o = self.blk_off
        return [self.phys_flat[o[r]:o[r] + int(m)] for r, m in enumerate(self.num_matched)]


class PutBatch:
    """Results of a batched put, flat per block of the batch (block offsets
    blk_off); per-request views on demand."""

    def __init__(self, num_skipped, num_transferred, cpu_flat, gpu_flat, hashes_flat, blk_off):
        self.num_skipped = num_skipped          # [R] leading blocks already cached, not copied
        self.num_transferred = num_transferred  # [R] blocks copied (0: empty put)
        self.cpu_flat = cpu_flat                # per block: pool block it went to, -1 if not copied
        self.gpu_flat = gpu_flat                # per block: its GPU block
        self.hashes_flat = hashes_flat          # per block: its hash (uint64)
        self.blk_off = blk_off

    def _moved(self, flat) -> List[np.ndarray]:
        o = self.blk_off
        return [flat[o[r] + int(s):o[r] + int(s) + int(t)]
                for r, (s, t) in enumerate(zip(self.num_skipped, self.num_transferred))]

    @property
    def cpu_blocks(self) -> List[np.ndarray]:
        """Per request: pool blocks the copied blocks went to."""
        return self._moved(self.cpu_flat)

    @property
    def gpu_blocks(self) -> List[np.ndarray]:
        """Per request: the GPU blocks copied."""
        return self._moved(self.gpu_flat)

    @property
    def block_hashes(self) -> List[np.ndarray]:
        """Per request: every full block's hash."""
        o = self.blk_off
        return [self.hashes_flat[o[r]:o[r + 1]] for r in range(len(o) - 1)]

    def return_mask(self, r: int, num_tokens: int, tokens_per_block: int) -> torch.Tensor:
        """The reference put's return mask: True over the copied tokens
        (cache_engine.py:600-602)."""
        m = torch.zeros(num_tokens, dtype=torch.bool)
        a = int(self.num_skipped[r]) * tokens_per_block
        m[a:a + int(self.num_transferred[r]) * tokens_per_block] = True
        return m


class GetBatch:
    """Results of a batched get: per request the first block read
    (block_starts) and how many were read, and per GPU entry the pool block
    read into it (-1 if none; offsets goff)."""

    def __init__(self, block_starts, num_transferred, cpu_flat, gpu_flat, goff):
        self.block_starts = block_starts
        self.num_transferred = num_transferred
        self.cpu_flat = cpu_flat
        self.gpu_flat = gpu_flat
        self.goff = goff

    @property
    def cpu_blocks(self) -> List[np.ndarray]:
        """Per request: the pool blocks read."""
        return [self.cpu_flat[self.goff[r]:self.goff[r] + int(t)] for r, t in enumerate(self.num_transferred)]

    @property
    def gpu_blocks(self) -> List[np.ndarray]:
        """Per request: the GPU blocks written."""
        return [self.gpu_flat[self.goff[r]:self.goff[r] + int(t)] for r, t in enumerate(self.num_transferred)]

    def return_mask(self, r: int, num_tokens: int, tokens_per_block: int) -> torch.Tensor:
        """The reference get's return mask (cache_engine.py:201-203)."""
        m = torch.zeros(num_tokens, dtype=torch.bool)
        a = int(self.block_starts[r]) * tokens_per_block
        m[a:a + int(self.num_transferred[r]) * tokens_per_block] = True
        return m


class TwoTierPutBatch(PutBatch):
    """A put with the SSD tier on: PutBatch plus, per block, the new SSD
    block (-1 if the SSD tier already held it or the put was empty)."""

    def __init__(self, num_skipped, num_transferred, num_to_ssd, cpu_flat, gpu_flat, ssd_flat, hashes_flat,
                 blk_off):
        super().__init__(num_skipped, num_transferred, cpu_flat, gpu_flat, hashes_flat, blk_off)
        self.num_to_ssd = num_to_ssd
        self.ssd_flat = ssd_flat

    def _to_ssd(self, flat) -> List[np.ndarray]:
        o = self.blk_off
        return [flat[o[r + 1] - int(f):o[r + 1]] for r, f in enumerate(self.num_to_ssd)]

    @property
    def ssd_blocks(self) -> List[np.ndarray]:
        """Per request: the new SSD blocks (the H2DISK destinations)."""
        return self._to_ssd(self.ssd_flat)

    @property
    def h2disk_cpu_blocks(self) -> List[np.ndarray]:
        """Per request: the CPU blocks written to them (the H2DISK sources)."""
        return self._to_ssd(self.cpu_flat)


@dataclass
class SsdTier:
    """The SSD tier of a two-tier put: its index, its SSD context and the
    arguments of c_ext.transfer_kv_blocks_ssd (worker.py:512-575)."""

    index: "CpuCacheIndex"
    ioctx: object              # c_ext.SSDIOCTX
    strides: object            # flexkv_b200.ssd.SsdStrides
    num_layers: int
    num_blocks_per_file: int
    round_robin: int = 1
    threads_per_device: int = 16
    is_mla: bool = False


def _pack_tokens(token_ids: Sequence) -> Tuple[object, np.ndarray, int]:
    """Concatenate a batch of token sequences (int64; numpy, host or CUDA
    tensors) and give the token offsets.  Returns (buffer kept alive,
    offsets, pointer)."""
    if all(isinstance(t, np.ndarray) for t in token_ids):
        lens = np.fromiter((t.size for t in token_ids), dtype=np.int64, count=len(token_ids))
        buf = np.ascontiguousarray(np.concatenate(token_ids).astype(np.int64, copy=False)) \
            if len(token_ids) and lens.sum() else np.zeros(1, dtype=np.int64)
        offsets = np.zeros(len(token_ids) + 1, dtype=np.int64)
        np.cumsum(lens, out=offsets[1:])
        return buf, offsets, buf.ctypes.data
    seqs = [t if isinstance(t, torch.Tensor) else torch.as_tensor(np.asarray(t, dtype=np.int64))
            for t in token_ids]
    lens = np.array([int(t.numel()) for t in seqs], dtype=np.int64)
    offsets = np.zeros(len(seqs) + 1, dtype=np.int64)
    np.cumsum(lens, out=offsets[1:])
    dev = next((t.device for t in seqs if t.is_cuda), torch.device("cpu"))
    parts = [t.reshape(-1).to(dtype=torch.int64, device=dev) for t in seqs]
    buf = torch.cat(parts) if parts and offsets[-1] > 0 else torch.zeros(1, dtype=torch.int64, device=dev)
    return buf, offsets, buf.data_ptr()


def _blk_off(offsets: np.ndarray, tpb: int) -> np.ndarray:
    out = np.zeros(len(offsets), dtype=np.int64)
    np.cumsum((offsets[1:] - offsets[:-1]) // tpb, out=out[1:])
    return out


class CpuCacheIndex:
    """Block index + block pool of the CPU tier, resident on one GPU."""

    def __init__(self, num_total_blocks: int, tokens_per_block: int, device: Optional[int] = None):
        if tokens_per_block <= 0:
            raise ValueError("tokens_per_block must be positive")
        self.tokens_per_block = int(tokens_per_block)
        self.num_total_blocks = int(num_total_blocks)
        dev = torch.cuda.current_device() if device is None else int(device)
        self.device = dev
        h = ctypes.c_void_p()
        check(_lib.load().fkv_cache_index_create(dev, self.num_total_blocks, self.tokens_per_block,
                                                 ctypes.byref(h)), "CpuCacheIndex")
        self._h = h

    def _stream(self) -> int:
        with torch.cuda.device(self.device):
            return int(torch.cuda.current_stream().cuda_stream)

    def match(self, token_ids: Sequence) -> MatchBatch:
        """match_prefix of every sequence (radixtree.py:143-195)."""
        buf, offsets, ptr = _pack_tokens(token_ids)
        return self.match_packed(ptr, offsets)

    def match_packed(self, token_ptr: int, seq_offsets: np.ndarray) -> MatchBatch:
        """match over a packed batch: token_ptr addresses the int64 tokens of
        all sequences (host or device), seq_offsets (R+1, host) delimits
        them."""
        offsets = np.ascontiguousarray(seq_offsets, dtype=np.int64)
        R = len(offsets) - 1
        blk = _blk_off(offsets, self.tokens_per_block)
        nb = int(blk[-1])
        nm = np.zeros(R, dtype=np.int64)
        nr = np.zeros(R, dtype=np.int64)
        phys = np.full(max(nb, 1), -1, dtype=np.int64)
        check(_lib.load().fkv_cache_index_match(self._h, token_ptr, offsets.ctypes.data, R, nm.ctypes.data,
                                                nr.ctypes.data, phys.ctypes.data, self._stream()),
              "CpuCacheIndex.match")
        return MatchBatch(nm, nr, phys[:nb], blk)

    def put(self, token_ids: Sequence, gpu_block_ids: Sequence, layout: KVLayout,
            mark_ready: bool = True, synchronous: bool = True) -> PutBatch:
        """Puts of the CPU tier for a batch of requests, in order
        (cache_engine.py:787-902): request r's full blocks are hashed, its
        cached prefix is skipped, pool blocks are taken for the rest, which
        are inserted (not ready), copied from the GPU blocks
        gpu_block_ids[r] (one per full block) and, with mark_ready, marked
        ready once the copy is done (the put callback).  Returns when the
        copies are complete, or with synchronous=False as soon as the
        decisions are known, the copies still running on the current
        stream (wait on it before reusing the blocks)."""
        if len(token_ids) != len(gpu_block_ids):
            raise ValueError("one gpu block list per request")
        buf, offsets, ptr = _pack_tokens(token_ids)
        nblk = (offsets[1:] - offsets[:-1]) // self.tokens_per_block
        glen = np.fromiter((len(g) for g in gpu_block_ids), dtype=np.int64, count=len(gpu_block_ids))
        bad = np.flatnonzero(glen != nblk)
        if len(bad):
            r = int(bad[0])
            raise ValueError(f"request {r}: {glen[r]} gpu blocks for {nblk[r]} full blocks")
        parts = [np.asarray(g.cpu() if isinstance(g, torch.Tensor) else g, dtype=np.int64).reshape(-1)
                 for g in gpu_block_ids]
        gids = np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)
        return self.put_packed(ptr, offsets, gids, layout, mark_ready, synchronous)

    def put_packed(self, token_ptr: int, seq_offsets: np.ndarray, gpu_block_ids: np.ndarray,
                   layout: KVLayout, mark_ready: bool = True, synchronous: bool = True) -> PutBatch:
        """put over a packed batch: token_ptr addresses the int64 tokens of
        all sequences (host or device), seq_offsets (R+1, host) delimits
        them, gpu_block_ids holds one GPU block per full block of the batch,
        sequence by sequence."""
        offsets = np.ascontiguousarray(seq_offsets, dtype=np.int64)
        R = len(offsets) - 1
        blk = _blk_off(offsets, self.tokens_per_block)
        nb = int(blk[-1])
        gids = np.ascontiguousarray(gpu_block_ids, dtype=np.int64).reshape(-1)
        if len(gids) != nb:
            raise ValueError(f"{len(gids)} gpu blocks for {nb} full blocks in the batch")
        if nb == 0:
            gids = np.zeros(1, dtype=np.int64)
        nsk = np.zeros(R, dtype=np.int64)
        ntr = np.zeros(R, dtype=np.int64)
        cpu = np.empty(max(nb, 1), dtype=np.int64)
        hashes = np.empty(max(nb, 1), dtype=np.uint64)
        d = layout.desc()
        check(_lib.load().fkv_cache_index_put(self._h, token_ptr, offsets.ctypes.data, R, gids.ctypes.data,
                                              ctypes.byref(d), int(bool(mark_ready)), int(bool(synchronous)),
                                              nsk.ctypes.data,
                                              ntr.ctypes.data, cpu.ctypes.data, hashes.ctypes.data,
                                              self._stream()),
              "CpuCacheIndex.put")
        return PutBatch(nsk, ntr, cpu[:nb], gids[:nb], hashes[:nb], blk)

    def get(self, token_ids: Sequence, gpu_block_ids: Sequence, layout: KVLayout,
            block_starts: Optional[Sequence[int]] = None, synchronous: bool = True,
            layer_granularity: int = -1, group_events: Optional[Sequence] = None) -> GetBatch:
        """Gets of the CPU tier for a batch of requests (cache_engine.py:
        412-548, SSD off): request r selects its full blocks from
        block_starts[r] (default 0) on and brings one GPU block per selected
        block; its ready cached blocks in that range are read into the
        leading GPU blocks.  Returns when the copies are complete (or, with
        synchronous=False, once the decisions are known).  layer_granularity
        copies the layers in groups of that many, in order, and records
        group_events[i] (torch.cuda.Event) after group i, for a prefill
        that starts on the first layers while later ones load."""
        if len(token_ids) != len(gpu_block_ids):
            raise ValueError("one gpu block list per request")
        buf, offsets, ptr = _pack_tokens(token_ids)
        parts = [np.asarray(g.cpu() if isinstance(g, torch.Tensor) else g, dtype=np.int64).reshape(-1)
                 for g in gpu_block_ids]
        gids = np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)
        return self.get_packed(ptr, offsets, gids, layout, block_starts, synchronous, layer_granularity,
                               group_events)

    def get_packed(self, token_ptr: int, seq_offsets: np.ndarray, gpu_block_ids: np.ndarray, layout: KVLayout,
                   block_starts: Optional[Sequence[int]] = None, synchronous: bool = True,
                   layer_granularity: int = -1, group_events: Optional[Sequence] = None) -> GetBatch:
        """get over a packed batch (as put_packed; gpu_block_ids holds
        n_r - block_starts[r] GPU blocks per request)."""
        offsets = np.ascontiguousarray(seq_offsets, dtype=np.int64)
        R = len(offsets) - 1
        nblk = (offsets[1:] - offsets[:-1]) // self.tokens_per_block
        starts = np.zeros(R, dtype=np.int64) if block_starts is None else \
            np.ascontiguousarray(block_starts, dtype=np.int64).reshape(-1)
        if len(starts) != R:
            raise ValueError("one block start per request")
        starts = np.where(nblk > 0, starts, 0)
        if ((starts < 0) | ((nblk > 0) & (starts >= nblk))).any():
            raise ValueError("block starts must lie in [0, blocks)")
        goff = np.zeros(R + 1, dtype=np.int64)
        np.cumsum(nblk - starts, out=goff[1:])
        gids = np.ascontiguousarray(gpu_block_ids, dtype=np.int64).reshape(-1)
        if len(gids) != goff[-1]:
            raise ValueError(f"{len(gids)} gpu blocks for {goff[-1]} selected blocks in the batch")
        ng = int(goff[-1])
        gbuf = gids if ng else np.zeros(1, dtype=np.int64)
        moved = np.zeros(R, dtype=np.int64)
        cpu = np.full(max(ng, 1), -1, dtype=np.int64)
        d = layout.desc(host_to_device=True)
        ev = None
        if group_events is not None:
            handles = []
            for e in group_events:
                if not e.cuda_event:  # torch creates the CUDA event on its first record
                    e.record()
                handles.append(e.cuda_event)
            ev = (ctypes.c_void_p * len(handles))(*handles)
        check(_lib.load().fkv_cache_index_get(self._h, token_ptr, offsets.ctypes.data, R, starts.ctypes.data,
                                              gbuf.ctypes.data, ctypes.byref(d), int(layer_granularity), ev,
                                              int(bool(synchronous)), moved.ctypes.data,
                                              cpu.ctypes.data, self._stream()),
              "CpuCacheIndex.get")
        return GetBatch(starts, moved, cpu[:ng], gids, goff)

    def get_requests(self, requests: Sequence[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
                     layout: KVLayout, synchronous: bool = True, layer_granularity: int = -1,
                     group_events: Optional[Sequence] = None) -> Tuple[List[torch.Tensor], GetBatch]:
        """``GlobalCacheEngine.get(request_id, token_ids, token_mask,
        slot_mapping)`` for a batch (cache_engine.py:150-219, CPU tier):
        the mask selects a suffix of the full blocks that ends at the last
        full block; the GPU block of each selected block is
        slot_mapping[::tpb] // tpb.  Returns the reference's return masks and
        the batch result."""
        tpb = self.tokens_per_block
        toks, gids, starts, lens = [], [], [], []
        for r, (token_ids, token_mask, slot_mapping) in enumerate(requests):
            token_ids = torch.as_tensor(token_ids)
            token_mask = torch.as_tensor(token_mask, dtype=torch.bool).clone()
            slot_mapping = torch.as_tensor(slot_mapping)
            if len(token_ids) != len(token_mask) or len(slot_mapping) != int(token_mask.sum()):
                raise ValueError(f"request {r}: lengths of token_ids, token_mask and slot_mapping disagree")
            aligned = (len(token_ids) // tpb) * tpb
            token_mask[aligned:] = False
            idx = torch.nonzero(token_mask).flatten()
            bs = int(idx[0]) // tpb if len(idx) else 0
            be = int(idx[-1]) // tpb + 1 if len(idx) else 0
            if be != aligned // tpb:  # cache_engine.py:169
                raise ValueError(f"request {r}: the token mask must reach the last full block")
            lens.append(len(token_ids))
            toks.append(token_ids[:aligned].to(torch.int64).numpy())
            starts.append(bs)
            gids.append((slot_mapping[::tpb][:be - bs] // tpb).cpu().numpy().astype(np.int64))
        res = self.get(toks, gids, layout, starts, synchronous, layer_granularity, group_events)
        return [res.return_mask(r, lens[r], tpb) for r in range(len(lens))], res

    def put_two_tier(self, ssd: SsdTier, token_ids: Sequence, gpu_block_ids: Sequence, layout: KVLayout,
                     mark_ready: bool = True) -> TwoTierPutBatch:
        """Puts with the SSD tier on (cache_engine.py:787-902): the decisions
        of both tiers on the device (this index is the CPU tier's), the D2H
        copy, then the H2DISK leg through the SSD tier for the blocks the SSD
        tier lacked, and with mark_ready both tiers' blocks marked ready (the
        put callback).  Returns when the SSD writes are done.  If the SSD
        writes fail, the SSD tier's new entries are removed and their blocks
        recycled before the error propagates; the CPU tier keeps its part."""
        from . import c_ext
        if len(token_ids) != len(gpu_block_ids):
            raise ValueError("one gpu block list per request")
        buf, offsets, ptr = _pack_tokens(token_ids)
        nblk = (offsets[1:] - offsets[:-1]) // self.tokens_per_block
        parts = [np.asarray(g.cpu() if isinstance(g, torch.Tensor) else g, dtype=np.int64).reshape(-1)
                 for g in gpu_block_ids]
        if any(len(g) != n for g, n in zip(parts, nblk)):
            raise ValueError("one gpu block per full block")
        gids = np.ascontiguousarray(np.concatenate(parts) if parts else np.zeros(0, np.int64))
        R = len(offsets) - 1
        blk = _blk_off(offsets, self.tokens_per_block)
        nb = int(blk[-1])
        gbuf = gids if nb else np.zeros(1, dtype=np.int64)
        nsk, ntr, nss = (np.zeros(R, dtype=np.int64) for _ in range(3))
        cpu = np.full(max(nb, 1), -1, dtype=np.int64)
        ssd_ids = np.full(max(nb, 1), -1, dtype=np.int64)
        hashes = np.zeros(max(nb, 1), dtype=np.uint64)
        d = layout.desc()
        check(_lib.load().fkv_cache_index_put2(self._h, ssd.index._h, ptr, offsets.ctypes.data, R, gbuf.ctypes.data,
                                               ctypes.byref(d), int(bool(mark_ready)), nsk.ctypes.data,
                                               ntr.ctypes.data, nss.ctypes.data, cpu.ctypes.data,
                                               ssd_ids.ctypes.data, hashes.ctypes.data, self._stream()),
              "CpuCacheIndex.put_two_tier")
        res = TwoTierPutBatch(nsk, ntr, nss, cpu[:nb], gids[:nb], ssd_ids[:nb], hashes[:nb], blk)
        sel = np.flatnonzero(ssd_ids[:nb] >= 0)
        if len(sel):
            st = ssd.strides
            try:
                c_ext.transfer_kv_blocks_ssd(
                    ssd.ioctx, list(range(ssd.num_layers)), layout.cpu_tensor.data_ptr(),
                    np.ascontiguousarray(ssd_ids[sel]), np.ascontiguousarray(cpu[sel]),
                    st.cpu_layer_stride_in_bytes, st.cpu_kv_stride_in_bytes, st.ssd_layer_stride_in_bytes,
                    st.ssd_kv_stride_in_bytes, st.chunk_size_in_bytes, st.block_stride_in_bytes, False,
                    ssd.num_blocks_per_file, ssd.round_robin, ssd.threads_per_device, ssd.is_mla,
                    cpu_pool_bytes=layout.cpu_tensor.numel() * layout.cpu_tensor.element_size())
            except Exception:
                # The SSD tier never received these blocks: take its new
                # entries out again and give their SSD blocks back, so no
                # entry points at a block that was never written.  The CPU
                # tier's part of the put (D2H, ready marks) stands.
                held = ssd.index.remove(hashes[sel])
                ssd.index.recycle(held[held >= 0])
                raise
            if mark_ready:
                ssd.index.set_ready(hashes[sel])
        return res

    def put_requests(self, requests: Sequence[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
                     layout: KVLayout, mark_ready: bool = True,
                     synchronous: bool = True) -> Tuple[List[torch.Tensor], PutBatch]:
        """``GlobalCacheEngine.put(request_id, token_ids, token_mask,
        slot_mapping)`` for a batch (cache_engine.py:550-615, CPU tier):
        tokens past the last full block are ignored, the mask must select a
        prefix of the full blocks, and the GPU block of each block is
        slot_mapping[::tpb] // tpb.  Returns the reference's return masks
        and the batch result."""
        tpb = self.tokens_per_block
        toks, gids, lens = [], [], []
        for r, (token_ids, token_mask, slot_mapping) in enumerate(requests):
            token_ids = torch.as_tensor(token_ids)
            token_mask = torch.as_tensor(token_mask, dtype=torch.bool).clone()
            slot_mapping = torch.as_tensor(slot_mapping)
            if token_ids.ndim != 1 or token_mask.ndim != 1 or slot_mapping.ndim != 1:
                raise ValueError(f"request {r}: token_ids, token_mask and slot_mapping must be 1-D")
            if len(token_ids) != len(token_mask) or len(slot_mapping) != int(token_mask.sum()):
                raise ValueError(f"request {r}: lengths of token_ids, token_mask and slot_mapping disagree")
            aligned = (len(token_ids) // tpb) * tpb
            token_mask[aligned:] = False
            idx = torch.nonzero(token_mask).flatten()
            end = int(idx[-1]) // tpb + 1 if len(idx) else 0
            if len(idx) and int(idx[0]) // tpb != 0:
                raise ValueError(f"request {r}: the token mask must start at the first block")
            nfull = aligned // tpb
            if end not in (0, nfull):
                raise ValueError(f"request {r}: the token mask must cover every full block or none")
            lens.append(len(token_ids))
            if end == 0:  # nothing selected: an empty put
                toks.append(torch.zeros(0, dtype=torch.int64))
                gids.append(np.zeros(0, dtype=np.int64))
                continue
            toks.append(token_ids[:aligned].to(torch.int64))
            gids.append((slot_mapping[::tpb][:nfull] // tpb).cpu().numpy().astype(np.int64))
        res = self.put(toks, gids, layout, mark_ready=mark_ready, synchronous=synchronous)
        masks = [res.return_mask(r, lens[r], tpb) for r in range(len(lens))]
        return masks, res

    def set_ready(self, block_hashes, ready: bool = True) -> int:
        h = np.ascontiguousarray(np.asarray(block_hashes, dtype=np.uint64).reshape(-1))
        found = ctypes.c_int64(0)
        check(_lib.load().fkv_cache_index_set_ready(self._h, h.ctypes.data, len(h), int(bool(ready)),
                                                    ctypes.byref(found), self._stream()),
              "CpuCacheIndex.set_ready")
        return int(found.value)

    def remove(self, block_hashes) -> np.ndarray:
        """Drop cached blocks (the caller's eviction); returns the pool block
        each held (-1 if not cached).  Recycle them to free them."""
        h = np.ascontiguousarray(np.asarray(block_hashes, dtype=np.uint64).reshape(-1))
        out = np.full(max(len(h), 1), -1, dtype=np.int64)
        check(_lib.load().fkv_cache_index_remove(self._h, h.ctypes.data, len(h), out.ctypes.data,
                                                 self._stream()), "CpuCacheIndex.remove")
        return out[:len(h)]

    def recycle(self, block_ids) -> None:
        """Mempool.recycle_blocks (mempool.py:44-51)."""
        ids = np.ascontiguousarray(np.asarray(block_ids.cpu() if isinstance(block_ids, torch.Tensor)
                                              else block_ids, dtype=np.int64).reshape(-1))
        check(_lib.load().fkv_cache_index_recycle(self._h, ids.ctypes.data, len(ids), self._stream()),
              "CpuCacheIndex.recycle")

    def take(self, num: int) -> np.ndarray:
        """CacheEngine.take(num, strict=False) with nothing to evict."""
        out = np.zeros(max(int(num), 1), dtype=np.int64)
        got = ctypes.c_int64(0)
        check(_lib.load().fkv_cache_index_take(self._h, int(num), out.ctypes.data, ctypes.byref(got),
                                               self._stream()), "CpuCacheIndex.take")
        return out[:got.value].copy()

    def stats(self) -> dict:
        out = np.zeros(7, dtype=np.int64)
        check(_lib.load().fkv_cache_index_stats(self._h, out.ctypes.data, self._stream()),
              "CpuCacheIndex.stats")
        keys = ("num_free_blocks", "total_cached_blocks", "total_ready_blocks", "pool_snapshot_len",
                "pool_snapshot_offset", "deleted_slots", "table_slots")
        return dict(zip(keys, (int(x) for x in out)))

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            _lib.load().fkv_cache_index_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
