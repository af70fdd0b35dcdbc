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

    def desc(self) -> TransferDesc:
        ptrs = self.gpu_layer_ptrs
        if ptrs.dtype != torch.int64 or ptrs.is_cuda:
            raise RuntimeError("gpu_layer_ptrs must be an int64 CPU tensor")
        ptrs = ptrs.contiguous()
        self._ptrs = ptrs  # keep alive for the call
        d = TransferDesc()
        _lib.load().fkv_transfer_desc_init(ctypes.byref(d))
        d.num_layers = ptrs.numel()
        d.is_host_to_device = 0
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


@dataclass
class MatchBatch:
    num_matched: np.ndarray        # [R] leading blocks cached (num_matched_blocks)
    num_ready: np.ndarray          # [R] of them ready (num_ready_matched_blocks)
    physical_blocks: List[np.ndarray]  # per request: pool blocks of the matched prefix


@dataclass
class PutBatch:
    num_skipped: np.ndarray        # [R] leading blocks already cached, not copied
    num_transferred: np.ndarray    # [R] blocks copied (0: empty put)
    cpu_blocks: List[np.ndarray]   # per request: pool blocks the copied blocks went to
    gpu_blocks: List[np.ndarray]   # per request: the GPU blocks copied
    block_hashes: List[np.ndarray]  # per request: every block's hash (uint64)

    def return_mask(self, r: int, num_tokens: int, tokens_per_block: int) -> torch.Tensor:
        """The reference put's return mask: True over the copied tokens
        (cache_engine.py:600-602)."""
        m = torch.zeros(num_tokens, dtype=torch.bool)
        a = int(self.num_skipped[r]) * tokens_per_block
        m[a:a + int(self.num_transferred[r]) * tokens_per_block] = True
        return m


def _pack_tokens(token_ids: Sequence) -> Tuple[object, np.ndarray, object]:
    """Concatenate a batch of token sequences (int64; host or CUDA) and give
    the token offsets.  Returns (buffer kept alive, offsets, pointer)."""
    seqs = [t if isinstance(t, torch.Tensor) else torch.as_tensor(np.asarray(t, dtype=np.int64))
            for t in token_ids]
    lens = np.array([int(t.numel()) for t in seqs], dtype=np.int64)
    offsets = np.zeros(len(seqs) + 1, dtype=np.int64)
    np.cumsum(lens, out=offsets[1:])
    on_gpu = any(t.is_cuda for t in seqs)
    dev = next((t.device for t in seqs if t.is_cuda), None)
    parts = [t.reshape(-1).to(dtype=torch.int64, device=dev if on_gpu else "cpu") for t in seqs]
    buf = torch.cat(parts) if parts and offsets[-1] > 0 else torch.zeros(1, dtype=torch.int64,
                                                                        device=dev if on_gpu else "cpu")
    return buf, offsets, buf.data_ptr()


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

    def _split(self, flat: np.ndarray, offsets: np.ndarray) -> List[np.ndarray]:
        tpb = self.tokens_per_block
        blk = np.concatenate([[0], np.cumsum((offsets[1:] - offsets[:-1]) // tpb)])
        return [flat[blk[r]:blk[r + 1]] for r in range(len(offsets) - 1)]

    def match(self, token_ids: Sequence) -> MatchBatch:
        """match_prefix of every sequence (radixtree.py:143-195)."""
        buf, offsets, ptr = _pack_tokens(token_ids)
        R = len(offsets) - 1
        nb = int(((offsets[1:] - offsets[:-1]) // self.tokens_per_block).sum())
        nm = np.zeros(R, dtype=np.int64)
        nr = np.zeros(R, dtype=np.int64)
        phys = np.full(max(nb, 1), -1, dtype=np.int64)
        check(_lib.load().fkv_cache_index_match(self._h, ptr, offsets.ctypes.data, R, nm.ctypes.data,
                                                nr.ctypes.data, phys.ctypes.data, self._stream()),
              "CpuCacheIndex.match")
        per = self._split(phys[:nb], offsets)
        return MatchBatch(nm, nr, [p[:int(m)].copy() for p, m in zip(per, nm)])

    def put(self, token_ids: Sequence, gpu_block_ids: Sequence, layout: KVLayout,
            mark_ready: bool = True) -> PutBatch:
        """Puts of the CPU tier for a batch of requests, in order
        (cache_engine.py:787-902): request r's full blocks are hashed, its
        cached prefix is skipped, pool blocks are taken for the rest, which
        are inserted (not ready), copied from the GPU blocks
        gpu_block_ids[r] (one per full block) and, with mark_ready, marked
        ready once the copy is done (the put callback).  Returns when the
        copies are complete."""
        tpb = self.tokens_per_block
        if len(token_ids) != len(gpu_block_ids):
            raise ValueError("one gpu block list per request")
        buf, offsets, ptr = _pack_tokens(token_ids)
        R = len(offsets) - 1
        nblk = (offsets[1:] - offsets[:-1]) // tpb
        gparts = []
        for r, g in enumerate(gpu_block_ids):
            g = np.asarray(g.cpu() if isinstance(g, torch.Tensor) else g, dtype=np.int64).reshape(-1)
            if len(g) != nblk[r]:
                raise ValueError(f"request {r}: {len(g)} gpu blocks for {nblk[r]} full blocks")
            gparts.append(g)
        nb = int(nblk.sum())
        gids = np.ascontiguousarray(np.concatenate(gparts) if gparts else np.zeros(0, np.int64))
        if nb == 0:
            gids = np.zeros(1, dtype=np.int64)
        nsk = np.zeros(R, dtype=np.int64)
        ntr = np.zeros(R, dtype=np.int64)
        cpu = np.full(max(nb, 1), -1, dtype=np.int64)
        hashes = np.zeros(max(nb, 1), dtype=np.uint64)
        d = layout.desc()
        check(_lib.load().fkv_cache_index_put(self._h, ptr, offsets.ctypes.data, R, gids.ctypes.data,
                                              ctypes.byref(d), int(bool(mark_ready)), nsk.ctypes.data,
                                              ntr.ctypes.data, cpu.ctypes.data, hashes.ctypes.data,
                                              self._stream()),
              "CpuCacheIndex.put")
        cpu_per = self._split(cpu[:nb], offsets)
        g_per = self._split(gids[:nb], offsets)
        h_per = self._split(hashes[:nb], offsets)
        cpu_blocks = [c[int(s):int(s) + int(t)].copy() for c, s, t in zip(cpu_per, nsk, ntr)]
        gpu_blocks = [g[int(s):int(s) + int(t)].copy() for g, s, t in zip(g_per, nsk, ntr)]
        return PutBatch(nsk, ntr, cpu_blocks, gpu_blocks, [h.copy() for h in h_per])

    def put_requests(self, requests: Sequence[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
                     layout: KVLayout, mark_ready: bool = True) -> Tuple[List[torch.Tensor], PutBatch]:
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
        res = self.put(toks, gids, layout, mark_ready=mark_ready)
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
