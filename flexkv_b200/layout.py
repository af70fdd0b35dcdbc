"""KV-cache byte layouts on either side of the transfer path — the shapes
and strides of FlexKV's KVCacheLayout (flexkv/common/storage.py:22-155).

GPU side (always LAYERWISE, one tensor per layer): [kv, num_blocks, tpb,
heads, head_dim].  CPU side: one flat tensor viewed as LAYERWISE
[layers, kv, blocks, tpb, heads, head_dim] or BLOCKWISE
[blocks, layers, kv, tpb, heads, head_dim].  kv = 1 for MLA.  Strides are
in elements; multiply by the element size for the byte strides the
transfer entry points take (worker.py:240-246, 383-390).
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from math import prod
from typing import Tuple


class KVCacheLayoutType(Enum):
    LAYERWISE = "LAYERWISE"
    BLOCKWISE = "BLOCKWISE"


@dataclass(frozen=True)
class KVCacheLayout:
    type: KVCacheLayoutType
    num_layer: int
    num_block: int
    tokens_per_block: int
    num_head: int
    head_size: int
    is_mla: bool = False

    @property
    def kv_dim(self) -> int:
        return 1 if self.is_mla else 2

    @property
    def kv_shape(self) -> Tuple[int, ...]:
        t, n, l, kv = self.tokens_per_block, self.num_block, self.num_layer, self.kv_dim
        if self.type == KVCacheLayoutType.LAYERWISE:
            return (l, kv, n, t, self.num_head, self.head_size)
        return (n, l, kv, t, self.num_head, self.head_size)

    def div_head(self, n: int) -> "KVCacheLayout":
        assert self.num_head % n == 0, f"num_head {self.num_head} not divisible by {n}"
        return KVCacheLayout(self.type, self.num_layer, self.num_block, self.tokens_per_block,
                             self.num_head // n, self.head_size, self.is_mla)

    def div_layer(self, n: int) -> "KVCacheLayout":
        assert self.num_layer % n == 0, f"num_layer {self.num_layer} not divisible by {n}"
        return KVCacheLayout(self.type, self.num_layer // n, self.num_block, self.tokens_per_block,
                             self.num_head, self.head_size, self.is_mla)

    def div_block(self, num_chunks: int, padding: bool = False) -> "KVCacheLayout":
        """Per-file layout of a pool split over num_chunks files
        (storage.py:78-94): ceil when padding, else exact."""
        if padding:
            nb = (self.num_block + num_chunks - 1) // num_chunks
        else:
            assert self.num_block % num_chunks == 0, \
                f"num_block {self.num_block} must be divisible by num_chunks {num_chunks}"
            nb = self.num_block // num_chunks
        return KVCacheLayout(self.type, self.num_layer, nb, self.tokens_per_block, self.num_head,
                             self.head_size, self.is_mla)

    def get_elements_per_block(self) -> int:
        return self.num_layer * self.kv_dim * self.get_chunk_size()

    def get_chunk_size(self) -> int:
        return self.tokens_per_block * self.num_head * self.head_size

    def get_layer_stride(self) -> int:
        s = self.kv_shape
        return prod(s[1:]) if self.type == KVCacheLayoutType.LAYERWISE else prod(s[2:])

    def get_block_stride(self) -> int:
        s = self.kv_shape
        return prod(s[3:]) if self.type == KVCacheLayoutType.LAYERWISE else prod(s[1:])

    def get_kv_stride(self) -> int:
        s = self.kv_shape
        return prod(s[2:]) if self.type == KVCacheLayoutType.LAYERWISE else prod(s[3:])

    def get_total_elements(self) -> int:
        return prod(self.kv_shape)


def gpu_byte_strides(gpu_layout: KVCacheLayout, itemsize: int) -> dict:
    """Per-layer GPU strides as GPUCPUTransferWorker computes them
    (worker.py:236-242): chunk, kv and block strides in bytes."""
    per_layer = gpu_layout.div_layer(gpu_layout.num_layer)
    return {
        "chunk": per_layer.get_chunk_size() * itemsize,
        "kv": per_layer.get_kv_stride() * itemsize,
        "block": per_layer.get_block_stride() * itemsize,
    }


def cpu_byte_strides(cpu_layout: KVCacheLayout, itemsize: int) -> dict:
    """CPU pool strides in bytes (worker.py:244-246, 387-390)."""
    return {
        "chunk": cpu_layout.get_chunk_size() * itemsize,
        "layer": cpu_layout.get_layer_stride() * itemsize,
        "kv": cpu_layout.get_kv_stride() * itemsize,
        "block": cpu_layout.get_block_stride() * itemsize,
    }
