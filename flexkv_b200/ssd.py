"""SSD tier helpers: the cache files and the byte strides of the SSD worker.

``allocate_ssd_files`` creates the files the way SSDAllocator.allocate
does (flexkv/storage/allocator.py:132-200): ``num_block`` must split evenly
over the cache directories (one directory per SSD device); each device
gets ceil(blocks_per_device / blocks_per_file) files named
``{prefix}_{device}_{file}.bin`` of blocks_per_file * block_bytes bytes,
blocks_per_file bounded by the free space of the first directory and by
``max_blocks_per_file``.

``SsdStrides`` derives the arguments of transfer_kv_blocks_ssd as
CPUSSDDiskTransferWorker does (flexkv/transfer/worker.py:512-520): chunk,
block stride and CPU strides from the CPU layout, SSD strides from the
SSD layout divided over all files with padding.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple, Union

from .layout import KVCacheLayout


def allocate_ssd_files(layout: KVCacheLayout, itemsize: int, cache_dir: Union[str, Sequence[str]],
                       file_prefix: str = "flexkv_ssd_cache",
                       max_blocks_per_file: int = -1) -> Tuple[Dict[int, List[str]], int]:
    """Create the SSD cache files; returns (files per device, blocks per file)."""
    dirs = [cache_dir] if isinstance(cache_dir, str) else list(cache_dir)
    for d in dirs:
        os.makedirs(d, exist_ok=True)
        if not os.path.isdir(d):
            raise ValueError("cache_dir must be a directory")
    if layout.num_block % len(dirs) != 0:
        raise ValueError(f"num_ssd_blocks ({layout.num_block}) must be a multiple of "
                         f"num_ssd_devices ({len(dirs)})")
    per_device = layout.num_block // len(dirs)
    block_bytes = layout.get_elements_per_block() * itemsize
    st = os.statvfs(dirs[0])
    fs_max = (st.f_frsize * st.f_bavail) // block_bytes
    cap = int(1e9) if max_blocks_per_file == -1 else max_blocks_per_file
    per_file = min(fs_max, cap)
    if per_file <= 0:
        raise ValueError("no room for a single block in the SSD cache directory")
    files_per_device = (per_device + per_file - 1) // per_file
    files: Dict[int, List[str]] = {}
    for i, d in enumerate(dirs):
        files[i] = []
        for j in range(files_per_device):
            path = os.path.join(d, f"{file_prefix}_{i}_{j}.bin")
            with open(path, "wb+", buffering=0) as f:
                os.truncate(f.fileno(), per_file * block_bytes)
                f.flush()
                os.fsync(f.fileno())
            files[i].append(path)
    return files, per_file


@dataclass(frozen=True)
class SsdStrides:
    chunk_size_in_bytes: int
    block_stride_in_bytes: int
    cpu_layer_stride_in_bytes: int
    cpu_kv_stride_in_bytes: int
    ssd_layer_stride_in_bytes: int
    ssd_kv_stride_in_bytes: int

    @classmethod
    def of(cls, cpu_layout: KVCacheLayout, ssd_layout: KVCacheLayout, num_files: int,
           itemsize: int) -> "SsdStrides":
        if cpu_layout.type != ssd_layout.type:
            raise ValueError("no support for different CPU and SSD KV cache layout type")
        per_file = ssd_layout.div_block(num_files, padding=True)
        e = itemsize
        return cls(cpu_layout.get_chunk_size() * e, cpu_layout.get_block_stride() * e,
                   cpu_layout.get_layer_stride() * e, cpu_layout.get_kv_stride() * e,
                   per_file.get_layer_stride() * e, per_file.get_kv_stride() * e)
