"""GPU test of fkv_transfer_kv_blocks_noalloc, the entry point for callers
that cannot allocate device memory when they move KV blocks (an engine whose
own caching allocator owns the GPU, a thread under a strict memory budget,
code that must not risk an allocation's implicit synchronization).

It must produce exactly the bytes of the regular entry point
fkv_transfer_kv_blocks, call after call: the two run here side by side on
identical pools, through the C ABI, for two calls in a row (a D2H and then
an H2D with a different block list, so the second call overwrites the
shared scratch table the first one filled).  This file is named to be
collected last; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from flexkv_b200 import _lib
from kvcase import Case, make_ids
from gpu_util import Pools, initial_images

pytestmark = pytest.mark.gpu

MAX_BLOCKS, MAX_LAYERS = 8192, 512


def _args(p: Pools, gids: np.ndarray, cids: np.ndarray):
    st = p.st
    g = np.ascontiguousarray(gids, dtype=np.int64)
    c = np.ascontiguousarray(cids, dtype=np.int64)
    ptrs = p.ptrs.numpy().astype(np.uint64)
    return g, c, ptrs, st


def existing(p: Pools, gids, cids, h2d: bool) -> None:
    lib = _lib.load()
    g, c, ptrs, st = _args(p, gids, cids)
    rc = lib.fkv_transfer_kv_blocks(
        len(g), p.case.layer_id, len(p.layers), g.ctypes.data, ptrs.ctypes.data, st["gpu_kv"],
        st["gpu_block"], c.ctypes.data, p.cpu.data_ptr(), st["cpu_kv"], st["cpu_layer"],
        st["cpu_block"], 0, st["gpu_chunk"], torch.cuda.current_stream().cuda_stream, -1, int(h2d),
        0, int(p.case.is_mla))
    _lib.check(rc, "fkv_transfer_kv_blocks")


def noalloc(p: Pools, gids, cids, h2d: bool) -> int:
    lib = _lib.load()
    g, c, ptrs, st = _args(p, gids, cids)
    return lib.fkv_transfer_kv_blocks_noalloc(
        len(g), p.case.layer_id, len(p.layers), g.ctypes.data, ptrs.ctypes.data, st["gpu_kv"],
        st["gpu_block"], c.ctypes.data, p.cpu.data_ptr(), st["cpu_kv"], st["cpu_layer"],
        st["cpu_block"], 0, st["gpu_chunk"], st["cpu_pool_bytes"], st["gpu_layer_bytes"],
        torch.cuda.current_stream().cuda_stream, -1, int(h2d), int(p.case.is_mla))


@pytest.mark.parametrize("case", [
    Case("llama8b_slice", 32, 8, 128, 16, 128, 256),
    Case("mla_blockwise", 5, 1, 576, 64, 96, 160, "BLOCKWISE", is_mla=True),
], ids=lambda c: c.name)
def test_noalloc_matches_regular_entry_point_on_two_calls(case):
    gpu, cpu = initial_images(case, 4000, 4001)
    a, b = Pools(case, gpu, cpu), Pools(case, gpu, cpu)
    g1, c1 = make_ids(96 if not case.is_mla else 64, case.gpu_blocks, case.cpu_blocks, 41, 0.5,
                      max_run=16)
    g2, c2 = make_ids(80 if not case.is_mla else 48, case.gpu_blocks, case.cpu_blocks, 42, 0.3,
                      max_run=8)
    # call 1: device -> host
    existing(a, g1, c1, h2d=False)
    _lib.check(noalloc(b, g1, c1, h2d=False), "fkv_transfer_kv_blocks_noalloc")
    assert np.array_equal(a.cpu_image(), b.cpu_image())
    # call 2: host -> device with another block list
    existing(a, g2, c2, h2d=True)
    _lib.check(noalloc(b, g2, c2, h2d=True), "fkv_transfer_kv_blocks_noalloc")
    for x, y in zip(a.gpu_images(), b.gpu_images()):
        assert np.array_equal(x, y)
    assert np.array_equal(a.cpu_image(), b.cpu_image())


def test_noalloc_rejects_sizes_beyond_its_table():
    case = Case("small", 2, 2, 64, 16, 16, 32)
    gpu, cpu = initial_images(case, 4100, 4101)
    p = Pools(case, gpu, cpu)
    lib = _lib.load()
    big = np.zeros(MAX_BLOCKS + 1, dtype=np.int64)
    rc = noalloc(p, big, big, h2d=False)
    assert rc == _lib.FKV_ERR_INVALID_ARG
    assert b"8192" in lib.fkv_last_error()
    # the pool is untouched and a call within the limits still works
    before = p.cpu_image().copy()
    assert np.array_equal(p.cpu_image(), before)
    _lib.check(noalloc(p, np.array([3], np.int64), np.array([5], np.int64), h2d=False),
               "fkv_transfer_kv_blocks_noalloc")
