"""GPU test of fkv_transfer_kv_blocks_noalloc, the entry point for callers
that cannot allocate device memory when they move KV blocks (an engine whose
own caching allocator owns the GPU, a thread under a strict memory budget,
code that must not risk an allocation's implicit synchronization).

It must produce exactly the bytes of the regular entry point
fkv_transfer_kv_blocks and of the CPU oracle, call after call: the two entry
points run here side by side on identical pools, through the C ABI, for two
calls in a row (a D2H and then an H2D with a different block list, so the
second call overwrites the shared scratch table the first one filled), and
the oracle replays both calls on host images.  The cases cover a layer
slice (start_layer_id > 0) and a tensor-parallel rank's byte offset inside
the host chunk.  A warm call must leave the device's free memory unchanged,
and a call refused for its size must leave both pools untouched.  This file
is named to be collected last; it also passes when run alone in a fresh
process.
"""
import numpy as np
import pytest
import torch

from flexkv_b200 import _lib
from gpu_util import Pools, initial_images, oracle_transfer
from kvcase import Case, make_ids

pytestmark = pytest.mark.gpu

MAX_BLOCKS, MAX_LAYERS = 8192, 512


def _args(p: Pools, gids: np.ndarray, cids: np.ndarray):
    g = np.ascontiguousarray(gids, dtype=np.int64)
    c = np.ascontiguousarray(cids, dtype=np.int64)
    ptrs = p.ptrs.numpy().astype(np.uint64)
    return g, c, ptrs, p.st


def existing(p: Pools, gids, cids, h2d: bool, off: int = 0) -> None:
    lib = _lib.load()
    g, c, ptrs, st = _args(p, gids, cids)
    rc = lib.fkv_transfer_kv_blocks(
        len(g), p.case.layer_id, len(p.layers), g.ctypes.data, ptrs.ctypes.data, st["gpu_kv"],
        st["gpu_block"], c.ctypes.data, p.cpu.data_ptr(), st["cpu_kv"], st["cpu_layer"],
        st["cpu_block"], off, st["gpu_chunk"], torch.cuda.current_stream().cuda_stream, -1, int(h2d),
        0, int(p.case.is_mla))
    _lib.check(rc, "fkv_transfer_kv_blocks")


def noalloc(p: Pools, gids, cids, h2d: bool, off: int = 0) -> int:
    lib = _lib.load()
    g, c, ptrs, st = _args(p, gids, cids)
    return lib.fkv_transfer_kv_blocks_noalloc(
        len(g), p.case.layer_id, len(p.layers), g.ctypes.data, ptrs.ctypes.data, st["gpu_kv"],
        st["gpu_block"], c.ctypes.data, p.cpu.data_ptr(), st["cpu_kv"], st["cpu_layer"],
        st["cpu_block"], off, st["gpu_chunk"], st["cpu_pool_bytes"], st["gpu_layer_bytes"],
        torch.cuda.current_stream().cuda_stream, -1, int(h2d), int(p.case.is_mla))


CASES = [
    (Case("llama8b_slice", 32, 8, 128, 16, 128, 256), 0),
    (Case("mla_blockwise", 5, 1, 576, 64, 96, 160, "BLOCKWISE", is_mla=True), 0),
    (Case("layer_slice", 12, 4, 64, 16, 64, 128, layer_id=4, layer_gran=5), 0),
    (Case("tp_rank1_of_2", 4, 2, 64, 16, 64, 128, "BLOCKWISE", tp=2), 1),
]


@pytest.mark.parametrize("case,rank", CASES, ids=[c.name for c, _ in CASES])
def test_noalloc_matches_regular_entry_point_and_oracle_on_two_calls(case, rank):
    gpu, cpu = initial_images(case, 4000, 4001)
    a, b = Pools(case, gpu, cpu), Pools(case, gpu, cpu)
    want_gpu, want_cpu = [x.copy() for x in gpu], cpu.copy()
    off = 0 if case.is_mla else rank * a.st["gpu_chunk"]
    n1, n2 = (64, 48) if case.is_mla else (min(96, case.gpu_blocks), min(80, case.gpu_blocks))
    g1, c1 = make_ids(n1, case.gpu_blocks, case.cpu_blocks, 41, 0.5, max_run=16)
    g2, c2 = make_ids(n2, case.gpu_blocks, case.cpu_blocks, 42, 0.3, max_run=8)
    # call 1: device -> host
    existing(a, g1, c1, h2d=False, off=off)
    _lib.check(noalloc(b, g1, c1, h2d=False, off=off), "fkv_transfer_kv_blocks_noalloc")
    oracle_transfer(case, want_gpu, want_cpu, g1, c1, False, rank=rank)
    assert np.array_equal(b.cpu_image(), want_cpu), "noalloc D2H differs from the oracle"
    assert np.array_equal(a.cpu_image(), b.cpu_image())
    # call 2: host -> device with another block list
    existing(a, g2, c2, h2d=True, off=off)
    _lib.check(noalloc(b, g2, c2, h2d=True, off=off), "fkv_transfer_kv_blocks_noalloc")
    oracle_transfer(case, want_gpu, want_cpu, g2, c2, True, rank=rank)
    for x, y, w in zip(a.gpu_images(), b.gpu_images(), want_gpu):
        assert np.array_equal(y, w), "noalloc H2D differs from the oracle"
        assert np.array_equal(x, y)
    assert np.array_equal(a.cpu_image(), b.cpu_image())


def test_noalloc_warm_call_allocates_no_device_memory():
    case = Case("budget", 8, 4, 64, 16, 256, 512)
    gpu, cpu = initial_images(case, 4200, 4201)
    p = Pools(case, gpu, cpu)
    g, c = make_ids(200, case.gpu_blocks, case.cpu_blocks, 43, 0.4, max_run=8)
    _lib.check(noalloc(p, g, c, h2d=False), "fkv_transfer_kv_blocks_noalloc")  # first call: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for h2d in (True, False, True):
        _lib.check(noalloc(p, g, c, h2d=h2d), "fkv_transfer_kv_blocks_noalloc")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"


def test_noalloc_rejects_sizes_beyond_its_table():
    case = Case("small", 2, 2, 64, 16, 16, 32)
    gpu, cpu = initial_images(case, 4100, 4101)
    p = Pools(case, gpu, cpu)
    lib = _lib.load()
    cpu_before = p.cpu_image().copy()
    gpu_before = [x.copy() for x in p.gpu_images()]
    big = np.zeros(MAX_BLOCKS + 1, dtype=np.int64)
    for h2d in (False, True):
        rc = noalloc(p, big, big, h2d=h2d)
        assert rc == _lib.FKV_ERR_INVALID_ARG
        assert b"8192" in lib.fkv_last_error()
    torch.cuda.synchronize()
    assert np.array_equal(p.cpu_image(), cpu_before), "a refused call changed the host pool"
    for x, y in zip(p.gpu_images(), gpu_before):
        assert np.array_equal(x, y), "a refused call changed a GPU layer"
    # a call within the limits still works, and moves exactly the oracle's bytes
    want_gpu, want_cpu = [x.copy() for x in gpu_before], cpu_before.copy()
    g, c = np.array([3], np.int64), np.array([5], np.int64)
    _lib.check(noalloc(p, g, c, h2d=False), "fkv_transfer_kv_blocks_noalloc")
    oracle_transfer(case, want_gpu, want_cpu, g, c, False)
    assert np.array_equal(p.cpu_image(), want_cpu)
