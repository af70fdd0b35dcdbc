"""The CUDA-IPC registration boundary on the GPU: a spawned process maps
this process's KV layers through TensorSharedHandle (the mirror of
flexkv/common/memory_handle.py:17-56) and moves blocks with the library;
both sides check the bytes against the oracle."""
import gc
import multiprocessing as mp
import pickle

import numpy as np
import pytest
import torch

import ipc_peer
from flexkv_b200.memory_handle import TensorSharedHandle, ipc_open_count
from gpu_util import Pools, initial_images, oracle_transfer
from kvcase import Case, fill_bytes, make_ids

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("alloc", ["separate", "contiguous"])
def test_cross_process_transfer_through_ipc_handles(alloc):
    """The exporter owns the cache; the importer reads it (D2H through the C
    ABI) and writes it (H2D through a TransferEngine on the imported
    tensors); the exporter sees exactly the oracle's bytes afterwards."""
    case = Case("ipc", 8, 2, 64, 16, 64, 128)
    st = case.strides()
    gids, cids = make_ids(40, case.gpu_blocks, case.cpu_blocks, 31, 0.5, max_run=8)
    gpu, cpu = initial_images(case, 1300, 1301)
    p = Pools(case, gpu, cpu, alloc=alloc)
    torch.cuda.synchronize()
    handles = [TensorSharedHandle(t) for t in p.layers]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    proc = ctx.Process(target=ipc_peer.child_main,
                       args=(handles, case, gids, cids, 1301, 1302, 1300, q))
    proc.start()
    try:  # well inside the per-test limit, so a stuck child fails this test alone
        status, info = q.get(timeout=150)
    finally:
        proc.join(timeout=30)
        if proc.is_alive():
            proc.kill()
            proc.join()
    assert status == "ok", info
    assert info["d2h_ok"], "importer read different bytes than the oracle"
    assert info["h2d_done"] and not info["failed"]
    assert info["open_after_release"] == 0
    if alloc == "contiguous":
        assert info["opened"] == 1  # every layer is a view of one allocation: one mapping
    want = [g.copy() for g in gpu]
    oracle_transfer(case, want, fill_bytes(st["cpu_pool_bytes"], 1302), gids, cids, True)
    for a, b in zip(p.gpu_images(), want):
        assert np.array_equal(a, b)


def test_same_process_handle_is_a_view_of_the_original():
    base = torch.arange(4000, dtype=torch.float32, device="cuda").view(40, 100)
    t = base[:, 10:60]  # strided view
    h = pickle.loads(pickle.dumps(TensorSharedHandle(t)))
    u = h.get_tensor()
    assert u.shape == t.shape and u.stride() == t.stride() and u.dtype == t.dtype
    assert u.data_ptr() == t.data_ptr()
    assert torch.equal(u, t)
    u.fill_(7.0)
    assert float(base[:, 10:60].sum()) == 7.0 * t.numel()
    assert float(base[:, :10].sum()) == float(torch.arange(4000.0).view(40, 100)[:, :10].sum())
    del u
    gc.collect()
    assert ipc_open_count() == 0


def test_empty_and_bf16_tensors():
    e = TensorSharedHandle(torch.empty(0, 5, device="cuda", dtype=torch.bfloat16)).get_tensor()
    assert e.shape == (0, 5) and e.dtype == torch.bfloat16
    x = torch.randn(3, 7, device="cuda").to(torch.bfloat16)
    y = TensorSharedHandle(x).get_tensor()
    assert torch.equal(x, y)
