"""CPU, world_size 2 over gloo: the data-parallel and tensor-parallel
sharding of the path, with no collective on the data path.

* DP: each rank derives its own batches (bench.rank_steps) and moves them
  with the oracle on its own pools; only the timing reductions cross ranks.
* TP: both ranks write their own byte slice (offset rank*gpu_chunk) of every
  CPU chunk of one shared host pool (a file-backed mapping standing in for
  the shared pinned pool); the union equals the view-based restatement.
"""
import os
import sys
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _dp_worker(rank, world, port, out_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]
    import bench
    from oracle import oracle as O
    from kvcase import Case, fill_bytes
    _init(rank, world, port)
    try:
        cfg = dict(layers=3, heads=2, head_dim=64, tpb=16, gpu_blocks=64, cpu_blocks=128, batch=24,
                   run_frac=0.5, max_run=8)
        steps = bench.rank_steps(dict(cfg, kind="batch"), cfg["cpu_blocks"], rank, nsteps=1)
        batches = [(g, c) for g, c, h in steps[0]]
        case = Case("dp", 3, 2, 64, 16, 64, 128)
        st = case.strides()
        gpu = [fill_bytes(st["gpu_layer_bytes"], 10 * rank + l) for l in range(3)]
        cpu = np.zeros(st["cpu_pool_bytes"], dtype=np.uint8)
        moved = 0
        for g, c in batches:
            O.transfer(len(g), 0, g, gpu, st["gpu_kv"], st["gpu_block"], c, cpu, st["cpu_kv"],
                       st["cpu_layer"], st["cpu_block"], 0, st["gpu_chunk"], False, False)
            moved += len(g) * 3 * 2 * st["gpu_chunk"]
        total = bench.sum_over_ranks(world, float(moved))
        slowest = bench.max_over_ranks(world, float(rank + 1))
        np.save(os.path.join(out_dir, f"dp{rank}.npy"),
                np.array([total, slowest] + [int(x) for g, c in batches for x in g[:4]], dtype=np.float64))
        np.save(os.path.join(out_dir, f"dp{rank}_cpu.npy"), cpu)
        bench.barrier(world)
    finally:
        dist.destroy_process_group()


def _tp_worker(rank, world, port, pool_path, out_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]
    from oracle import oracle as O
    from kvcase import Case, fill_bytes, make_ids
    _init(rank, world, port)
    try:
        case = Case("tp", 4, 1, 64, 16, 32, 64, "BLOCKWISE", tp=world)
        st = case.strides()
        pool = np.memmap(pool_path, dtype=np.uint8, mode="r+", shape=(st["cpu_pool_bytes"],))
        gids, cids = make_ids(12, 32, 64, 5, 0.5, max_run=4)  # the same op on every rank
        gpu = [fill_bytes(st["gpu_layer_bytes"], 100 * rank + l) for l in range(4)]
        O.transfer(len(gids), 0, gids, gpu, st["gpu_kv"], st["gpu_block"], cids, pool,
                   st["cpu_kv"], st["cpu_layer"], st["cpu_block"], rank * st["gpu_chunk"],
                   st["gpu_chunk"], False, False)
        pool.flush()
        dist.barrier()  # completion of every rank's slice, host-side
    finally:
        dist.destroy_process_group()


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_dp_ranks_shard_without_data_collective():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_dp_worker, args=(2, _free_port(), d), nprocs=2, join=True,
                           start_method="spawn")
        a, b = np.load(os.path.join(d, "dp0.npy")), np.load(os.path.join(d, "dp1.npy"))
        assert a[0] == b[0] == 2 * 2 * 24 * 3 * 2 * 4096  # bytes summed over ranks (4 KiB chunks)
        assert a[1] == b[1] == 2.0                          # max over ranks
        assert not np.array_equal(a[2:], b[2:])             # each rank has its own ids
        ca, cb = np.load(os.path.join(d, "dp0_cpu.npy")), np.load(os.path.join(d, "dp1_cpu.npy"))
        assert ca.any() and cb.any() and not np.array_equal(ca, cb)


def test_tp_ranks_write_disjoint_slices_of_shared_pool():
    sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]
    from kvcase import Case, fill_bytes, make_ids, view_transfer
    world = 2
    case = Case("tp", 4, 1, 64, 16, 32, 64, "BLOCKWISE", tp=world)
    st = case.strides()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "pool.bin")
        np.zeros(st["cpu_pool_bytes"], dtype=np.uint8).tofile(path)
        mp.start_processes(_tp_worker, args=(world, _free_port(), path, d), nprocs=world,
                           join=True, start_method="spawn")
        got = np.fromfile(path, dtype=np.uint8)
    want = np.zeros(st["cpu_pool_bytes"], dtype=np.uint8)
    gids, cids = make_ids(12, 32, 64, 5, 0.5, max_run=4)
    for r in range(world):
        gpu = [fill_bytes(st["gpu_layer_bytes"], 100 * r + l) for l in range(4)]
        view_transfer(case, gpu, want, gids, cids, h2d=False, rank=r)
    assert np.array_equal(got, want)
