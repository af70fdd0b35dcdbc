"""GPU, world_size 2 over gloo: the product's data-parallel sharding in
separate processes.

Each rank is its own process with its own GPU layers and page-locked pool
(on cuda:rank when the box has two GPUs, both on cuda:0 otherwise), derives
its own batches (bench.rank_steps, the bench's DP sharding) and moves them
through flexkv_b200.c_ext.transfer_kv_blocks: a D2H batch, then an H2D
batch, per step, synchronous per op as FlexKV's worker calls it.  Every byte
of both pools is checked against the oracle on the rank's host images.  The
ranks exchange only timing-style reductions (gloo), never data: the path
has no collective.
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

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]
    import bench
    from flexkv_b200 import c_ext
    from oracle import oracle as O
    from kvcase import Case, fill_bytes
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ok, moved = False, 0
    try:
        torch.cuda.set_device(rank % torch.cuda.device_count())
        case = Case("dp", 4, 2, 64, 16, 64, 128)
        st = case.strides()
        cfg = dict(layers=4, heads=2, head_dim=64, tpb=16, gpu_blocks=64, cpu_blocks=128, batch=24,
                   run_frac=0.5, max_run=8, kind="batch")
        steps = bench.rank_steps(cfg, cfg["cpu_blocks"], rank, nsteps=2)
        gpu_img = [fill_bytes(st["gpu_layer_bytes"], 500 + 10 * rank + l) for l in range(4)]
        cpu_img = fill_bytes(st["cpu_pool_bytes"], 600 + rank)
        layers = [torch.from_numpy(x.copy()).cuda() for x in gpu_img]
        ptrs = torch.tensor([t.data_ptr() for t in layers], dtype=torch.int64)
        cpu = torch.from_numpy(cpu_img.copy())
        c_ext.cudaHostRegister(cpu)
        try:
            for ops in steps:
                for g, c, h2d in ops:
                    c_ext.transfer_kv_blocks(torch.from_numpy(g), ptrs, st["gpu_kv"], st["gpu_block"],
                                             torch.from_numpy(c), cpu, st["cpu_kv"], st["cpu_layer"],
                                             st["cpu_block"], st["gpu_chunk"], 0, 8, h2d, False, False)
                    O.transfer(len(g), 0, g, gpu_img, st["gpu_kv"], st["gpu_block"], c, cpu_img, st["cpu_kv"],
                               st["cpu_layer"], st["cpu_block"], 0, st["gpu_chunk"], h2d, False)
                    moved += len(g) * 4 * 2 * st["gpu_chunk"]
            torch.cuda.synchronize()
            ok = np.array_equal(cpu.numpy(), cpu_img) and all(
                np.array_equal(t.cpu().numpy(), w) for t, w in zip(layers, gpu_img))
        finally:
            c_ext.cudaHostUnregister(cpu)
        total = bench.sum_over_ranks(world, float(moved))
        np.save(os.path.join(out_dir, f"rank{rank}.npy"),
                np.array([float(ok), float(moved), total] + [float(x) for x in steps[0][0][0]], dtype=np.float64))
        bench.barrier(world)
    finally:
        dist.destroy_process_group()


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_dp_ranks_in_separate_processes_move_their_own_batches():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d), nprocs=2, join=True, start_method="spawn")
        a, b = np.load(os.path.join(d, "rank0.npy")), np.load(os.path.join(d, "rank1.npy"))
    assert a[0] == 1.0 and b[0] == 1.0, "a rank's pools differ from the oracle"
    assert a[1] == b[1] > 0 and a[2] == b[2] == a[1] + b[1]  # each rank's bytes, summed over ranks
    assert not np.array_equal(a[3:], b[3:])  # each rank drew its own block ids
