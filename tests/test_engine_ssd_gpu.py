"""GPU: the TransferEngine across three tiers (GPU <-> CPU <-> SSD), ports
of test_ssd_round_trip and test_concurrent_mixed_transfers
(tests/test_transfer_engine.py:163-255, 258-400).  Stronger than the
originals: the CPU pool is zeroed between the write and the read graphs,
so the bytes that reach the GPU can only come back from the files, and an
H2D that ran ahead of its DISK2H predecessor would show as zeros."""
import time

import pytest
import torch

from flexkv_b200.engine import TransferDescriptor, TransferEngine, TransferOp, TransferOpGraph, TransferType
from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
from flexkv_b200.ssd import allocate_ssd_files

pytestmark = pytest.mark.gpu


def wait_graphs(engine, graph_ids, max_wait=60.0):
    done = set()
    t0 = time.time()
    while done != set(graph_ids) and time.time() - t0 < max_wait:
        for g, o in engine.get_completed_graphs_and_ops(timeout=0.05):
            if o == -1:
                done.add(g)
    assert done == set(graph_ids), f"graphs not finished: {set(graph_ids) - done}"


def op(graph, kind, src, dst, layers):
    o = TransferOp(graph_id=graph.graph_id, transfer_type=kind, layer_id=0, layer_granularity=layers,
                   src_descriptor=TransferDescriptor(torch.as_tensor(src, dtype=torch.int64)),
                   dst_descriptor=TransferDescriptor(torch.as_tensor(dst, dtype=torch.int64)))
    graph.add_transfer_op(o)
    return o


def write_graph(gpu_ids, cpu_ids, ssd_ids, layers):
    """create_write_graph_cpu_storage (transfer_pattern.py:245-300): D2H,
    then H2DISK depending on it."""
    g = TransferOpGraph()
    d2h = op(g, TransferType.D2H, gpu_ids, cpu_ids, layers)
    h2disk = op(g, TransferType.H2DISK, cpu_ids, ssd_ids, layers)
    g.add_dependency(h2disk.op_id, d2h.op_id)
    return g


def read_graph(gpu_ids, cpu_ids, ssd_ids, layers):
    """create_read_graph_cpu_storage (transfer_pattern.py:27-120), all
    blocks on the SSD: DISK2H, then H2D depending on it."""
    g = TransferOpGraph()
    disk2h = op(g, TransferType.DISK2H, ssd_ids, cpu_ids, layers)
    h2d = op(g, TransferType.H2D, cpu_ids, gpu_ids, layers)
    g.add_dependency(h2d.op_id, disk2h.op_id)
    return g


def make(tmp_path, num_gpu_blocks, use_mla, layout_type=KVCacheLayoutType.BLOCKWISE, L=4, H=8, D=128,
         tpb=16, n_cpu=None, n_ssd=None, seed=0):
    n_cpu = n_cpu or num_gpu_blocks
    n_ssd = n_ssd or num_gpu_blocks
    h = 1 if use_mla else H
    gpu_layout = KVCacheLayout(KVCacheLayoutType.LAYERWISE, L, num_gpu_blocks, tpb, h, D, use_mla)
    cpu_layout = KVCacheLayout(layout_type, L, n_cpu, tpb, h, D, use_mla)
    ssd_layout = KVCacheLayout(layout_type, L, n_ssd, tpb, h, D, use_mla)
    gen = torch.Generator().manual_seed(seed)
    gt = [torch.randn(gpu_layout.kv_shape[1:], generator=gen).to(torch.float16) for _ in range(L)]
    layers = [x.clone().cuda() for x in gt]
    cpu = torch.zeros(cpu_layout.get_total_elements(), dtype=torch.float16).pin_memory()
    files, per_file = allocate_ssd_files(ssd_layout, 2, str(tmp_path / "ssd"), max_blocks_per_file=n_ssd)
    eng = TransferEngine([layers], cpu, gpu_layout, cpu_layout, ssd_files=files, ssd_layout=ssd_layout,
                         ssd_num_blocks_per_file=per_file)
    return eng, gt, layers, cpu


@pytest.mark.parametrize("layout_type", [KVCacheLayoutType.BLOCKWISE, KVCacheLayoutType.LAYERWISE])
@pytest.mark.parametrize("use_mla", [True, False])
@pytest.mark.parametrize("transfer_block_num", [8, 16])
@pytest.mark.parametrize("num_gpu_blocks", [64, 128])
def test_ssd_round_trip(tmp_path, num_gpu_blocks, transfer_block_num, use_mla, layout_type):
    eng, gt, layers, cpu = make(tmp_path, num_gpu_blocks, use_mla, layout_type)
    try:
        ids = torch.arange(0, transfer_block_num, dtype=torch.int64)
        g = write_graph(ids, ids, ids, len(layers))
        eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id])
        assert not eng.failed_ops
        for x in layers:
            x[:, ids.cuda()].zero_()
        cpu.zero_()
        g = read_graph(ids, ids, ids, len(layers))
        eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id])
        assert not eng.failed_ops
        torch.cuda.synchronize()
        for x, y in zip(layers, gt):
            assert torch.equal(x.cpu(), y)
    finally:
        eng.shutdown()


@pytest.mark.parametrize("use_mla", [True, False])
def test_concurrent_mixed_transfers_with_ssd(tmp_path, use_mla):
    """Four write graphs in flight at once, then four read graphs in flight
    at once, on disjoint blocks with shuffled SSD placement."""
    n, per = 4, 16
    eng, gt, layers, cpu = make(tmp_path, 128, use_mla, n_cpu=128, n_ssd=256, seed=3)
    try:
        rng = torch.Generator().manual_seed(9)
        gpu_ids = torch.randperm(128, generator=rng)[:n * per]
        cpu_ids = torch.randperm(128, generator=rng)[:n * per]
        ssd_ids = torch.randperm(256, generator=rng)[:n * per]
        parts = lambda t, i: t[i * per:(i + 1) * per]
        ws = [write_graph(parts(gpu_ids, i), parts(cpu_ids, i), parts(ssd_ids, i), len(layers)) for i in range(n)]
        for g in ws:
            eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id for g in ws])
        for x in layers:
            x[:, gpu_ids.cuda()].zero_()
        cpu.zero_()
        rs = [read_graph(parts(gpu_ids, i), parts(cpu_ids, i), parts(ssd_ids, i), len(layers)) for i in range(n)]
        for g in rs:
            eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id for g in rs])
        assert not eng.failed_ops
        torch.cuda.synchronize()
        for x, y in zip(layers, gt):
            assert torch.equal(x.cpu(), y)
    finally:
        eng.shutdown()


def test_ssd_op_failure_is_reported_and_successor_still_runs(tmp_path):
    """A DISK2H that reads past the end of its file fails with its status;
    the dependent H2D is still run (the engine does not hold successors of a
    failed op) and the graph reports the failure."""
    eng, gt, layers, cpu = make(tmp_path, 64, False)
    try:
        g = read_graph(torch.tensor([0]), torch.tensor([0]), torch.tensor([10_000]), len(layers))
        eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id])
        assert len(eng.failed_ops) == 1
    finally:
        eng.shutdown()


def test_ssd_ops_need_an_ssd_context():
    L = 2
    gl = KVCacheLayout(KVCacheLayoutType.LAYERWISE, L, 8, 16, 2, 64)
    cl = KVCacheLayout(KVCacheLayoutType.BLOCKWISE, L, 8, 16, 2, 64)
    layers = [torch.zeros(gl.kv_shape[1:], dtype=torch.float16, device="cuda") for _ in range(L)]
    cpu = torch.zeros(cl.get_total_elements(), dtype=torch.float16).pin_memory()
    eng = TransferEngine([layers], cpu, gl, cl)
    try:
        g = read_graph(torch.tensor([0]), torch.tensor([0]), torch.tensor([0]), L)
        with pytest.raises(RuntimeError):
            eng.submit_transfer_graph(g)
    finally:
        eng.shutdown()


def test_from_handles_configures_the_ssd_tier(tmp_path):
    """TransferEngine.from_handles takes the reference constructor's
    arguments (transfer_engine.py:43-49) including an SSD StorageHandle
    (file list, layout, blocks per file; storage.py:159-200), by duck typing."""
    from enum import Enum
    from types import SimpleNamespace as NS

    class LT(Enum):
        LAYERWISE = "LAYERWISE"
        BLOCKWISE = "BLOCKWISE"

    L, H, D, tpb, ng, nc, ns = 2, 4, 64, 16, 32, 64, 64
    gpu_l = NS(type=LT.LAYERWISE, num_layer=L, num_block=ng, tokens_per_block=tpb, num_head=H, head_size=D,
               is_mla=False)
    cpu_l = NS(type=LT.BLOCKWISE, num_layer=L, num_block=nc, tokens_per_block=tpb, num_head=H, head_size=D,
               is_mla=False)
    ssd_l = NS(type=LT.BLOCKWISE, num_layer=L, num_block=ns, tokens_per_block=tpb, num_head=H, head_size=D,
               is_mla=False)
    files, per_file = allocate_ssd_files(
        KVCacheLayout(KVCacheLayoutType.BLOCKWISE, L, ns, tpb, H, D), 2, str(tmp_path / "ssd"),
        max_blocks_per_file=16)
    gen = torch.Generator().manual_seed(4)
    gt = [torch.randn(2, ng, tpb, H, D, generator=gen).to(torch.float16) for _ in range(L)]
    layers = [x.cuda() for x in gt]
    cpu = torch.zeros(nc * L * 2 * tpb * H * D, dtype=torch.float16)
    gh = NS(get_tensor_list=lambda: layers, kv_layout=gpu_l)
    ch = NS(get_tensor=lambda: cpu, kv_layout=cpu_l)
    sh = NS(get_file_list=lambda: files, kv_layout=ssd_l, num_blocks_per_file=per_file)
    mc = NS(tp_size=1, dp_size=1)
    cc = NS(transfer_sms_h2d=-1, transfer_sms_d2h=-1, use_ce_transfer_h2d=False, use_ce_transfer_d2h=False,
            ssd_cache_iouring_entries=512, ssd_cache_iouring_flags=0)
    eng = TransferEngine.from_handles([gh], mc, cc, ch, ssd_handle=sh)
    try:
        ids = torch.arange(3, 19, dtype=torch.int64)
        g = write_graph(ids, ids + 7, ids * 3, L)  # SSD ids spread over all four files
        eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id])
        for x in layers:
            x[:, ids.cuda()].zero_()
        cpu.zero_()
        g = read_graph(ids, ids + 7, ids * 3, L)
        eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id])
        assert not eng.failed_ops
        torch.cuda.synchronize()
        for x, y in zip(layers, gt):
            assert torch.equal(x.cpu(), y)
    finally:
        eng.shutdown()
