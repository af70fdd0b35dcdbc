"""GPU tests of the native TransferEngine (flexkv_b200.engine): the
reference's round-trip acceptance test driven through the engine, dependency
ordering, both directions in flight, failures and rejected graphs."""
import time

import numpy as np
import pytest
import torch

from flexkv_b200.engine import TransferDescriptor, TransferEngine, TransferOp, TransferOpGraph, TransferType
from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
from kvcase import Case, fill_bytes, make_ids
from gpu_util import oracle_transfer

pytestmark = pytest.mark.gpu


def dev(i):
    return torch.device(f"cuda:{i}" if i < torch.cuda.device_count() else "cuda:0")


def wait_graphs(engine, graph_ids, max_wait=30.0):
    """(graph_id, op_id) pairs seen until every graph in graph_ids finished."""
    seen, done = [], set()
    t0 = time.time()
    while done != set(graph_ids) and time.time() - t0 < max_wait:
        for g, o in engine.get_completed_graphs_and_ops(timeout=0.05):
            seen.append((g, o))
            if o == -1:
                done.add(g)
    assert done == set(graph_ids), f"graphs not finished: {set(graph_ids) - done}"
    return seen


def one_op_graph(kind, gpu_ids, cpu_ids, layer_id=-1, gran=-1, dp_id=0):
    g = TransferOpGraph()
    src, dst = (cpu_ids, gpu_ids) if kind == TransferType.H2D else (gpu_ids, cpu_ids)
    op = TransferOp(graph_id=g.graph_id, transfer_type=kind, layer_id=layer_id, layer_granularity=gran,
                    src_descriptor=TransferDescriptor(torch.as_tensor(src, dtype=torch.int64)),
                    dst_descriptor=TransferDescriptor(torch.as_tensor(dst, dtype=torch.int64)))
    g.add_transfer_op(op)
    g.bind_to_dp_group(dp_id)
    return g, op


@pytest.mark.parametrize("tp_size,dp_size", [(1, 1), (2, 1), (2, 2)])
@pytest.mark.parametrize("use_mla", [False, True])
@pytest.mark.parametrize("layout_type", ["LAYERWISE", "BLOCKWISE"])
def test_engine_round_trip(tp_size, dp_size, use_mla, layout_type):
    """test_gpu_cpu_round_trip (tests/test_transfer_engine.py:55-161) through
    the engine: write GPU->CPU, zero the GPU blocks, read CPU->GPU, compare
    bit for bit with the ground truth."""
    L, H, D, tpb, n_gpu, n_cpu, n = 4, 32, 128, 16, 128, 128, 16
    gen = torch.Generator().manual_seed(1)
    full = KVCacheLayout(KVCacheLayoutType.LAYERWISE, L, n_gpu, tpb, H, D, use_mla)
    gpu_layout = full if use_mla else full.div_head(tp_size)
    cpu_layout = KVCacheLayout(KVCacheLayoutType[layout_type], L, n_cpu, tpb, H, D, use_mla)
    hp = H // tp_size
    gt, gpu_blocks = [], []
    for d in range(dp_size):
        layers = [torch.randn(full.kv_shape[1:], generator=gen).to(torch.float16) for _ in range(L)]
        gt.append(layers)
        for t in range(tp_size):
            sl = slice(0, H) if use_mla else slice(t * hp, (t + 1) * hp)
            gpu_blocks.append([x[:, :, :, sl, :].contiguous().to(dev(d * tp_size + t)) for x in layers])
    cpu = torch.zeros(cpu_layout.get_total_elements(), dtype=torch.float16)
    eng = TransferEngine(gpu_blocks, cpu, gpu_layout, cpu_layout, tp_size, dp_size)
    try:
        for d in range(dp_size):
            gids = torch.arange(0, n)
            cids = torch.arange(d * n, (d + 1) * n)
            g, _ = one_op_graph(TransferType.D2H, gids, cids, dp_id=d)
            eng.submit_transfer_graph(g)
            wait_graphs(eng, [g.graph_id])
            for t in range(tp_size):
                for x in gpu_blocks[d * tp_size + t]:
                    x[:, gids.to(x.device)].zero_()
            g, _ = one_op_graph(TransferType.H2D, gids, cids, dp_id=d)
            eng.submit_transfer_graph(g)
            wait_graphs(eng, [g.graph_id])
        assert not eng.failed_ops
        for d in range(dp_size):
            for t in range(tp_size):
                sl = slice(0, H) if use_mla else slice(t * hp, (t + 1) * hp)
                for layer in range(L):
                    assert torch.equal(gpu_blocks[d * tp_size + t][layer].cpu(),
                                       gt[d][layer][:, :, :, sl, :])
    finally:
        eng.shutdown()


def _pools(case, seed):
    st = case.strides()
    imgs = [fill_bytes(st["gpu_layer_bytes"], seed + l) for l in range(case.num_layers)]
    cpu_img = fill_bytes(st["cpu_pool_bytes"], seed + 99)
    layers = [torch.from_numpy(x.copy()).cuda() for x in imgs]
    cpu = torch.from_numpy(cpu_img.copy()).pin_memory()
    return st, imgs, cpu_img, layers, cpu


def test_layerwise_read_graph_orders_ops_and_matches_oracle():
    """A layer-group chain (convert_read_graph_to_layer_wise_graph,
    transfer_pattern.py:370-428): op k reads layers [2k, 2k+2) and depends on
    op k-1; a virtual op ends the graph.  Completions come in dependency
    order and the bytes equal the oracle's."""
    case = Case("chain", 8, 2, 64, 16, 64, 128)
    st, imgs, cpu_img, layers, cpu = _pools(case, 500)
    gl, cl = case.gpu_layout(), case.cpu_layout_obj()
    eng = TransferEngine([[t.view(torch.bfloat16) for t in layers]], cpu.view(torch.bfloat16), gl, cl)
    try:
        gids, cids = make_ids(20, 64, 128, 3, 0.4, max_run=4)
        g = TransferOpGraph()
        ops = []
        for k in range(4):
            op = TransferOp(graph_id=g.graph_id, transfer_type=TransferType.H2D, layer_id=2 * k,
                            layer_granularity=2,
                            src_descriptor=TransferDescriptor(torch.from_numpy(cids)),
                            dst_descriptor=TransferDescriptor(torch.from_numpy(gids)))
            g.add_transfer_op(op)
            if ops:
                g.add_dependency(op.op_id, ops[-1].op_id)
            ops.append(op)
        v = TransferOp(graph_id=g.graph_id, transfer_type=TransferType.VIRTUAL)
        g.add_virtual_op(v)
        for op in ops:
            g.add_dependency(v.op_id, op.op_id)
        eng.submit_transfer_graph(g)
        seen = wait_graphs(eng, [g.graph_id])
        order = [o for _, o in seen]
        idx = {o: i for i, o in enumerate(order)}
        for a, b in zip(ops, ops[1:]):
            assert idx[a.op_id] < idx[b.op_id]
        assert idx[v.op_id] > idx[ops[-1].op_id]
        assert order[-1] == -1
        want = [x.copy() for x in imgs]
        oracle_transfer(case, want, cpu_img.copy(), gids, cids, True)
        for t, w in zip(layers, want):
            assert np.array_equal(t.cpu().numpy(), w)
    finally:
        eng.shutdown()


def test_both_directions_in_flight_and_many_small_graphs():
    case = Case("mix", 4, 2, 64, 16, 512, 1024)
    st, imgs, cpu_img, layers, cpu = _pools(case, 700)
    gl, cl = case.gpu_layout(), case.cpu_layout_obj()
    eng = TransferEngine([[t.view(torch.bfloat16) for t in layers]], cpu.view(torch.bfloat16), gl, cl,
                         staging_bytes=1024)  # tiny ring: forces wraparound and waits
    try:
        gids, cids = make_ids(400, 512, 1024, 9, 0.3, max_run=8)
        half = 200  # first half read into the GPU, second half written out
        want_gpu = [x.copy() for x in imgs]
        want_cpu = cpu_img.copy()
        # D2H first in the oracle (it reads GPU blocks the H2D does not touch)
        oracle_transfer(case, [x.copy() for x in imgs], want_cpu, gids[half:], cids[half:], False)
        oracle_transfer(case, want_gpu, cpu_img.copy(), gids[:half], cids[:half], True)
        graphs = []
        for i in range(0, half, 5):
            g1, _ = one_op_graph(TransferType.H2D, gids[i:i + 5], cids[i:i + 5])
            g2, _ = one_op_graph(TransferType.D2H, gids[half + i:half + i + 5], cids[half + i:half + i + 5])
            eng.submit_transfer_graph(g1)
            eng.submit_transfer_graph(g2)
            graphs += [g1.graph_id, g2.graph_id]
        wait_graphs(eng, graphs)
        assert not eng.failed_ops
        assert eng.pending_ops() == 0
        for t, w in zip(layers, want_gpu):
            assert np.array_equal(t.cpu().numpy(), w)
        # D2H never writes CPU blocks of the H2D half's sources
        assert np.array_equal(cpu.numpy(), want_cpu)
    finally:
        eng.shutdown()


def test_failed_op_is_reported_and_engine_keeps_working():
    case = Case("fail", 2, 2, 64, 16, 16, 32)
    st, imgs, cpu_img, layers, cpu = _pools(case, 900)
    gl, cl = case.gpu_layout(), case.cpu_layout_obj()
    eng = TransferEngine([[t.view(torch.bfloat16) for t in layers]], cpu.view(torch.bfloat16), gl, cl)
    try:
        bad, bad_op = one_op_graph(TransferType.D2H, [0, 1], [3, 32])  # cpu id past the pool
        good, good_op = one_op_graph(TransferType.D2H, [2], [4])
        eng.submit_transfer_graph(bad)
        eng.submit_transfer_graph(good)
        wait_graphs(eng, [bad.graph_id, good.graph_id])
        assert bad_op.op_id in eng.failed_ops and good_op.op_id not in eng.failed_ops
        want = cpu_img.copy()
        oracle_transfer(case, [x.copy() for x in imgs], want, np.array([2]), np.array([4]), False)
        assert np.array_equal(cpu.numpy(), want)
        # a cyclic graph is rejected as a whole
        g = TransferOpGraph()
        a = TransferOp(graph_id=g.graph_id, transfer_type=TransferType.VIRTUAL)
        b = TransferOp(graph_id=g.graph_id, transfer_type=TransferType.VIRTUAL)
        g.add_virtual_op(a)
        g.add_virtual_op(b)
        g.add_dependency(a.op_id, b.op_id)
        g.add_dependency(b.op_id, a.op_id)
        eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id])
        assert a.op_id in eng.failed_ops and b.op_id in eng.failed_ops
    finally:
        eng.shutdown()


def test_from_reference_style_handles():
    """from_handles reads FlexKV StorageHandles / configs by duck typing."""
    from types import SimpleNamespace as NS
    from enum import Enum

    class LT(Enum):
        LAYERWISE = "LAYERWISE"
        BLOCKWISE = "BLOCKWISE"

    L, H, D, tpb = 2, 4, 64, 16
    gpu_l = NS(type=LT.LAYERWISE, num_layer=L, num_block=32, tokens_per_block=tpb, num_head=H,
               head_size=D, is_mla=False)
    cpu_l = NS(type=LT.BLOCKWISE, num_layer=L, num_block=64, tokens_per_block=tpb, num_head=H,
               head_size=D, is_mla=False)
    layers = [torch.randn(2, 32, tpb, H, D, device="cuda", dtype=torch.float16) for _ in range(L)]
    cpu = torch.zeros(64 * L * 2 * tpb * H * D, dtype=torch.float16)
    gh = NS(get_tensor_list=lambda: layers, kv_layout=gpu_l)
    ch = NS(get_tensor=lambda: cpu, kv_layout=cpu_l)
    mc = NS(tp_size=1, dp_size=1)
    cc = NS(transfer_sms_h2d=8, transfer_sms_d2h=8, use_ce_transfer_h2d=False, use_ce_transfer_d2h=True)
    eng = TransferEngine.from_handles([gh], mc, cc, ch)
    try:
        g, _ = one_op_graph(TransferType.D2H, [5, 6, 7], [10, 11, 12])
        eng.submit_transfer_graph(g)
        wait_graphs(eng, [g.graph_id])
        view = cpu.view(64, L, 2, tpb, H, D)
        for layer in range(L):
            assert torch.equal(view[10:13, layer].cpu(), layers[layer][:, 5:8].transpose(0, 1).cpu())
    finally:
        eng.shutdown()


def test_bounded_shutdown_drains_submitted_ops():
    case = Case("drain", 4, 2, 64, 16, 256, 512)
    st, imgs, cpu_img, layers, cpu = _pools(case, 1100)
    gl, cl = case.gpu_layout(), case.cpu_layout_obj()
    eng = TransferEngine([[t.view(torch.bfloat16) for t in layers]], cpu.view(torch.bfloat16), gl, cl)
    gids, cids = make_ids(128, 256, 512, 21, 0.5, max_run=8)
    g, _ = one_op_graph(TransferType.D2H, gids, cids)
    eng.submit_transfer_graph(g)
    eng.shutdown(timeout=30.0)  # returns once the op has drained
    want = cpu_img.copy()
    oracle_transfer(case, [x.copy() for x in imgs], want, gids, cids, False)
    assert np.array_equal(cpu.numpy(), want)


def test_shutdown_timeout_is_reported_and_the_engine_finishes_detached():
    """Host-side failure injection: a zero shutdown budget while a 1024-block
    D2H is in flight.  The call reports the timeout; the engine finishes its
    op detached (its tensors are kept alive for it), and the bytes land."""
    from flexkv_b200 import engine as engine_mod
    case = Case("detach", 4, 8, 128, 16, 1024, 2048)
    st, imgs, cpu_img, layers, cpu = _pools(case, 1300)
    gl, cl = case.gpu_layout(), case.cpu_layout_obj()
    eng = TransferEngine([[t.view(torch.bfloat16) for t in layers]], cpu.view(torch.bfloat16), gl, cl)
    gids, cids = make_ids(1024, 1024, 2048, 22, 0.5, max_run=16)
    g, _ = one_op_graph(TransferType.D2H, gids, cids)
    eng.submit_transfer_graph(g)
    before = len(engine_mod._DETACHED)
    with pytest.raises(RuntimeError, match="did not drain"):
        eng.shutdown(timeout=0.0)
    assert len(engine_mod._DETACHED) == before + 1
    want = cpu_img.copy()
    oracle_transfer(case, [x.copy() for x in imgs], want, gids, cids, False)
    for _ in range(100):  # the detached dispatcher launches and drains on its own
        torch.cuda.synchronize()
        if np.array_equal(cpu.numpy(), want):
            break
        time.sleep(0.05)
    assert np.array_equal(cpu.numpy(), want)
