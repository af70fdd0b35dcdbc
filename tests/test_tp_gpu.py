"""GPU: tensor-parallel group (TPTransferThreadGroup mirror) against the
oracle, and the port of the reference's round-trip acceptance test
(tests/test_transfer_engine.py:55-161) with bit equality instead of allclose.
Ranks run on distinct GPUs when present, else all on cuda:0 (the reference
test falls back the same way, tests/test_utils.py:164-167)."""
import numpy as np
import pytest
import torch

from flexkv_b200 import c_ext
from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
from kvcase import Case, fill_bytes, make_ids
from gpu_util import oracle_transfer

pytestmark = pytest.mark.gpu


def dev(i):
    return torch.device(f"cuda:{i}" if i < torch.cuda.device_count() else "cuda:0")


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
@pytest.mark.parametrize("layout", ["LAYERWISE", "BLOCKWISE"])
@pytest.mark.parametrize("mla", [False, True])
def test_tp_group_vs_oracle(tp, layout, mla):
    heads_total = 8
    case = Case("tp", 4, heads_total if mla else heads_total // tp, 64, 16, 64, 128, layout,
                is_mla=mla, tp=tp)
    if mla:
        case = Case("tp", 4, 1, 576, 16, 64, 128, layout, is_mla=True, tp=tp)
    st = case.strides()
    gids, cids = make_ids(40, case.gpu_blocks, case.cpu_blocks, 50 + tp, 0.4, max_run=8)
    imgs = [[fill_bytes(st["gpu_layer_bytes"], 1000 * r + l) for l in range(case.num_layers)]
            for r in range(tp)]
    cpu_img = fill_bytes(st["cpu_pool_bytes"], 7)
    layers = [[torch.from_numpy(x.copy()).to(dev(r)) for x in imgs[r]] for r in range(tp)]
    cpu = torch.from_numpy(cpu_img.copy()).pin_memory()
    grp = c_ext.TPTransferThreadGroup(tp, layers, cpu, 0)
    args = dict(gpu_kv_stride_in_bytes=st["gpu_kv"], gpu_block_stride_in_bytes=st["gpu_block"],
                gpu_chunk_size_in_bytes=st["gpu_chunk"], cpu_kv_stride_in_bytes=st["cpu_kv"],
                cpu_layer_stride_in_bytes=st["cpu_layer"],
                cpu_block_stride_in_bytes=st["cpu_block"], cpu_chunk_size_in_bytes=st["cpu_chunk"],
                transfer_sms=8, use_ce_transfer=False, layer_id=0,
                layer_granularity=case.num_layers, is_mla=mla)
    grp.tp_group_transfer(torch.from_numpy(gids), cpu_block_id_tensor=torch.from_numpy(cids),
                          is_host_to_device=False, **args)
    # Oracle: rank by rank (MLA ranks write identical bytes at offset 0 only
    # when their data is identical; here data differs, so MLA is order-
    # dependent: compare MLA against the last rank's data in rank order only
    # for a single rank).
    if not mla or tp == 1:
        for r in range(tp):
            oracle_transfer(case, imgs[r], cpu_img, gids, cids, False, rank=r)
        assert np.array_equal(cpu.numpy(), cpu_img)
    # H2D back into zeroed layers: every rank reads its own slice.
    for r in range(tp):
        for t in layers[r]:
            t.zero_()
    grp.tp_group_transfer(torch.from_numpy(gids), cpu_block_id_tensor=torch.from_numpy(cids),
                          is_host_to_device=True, **args)
    for r in range(tp):
        want = [np.zeros_like(x) for x in imgs[r]]
        oracle_transfer(case, want, cpu.numpy().copy(), gids, cids, True, rank=r)
        for a, b in zip(layers[r], want):
            assert np.array_equal(a.cpu().numpy(), b), f"rank {r}"
    grp.close()


def test_tp_layer_slice_uses_full_layer_rows():
    """Layer-granular op (layer_id>0): rank i reads pointer row i of the
    [num_gpus][num_layers] table at layer_id+l."""
    tp, L = 2, 6
    case = Case("tpl", L, 2, 64, 16, 32, 64, "LAYERWISE", tp=tp, layer_id=2, layer_gran=3)
    st = case.strides()
    gids, cids = make_ids(10, 32, 64, 3, 0.0)
    imgs = [[fill_bytes(st["gpu_layer_bytes"], 77 * r + l) for l in range(L)] for r in range(tp)]
    layers = [[torch.from_numpy(x.copy()).to(dev(r)) for x in imgs[r]] for r in range(tp)]
    cpu_img = fill_bytes(st["cpu_pool_bytes"], 8)
    cpu = torch.from_numpy(cpu_img.copy()).pin_memory()
    grp = c_ext.TPTransferThreadGroup(tp, layers, cpu, 0)
    grp.tp_group_transfer(torch.from_numpy(gids), st["gpu_kv"], st["gpu_block"], st["gpu_chunk"],
                          torch.from_numpy(cids), st["cpu_kv"], st["cpu_layer"], st["cpu_block"],
                          st["cpu_chunk"], -1, False, False, 2, 3, False)
    for r in range(tp):
        oracle_transfer(case, imgs[r][2:5], cpu_img, gids, cids, False, rank=r)
    assert np.array_equal(cpu.numpy(), cpu_img)
    grp.close()


def test_tp_group_reports_rank_errors():
    case = Case("tperr", 2, 1, 64, 16, 8, 8, tp=2)
    st = case.strides()
    layers = [[torch.zeros(st["gpu_layer_bytes"], dtype=torch.uint8, device=dev(r))
               for _ in range(2)] for r in range(2)]
    cpu = torch.zeros(st["cpu_pool_bytes"], dtype=torch.uint8).pin_memory()
    grp = c_ext.TPTransferThreadGroup(2, layers, cpu, 0)
    with pytest.raises(RuntimeError, match="tp_group_transfer failed"):
        grp.tp_group_transfer(torch.tensor([0]), st["gpu_kv"], st["gpu_block"], st["gpu_chunk"],
                              torch.tensor([8]), st["cpu_kv"], st["cpu_layer"], st["cpu_block"],
                              st["cpu_chunk"], -1, False, False, 0, 2, False)
    grp.close()


@pytest.mark.parametrize("tp_size,dp_size", [(1, 1), (2, 1), (2, 2)])
@pytest.mark.parametrize("use_mla", [False, True])
@pytest.mark.parametrize("layout_type", ["LAYERWISE", "BLOCKWISE"])
def test_gpu_cpu_round_trip(tp_size, dp_size, use_mla, layout_type):
    """Port of test_gpu_cpu_round_trip: GPU->CPU for blocks 0..15 of each DP
    group, zero them on the GPU, CPU->GPU, compare with the ground truth."""
    num_layers, num_kv_heads, head_size, tpb = 4, 32, 128, 16
    num_gpu_blocks, n, num_cpu_blocks = 128, 16, 128
    g = torch.Generator().manual_seed(0)
    gpu_layout = KVCacheLayout(KVCacheLayoutType.LAYERWISE, num_layers, num_gpu_blocks, tpb,
                               num_kv_heads, head_size, use_mla)
    cpu_layout = KVCacheLayout(KVCacheLayoutType[layout_type], num_layers, num_cpu_blocks, tpb,
                               num_kv_heads, head_size, use_mla)
    rank_layout = gpu_layout if use_mla else gpu_layout.div_head(tp_size)
    per = rank_layout.div_layer(num_layers)
    e = 2
    gt, gpu_blocks = [], {}
    for dp in range(dp_size):
        layers_gt = [torch.randn(gpu_layout.kv_shape[1:], generator=g).to(torch.float16)
                     for _ in range(num_layers)]
        gt.append(layers_gt)
        hp = num_kv_heads // tp_size
        for tp in range(tp_size):
            gid = dp * tp_size + tp
            sl = slice(0, num_kv_heads) if use_mla else slice(tp * hp, (tp + 1) * hp)
            gpu_blocks[gid] = [x[:, :, :, sl, :].contiguous().to(dev(gid)) for x in layers_gt]
    cpu = torch.empty(cpu_layout.get_total_elements(), dtype=torch.float16)
    c_ext.cudaHostRegister(cpu)
    try:
        for dp in range(dp_size):
            ranks = [gpu_blocks[dp * tp_size + t] for t in range(tp_size)]
            gids = torch.arange(0, n, dtype=torch.int64)
            cids = torch.arange(dp * n, (dp + 1) * n, dtype=torch.int64)
            kw = dict(gpu_kv_stride_in_bytes=per.get_kv_stride() * e,
                      gpu_block_stride_in_bytes=per.get_block_stride() * e,
                      gpu_chunk_size_in_bytes=per.get_chunk_size() * e,
                      cpu_kv_stride_in_bytes=cpu_layout.get_kv_stride() * e,
                      cpu_layer_stride_in_bytes=cpu_layout.get_layer_stride() * e,
                      cpu_block_stride_in_bytes=cpu_layout.get_block_stride() * e,
                      cpu_chunk_size_in_bytes=cpu_layout.get_chunk_size() * e,
                      transfer_sms=4, use_ce_transfer=False, layer_id=0,
                      layer_granularity=num_layers, is_mla=use_mla)
            grp = c_ext.TPTransferThreadGroup(tp_size, ranks, cpu, dp)
            grp.tp_group_transfer(gids, cpu_block_id_tensor=cids, is_host_to_device=False, **kw)
            for r in ranks:
                for x in r:
                    x[:, gids.to(x.device)].zero_()
            grp.tp_group_transfer(gids, cpu_block_id_tensor=cids, is_host_to_device=True, **kw)
            grp.close()
        hp = num_kv_heads // tp_size
        for dp in range(dp_size):
            for tp in range(tp_size):
                sl = slice(0, num_kv_heads) if use_mla else slice(tp * hp, (tp + 1) * hp)
                for layer in range(num_layers):
                    assert torch.equal(gpu_blocks[dp * tp_size + tp][layer].cpu(),
                                       gt[dp][layer][:, :, :, sl, :])
    finally:
        c_ext.cudaHostUnregister(cpu)


def test_concurrent_callers_take_turns():
    """Two host threads drive one group at once on disjoint blocks (D2H); the
    group serializes them and both land exactly."""
    import threading
    tp = 2
    case = Case("tpc", 4, 4, 64, 16, 128, 256, "BLOCKWISE", tp=tp)
    st = case.strides()
    gids, cids = make_ids(96, case.gpu_blocks, case.cpu_blocks, 61, 0.4, max_run=8)
    imgs = [[fill_bytes(st["gpu_layer_bytes"], 300 * r + l) for l in range(case.num_layers)] for r in range(tp)]
    cpu_img = fill_bytes(st["cpu_pool_bytes"], 9)
    layers = [[torch.from_numpy(x.copy()).to(dev(r)) for x in imgs[r]] for r in range(tp)]
    cpu = torch.from_numpy(cpu_img.copy()).pin_memory()
    grp = c_ext.TPTransferThreadGroup(tp, layers, cpu, 0)
    args = dict(gpu_kv_stride_in_bytes=st["gpu_kv"], gpu_block_stride_in_bytes=st["gpu_block"],
                gpu_chunk_size_in_bytes=st["gpu_chunk"], cpu_kv_stride_in_bytes=st["cpu_kv"],
                cpu_layer_stride_in_bytes=st["cpu_layer"], cpu_block_stride_in_bytes=st["cpu_block"],
                cpu_chunk_size_in_bytes=st["cpu_chunk"], transfer_sms=8, use_ce_transfer=False, layer_id=0,
                layer_granularity=case.num_layers, is_mla=False, is_host_to_device=False)
    errors = []

    def run(part):
        try:
            for _ in range(5):
                grp.tp_group_transfer(torch.from_numpy(gids[part]), cpu_block_id_tensor=torch.from_numpy(cids[part]),
                                      **args)
        except Exception as e:  # reported below
            errors.append(e)

    halves = [slice(0, 48), slice(48, 96)]
    threads = [threading.Thread(target=run, args=(h,)) for h in halves]
    for t in threads:
        t.start()
    for t in threads:
        t.join(60)
    assert not errors and not any(t.is_alive() for t in threads)
    for r in range(tp):
        oracle_transfer(case, imgs[r], cpu_img, gids, cids, False, rank=r)
    assert np.array_equal(cpu.numpy(), cpu_img)
    grp.close()
