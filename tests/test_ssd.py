"""CPU: the SSD tier (SSDIOCTX / transfer_kv_blocks_ssd mirror) against the
oracle's restatement of csrc/transfer_ssd.cpp on in-memory file images.
Every byte of every file and of the pool is compared.  No GPU needed: the
tier moves bytes between the host pool and files."""
import os

import numpy as np
import pytest
import torch

from flexkv_b200 import c_ext
from flexkv_b200._lib import FKV_ERR_IO, FKV_ERR_OUT_OF_RANGE, FlexKVError
from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
from flexkv_b200.ssd import SsdStrides, allocate_ssd_files
from kvcase import fill_bytes, make_ids
from oracle import oracle as O

BW, LW = KVCacheLayoutType.BLOCKWISE, KVCacheLayoutType.LAYERWISE

# name, layout, L, tpb, H, D, mla, cpu_blocks, ssd_blocks, devices, max_blocks_per_file,
# round_robin, (start_layer, num_layers), blocks moved
CASES = [
    ("bw_1dev", BW, 4, 16, 2, 64, False, 64, 64, 1, 64, 1, (0, 4), 24),
    ("bw_2dev_3files_rr4", BW, 4, 16, 2, 64, False, 64, 96, 2, 16, 4, (0, 4), 40),
    ("bw_partial_layers", BW, 5, 16, 2, 64, False, 48, 48, 1, 20, 1, (1, 3), 20),
    ("lw_2dev_partial_layers", LW, 6, 16, 2, 64, False, 64, 64, 2, 12, 1, (2, 3), 30),
    ("bw_mla_direct_reads", BW, 3, 64, 1, 64, True, 48, 48, 1, 48, 1, (0, 3), 20),
    ("lw_mla_rr2", LW, 3, 16, 1, 72, True, 48, 64, 2, 10, 2, (1, 2), 20),
]


def aligned(nbytes, fill_seed=None, align=4096):
    raw = np.zeros(nbytes + align, np.uint8)
    off = (-raw.ctypes.data) % align
    a = raw[off:off + nbytes]
    if fill_seed is not None:
        a[:] = fill_bytes(nbytes, fill_seed)
    return a


def images(files):
    return [[np.fromfile(p, dtype=np.uint8) for p in files[d]] for d in sorted(files)]


def setup(case, tmp_path):
    name, typ, L, tpb, H, D, mla, ncpu, nssd, ndev, mbpf, rr, (l0, nl), n = case
    cpu_layout = KVCacheLayout(typ, L, ncpu, tpb, H, D, mla)
    ssd_layout = KVCacheLayout(typ, L, nssd, tpb, H, D, mla)
    files, per_file = allocate_ssd_files(ssd_layout, 2, [str(tmp_path / f"dev{i}") for i in range(ndev)],
                                         max_blocks_per_file=mbpf)
    nfiles = sum(len(v) for v in files.values())
    st = SsdStrides.of(cpu_layout, ssd_layout, nfiles, 2)
    cids, sids = make_ids(n, ncpu, nssd, 4242 + n, 0.5, max_run=8)
    return cpu_layout, files, per_file, st, cids, sids


def run(ctx, st, pool, sids, cids, l0, nl, is_read, per_file, rr, mla, threads=16, layer_dtype=torch.int32):
    c_ext.transfer_kv_blocks_ssd(
        ioctx=ctx, cpu_layer_id_list=torch.arange(l0, l0 + nl, dtype=layer_dtype),
        cpu_tensor_ptr=pool.ctypes.data, ssd_block_ids=torch.from_numpy(sids),
        cpu_block_ids=torch.from_numpy(cids), cpu_layer_stride_in_bytes=st.cpu_layer_stride_in_bytes,
        cpu_kv_stride_in_bytes=st.cpu_kv_stride_in_bytes, ssd_layer_stride_in_bytes=st.ssd_layer_stride_in_bytes,
        ssd_kv_stride_in_bytes=st.ssd_kv_stride_in_bytes, chunk_size_in_bytes=st.chunk_size_in_bytes,
        block_stride_in_bytes=st.block_stride_in_bytes, is_read=is_read, num_blocks_per_file=per_file,
        round_robin=rr, num_threads_per_device=threads, is_mla=mla)


def oracle(imgs, st, pool, sids, cids, l0, nl, is_read, rr, mla):
    O.ssd_transfer(imgs, l0, nl, pool, sids, cids, st.cpu_layer_stride_in_bytes, st.cpu_kv_stride_in_bytes,
                   st.ssd_layer_stride_in_bytes, st.ssd_kv_stride_in_bytes, st.chunk_size_in_bytes,
                   st.block_stride_in_bytes, is_read, rr, mla)


def io_uring_available() -> bool:
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "f")
        open(p, "wb").close()
        ctx = c_ext.SSDIOCTX({0: [p]}, 1, 8, 0)
        ok = ctx.uses_io_uring
        ctx.close()
    return ok


@pytest.mark.parametrize("engine", ["threads1", "threads16", "io_uring"])
@pytest.mark.parametrize("ci", range(len(CASES)), ids=[c[0] for c in CASES])
def test_write_then_read_matches_oracle(ci, engine, tmp_path):
    """Both request engines: the thread pool (1 or 16 threads per device)
    and io_uring (64 entries)."""
    if engine == "io_uring" and not io_uring_available():
        pytest.skip("io_uring not available on this kernel")
    threads = 1 if engine == "threads1" else 16
    case = CASES[ci]
    mla, rr, (l0, nl) = case[6], case[11], case[12]
    cpu_layout, files, per_file, st, cids, sids = setup(case, tmp_path)
    pool = aligned(cpu_layout.get_total_elements() * 2, 77 + ci)
    want = images(files)  # fresh files are all zero
    ctx = c_ext.SSDIOCTX(files, len(files), 64 if engine == "io_uring" else 0, 0)
    assert ctx.uses_io_uring == (engine == "io_uring")
    run(ctx, st, pool, sids, cids, l0, nl, False, per_file, rr, mla, threads)
    oracle(want, st, pool, sids, cids, l0, nl, False, rr, mla)
    got = images(files)
    for gd, wd in zip(got, want):
        for g, w in zip(gd, wd):
            assert g.size == w.size and np.array_equal(g, w)
    back = aligned(pool.size)
    run(ctx, st, back, sids, cids, l0, nl, True, per_file, rr, mla, threads)
    ref = np.zeros_like(back)
    oracle(want, st, ref, sids, cids, l0, nl, True, rr, mla)
    assert np.array_equal(back, ref)
    ctx.close()


def test_requests_are_merged(tmp_path):
    """A joint run of 8 blocks: one request for all layers of all 8 blocks
    in a BLOCKWISE file, one per (layer, kv) in a LAYERWISE one."""
    for typ, want in ((BW, 1), (LW, 4 * 2)):
        cpu_layout = KVCacheLayout(typ, 4, 32, 16, 2, 64)
        ssd_layout = KVCacheLayout(typ, 4, 32, 16, 2, 64)
        files, per_file = allocate_ssd_files(ssd_layout, 2, str(tmp_path / typ.value), max_blocks_per_file=32)
        st = SsdStrides.of(cpu_layout, ssd_layout, 1, 2)
        pool = aligned(cpu_layout.get_total_elements() * 2, 5)
        ctx = c_ext.SSDIOCTX(files, 1)
        ids = np.arange(8, 16, dtype=np.int64)
        run(ctx, st, pool, ids, ids + 4, 0, 4, False, per_file, 1, False)
        n_ios, n_bytes = ctx.last_stats()
        assert n_ios == want and n_bytes == 8 * 4 * 2 * st.chunk_size_in_bytes
        ctx.close()


def test_empty_transfer_is_a_no_op(tmp_path):
    case = CASES[0]
    cpu_layout, files, per_file, st, _, _ = setup(case, tmp_path)
    pool = aligned(cpu_layout.get_total_elements() * 2, 1)
    before = images(files)
    ctx = c_ext.SSDIOCTX(files, 1)
    e = np.zeros(0, np.int64)
    run(ctx, st, pool, e, e, 0, 4, False, per_file, 1, False)
    for gd, wd in zip(images(files), before):
        for g, w in zip(gd, wd):
            assert np.array_equal(g, w)


def test_errors(tmp_path):
    case = CASES[0]
    cpu_layout, files, per_file, st, cids, sids = setup(case, tmp_path)
    pool = aligned(cpu_layout.get_total_elements() * 2, 1)
    ctx = c_ext.SSDIOCTX(files, 1)
    # a read past the end of the file
    far = np.array([per_file + 3], np.int64)
    with pytest.raises(FlexKVError) as ei:
        run(ctx, st, pool, far, np.array([0], np.int64), 0, 4, True, per_file, 1, False)
    assert ei.value.code == FKV_ERR_IO
    # ids outside [0, 2^31)
    with pytest.raises(FlexKVError) as ei:
        run(ctx, st, pool, np.array([-1], np.int64), np.array([0], np.int64), 0, 4, False, per_file, 1, False)
    assert ei.value.code == FKV_ERR_OUT_OF_RANGE
    # int64 ids required, as the reference's TORCH_CHECK
    with pytest.raises(RuntimeError):
        c_ext.transfer_kv_blocks_ssd(ctx, torch.arange(0, 4, dtype=torch.int32), pool.ctypes.data,
                                     torch.zeros(1, dtype=torch.int32), torch.zeros(1, dtype=torch.int64),
                                     0, 0, 0, 0, 4096, 4096, False, per_file)
    # the optional CPU bound
    with pytest.raises(FlexKVError) as ei:
        c_ext.transfer_kv_blocks_ssd(ctx, torch.arange(0, 4, dtype=torch.int32), pool.ctypes.data,
                                     torch.from_numpy(sids[:1]), torch.tensor([cpu_layout.num_block]),
                                     st.cpu_layer_stride_in_bytes, st.cpu_kv_stride_in_bytes,
                                     st.ssd_layer_stride_in_bytes, st.ssd_kv_stride_in_bytes,
                                     st.chunk_size_in_bytes, st.block_stride_in_bytes, True, per_file,
                                     cpu_pool_bytes=pool.size)
    assert ei.value.code == FKV_ERR_OUT_OF_RANGE
    ctx.close()
    with pytest.raises(FlexKVError) as ei:
        c_ext.SSDIOCTX({0: [str(tmp_path / "missing.bin")]}, 1)
    assert ei.value.code == FKV_ERR_IO


@pytest.mark.parametrize("ci", [1, 3, 5], ids=[CASES[i][0] for i in (1, 3, 5)])
def test_reference_style_loop_agrees(ci, tmp_path):
    """The C restatement of the reference's per-chunk loop (the bench's
    reference arm) writes the same files and reads the same pool."""
    case = CASES[ci]
    mla, rr, (l0, nl) = case[6], case[11], case[12]
    cpu_layout, files, per_file, st, cids, sids = setup(case, tmp_path)
    pool = aligned(cpu_layout.get_total_elements() * 2, 500 + ci)
    ref = O.SsdRefContext(files, len(files))
    ref.transfer(l0, nl, pool.ctypes.data, sids, cids, st, False, rr, 4, mla)
    want = images(files)
    back_ref = aligned(pool.size)
    ref.transfer(l0, nl, back_ref.ctypes.data, sids, cids, st, True, rr, 4, mla)
    ref.close()
    for d in files.values():
        for p in d:
            with open(p, "r+b") as f:
                f.truncate(0)
                f.truncate(per_file * cpu_layout.get_elements_per_block() * 2)
    ctx = c_ext.SSDIOCTX(files, len(files))
    run(ctx, st, pool, sids, cids, l0, nl, False, per_file, rr, mla)
    for gd, wd in zip(images(files), want):
        for g, w in zip(gd, wd):
            assert np.array_equal(g, w)
    back = aligned(pool.size)
    run(ctx, st, back, sids, cids, l0, nl, True, per_file, rr, mla)
    assert np.array_equal(back, back_ref)
    ctx.close()


def test_allocation_and_stride_helpers(tmp_path):
    """allocate_ssd_files follows SSDAllocator.allocate (allocator.py:132-200);
    SsdStrides follows the SSD worker (worker.py:512-520)."""
    lay = KVCacheLayout(LW, 4, 30, 16, 2, 64)
    with pytest.raises(ValueError):  # blocks must split evenly over the devices
        allocate_ssd_files(lay, 2, [str(tmp_path / "a"), str(tmp_path / "b"), str(tmp_path / "c"),
                                    str(tmp_path / "d")], max_blocks_per_file=8)
    files, per_file = allocate_ssd_files(lay, 2, [str(tmp_path / "a"), str(tmp_path / "b")],
                                         max_blocks_per_file=4)
    assert per_file == 4 and [len(v) for v in files.values()] == [4, 4]  # ceil(15 / 4) per device
    block_bytes = lay.get_elements_per_block() * 2
    for v in files.values():
        for p in v:
            assert os.path.getsize(p) == per_file * block_bytes
    st = SsdStrides.of(lay, lay, 8, 2)
    per = lay.div_block(8, padding=True)  # ceil(30 / 8) = 4 blocks per file
    assert per.num_block == 4
    assert st.ssd_layer_stride_in_bytes == per.get_layer_stride() * 2
    assert st.ssd_kv_stride_in_bytes == per.get_kv_stride() * 2
    assert st.block_stride_in_bytes == lay.get_block_stride() * 2
    with pytest.raises(ValueError):  # one layout type on both sides, as the reference requires
        SsdStrides.of(lay, KVCacheLayout(BW, 4, 30, 16, 2, 64), 8, 2)


def test_io_uring_errors_and_stats(tmp_path):
    """The io_uring path reports a read past the end of a file like the
    thread pool, and merges requests the same way."""
    if not io_uring_available():
        pytest.skip("io_uring not available on this kernel")
    case = CASES[0]
    cpu_layout, files, per_file, st, cids, sids = setup(case, tmp_path)
    pool = aligned(cpu_layout.get_total_elements() * 2, 1)
    ctx = c_ext.SSDIOCTX(files, 1, 16, 0)
    with pytest.raises(FlexKVError) as ei:
        run(ctx, st, pool, np.array([per_file + 3], np.int64), np.array([0], np.int64), 0, 4, True,
            per_file, 1, False)
    assert ei.value.code == FKV_ERR_IO
    ids = np.arange(8, 16, dtype=np.int64)
    run(ctx, st, pool, ids, ids + 4, 0, 4, False, per_file, 1, False)
    assert ctx.last_stats()[0] == 1  # BLOCKWISE joint run of 8 blocks: one request
    ctx.close()
