"""CPU: flexkv_b200's SSD tier against the reference's own SSD code.

The reference's csrc/transfer_ssd.cpp (thread-pool path) is compiled
unmodified from its tree into oracle/_ref/libref_ssd.so (oracle/Makefile,
with header stand-ins for libtorch and liburing).  For every case the two
implementations write the same pool into two separate sets of SSD files:
every byte of every file must agree.  Each then reads its files back into a
zeroed pool, and the reference also reads the files flexkv_b200 wrote (the
on-disk format is shared): the pools must agree byte for byte.  Skipped
when the reference library was not built (FLEXKV_REFERENCE unset at build
time)."""
import numpy as np
import pytest

from flexkv_b200 import c_ext
from oracle import oracle as O
from test_ssd import CASES, aligned, images, run, setup

pytestmark = pytest.mark.skipif(not O.reference_ssd_available(),
                                reason="oracle/_ref/libref_ssd.so not built (set FLEXKV_REFERENCE and build)")


def ref_run(ctx, st, pool, sids, cids, l0, nl, is_read, per_file, rr, mla, threads=16):
    ctx.transfer(l0, nl, pool.ctypes.data, sids, cids, st.cpu_layer_stride_in_bytes, st.cpu_kv_stride_in_bytes,
                 st.ssd_layer_stride_in_bytes, st.ssd_kv_stride_in_bytes, st.chunk_size_in_bytes,
                 st.block_stride_in_bytes, is_read, per_file, rr, threads, mla)


@pytest.mark.parametrize("threads", [1, 16])
@pytest.mark.parametrize("ci", range(len(CASES)), ids=[c[0] for c in CASES])
def test_files_and_pools_match_the_reference(ci, threads, tmp_path):
    case = CASES[ci]
    mla, rr, (l0, nl) = case[6], case[11], case[12]
    cpu_layout, f_ours, per_file, st, cids, sids = setup(case, tmp_path / "ours")
    _, f_ref, per_file_r, st_r, _, _ = setup(case, tmp_path / "ref")
    assert per_file == per_file_r and st == st_r
    pool = aligned(cpu_layout.get_total_elements() * 2, 177 + ci)
    ours = c_ext.SSDIOCTX(f_ours, len(f_ours), 0, 0)
    ref = O.RefSSDContext(f_ref)
    try:
        run(ours, st, pool, sids, cids, l0, nl, False, per_file, rr, mla, threads)
        ref_run(ref, st, pool, sids, cids, l0, nl, False, per_file, rr, mla, threads)
        for d_ours, d_ref in zip(images(f_ours), images(f_ref)):
            for a, b in zip(d_ours, d_ref):
                assert a.size == b.size and np.array_equal(a, b), "SSD files differ from the reference's"
        back_ours, back_ref, back_cross = (aligned(pool.size) for _ in range(3))
        run(ours, st, back_ours, sids, cids, l0, nl, True, per_file, rr, mla, threads)
        ref_run(ref, st, back_ref, sids, cids, l0, nl, True, per_file, rr, mla, threads)
        assert np.array_equal(back_ours, back_ref), "pool read back differs from the reference's"
        cross = O.RefSSDContext(f_ours)  # the reference reads the files flexkv_b200 wrote
        try:
            ref_run(cross, st, back_cross, sids, cids, l0, nl, True, per_file, rr, mla, threads)
        finally:
            cross.close()
        assert np.array_equal(back_cross, back_ref)
    finally:
        ours.close()
        ref.close()


def test_second_write_over_the_first_matches_the_reference(tmp_path):
    """Two writes in a row over overlapping SSD blocks (the later one wins),
    then a read of a different subset, against the reference."""
    case = CASES[1]
    mla, rr, (l0, nl) = case[6], case[11], case[12]
    cpu_layout, f_ours, per_file, st, cids, sids = setup(case, tmp_path / "ours")
    _, f_ref, _, _, _, _ = setup(case, tmp_path / "ref")
    pool1 = aligned(cpu_layout.get_total_elements() * 2, 501)
    pool2 = aligned(cpu_layout.get_total_elements() * 2, 502)
    ours, ref = c_ext.SSDIOCTX(f_ours, len(f_ours), 0, 0), O.RefSSDContext(f_ref)
    try:
        half = len(sids) // 2
        for pool, s_, c_ in ((pool1, sids, cids), (pool2, sids[half:], cids[:len(sids) - half])):
            run(ours, st, pool, s_, c_, l0, nl, False, per_file, rr, mla)
            ref_run(ref, st, pool, s_, c_, l0, nl, False, per_file, rr, mla)
        for d_ours, d_ref in zip(images(f_ours), images(f_ref)):
            for a, b in zip(d_ours, d_ref):
                assert np.array_equal(a, b)
        a, b = aligned(pool1.size), aligned(pool1.size)
        sub = slice(1, None, 2)
        run(ours, st, a, sids[sub], cids[sub], l0, nl, True, per_file, rr, mla)
        ref_run(ref, st, b, sids[sub], cids[sub], l0, nl, True, per_file, rr, mla)
        assert np.array_equal(a, b)
    finally:
        ours.close()
        ref.close()
