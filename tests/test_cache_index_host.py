"""CPU tests of the host side of flexkv_b200.cache_index: how the
reference-facing put_requests / get_requests turn (token_ids, token_mask,
slot_mapping) into blocks and GPU block ids (cache_engine.py:150-203,
550-602), the return masks they build, their argument errors, and the
batch packing.  The device calls are replaced by recorders; no GPU."""
import numpy as np
import pytest
import torch

from flexkv_b200 import cache_index as C


def index(tpb=4):
    ci = object.__new__(C.CpuCacheIndex)  # no device index: the packed calls are recorded below
    ci.tokens_per_block = tpb
    ci.num_total_blocks = 64
    ci.device = 0
    ci.calls = []

    def put_packed(ptr, offsets, gids, layout, mark_ready=True, synchronous=True):
        ci.calls.append(("put", offsets.copy(), np.asarray(gids).copy()))
        R = len(offsets) - 1
        blk = C._blk_off(offsets, tpb)
        nb = int(blk[-1])
        # pretend every request skipped one block and moved the rest
        n = blk[1:] - blk[:-1]
        sk = np.minimum(n, 1)
        return C.PutBatch(sk, n - sk, np.arange(nb), np.asarray(gids)[:nb], np.zeros(nb, np.uint64), blk)

    def get_packed(ptr, offsets, gids, layout, block_starts=None, synchronous=True, layer_granularity=-1,
                   group_events=None):
        ci.calls.append(("get", offsets.copy(), np.asarray(gids).copy(), list(block_starts)))
        R = len(offsets) - 1
        goff = np.zeros(R + 1, dtype=np.int64)
        n = (offsets[1:] - offsets[:-1]) // tpb
        np.cumsum(n - np.asarray(block_starts), out=goff[1:])
        moved = (n - np.asarray(block_starts)) // 2
        return C.GetBatch(np.asarray(block_starts), moved, np.arange(int(goff[-1])), np.asarray(gids), goff)

    ci.put_packed = put_packed
    ci.get_packed = get_packed
    return ci


def slots_for(gpu_blocks, tpb, tail):
    g = np.asarray(gpu_blocks, dtype=np.int64)
    s = np.concatenate([np.repeat(g, tpb) * tpb + np.tile(np.arange(tpb), len(g)), 900 * tpb + np.arange(tail)])
    return torch.from_numpy(s.astype(np.int64))


def test_put_requests_maps_slots_to_blocks_and_ignores_the_partial_block():
    ci = index(4)
    tok = torch.arange(4 * 3 + 2, dtype=torch.int64)  # 3 full blocks + 2 tokens
    masks, res = ci.put_requests([(tok, torch.ones(len(tok), dtype=torch.bool), slots_for([7, 2, 9], 4, 2))],
                                 layout=None)
    kind, offsets, gids = ci.calls[0]
    assert kind == "put" and offsets.tolist() == [0, 12] and gids.tolist() == [7, 2, 9]
    # skipped 1, moved 2 -> tokens [4, 12) of 14
    assert masks[0].tolist() == [False] * 4 + [True] * 8 + [False] * 2


def test_put_requests_empty_mask_and_short_requests():
    ci = index(4)
    tok = torch.arange(10, dtype=torch.int64)
    short = torch.arange(3, dtype=torch.int64)
    masks, _ = ci.put_requests([(tok, torch.zeros(10, dtype=torch.bool), torch.zeros(0, dtype=torch.int64)),
                                (short, torch.ones(3, dtype=torch.bool), torch.arange(3))], layout=None)
    _, offsets, gids = ci.calls[0]
    assert offsets.tolist() == [0, 0, 0] and gids.tolist() == []
    assert not masks[0].any() and not masks[1].any()


@pytest.mark.parametrize("mask,err", [
    ([False] * 4 + [True] * 8, "first block"),        # starts at block 1
    ([True] * 4 + [False] * 8, "every full block"),   # stops before the last full block
])
def test_put_requests_rejects_masks_the_reference_cannot_insert(mask, err):
    ci = index(4)
    tok = torch.arange(12, dtype=torch.int64)
    m = torch.tensor(mask)
    with pytest.raises(ValueError, match=err):
        ci.put_requests([(tok, m, torch.arange(int(m.sum())))], layout=None)


def test_put_requests_checks_lengths():
    ci = index(4)
    tok = torch.arange(8, dtype=torch.int64)
    with pytest.raises(ValueError, match="disagree"):
        ci.put_requests([(tok, torch.ones(8, dtype=torch.bool), torch.arange(7))], layout=None)


def test_get_requests_reads_from_the_first_masked_block():
    ci = index(4)
    tok = torch.arange(4 * 5 + 1, dtype=torch.int64)  # 5 full blocks + 1 token
    mask = torch.zeros(len(tok), dtype=torch.bool)
    mask[8:] = True                                   # blocks 2..4 (and the partial token)
    masks, res = ci.get_requests([(tok, mask, slots_for([11, 12, 13], 4, 1))], layout=None)
    kind, offsets, gids, starts = ci.calls[0]
    assert kind == "get" and offsets.tolist() == [0, 20] and gids.tolist() == [11, 12, 13] and starts == [2]
    # moved (5-2)//2 = 1 block from block 2 -> tokens [8, 12)
    assert masks[0].tolist() == [False] * 8 + [True] * 4 + [False] * 9


def test_get_requests_mask_must_reach_the_last_full_block():
    ci = index(4)
    tok = torch.arange(16, dtype=torch.int64)
    mask = torch.zeros(16, dtype=torch.bool)
    mask[4:8] = True
    with pytest.raises(ValueError, match="last full block"):
        ci.get_requests([(tok, mask, torch.arange(4))], layout=None)


def test_pack_tokens_numpy_tensor_and_empty():
    a, b = np.arange(5, dtype=np.int32), np.arange(7, dtype=np.int64)
    buf, off, ptr = C._pack_tokens([a, b])
    assert off.tolist() == [0, 5, 12] and buf.dtype == np.int64 and buf.tolist() == a.tolist() + b.tolist()
    buf, off, ptr = C._pack_tokens([torch.arange(3), torch.arange(2)])
    assert off.tolist() == [0, 3, 5] and buf.tolist() == [0, 1, 2, 0, 1]
    buf, off, ptr = C._pack_tokens([])
    assert off.tolist() == [0] and ptr != 0
    buf, off, ptr = C._pack_tokens([np.zeros(0, np.int64)])
    assert off.tolist() == [0, 0] and ptr != 0


def test_batch_views_slice_per_request():
    blk = np.array([0, 3, 3, 5])
    pb = C.PutBatch(np.array([1, 0, 0]), np.array([2, 0, 2]), np.arange(10, 15), np.arange(20, 25),
                    np.arange(5, dtype=np.uint64), blk)
    assert [x.tolist() for x in pb.cpu_blocks] == [[11, 12], [], [13, 14]]
    assert [x.tolist() for x in pb.gpu_blocks] == [[21, 22], [], [23, 24]]
    assert [x.tolist() for x in pb.block_hashes] == [[0, 1, 2], [], [3, 4]]
    mb = C.MatchBatch(np.array([2, 0, 1]), np.array([1, 0, 1]), np.array([4, 5, -1, 6, -1]), blk)
    assert [x.tolist() for x in mb.physical_blocks] == [[4, 5], [], [6]]
