"""CPU: the oracle (oracle/oracle.c) pinned against the golden vectors.

hash.json comes from the xxHash library the reference links (python xxhash,
cross-checked with libxxhash.so.0); transfer.json from a view-based
restatement over the reference's own KVCacheLayout strides; layouts.json from
the reference's KVCacheLayout itself.
"""
import json
import os

import numpy as np
import pytest

from kvcase import Case, fill_bytes, sha, tokens
from oracle import oracle as O
from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    with open(os.path.join(GOLD, name)) as f:
        return json.load(f)


def test_xxh64_empty_is_spec_value():
    assert O.xxh64(b"") == 0xEF46DB3751D8E999


def test_xxh64_oneshot_golden():
    for v in load("hash.json")["oneshot"]:
        assert O.xxh64(bytes.fromhex(v["hex"])) == v["xxh64"], len(v["hex"]) // 2


def test_xxh64_streaming_any_split():
    data = fill_bytes(777, 5).tobytes()
    want = O.xxh64(data)
    rng = np.random.default_rng(0)
    for _ in range(50):
        cuts = sorted(rng.integers(0, len(data) + 1, rng.integers(1, 8)).tolist())
        h = O.XXH64()
        prev = 0
        for c in cuts + [len(data)]:
            h.update(data[prev:c])
            prev = c
        assert h.digest() == want


@pytest.mark.parametrize("idx", range(9))
def test_gen_hashes_golden(idx):
    g = load("hash.json")["gen_hashes"][idx]
    toks = tokens(g["n_tokens"], g["vocab"], g["seed"])
    h = O.XXH64()
    h.update(bytes.fromhex(g["prefix_hex"]))
    out = h.gen_hashes(toks, g["tpb"])
    assert out.size == g["num_blocks"]
    assert sha(out) == g["sha256"], g["name"]
    if "hashes" in g:
        assert out.tolist() == g["hashes"]
    # hash.cpp:61-65 leaves the hasher after the last block
    assert h.digest() == g["final_digest_after"]


def test_gen_hashes_batched_golden():
    b = load("hash.json")["batched"]
    toks = tokens(sum(b["lens"]), b["vocab"], b["seed"])
    offs = np.concatenate([[0], np.cumsum(b["lens"])])
    assert O.gen_hashes_batched(toks, offs, b["tpb"]).tolist() == b["hashes"]


def test_prefix_property_matches_oneshot():
    toks = tokens(16 * 10, 32000, 3)
    hs = O.gen_hashes(toks, 16)
    for i in range(10):
        assert hs[i] == O.xxh64(toks[:(i + 1) * 16].tobytes())


@pytest.mark.parametrize("idx", range(11))
def test_transfer_oracle_golden(idx):
    g = load("transfer.json")[idx]
    case = Case(**g["case"])
    st = case.strides()
    gids = np.array(g["gpu_ids"], dtype=np.int64)
    cids = np.array(g["cpu_ids"], dtype=np.int64)
    gpu = [fill_bytes(st["gpu_layer_bytes"], g["gpu_seed_base"] + l) for l in range(case.gran)]
    cpu = fill_bytes(st["cpu_pool_bytes"], g["cpu_seed"])
    off = 0 if case.is_mla else g["rank"] * st["gpu_chunk"]
    args = dict(gpu_kv_stride=st["gpu_kv"], gpu_block_stride=st["gpu_block"],
                cpu_kv_stride=st["cpu_kv"], cpu_layer_stride=st["cpu_layer"],
                cpu_block_stride=st["cpu_block"], cpu_startoff=off, chunk=st["gpu_chunk"],
                is_mla=case.is_mla)
    O.transfer(len(gids), case.layer_id, gids, gpu, cpu_block_ids=cids, cpu_pool=cpu,
               is_host_to_device=False, num_threads=3, **args)
    assert sha(cpu) == g["d2h_cpu_sha256"], g["name"]
    gpu2 = [np.zeros(st["gpu_layer_bytes"], dtype=np.uint8) for _ in range(case.gran)]
    O.transfer(len(gids), case.layer_id, gids, gpu2, cpu_block_ids=cids, cpu_pool=cpu,
               is_host_to_device=True, num_threads=1, **args)
    assert [sha(x) for x in gpu2] == g["h2d_gpu_sha256"], g["name"]


def test_layout_mirror_matches_reference():
    for key, v in load("layouts.json").items():
        if "/cpu/" in key:
            lt, L, n, tpb, H, D, mla = v["args"]
            lay = KVCacheLayout(KVCacheLayoutType[lt], L, n, tpb, H, D, mla)
            assert list(lay.kv_shape) == v["kv_shape"], key
            assert lay.get_chunk_size() == v["chunk"]
            assert lay.get_layer_stride() == v["layer_stride"], key
            assert lay.get_kv_stride() == v["kv_stride"], key
            assert lay.get_block_stride() == v["block_stride"], key
            assert lay.get_total_elements() == v["total"], key
        else:
            lt, L, n, tpb, H, D, mla, tp = v["args"]
            lay = KVCacheLayout(KVCacheLayoutType[lt], L, n, tpb, H, D, mla)
            lay = lay.div_head(tp) if not mla else lay
            per = lay.div_layer(L)
            assert list(lay.kv_shape) == v["kv_shape"], key
            assert per.get_chunk_size() == v["chunk"]
            assert per.get_kv_stride() == v["kv_stride"], key
            assert per.get_block_stride() == v["block_stride"], key
            assert per.get_total_elements() == v["total_per_layer"], key


def test_batched_hash_threads_agree():
    """The n-core CPU baseline of the batched hash gives the same digests."""
    rng = np.random.default_rng(12)
    sizes = rng.integers(0, 40, 97) * 3 + rng.integers(0, 5, 97)  # ragged, some shorter than a block
    offs = np.concatenate([[0], np.cumsum(sizes)])
    toks = rng.integers(0, 152064, int(sizes.sum())).astype(np.int64)
    one = O.gen_hashes_batched(toks, offs, 16)
    for n in (2, 5, 200):
        assert np.array_equal(O.gen_hashes_batched(toks, offs, 16, n), one)
