"""GPU XXH64 (flexkv_b200 C ABI) against the golden vectors of the xxHash
library the reference links, and against the oracle."""
import json
import os

import numpy as np
import pytest
import torch

from flexkv_b200 import c_ext
from kvcase import fill_bytes, sha, tokens

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "hash.json")))


def test_get_hash_size():
    assert c_ext.get_hash_size() == 8


def test_oneshot_vectors_via_hasher():
    h = c_ext.Hasher()
    for v in GOLD["oneshot"]:
        h.reset()
        data = np.frombuffer(bytes.fromhex(v["hex"]), dtype=np.uint8)
        if data.size:
            h.update(torch.from_numpy(data.copy()))
        assert h.digest() == v["xxh64"], data.size


@pytest.mark.parametrize("where", ["host", "device"])
@pytest.mark.parametrize("idx", range(len(GOLD["gen_hashes"])),
                         ids=[g["name"] for g in GOLD["gen_hashes"]])
def test_gen_hashes_golden(idx, where):
    g = GOLD["gen_hashes"][idx]
    toks = torch.from_numpy(tokens(g["n_tokens"], g["vocab"], g["seed"]))
    h = c_ext.Hasher()
    pre = bytes.fromhex(g["prefix_hex"])
    if pre:
        h.update(torch.frombuffer(bytearray(pre), dtype=torch.uint8))
    nb = g["num_blocks"]
    if where == "device":
        toks = toks.cuda()
        out = torch.zeros(nb, dtype=torch.uint64, device="cuda")
    else:
        out = torch.zeros(nb, dtype=torch.uint64)
    c_ext.gen_hashes(h, toks, g["tpb"], out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert sha(got) == g["sha256"], g["name"]
    assert h.digest() == g["final_digest_after"]


def test_streaming_odd_splits_and_raw_pointers():
    from oracle import oracle as O
    data = fill_bytes(5000, 42)
    rng = np.random.default_rng(3)
    host = torch.from_numpy(data.copy())
    dev = host.cuda()
    for trial in range(6):
        cuts = sorted(rng.integers(0, data.size + 1, 7).tolist())
        h = c_ext.Hasher()
        o = O.XXH64()
        prev = 0
        for i, c in enumerate(cuts + [data.size]):
            if c > prev:
                src = dev if (i + trial) % 2 else host
                h.update(src.data_ptr() + prev, c - prev)
                o.update(data[prev:c])
            prev = c
            assert h.digest() == o.digest()
        assert h.digest() == O.xxh64(data)


def test_gen_hashes_after_misaligned_update_matches_oracle():
    from oracle import oracle as O
    toks = tokens(16 * 37 + 5, 32000, 12)
    for pre_len in [1, 5, 8, 13, 24, 31, 32, 45]:
        pre = fill_bytes(pre_len, pre_len)
        h = c_ext.Hasher()
        h.update(torch.from_numpy(pre.copy()))
        out = torch.zeros(37, dtype=torch.uint64)
        c_ext.gen_hashes(h, torch.from_numpy(toks), 16, out)
        o = O.XXH64()
        o.update(pre)
        want = o.gen_hashes(toks, 16)
        assert np.array_equal(out.numpy(), want), pre_len
        assert h.digest() == o.digest()


def test_batched_golden_and_device_io():
    b = GOLD["batched"]
    toks = torch.from_numpy(tokens(sum(b["lens"]), b["vocab"], b["seed"]))
    offs = np.concatenate([[0], np.cumsum(b["lens"])]).tolist()
    out = c_ext.gen_hashes_batched(toks, offs, b["tpb"])
    assert out.tolist() == b["hashes"]
    out_d = c_ext.gen_hashes_batched(toks.cuda(), offs, b["tpb"])
    torch.cuda.synchronize()
    assert out_d.cpu().tolist() == b["hashes"]


def test_batched_many_requests_vs_oracle():
    from oracle import oracle as O
    rng = np.random.default_rng(5)
    lens = (rng.integers(1, 33, 256) * 16 + rng.integers(0, 16, 256)).tolist()
    toks = tokens(sum(lens), 152064, 21)
    offs = np.concatenate([[0], np.cumsum(lens)]).tolist()
    out = c_ext.gen_hashes_batched(torch.from_numpy(toks).cuda(), offs, 16)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.gen_hashes_batched(toks, offs, 16))


def test_hash_utils_style_usage():
    """flexkv/common/hash_utils.py:32-37 and block.py:41-57 usage."""
    from oracle import oracle as O
    toks = torch.randint(0, 10000, (32000,), dtype=torch.int64,
                         generator=torch.Generator().manual_seed(0))
    block_hashes = torch.zeros(toks.numel() // 16, dtype=torch.uint64)
    c_ext.gen_hashes(c_ext.Hasher(), toks, 16, block_hashes)
    assert np.array_equal(block_hashes.numpy(), O.gen_hashes(toks.numpy(), 16))
    h = c_ext.Hasher()
    h.update(toks[:5 * 16])
    assert h.digest() == int(block_hashes.numpy()[4])
