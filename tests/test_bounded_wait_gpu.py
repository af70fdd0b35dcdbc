"""GPU: a bounded device-side wait that runs out.

The XXH64 chain kernel hands 8 KiB token tiles from a producer warp to a
chain warp through mbarriers; every wait gives up after a time limit and
reports FKV_ERR_TIMEOUT through a host-mapped error word.  Here the producer
is told to stop early (fkv_hasher_update_bounded), so the chain warp waits
for a tile that never comes: the call must come back with FKV_ERR_TIMEOUT
within the short limit, the kernel must have returned (no fault, no hang),
the hasher must keep its state from before the call, and the same device
must then hash correctly against the CPU oracle.  No GPU fault is made: the
wait simply has nothing to wait for, and it is bounded.
"""
import time

import numpy as np
import pytest
import torch

from flexkv_b200 import _lib, c_ext
from kvcase import tokens
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms


def bounded_update(h, data: torch.Tensor, limit_ns: int, producer_tiles: int) -> int:
    lib = _lib.load()
    return lib.fkv_hasher_update_bounded(h._handle, data.data_ptr(), data.numel() * data.element_size(),
                                         limit_ns, producer_tiles, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("producer_tiles", [0, 1, 3])
def test_chain_wait_runs_out_and_the_context_stays_usable(producer_tiles):
    lib = _lib.load()
    toks = tokens(8192, 32000, 11)  # 64 KiB: 8 tiles of 8 KiB
    data = torch.from_numpy(toks).cuda()
    h = c_ext.Hasher()
    t0 = time.perf_counter()
    rc = bounded_update(h, data, LIMIT_NS, producer_tiles)
    dt = time.perf_counter() - t0
    assert rc == _lib.FKV_ERR_TIMEOUT
    assert b"timed out" in lib.fkv_last_error()
    assert dt < 1.0, f"the 1 ms limit held for {dt:.3f} s"
    # The hasher kept its state from before the call (empty): the same data
    # hashed in full now gives the one-shot digest.
    _lib.check(bounded_update(h, data, 2_000_000_000, -1), "fkv_hasher_update_bounded")
    assert h.digest() == O.xxh64(toks.view(np.uint8).tobytes())
    # The device still runs the product path bit-exactly.
    out = torch.zeros(len(toks) // 16, dtype=torch.uint64)
    c_ext.gen_hashes(c_ext.Hasher(), torch.from_numpy(toks), 16, out)
    assert np.array_equal(out.numpy(), O.gen_hashes(toks, 16))
    dev_out = torch.zeros(len(toks) // 16, dtype=torch.uint64, device="cuda")
    c_ext.gen_hashes(c_ext.Hasher(), data, 16, dev_out)
    assert np.array_equal(dev_out.cpu().numpy(), O.gen_hashes(toks, 16))


def test_bounded_update_rejects_limits_outside_its_range():
    h = c_ext.Hasher()
    data = torch.from_numpy(tokens(64, 32000, 12)).cuda()
    assert bounded_update(h, data, 0, -1) == _lib.FKV_ERR_INVALID_ARG
    assert bounded_update(h, data, 3_000_000_000, -1) == _lib.FKV_ERR_INVALID_ARG
    assert bounded_update(h, data, LIMIT_NS, -2) == _lib.FKV_ERR_INVALID_ARG
