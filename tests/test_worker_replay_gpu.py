"""GPU: the calls FlexKV's own workers and hash helpers make, replayed
argument for argument through flexkv_b200.c_ext, against the CPU oracle.

tests/golden/worker_calls.json was recorded by running the reference's
unchanged flexkv/transfer/worker.py (GPUCPUTransferWorker and
tpGPUCPUTransferWorker: __init__, then _transfer_impl per op, worker.py
:212-313, 335-451) and flexkv/common/hash_utils.py (gen_hashes,
hash_tensor, :29-37) with flexkv.c_ext pointed at flexkv_b200.c_ext
(tests/golden/make_worker_golden.py).  Each recorded call is made here with
the same positional arguments in the same order (the recorded ids, the
layer-pointer table rebuilt from the recorded layers, the worker's strides,
transfer_sms, direction and flags), on real GPU layers and a page-locked
host pool; every byte of every layer and of the pool is then compared with
the CPU oracle applying the same calls to host images.  The hash calls are
checked against the digests the xxHash library produced when recording.
"""
import json
import os

import numpy as np
import pytest
import torch

from flexkv_b200 import c_ext
from kvcase import fill_bytes
from oracle import oracle as O

pytestmark = pytest.mark.gpu

FIX = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "worker_calls.json")))
WORKERS = [s for s in FIX["scenarios"] if "worker" in s]


def _ids(rec):
    return torch.tensor(rec["values"], dtype=getattr(torch, rec["dtype"]))


class Pools:
    """Rank x layer GPU tensors and one page-locked pool, with host images."""

    def __init__(self, sc):
        kv = 1 if sc["is_mla"] else 2
        L, tp = sc["layers"], sc["tp"]
        chunk = sc["tokens_per_block"] * sc["heads"] * sc["head_dim"] * 2
        layer_bytes = kv * sc["gpu_blocks"] * chunk
        heads_total = sc["heads"] * (1 if sc["is_mla"] else tp)
        cpu_bytes = L * kv * sc["cpu_blocks"] * sc["tokens_per_block"] * heads_total * sc["head_dim"] * 2
        self.imgs = [[fill_bytes(layer_bytes, 300 + 50 * r + l) for l in range(L)] for r in range(tp)]
        self.cpu_img = fill_bytes(cpu_bytes, 299)
        self.layers = [[torch.from_numpy(x.copy()).cuda() for x in rank] for rank in self.imgs]
        self.cpu = torch.from_numpy(self.cpu_img.copy())
        c_ext.cudaHostRegister(self.cpu)

    def check(self, what):
        torch.cuda.synchronize()
        assert np.array_equal(self.cpu.numpy(), self.cpu_img), f"host pool differs from the oracle after {what}"
        for r, rank in enumerate(self.layers):
            for l, t in enumerate(rank):
                assert np.array_equal(t.cpu().numpy(), self.imgs[r][l]), f"rank {r} layer {l} after {what}"

    def close(self):
        c_ext.cudaHostUnregister(self.cpu)


@pytest.mark.parametrize("sc", WORKERS, ids=[s["name"] for s in WORKERS])
def test_worker_calls_replayed_through_the_drop_in_module(sc):
    p = Pools(sc)
    group = None
    try:
        for i, call in enumerate(sc["calls"]):
            what = f"call {i} ({call['fn']})"
            if call["fn"] == "transfer_kv_blocks":
                assert call["num_positional"] == 15 and call["keywords"] == []
                g, c = _ids(call["gpu_block_id_tensor"]), _ids(call["cpu_block_id_tensor"])
                table = call["gpu_layer_ptrs_tensor"]
                ptrs = torch.tensor([p.layers[r][l].data_ptr() for r, l in table], dtype=torch.int64).pin_memory()
                args = (g.pin_memory(), ptrs, call["gpu_kv_stride_in_bytes"], call["gpu_block_stride_in_bytes"],
                        c.pin_memory(), p.cpu, call["cpu_kv_stride_in_bytes"], call["cpu_layer_stride_in_bytes"],
                        call["cpu_block_stride_in_bytes"], call["chunk_size_in_bytes"], call["start_layer_id"],
                        call["transfer_sms"], call["is_host_to_device"], call["use_ce_transfer"], call["is_mla"])
                with torch.cuda.stream(torch.cuda.Stream()):  # the worker's private stream (worker.py:253)
                    c_ext.transfer_kv_blocks(*args)
                O.transfer(len(g), call["start_layer_id"], g.numpy(), [p.imgs[r][l] for r, l in table],
                           call["gpu_kv_stride_in_bytes"], call["gpu_block_stride_in_bytes"], c.numpy(), p.cpu_img,
                           call["cpu_kv_stride_in_bytes"], call["cpu_layer_stride_in_bytes"],
                           call["cpu_block_stride_in_bytes"], 0, call["chunk_size_in_bytes"],
                           call["is_host_to_device"], call["is_mla"])
            elif call["fn"] == "TPTransferThreadGroup":
                blocks = [[p.layers[r][l] for r, l in rank] for rank in call["gpu_blocks"]]
                group = c_ext.TPTransferThreadGroup(call["num_gpus"], blocks, p.cpu, call["dp_group_id"])
                continue
            elif call["fn"] == "tp_group_transfer":
                assert group is not None and call["num_positional"] == 15
                g, c = _ids(call["gpu_block_id_tensor"]), _ids(call["cpu_block_id_tensor"])
                group.tp_group_transfer(g.pin_memory(), call["gpu_kv_stride_in_bytes"],
                                        call["gpu_block_stride_in_bytes"], call["gpu_chunk_size_in_bytes"],
                                        c.pin_memory(), call["cpu_kv_stride_in_bytes"],
                                        call["cpu_layer_stride_in_bytes"], call["cpu_block_stride_in_bytes"],
                                        call["cpu_chunk_size_in_bytes"], call["transfer_sms"],
                                        call["is_host_to_device"], call["use_ce_transfer"], call["layer_id"],
                                        call["layer_granularity"], call["is_mla"])
                l0, n = call["layer_id"], call["layer_granularity"]
                for r in range(len(p.layers)):
                    off = 0 if call["is_mla"] else r * call["gpu_chunk_size_in_bytes"]
                    O.transfer(len(g), l0, g.numpy(), p.imgs[r][l0:l0 + n], call["gpu_kv_stride_in_bytes"],
                               call["gpu_block_stride_in_bytes"], c.numpy(), p.cpu_img,
                               call["cpu_kv_stride_in_bytes"], call["cpu_layer_stride_in_bytes"],
                               call["cpu_block_stride_in_bytes"], off, call["gpu_chunk_size_in_bytes"],
                               call["is_host_to_device"], call["is_mla"])
            else:
                raise AssertionError(f"unexpected recorded call {call['fn']}")
            p.check(what)
    finally:
        if group is not None:
            group.close()
        p.close()


def test_hash_utils_calls_replayed_through_the_drop_in_module():
    sc = next(s for s in FIX["scenarios"] if s["name"] == "hash_utils")
    for i, call in enumerate(sc["calls"]):
        if call["fn"] == "gen_hashes":
            # hash_utils.gen_hashes: a fresh Hasher, a zeroed uint64 tensor, then c_ext.gen_hashes
            out = torch.zeros(call["block_hashes_len"], dtype=getattr(torch, call["block_hashes_dtype"]))
            c_ext.gen_hashes(c_ext.Hasher(), _ids(call["token_ids"]), call["tokens_per_block"], out)
            got = out.view(torch.int64).numpy().view(np.uint64)
            assert [str(x) for x in got.tolist()] == call["want"], f"call {i}"
        elif call["fn"] == "Hasher.digest":
            # hash_utils.hash_tensor: Hasher().update(tensor) per update, then digest()
            h = c_ext.Hasher()
            for u in call["updates"]:
                h.update(_ids(u))
            assert str(h.digest()) == call["digest"], f"call {i}"
        else:
            raise AssertionError(f"unexpected recorded call {call['fn']}")
