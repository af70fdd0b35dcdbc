"""CPU: the C-ABI library loads, exports every entry point the header
declares, and its host-only logic works without a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

from flexkv_b200 import _lib
from kvcase import make_ids

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    txt = open(os.path.join(ROOT, "include", "flexkv_b200.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(fkv_\w+)\s*\(", txt)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ["fkv_transfer_kv_blocks", "fkv_transfer_kv_blocks_ex", "fkv_tp_group_create",
                 "fkv_tp_group_transfer", "fkv_hasher_create", "fkv_hasher_update",
                 "fkv_hasher_digest", "fkv_gen_hashes", "fkv_get_hash_size"]:
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes signature table covers them all
    assert set(declared_functions()) <= set(_lib._SIGNATURES)


def test_hash_size_and_version():
    lib = _lib.load()
    assert lib.fkv_get_hash_size() == 8
    assert b"sm_100a" in lib.fkv_version()


def test_desc_init_defaults_and_layout():
    d = _lib.TransferDesc()
    ctypes.memset(ctypes.byref(d), 0x5A, ctypes.sizeof(d))
    _lib.load().fkv_transfer_desc_init(ctypes.byref(d))
    assert (d.transfer_sms, d.synchronous, d.ce_min_run_bytes, d.num_ce_streams) == (-1, 1, -1, 0)
    assert d.num_blocks == 0 and d.cpu_pool_bytes == 0 and d.ce_schedule == -1 and d.is_host_to_device == 1


def py_runs(g, c):
    runs, i = [], 0
    while i < len(g):
        r = 1
        while i + r < len(g) and g[i + r] == g[i] + r and c[i + r] == c[i] + r:
            r += 1
        runs.append((int(g[i]), int(c[i]), r))
        i += r
    return runs


def test_coalesce_runs_matches_python():
    lib = _lib.load()
    for seed, frac in [(1, 0.0), (2, 0.5), (3, 1.0)]:
        g, c = make_ids(500, 4096, 8192, seed, frac, max_run=16)
        out = np.zeros(3 * 500, dtype=np.int64)
        n = lib.fkv_coalesce_runs(g.ctypes.data, c.ctypes.data, len(g), out.ctypes.data, 500)
        assert [tuple(x) for x in out[:3 * n].reshape(-1, 3).tolist()] == py_runs(g, c)
    # too-small output
    g = np.arange(10, dtype=np.int64)
    c = g[::-1].copy()
    out = np.zeros(3, dtype=np.int64)
    assert lib.fkv_coalesce_runs(g.ctypes.data, c.ctypes.data, 10, out.ctypes.data, 1) == -1
    assert lib.fkv_coalesce_runs(g.ctypes.data, g.ctypes.data, 10, out.ctypes.data, 1) == 1
    assert out.tolist() == [0, 0, 10]


def test_invalid_arguments_rejected_before_any_device_work():
    lib = _lib.load()
    d = _lib.TransferDesc()
    lib.fkv_transfer_desc_init(ctypes.byref(d))
    d.num_blocks = -1
    rc = lib.fkv_transfer_kv_blocks_ex(ctypes.byref(d), None)
    assert rc == _lib.FKV_ERR_INVALID_ARG
    assert b"non-negative" in lib.fkv_last_error()
    lib.fkv_transfer_desc_init(ctypes.byref(d))
    d.chunk_size_in_bytes = -16
    assert lib.fkv_transfer_kv_blocks_ex(ctypes.byref(d), None) == _lib.FKV_ERR_INVALID_ARG


def test_tp_group_rejects_bad_arguments():
    lib = _lib.load()
    h = ctypes.c_void_p()
    assert lib.fkv_tp_group_create(0, 0, None, None, 0, None, 0, ctypes.byref(h)) == _lib.FKV_ERR_INVALID_ARG
    assert lib.fkv_tp_group_transfer(None, None, None, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 0, 0, 0, 0) \
        == _lib.FKV_ERR_INVALID_ARG


def test_ipc_argument_checks_without_gpu():
    """IPC entry points reject bad arguments before touching CUDA, and the
    Python handle refuses host tensors like the reference's."""
    import ctypes
    import torch
    from flexkv_b200 import _lib
    from flexkv_b200.memory_handle import TensorSharedHandle
    L = _lib.load()
    h = _lib.IpcHandle()
    assert ctypes.sizeof(h) == 104
    assert L.fkv_ipc_export(None, 16, ctypes.byref(h)) == _lib.FKV_ERR_INVALID_ARG
    h.alloc_bytes, h.offset, h.bytes = 100, 96, 8  # range past the allocation
    out = ctypes.c_void_p()
    assert L.fkv_ipc_open(ctypes.byref(h), 0, ctypes.byref(out)) == _lib.FKV_ERR_INVALID_ARG
    assert L.fkv_ipc_close(ctypes.c_void_p(0x1000)) == _lib.FKV_ERR_INVALID_ARG
    assert L.fkv_ipc_open_count() == 0
    with pytest.raises(ValueError):
        TensorSharedHandle(torch.zeros(4))
