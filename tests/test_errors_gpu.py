"""GPU: invalid requests come back as RuntimeError before any launch; the
pools stay untouched (the reference kernel would fault or corrupt memory)."""
import numpy as np
import pytest
import torch

from flexkv_b200 import c_ext
from kvcase import Case
from gpu_util import Pools, initial_images

pytestmark = pytest.mark.gpu


def setup():
    case = Case("err", 2, 2, 64, 16, 16, 32)
    gpu, cpu = initial_images(case, 10, 11)
    return case, Pools(case, gpu, cpu)


def call(p, gids, cids, h2d=False, cpu=None, ptrs=None, **kw):
    st = p.st
    c_ext.transfer_kv_blocks(torch.tensor(gids, dtype=torch.int64),
                             p.ptrs if ptrs is None else ptrs, st["gpu_kv"], st["gpu_block"],
                             torch.tensor(cids, dtype=torch.int64), p.cpu if cpu is None else cpu,
                             st["cpu_kv"], st["cpu_layer"], st["cpu_block"], st["gpu_chunk"], 0,
                             -1, h2d, False, False, **kw)


def unchanged(p, before_cpu, before_gpu):
    assert np.array_equal(p.cpu_image(), before_cpu)
    for a, b in zip(p.gpu_images(), before_gpu):
        assert np.array_equal(a, b)


def test_cpu_id_past_pool():
    case, p = setup()
    bc, bg = p.cpu_image().copy(), [x.copy() for x in p.gpu_images()]
    with pytest.raises(RuntimeError, match="past the cpu pool"):
        call(p, [0, 1], [3, 32])
    with pytest.raises(RuntimeError, match="past the cpu pool"):
        call(p, [0, 1], [3, 32], h2d=True)
    unchanged(p, bc, bg)


def test_gpu_id_past_layer_and_negative_ids():
    case, p = setup()
    bc, bg = p.cpu_image().copy(), [x.copy() for x in p.gpu_images()]
    with pytest.raises(RuntimeError, match="past the gpu layer"):
        call(p, [16], [0], h2d=True, gpu_layer_bytes=p.st["gpu_layer_bytes"])
    with pytest.raises(RuntimeError, match="out of"):
        call(p, [-1], [0])
    with pytest.raises(RuntimeError, match="out of"):
        call(p, [0], [1 << 31])
    unchanged(p, bc, bg)


def test_misaligned_and_unpinned():
    case, p = setup()
    with pytest.raises(RuntimeError, match="aligned"):
        call(p, [0], [0], ptrs=p.ptrs + 8)
    pageable = torch.zeros_like(p.cpu, pin_memory=False)
    with pytest.raises(RuntimeError, match="page-locked"):
        call(p, [0], [0], cpu=pageable)
    with pytest.raises(RuntimeError, match="differ in length"):
        call(p, [0, 1], [0])
    with pytest.raises(RuntimeError, match="int64"):
        c_ext.transfer_kv_blocks(torch.tensor([0], dtype=torch.int32), p.ptrs, 0, 0,
                                 torch.tensor([0]), p.cpu, 0, 0, 0, 16, 0)


def test_context_survives_errors():
    """After the rejected calls a valid transfer still runs."""
    case, p = setup()
    with pytest.raises(RuntimeError):
        call(p, [0], [99])
    call(p, [1], [2])
    torch.cuda.synchronize()
