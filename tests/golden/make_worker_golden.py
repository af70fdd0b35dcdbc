"""Record the calls FlexKV's own transfer workers and hash helpers make into
the native module, with flexkv_b200.c_ext standing in for flexkv.c_ext
(run where the reference tree is; the fixture travels without it):

    python tests/golden/make_worker_golden.py --reference /path/to/FlexKV

The reference's flexkv/transfer/worker.py and flexkv/common/hash_utils.py are
imported unchanged, after `sys.modules["flexkv.c_ext"]` is pointed at a
recording front of flexkv_b200.c_ext: every call the reference code makes
is bound to flexkv_b200.c_ext's own signature (inspect.Signature.bind, so a
call the drop-in module would not accept fails here) and recorded.  The
workers are built through their own __init__ (GPUCPUTransferWorker,
worker.py:212-258; tpGPUCPUTransferWorker, :335-400): their strides come
from the reference's KVCacheLayout.  This container has no GPU, so the few
CUDA-only calls around the native module are stood in for while recording:
the worker's own cudaHostRegister (a ctypes call into libcudart), pin_memory
(identity), torch.cuda.Stream (a dummy); the GPU KV layers are host tensors
whose data pointers identify the layer in the record.  Then each op is run
through the worker's _transfer_impl (worker.py:259-313, 402-451) and each
sequence through hash_utils.gen_hashes / hash_tensor (hash_utils.py:29-37).

tests/test_worker_replay_gpu.py replays the recorded calls, argument for
argument, through flexkv_b200.c_ext on the GPU and checks the bytes against
the CPU oracle; tests/test_c_ext_surface.py checks, on the CPU, that every
recorded call still binds and that c_ext keeps the names, keyword names and
defaults of the reference's pybind module (bindings.cpp:107-171), which this
script also extracts into the fixture.

Writes tests/golden/worker_calls.json.
"""
from __future__ import annotations

import argparse
import contextlib
import inspect
import json
import os
import re
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.dirname(HERE))

import torch  # noqa: E402

from flexkv_b200 import c_ext as ours  # noqa: E402
from kvcase import make_ids, tokens  # noqa: E402


class Recorder:
    """The recording front of flexkv_b200.c_ext."""

    def __init__(self):
        self.calls = []
        self.layer_ids = {}   # data_ptr of a fake GPU layer -> [rank, layer]
        self.cpu_ptr = None

    def tensor(self, t):
        return {"dtype": str(t.dtype).replace("torch.", ""), "values": t.tolist()}

    def layer_table(self, t):
        return [self.layer_ids[int(p)] for p in t.tolist()]

    def module(self):
        rec = self
        m = types.ModuleType("flexkv.c_ext")

        def transfer_kv_blocks(*args, **kwargs):
            b = inspect.signature(ours.transfer_kv_blocks).bind(*args, **kwargs)
            a = b.arguments
            assert a["cpu_tensor"].data_ptr() == rec.cpu_ptr, "the worker passed another CPU tensor"
            rec.calls.append({
                "fn": "transfer_kv_blocks", "num_positional": len(args), "keywords": sorted(kwargs),
                "gpu_block_id_tensor": rec.tensor(a["gpu_block_id_tensor"]),
                "gpu_layer_ptrs_tensor": rec.layer_table(a["gpu_layer_ptrs_tensor"]),
                "cpu_block_id_tensor": rec.tensor(a["cpu_block_id_tensor"]),
                **{k: (bool(v) if isinstance(v, bool) else int(v)) for k, v in a.items()
                   if k not in ("gpu_block_id_tensor", "gpu_layer_ptrs_tensor", "cpu_block_id_tensor",
                                "cpu_tensor")}})

        class TPTransferThreadGroup:
            def __init__(self, *args, **kwargs):
                sig = inspect.signature(ours.TPTransferThreadGroup.__init__)
                b = sig.bind(None, *args, **kwargs)
                a = b.arguments
                assert a["cpu_blocks"].data_ptr() == rec.cpu_ptr
                rec.calls.append({"fn": "TPTransferThreadGroup", "num_gpus": int(a["num_gpus"]),
                                  "gpu_blocks": [[rec.layer_ids[int(t.data_ptr())] for t in r]
                                                 for r in a["gpu_blocks"]],
                                  "dp_group_id": int(a["dp_group_id"])})

            def tp_group_transfer(self, *args, **kwargs):
                sig = inspect.signature(ours.TPTransferThreadGroup.tp_group_transfer)
                a = sig.bind(None, *args, **kwargs).arguments
                rec.calls.append({
                    "fn": "tp_group_transfer", "num_positional": len(args), "keywords": sorted(kwargs),
                    "gpu_block_id_tensor": rec.tensor(a["gpu_block_id_tensor"]),
                    "cpu_block_id_tensor": rec.tensor(a["cpu_block_id_tensor"]),
                    **{k: (bool(v) if isinstance(v, bool) else int(v)) for k, v in a.items()
                       if k not in ("self", "gpu_block_id_tensor", "cpu_block_id_tensor")}})

        class Hasher:
            def __init__(self, *args):
                inspect.signature(ours.Hasher.__init__).bind(None, *args)
                import xxhash  # the library the reference's hash.cpp wraps
                self.h = xxhash.xxh64(seed=0)
                self.fed = []

            def reset(self):
                self.h.reset()
                self.fed = []

            def update(self, t, size=None):
                inspect.signature(ours.Hasher.update).bind(None, t, *([] if size is None else [size]))
                b = t.contiguous().numpy().tobytes()
                self.h.update(b)
                self.fed.append(rec.tensor(t.contiguous().view(-1)))

            def digest(self):
                d = self.h.intdigest()
                rec.calls.append({"fn": "Hasher.digest", "updates": self.fed, "digest": str(d)})
                return d

        def gen_hashes(hasher, token_ids, tokens_per_block, block_hashes):
            inspect.signature(ours.gen_hashes).bind(hasher, token_ids, tokens_per_block, block_hashes)
            import xxhash
            h = xxhash.xxh64(seed=0)
            t = token_ids.contiguous().numpy()
            out = []
            for i in range(block_hashes.numel()):
                h.update(t[i * tokens_per_block:(i + 1) * tokens_per_block].tobytes())
                out.append(h.intdigest())
            block_hashes.copy_(torch.tensor(np.array(out, dtype=np.uint64).view(np.int64)).view(torch.uint64))
            rec.calls.append({"fn": "gen_hashes", "token_ids": rec.tensor(token_ids),
                              "tokens_per_block": int(tokens_per_block),
                              "block_hashes_len": int(block_hashes.numel()),
                              "block_hashes_dtype": str(block_hashes.dtype).replace("torch.", ""),
                              "want": [str(x) for x in out]})

        m.transfer_kv_blocks = transfer_kv_blocks
        m.TPTransferThreadGroup = TPTransferThreadGroup
        m.Hasher = Hasher
        m.gen_hashes = gen_hashes
        m.get_hash_size = ours.get_hash_size
        m.transfer_kv_blocks_ssd = ours.transfer_kv_blocks_ssd
        m.SSDIOCTX = ours.SSDIOCTX
        return m


@contextlib.contextmanager
def host_stand_ins():
    """The CUDA-only calls around the native module, stood in for on a
    machine without a GPU while the reference code runs."""
    saved = (torch.Tensor.pin_memory, torch.zeros, torch.cuda.Stream)
    real_zeros = torch.zeros

    def zeros(*a, **k):
        k.pop("pin_memory", None)
        return real_zeros(*a, **k)

    class Stream:
        def __init__(self, *a, **k):
            pass

    torch.Tensor.pin_memory = lambda self, *a, **k: self
    torch.zeros = zeros
    torch.cuda.Stream = Stream
    try:
        yield
    finally:
        torch.Tensor.pin_memory, torch.zeros, torch.cuda.Stream = saved


class Handle:
    """Stands in for TensorSharedHandle (memory_handle.py:17-56)."""

    def __init__(self, t):
        self.t = t

    def get_tensor(self):
        return self.t


def binding_surface(ref: str) -> dict:
    """Names, keyword names and defaults the pybind module declares
    (csrc/bindings.cpp), and the positional arity of transfer_kv_blocks
    (bound without py::arg, so every argument is positional and required)."""
    src = open(os.path.join(ref, "csrc", "bindings.cpp")).read()
    body = src[src.index("PYBIND11_MODULE"):]
    body = re.sub(r"#ifdef FLEXKV_ENABLE_CFS.*?#endif", "", body, flags=re.S)
    out = {"functions": {}, "classes": {}}
    for m in re.finditer(r'm\.def\("(\w+)",\s*&([\w:]+)(.*?)\);', body, flags=re.S):
        args = re.findall(r'py::arg\("(\w+)"\)(\s*=\s*([\w.-]+))?', m.group(3))
        out["functions"][m.group(1)] = [[a, d or None] for a, _, d in args]
    for m in re.finditer(r'py::class_<[\w:]+>\(m,\s*"(\w+)"\)(.*?);', body, flags=re.S):
        methods = {}
        for d in re.finditer(r'\.def\("(\w+)",(.*?)\)\s*(?=\.def|$)', m.group(2), flags=re.S):
            args = re.findall(r'py::arg\("(\w+)"\)', d.group(2))
            methods.setdefault(d.group(1), []).append(args)
        out["classes"][m.group(1)] = methods
    sig = src[src.index("void transfer_kv_blocks_binding("):src.index(") {", src.index("void transfer_kv_blocks_binding("))]
    params = [p.strip() for p in sig[sig.index("(") + 1:].split(",")]
    out["transfer_kv_blocks_positional"] = [re.split(r"[\s&*]+", p.split("=")[0].strip())[-1] for p in params]
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FLEXKV_REFERENCE"),
                    help="the reference tree (default: $FLEXKV_REFERENCE)")
    a = ap.parse_args()
    if not a.reference or not os.path.isdir(a.reference):
        ap.error("the reference tree is needed: pass --reference or set FLEXKV_REFERENCE")
    sys.path.insert(0, a.reference)
    nv = types.ModuleType("nvtx")  # the reference imports nvtx (absent here) for its trace ranges
    nv.push_range = lambda *x, **k: None
    nv.pop_range = lambda *x, **k: None
    nv.annotate = lambda *x, **k: (lambda f: f)
    sys.modules.setdefault("nvtx", nv)
    rec = Recorder()
    sys.modules["flexkv.c_ext"] = rec.module()
    import flexkv  # reference package
    flexkv.c_ext = sys.modules["flexkv.c_ext"]
    import flexkv.transfer.worker as W  # reference code, unchanged
    from flexkv.common import hash_utils  # reference code, unchanged
    from flexkv.common.storage import KVCacheLayout, KVCacheLayoutType  # reference code
    from flexkv.common.transfer import TransferType  # reference code
    W.cudaHostRegister = lambda t: None  # its ctypes cudart call; the pool is registered on replay

    scenarios = []

    def gpu_worker(name, L, H, D, tpb, ngpu, ncpu, cpu_type, mla, ops):
        rec.calls = []
        kv = 1 if mla else 2
        gpu_layout = KVCacheLayout(KVCacheLayoutType.LAYERWISE, L, ngpu, tpb, H, D, mla)
        cpu_layout = KVCacheLayout(KVCacheLayoutType[cpu_type], L, ncpu, tpb, H, D, mla)
        layers = [torch.zeros((kv, ngpu, tpb, H, D), dtype=torch.bfloat16) for _ in range(L)]
        rec.layer_ids = {int(t[0].data_ptr()): [0, l] for l, t in enumerate(layers)}
        cpu = torch.zeros(cpu_layout.get_total_elements(), dtype=torch.bfloat16)
        rec.cpu_ptr = cpu.data_ptr()
        with host_stand_ins():
            w = W.GPUCPUTransferWorker(0, None, None, [Handle(t) for t in layers], cpu, gpu_layout, cpu_layout,
                                       torch.bfloat16, -1)
            for (src, dst, kind, layer_id, gran) in ops:
                w._transfer_impl(src, dst, kind, layer_id, gran)
        scenarios.append({"name": name, "worker": "GPUCPUTransferWorker", "layers": L, "heads": H, "head_dim": D,
                          "tokens_per_block": tpb, "gpu_blocks": ngpu, "cpu_blocks": ncpu, "cpu_layout": cpu_type,
                          "is_mla": mla, "tp": 1, "calls": rec.calls})

    def tp_worker(name, L, H_total, D, tpb, ngpu, ncpu, tp, ops):
        rec.calls = []
        gpu_layout = KVCacheLayout(KVCacheLayoutType.LAYERWISE, L, ngpu, tpb, H_total, D, False)
        cpu_layout = KVCacheLayout(KVCacheLayoutType.BLOCKWISE, L, ncpu, tpb, H_total, D, False)
        per_rank = gpu_layout.div_head(tp)
        ranks = [[torch.zeros((2, ngpu, tpb, H_total // tp, D), dtype=torch.bfloat16) for _ in range(L)]
                 for _ in range(tp)]
        rec.layer_ids = {int(t.data_ptr()): [r, l] for r, ls in enumerate(ranks) for l, t in enumerate(ls)}
        cpu = torch.zeros(cpu_layout.get_total_elements(), dtype=torch.bfloat16)
        rec.cpu_ptr = cpu.data_ptr()
        with host_stand_ins():
            w = W.tpGPUCPUTransferWorker(0, None, None, [[Handle(t) for t in ls] for ls in ranks], cpu, per_rank,
                                         cpu_layout, torch.bfloat16, tp, 0)
            for (src, dst, kind, layer_id, gran) in ops:
                w._transfer_impl(src, dst, kind, layer_id, gran)
        scenarios.append({"name": name, "worker": "tpGPUCPUTransferWorker", "layers": L, "heads": H_total // tp,
                          "head_dim": D, "tokens_per_block": tpb, "gpu_blocks": ngpu, "cpu_blocks": ncpu,
                          "cpu_layout": "BLOCKWISE", "is_mla": False, "tp": tp, "calls": rec.calls})

    H2D, D2H = TransferType.H2D, TransferType.D2H

    def op(kind, n, ngpu, ncpu, seed, layer_id, gran, run_frac=0.5):
        g, c = make_ids(n, ngpu, ncpu, seed, run_frac, max_run=8)
        return (c, g, kind, layer_id, gran) if kind == H2D else (g, c, kind, layer_id, gran)

    gpu_worker("layerwise_pool", 4, 2, 64, 16, 64, 128, "LAYERWISE", False, [
        op(D2H, 40, 64, 128, 1, 0, 4), op(H2D, 33, 64, 128, 2, 0, 4), op(D2H, 20, 64, 128, 3, 1, 2),
        op(H2D, 17, 64, 128, 4, 2, 2), op(H2D, 1, 64, 128, 5, 3, 1), op(D2H, 0, 64, 128, 6, 0, 4)])
    gpu_worker("blockwise_pool", 4, 2, 64, 16, 64, 96, "BLOCKWISE", False, [
        op(D2H, 48, 64, 96, 11, 0, 4), op(H2D, 30, 64, 96, 12, 0, 4), op(D2H, 16, 64, 96, 13, 2, 2),
        op(H2D, 24, 64, 96, 14, 1, 3)])
    gpu_worker("mla_blockwise", 3, 1, 576, 64, 32, 48, "BLOCKWISE", True, [
        op(D2H, 20, 32, 48, 21, 0, 3), op(H2D, 12, 32, 48, 22, 0, 3), op(D2H, 9, 32, 48, 23, 1, 1)])
    tp_worker("tp2_blockwise", 4, 4, 64, 16, 64, 96, 2, [
        op(D2H, 40, 64, 96, 31, 0, 4), op(H2D, 28, 64, 96, 32, 0, 4)])
    tp_worker("tp4_blockwise", 2, 8, 64, 16, 32, 64, 4, [
        op(D2H, 24, 32, 64, 41, 0, 2), op(H2D, 20, 32, 64, 42, 0, 2)])

    rec.calls = []
    for n, tpb, seed in ((64, 16, 51), (1000, 16, 52), (37, 4, 53), (5, 16, 54)):
        hash_utils.gen_hashes(torch.from_numpy(tokens(n, 32000, seed)), tpb)
    hash_utils.hash_tensor(torch.from_numpy(tokens(96, 32000, 55)))
    scenarios.append({"name": "hash_utils", "calls": rec.calls})

    out = {"scenarios": scenarios, "bindings": binding_surface(a.reference),
           "recorded_with": "flexkv_b200.c_ext signatures; reference worker.py and hash_utils.py unchanged"}
    with open(os.path.join(HERE, "worker_calls.json"), "w") as f:
        json.dump(out, f, indent=None, separators=(",", ":"))
    print("wrote worker_calls.json:", [(s["name"], len(s["calls"])) for s in scenarios])
    return 0


if __name__ == "__main__":
    sys.exit(main())
