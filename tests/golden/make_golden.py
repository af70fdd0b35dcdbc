"""Regenerate the golden fixtures in tests/golden/ (run in a container that
has the reference tree; the fixtures themselves travel without it):

    python tests/golden/make_golden.py --reference /path/to/FlexKV

* layouts.json  — shapes and element strides from the reference's own
  KVCacheLayout (flexkv/common/storage.py:22-155), imported from the
  reference tree, for the five benchmark configurations, both CPU layouts
  and the per-rank GPU layout (div_head for TP).
* hash.json     — XXH64 vectors from the xxHash library the reference links
  (csrc/hash.cpp via cache_utils.h), taken from python `xxhash` and checked
  against the system libxxhash.so.0 through ctypes: the empty-input value of
  the specification, one-shot vectors, and gen_hashes prefix vectors in the
  reference's semantics (update per block, digest after each, hash.cpp:61-65).
* transfer.json — sha256 digests of pools after D2H/H2D copies computed by
  the view-based restatement in tests/kvcase.py with the reference's
  KVCacheLayout strides, on splitmix64 data (stable across library versions).
"""
from __future__ import annotations

import argparse
import ctypes
import ctypes.util
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from kvcase import Case, fill_bytes, make_ids, sha, tokens, view_transfer  # noqa: E402

CONFIGS = {
    # name: (layers, kv heads total, head_dim, tpb, gpu blocks, cpu blocks, mla, tp list)
    "cfg1_tiny": (4, 8, 64, 16, 256, 1024, False, [1]),
    "cfg2_llama3_8b": (32, 8, 128, 16, 16384, 32768, False, [1]),
    "cfg3_llama3_70b_tp": (80, 8, 128, 64, 4096, 8192, False, [1, 2, 4, 8]),
    "cfg4_qwen2_7b": (28, 4, 128, 16, 8192, 16384, False, [1]),
    "cfg5_dsv3_mla": (61, 1, 576, 64, 8192, 16384, True, [1]),
}


def make_layouts(ref_root: str) -> dict:
    sys.path.insert(0, ref_root)
    from flexkv.common.storage import KVCacheLayout, KVCacheLayoutType  # reference code
    out = {}
    for name, (L, H, D, tpb, ng, nc, mla, tps) in CONFIGS.items():
        for lt in ("LAYERWISE", "BLOCKWISE"):
            cpu = KVCacheLayout(type=KVCacheLayoutType[lt], num_layer=L, num_block=nc,
                                tokens_per_block=tpb, num_head=H, head_size=D, is_mla=mla)
            out[f"{name}/cpu/{lt}"] = {
                "args": [lt, L, nc, tpb, H, D, mla],
                "kv_shape": list(cpu.kv_shape), "chunk": cpu.get_chunk_size(),
                "layer_stride": cpu.get_layer_stride(), "kv_stride": cpu.get_kv_stride(),
                "block_stride": cpu.get_block_stride(), "total": cpu.get_total_elements(),
            }
        for tp in tps:
            g = KVCacheLayout(type=KVCacheLayoutType.LAYERWISE, num_layer=L, num_block=ng,
                              tokens_per_block=tpb, num_head=H, head_size=D, is_mla=mla)
            g = g.div_head(tp) if not mla else g
            per_layer = g.div_layer(L)
            out[f"{name}/gpu/tp{tp}"] = {
                "args": ["LAYERWISE", L, ng, tpb, H, D, mla, tp],
                "kv_shape": list(g.kv_shape), "chunk": per_layer.get_chunk_size(),
                "kv_stride": per_layer.get_kv_stride(), "block_stride": per_layer.get_block_stride(),
                "total_per_layer": per_layer.get_total_elements(),
            }
    sys.path.remove(ref_root)
    return out


class LibXXH:
    """The installed xxHash C library (the library hash.cpp links)."""

    def __init__(self):
        name = ctypes.util.find_library("xxhash") or "libxxhash.so.0"
        L = ctypes.CDLL(name)
        L.XXH64_createState.restype = ctypes.c_void_p
        L.XXH64_reset.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
        L.XXH64_update.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        L.XXH64_digest.restype = ctypes.c_uint64
        L.XXH64_digest.argtypes = [ctypes.c_void_p]
        L.XXH64_freeState.argtypes = [ctypes.c_void_p]
        L.XXH_versionNumber.restype = ctypes.c_uint
        self.L = L

    def version(self) -> int:
        return int(self.L.XXH_versionNumber())

    def gen_hashes(self, prefix: bytes, toks: np.ndarray, tpb: int) -> list:
        st = self.L.XXH64_createState()
        self.L.XXH64_reset(st, 0)
        if prefix:
            self.L.XXH64_update(st, prefix, len(prefix))
        out = []
        t = np.ascontiguousarray(toks, dtype=np.int64)
        for b in range(t.size // tpb):
            blk = t[b * tpb:(b + 1) * tpb]
            self.L.XXH64_update(st, blk.ctypes.data, blk.nbytes)
            out.append(int(self.L.XXH64_digest(st)))
        self.L.XXH64_freeState(st)
        return out


def py_gen_hashes(prefix: bytes, toks: np.ndarray, tpb: int) -> list:
    import xxhash
    h = xxhash.xxh64(seed=0)
    if prefix:
        h.update(prefix)
    t = np.ascontiguousarray(toks, dtype=np.int64)
    out = []
    for b in range(t.size // tpb):
        h.update(t[b * tpb:(b + 1) * tpb].tobytes())
        out.append(h.intdigest())
    return out


def make_hash() -> dict:
    import xxhash
    lib = LibXXH()
    res = {"xxhash_py": xxhash.VERSION, "libxxhash_version": lib.version(), "oneshot": [],
           "gen_hashes": []}
    for n in list(range(0, 70)) + [100, 127, 128, 129, 255, 256, 257, 1000, 4099]:
        data = fill_bytes(n, 7000 + n).tobytes()
        res["oneshot"].append({"hex": data.hex(), "xxh64": xxhash.xxh64(data, seed=0).intdigest()})
    cases = [
        # name, n_tokens, vocab, seed, tpb, prefix bytes
        ("cfg1", 64 * 16, 32000, 1, 16, 0),
        ("tpb1", 40, 32000, 2, 1, 0),
        ("tpb3", 40 * 3, 32000, 3, 3, 0),
        ("tpb5", 40 * 5 + 2, 32000, 4, 5, 0),
        ("tpb17", 40 * 17, 32000, 5, 17, 0),
        ("prefix13_tpb16", 20 * 16, 32000, 6, 16, 13),
        ("prefix8_tpb2", 33 * 2, 32000, 7, 2, 8),
        ("prefix31_tpb16", 20 * 16 + 7, 32000, 8, 16, 31),
        ("cfg4_1M", 1 << 20, 152064, 4, 16, 0),
    ]
    for name, n, vocab, seed, tpb, npre in cases:
        toks = tokens(n, vocab, seed)
        prefix = fill_bytes(npre, 9000 + seed).tobytes()
        hs = py_gen_hashes(prefix, toks, tpb)
        assert hs == lib.gen_hashes(prefix, toks, tpb), f"libxxhash disagrees on {name}"
        entry = {"name": name, "n_tokens": n, "vocab": vocab, "seed": seed, "tpb": tpb,
                 "prefix_hex": prefix.hex(), "num_blocks": len(hs),
                 "sha256": hashlib.sha256(np.array(hs, dtype=np.uint64).tobytes()).hexdigest(),
                 "final_digest_after": hs[-1] if hs else None}
        if len(hs) <= 128:
            entry["hashes"] = hs
        else:
            entry["head"] = hs[:8]
            entry["tail"] = hs[-8:]
        res["gen_hashes"].append(entry)
    # Batched: independent sequences with fresh hashers.
    lens = [0, 1, 15, 16, 17, 31, 32, 33, 64, 100, 512, 16 * 32]
    toks = tokens(sum(lens), 152064, 11)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    allh = []
    for i in range(len(lens)):
        allh += py_gen_hashes(b"", toks[offs[i]:offs[i + 1]], 16)
    res["batched"] = {"lens": lens, "vocab": 152064, "seed": 11, "tpb": 16, "hashes": allh}
    return res


TRANSFER_CASES = [
    # Case fields + id generation (n, seed, run_frac)
    dict(case=Case("cfg1_layerwise", 4, 8, 64, 16, 256, 1024), n=64, seed=1, run_frac=0.0),
    dict(case=Case("cfg1_blockwise", 4, 8, 64, 16, 256, 1024, "BLOCKWISE"), n=64, seed=2, run_frac=0.0),
    dict(case=Case("runs_layerwise", 4, 8, 64, 16, 512, 1024), n=200, seed=3, run_frac=0.5),
    dict(case=Case("runs_blockwise", 4, 8, 64, 16, 512, 1024, "BLOCKWISE"), n=200, seed=4, run_frac=0.5),
    dict(case=Case("mla_blockwise", 3, 1, 576, 16, 128, 256, "BLOCKWISE", is_mla=True), n=40, seed=5, run_frac=0.5),
    dict(case=Case("mla_layerwise", 3, 1, 576, 16, 128, 256, "LAYERWISE", is_mla=True), n=40, seed=6, run_frac=0.0),
    dict(case=Case("layer_slice", 6, 2, 64, 16, 64, 128, "LAYERWISE", layer_id=2, layer_gran=3), n=24, seed=7, run_frac=0.3),
    dict(case=Case("layer_slice_blockwise", 6, 2, 64, 16, 64, 128, "BLOCKWISE", layer_id=1, layer_gran=4), n=24, seed=8, run_frac=0.3),
    dict(case=Case("tp2_rank1_blockwise", 4, 2, 64, 16, 64, 128, "BLOCKWISE", tp=2), n=20, seed=9, run_frac=0.4, rank=1),
    dict(case=Case("tp4_rank3_layerwise", 4, 1, 128, 16, 64, 128, "LAYERWISE", tp=4), n=20, seed=10, run_frac=0.4, rank=3),
    dict(case=Case("tail_dropped", 2, 1, 64, 16, 32, 64, "LAYERWISE", chunk_override=2040), n=10, seed=11, run_frac=0.0),
]


def run_transfer_case(spec: dict) -> dict:
    case: Case = spec["case"]
    st = case.strides()
    gids, cids = make_ids(spec["n"], case.gpu_blocks, case.cpu_blocks, spec["seed"],
                          spec["run_frac"], max_run=8)
    gpu = [fill_bytes(st["gpu_layer_bytes"], 100 + l) for l in range(case.gran)]
    cpu = fill_bytes(st["cpu_pool_bytes"], 99)
    rank = spec.get("rank", 0)
    view_transfer(case, gpu, cpu, gids, cids, h2d=False, rank=rank)
    d2h_cpu = sha(cpu)
    gpu2 = [np.zeros(st["gpu_layer_bytes"], dtype=np.uint8) for _ in range(case.gran)]
    view_transfer(case, gpu2, cpu, gids, cids, h2d=True, rank=rank)
    h2d_gpu = [sha(g) for g in gpu2]
    return {"name": case.name, "case": case.__dict__, "gpu_ids": gids.tolist(),
            "cpu_ids": cids.tolist(), "rank": rank, "gpu_seed_base": 100, "cpu_seed": 99,
            "d2h_cpu_sha256": d2h_cpu, "h2d_gpu_sha256": h2d_gpu}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FLEXKV_REFERENCE"),
                    help="the reference tree (default: $FLEXKV_REFERENCE)")
    a = ap.parse_args()
    if not a.reference or not os.path.isdir(a.reference):
        ap.error("the reference tree is needed: pass --reference or set FLEXKV_REFERENCE")
    with open(os.path.join(HERE, "layouts.json"), "w") as f:
        json.dump(make_layouts(a.reference), f, indent=1)
    with open(os.path.join(HERE, "hash.json"), "w") as f:
        json.dump(make_hash(), f, indent=1)
    with open(os.path.join(HERE, "transfer.json"), "w") as f:
        json.dump([run_transfer_case(s) for s in TRANSFER_CASES], f, indent=1)
    print("wrote", os.listdir(HERE))
    return 0


if __name__ == "__main__":
    sys.exit(main())
