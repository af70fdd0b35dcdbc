"""TEST INFRASTRUCTURE ONLY — ctypes wrapper of the CPU oracle (oracle.c)
and of the reference's own transfer.cu built into oracle/_ref.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs use this module, as the checker or the baseline.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_transfer.so")

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_vp = ctypes.c_void_p


def build(with_reference: bool = True) -> None:
    """Build liboracle.so (and the reference transfer.cu when its tree is
    present).  Outputs stay under oracle/_build and oracle/_ref."""
    target = "all" if with_reference else "_build/liboracle.so"
    subprocess.run(["make", "-s", "-C", HERE, target], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build(with_reference=False)
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_transfer_kv_blocks.restype = _c_int
        L.oracle_transfer_kv_blocks.argtypes = [
            _c_int, _c_int, _c_int, _vp, _vp, _c_i64, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64,
            _c_i64, _c_i64, _c_int, _c_int, _c_int]
        L.oracle_xxh64_state_size.restype = ctypes.c_size_t
        L.oracle_xxh64_reset.argtypes = [_vp, ctypes.c_uint64]
        L.oracle_xxh64_update.argtypes = [_vp, _vp, ctypes.c_size_t]
        L.oracle_xxh64_digest.restype = ctypes.c_uint64
        L.oracle_xxh64_digest.argtypes = [_vp]
        L.oracle_xxh64.restype = ctypes.c_uint64
        L.oracle_xxh64.argtypes = [_vp, ctypes.c_size_t, ctypes.c_uint64]
        L.oracle_gen_hashes.argtypes = [_vp, _vp, _c_int, _vp, _c_i64]
        L.oracle_gen_hashes_batched.argtypes = [_vp, _vp, _c_int, _c_int, _vp]
        L.oracle_gen_hashes_batched_mt.argtypes = [_vp, _vp, _c_int, _c_int, _vp, _c_int]
        L.oracle_ssd_transfer.restype = _c_int
        L.oracle_ssd_transfer.argtypes = [
            _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int, _c_i64, _c_i64, _c_i64,
            _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def transfer(num_blocks: int, start_layer_id: int, gpu_block_ids: np.ndarray,
             gpu_layers: Sequence[np.ndarray], gpu_kv_stride: int, gpu_block_stride: int,
             cpu_block_ids: np.ndarray, cpu_pool: np.ndarray, cpu_kv_stride: int,
             cpu_layer_stride: int, cpu_block_stride: int, cpu_startoff: int, chunk: int,
             is_host_to_device: bool, is_mla: bool, num_threads: int = 1) -> None:
    """Run the reference copy semantics on host arrays in place.  gpu_layers
    are byte images (uint8 arrays) of the per-layer GPU tensors."""
    g = np.ascontiguousarray(gpu_block_ids, dtype=np.int64)
    c = np.ascontiguousarray(cpu_block_ids, dtype=np.int64)
    ptrs = np.array([_ptr(x) for x in gpu_layers], dtype=np.uint64)
    lib().oracle_transfer_kv_blocks(
        int(num_blocks), int(start_layer_id), len(gpu_layers), _ptr(g), _ptr(ptrs),
        int(gpu_kv_stride), int(gpu_block_stride), _ptr(c), _ptr(cpu_pool), int(cpu_kv_stride),
        int(cpu_layer_stride), int(cpu_block_stride), int(cpu_startoff), int(chunk),
        int(bool(is_host_to_device)), int(bool(is_mla)), int(num_threads))


class XXH64:
    """Streaming XXH64 oracle."""

    def __init__(self, seed: int = 0):
        self._st = ctypes.create_string_buffer(int(lib().oracle_xxh64_state_size()))
        lib().oracle_xxh64_reset(self._st, seed)

    def update(self, data: bytes | np.ndarray) -> "XXH64":
        b = np.frombuffer(bytes(data), dtype=np.uint8) if isinstance(data, (bytes, bytearray)) \
            else np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        lib().oracle_xxh64_update(self._st, _ptr(b) if b.size else None, b.size)
        return self

    def digest(self) -> int:
        return int(lib().oracle_xxh64_digest(self._st))

    def gen_hashes(self, token_ids: np.ndarray, tokens_per_block: int) -> np.ndarray:
        t = np.ascontiguousarray(token_ids, dtype=np.int64)
        nb = t.size // tokens_per_block
        out = np.zeros(nb, dtype=np.uint64)
        if nb:
            lib().oracle_gen_hashes(self._st, _ptr(t), int(tokens_per_block), _ptr(out), nb)
        return out


def xxh64(data: bytes | np.ndarray, seed: int = 0) -> int:
    return XXH64(seed).update(data).digest()


def gen_hashes(token_ids: np.ndarray, tokens_per_block: int) -> np.ndarray:
    return XXH64(0).gen_hashes(token_ids, tokens_per_block)


def gen_hashes_batched(token_ids: np.ndarray, seq_offsets: Sequence[int],
                       tokens_per_block: int, num_threads: int = 1) -> np.ndarray:
    t = np.ascontiguousarray(token_ids, dtype=np.int64)
    offs = np.ascontiguousarray(seq_offsets, dtype=np.int64)
    n = offs.size - 1
    total = int(((offs[1:] - offs[:-1]) // tokens_per_block).sum()) if n > 0 else 0
    out = np.zeros(max(total, 1), dtype=np.uint64)
    if num_threads > 1:
        lib().oracle_gen_hashes_batched_mt(_ptr(t), _ptr(offs), n, int(tokens_per_block), _ptr(out),
                                           int(num_threads))
    else:
        lib().oracle_gen_hashes_batched(_ptr(t), _ptr(offs), n, int(tokens_per_block), _ptr(out))
    return out[:total]


# ---- the reference's own transfer.cu (GPU), built by oracle/Makefile ------

_ref = None


def reference_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not reference_available():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference tree at build time)")
        L = ctypes.CDLL(REF_SO)
        L.ref_transfer_kv_blocks.restype = _c_int
        L.ref_transfer_kv_blocks.argtypes = [
            _c_int, _c_int, _c_int, _vp, _vp, _c_i64, _c_i64, _vp, _vp, _c_i64, _c_i64, _c_i64,
            _c_i64, _c_i64, _vp, _c_int, _c_int, _c_int, _c_int]
        _ref = L
    return _ref


REF_SSD_SO = os.path.join(HERE, "_ref", "libref_ssd.so")
_ref_ssd = None


def reference_ssd_available() -> bool:
    return os.path.exists(REF_SSD_SO)


def ref_ssd_lib() -> ctypes.CDLL:
    """The reference's own SSD tier (csrc/transfer_ssd.cpp), built into
    oracle/_ref/libref_ssd.so by oracle/Makefile (ref_ssd_shim.cpp)."""
    global _ref_ssd
    if _ref_ssd is None:
        if not reference_ssd_available():
            raise FileNotFoundError(f"{REF_SSD_SO} not built (needs FLEXKV_REFERENCE at build time)")
        L = ctypes.CDLL(REF_SSD_SO)
        L.ref_ssd_ctx_create.restype = _c_int
        L.ref_ssd_ctx_create.argtypes = [_vp, _c_int, _c_int, ctypes.POINTER(_vp)]
        L.ref_ssd_ctx_destroy.restype = None
        L.ref_ssd_ctx_destroy.argtypes = [_vp]
        L.ref_ssd_transfer.restype = _c_int
        L.ref_ssd_transfer.argtypes = [
            _vp, _c_int, _c_int, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
            _c_int, _c_int, _c_int, _c_int, _c_int]
        _ref_ssd = L
    return _ref_ssd


class RefSSDContext:
    """flexkv::SSDIOCTX of the reference (thread-pool path): files[d] lists
    the file paths of SSD device d, every device with as many files."""

    def __init__(self, files: dict):
        nd, nf = len(files), len(files[0])
        paths = [str(files[d][f]).encode() for d in range(nd) for f in range(nf)]
        arr = (ctypes.c_char_p * len(paths))(*paths)
        h = _vp()
        if ref_ssd_lib().ref_ssd_ctx_create(ctypes.cast(arr, _vp), nd, nf, ctypes.byref(h)) != 0:
            raise RuntimeError("reference SSDIOCTX failed to open its files")
        self._h = h

    def transfer(self, start_layer: int, num_layers: int, cpu_ptr: int, ssd_block_ids: np.ndarray,
                 cpu_block_ids: np.ndarray, cpu_layer_stride: int, cpu_kv_stride: int, ssd_layer_stride: int,
                 ssd_kv_stride: int, chunk: int, block_stride: int, is_read: bool, num_blocks_per_file: int,
                 round_robin: int = 1, threads_per_device: int = 16, is_mla: bool = False) -> None:
        s = np.ascontiguousarray(ssd_block_ids, dtype=np.int64)
        c = np.ascontiguousarray(cpu_block_ids, dtype=np.int64)
        rc = ref_ssd_lib().ref_ssd_transfer(
            self._h, int(start_layer), int(num_layers), _vp(int(cpu_ptr)), _ptr(s), _ptr(c), len(s),
            int(cpu_layer_stride), int(cpu_kv_stride), int(ssd_layer_stride), int(ssd_kv_stride), int(chunk),
            int(block_stride), int(bool(is_read)), int(num_blocks_per_file), int(round_robin),
            int(threads_per_device), int(bool(is_mla)))
        if rc != 0:
            raise RuntimeError("reference transfer_kv_blocks_ssd threw")

    def close(self) -> None:
        if self._h:
            ref_ssd_lib().ref_ssd_ctx_destroy(self._h)
            self._h = None


def ssd_transfer(files: List[List[np.ndarray]], start_layer: int, num_layers: int, cpu: np.ndarray,
                 ssd_block_ids: np.ndarray, cpu_block_ids: np.ndarray, cpu_layer_stride: int,
                 cpu_kv_stride: int, ssd_layer_stride: int, ssd_kv_stride: int, chunk: int,
                 block_stride: int, is_read: bool, round_robin: int = 1, is_mla: bool = False) -> None:
    """Restatement of flexkv::transfer_kv_blocks_ssd on in-memory file
    images: files[d][f] is the byte image of file f of SSD device d.
    Device/file mapping: transfer_ssd.cpp:17-32 (partition_and_remap);
    per-chunk offsets and the K-then-V order: transfer_ssd.cpp:133-176
    (_transfer_single_thread_impl).  Block ids are cast to int there
    (std::vector<int>), so ids must fit in 31 bits."""
    D, F = len(files), len(files[0])
    kv = 1 if is_mla else 2
    for s_id, c_id in zip(ssd_block_ids.tolist(), cpu_block_ids.tolist()):
        assert 0 <= s_id < 2 ** 31 and 0 <= c_id < 2 ** 31
        d = (s_id // round_robin) % D
        in_dev = ((s_id // round_robin) // D) * round_robin + s_id % round_robin
        img = files[d][in_dev % F]
        b = in_dev // F
        for l in range(start_layer, start_layer + num_layers):
            for k in range(kv):
                so = b * block_stride + l * ssd_layer_stride + k * ssd_kv_stride
                co = c_id * block_stride + l * cpu_layer_stride + k * cpu_kv_stride
                if is_read:
                    if so + chunk > img.size:
                        raise IOError("short read past the end of the file")
                    cpu[co:co + chunk] = img[so:so + chunk]
                else:
                    img[so:so + chunk] = cpu[co:co + chunk]


class SsdRefContext:
    """Files opened the way the reference's SSDIOCTX opens them (buffered
    and O_DIRECT, transfer_ssd.h:196-220) for oracle_ssd_transfer, the C
    restatement of its per-chunk loop."""

    def __init__(self, ssd_files, num_devices: int):
        self.nd = num_devices
        self.nf = len(ssd_files[0])
        paths = [ssd_files[d][f] for d in range(num_devices) for f in range(self.nf)]
        self.buf = np.array([os.open(p, os.O_RDWR) for p in paths], dtype=np.int32)
        direct = []
        for p in paths:
            try:
                direct.append(os.open(p, os.O_RDWR | getattr(os, "O_DIRECT", 0)))
            except OSError:  # a filesystem without O_DIRECT: the reference would throw here
                direct.append(os.open(p, os.O_RDWR))
        self.direct = np.array(direct, dtype=np.int32)

    def transfer(self, start_layer, num_layers, cpu_ptr, ssd_ids, cpu_ids, st, is_read, round_robin=1,
                 threads_per_device=32, is_mla=False) -> None:
        s = np.ascontiguousarray(ssd_ids, dtype=np.int64)
        c = np.ascontiguousarray(cpu_ids, dtype=np.int64)
        rc = lib().oracle_ssd_transfer(
            self.buf.ctypes.data, self.direct.ctypes.data, self.nd, self.nf, start_layer, num_layers,
            cpu_ptr, s.ctypes.data, c.ctypes.data, len(s), st.cpu_layer_stride_in_bytes,
            st.cpu_kv_stride_in_bytes, st.ssd_layer_stride_in_bytes, st.ssd_kv_stride_in_bytes,
            st.chunk_size_in_bytes, st.block_stride_in_bytes, int(is_read), round_robin,
            threads_per_device, int(is_mla))
        if rc:
            raise IOError("reference-style SSD transfer: a request failed or came up short")

    def close(self) -> None:
        for fd in list(self.buf) + list(self.direct):
            os.close(int(fd))
        self.buf = self.direct = np.zeros(0, np.int32)
