"""Drop-in mirror of FlexKV's native module ``flexkv.c_ext`` for the transfer
data plane (linhu-nv/FlexKV csrc/bindings.cpp:107-171).

Same names, argument order, defaults and keyword names as the pybind11
module, so FlexKV's transfer workers (flexkv/transfer/worker.py:17-30,
297-313, 400, 425-441) and hash helpers (flexkv/common/hash_utils.py:6-37)
run unchanged on top of it.  Every call goes through the C ABI of
libflexkv_b200.so (include/flexkv_b200.h); failures raise RuntimeError as
the reference does (bindings.cpp:51-54, tp_transfer_thread_group.cpp:106-108).

Differences a caller can observe, all on inputs the reference mishandles:
  * ids and alignment are validated on the host before launch: an id that
    addresses past the CPU pool, a negative id or a misaligned chunk raises
    instead of faulting the GPU or corrupting host memory;
  * the id tensors need not be pinned (they are read on the host), and may
    be CUDA tensors (copied to the host first);
  * the GIL is released during the copy (ctypes), the reference holds it;
  * TPTransferThreadGroup keeps persistent rank threads, uses each rank's
    tensor device instead of dp_group_id*num_gpus+i, and indexes rank i's
    layer pointers with the full layer count (tp_transfer_thread_group.cpp
    :70,77 use layer_granularity; identical for full-layer ops).
Extra keyword-only options (ce_min_run_bytes, ce_schedule, synchronous,
gpu_layer_bytes) default to the reference behaviour.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import TransferDesc, check

__all__ = [
    "transfer_kv_blocks", "TPTransferThreadGroup", "Hasher", "gen_hashes", "gen_hashes_batched",
    "get_hash_size", "transfer_kv_blocks_ssd", "SSDIOCTX", "cudaHostRegister",
    "cudaHostUnregister", "TransferPlan", "kernel_launch_count",
]


def _stream_handle() -> int:
    return int(torch.cuda.current_stream().cuda_stream)


def _host_i64(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != torch.int64:
        raise RuntimeError(f"{name} must be an int64 tensor, got {t.dtype}")
    if t.is_cuda:
        t = t.cpu()
    return t.contiguous()


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def kernel_launch_count() -> int:
    """Kernels launched by libflexkv_b200 in this process so far."""
    return int(_lib.load().fkv_kernel_launch_count())


def cudaHostRegister(tensor: torch.Tensor, advise_hugepages: bool = False) -> None:
    """Page-lock a CPU tensor for zero-copy device access (worker.py:35-41)."""
    lib = _lib.load()
    check(lib.fkv_host_register(tensor.data_ptr(), _nbytes(tensor), int(advise_hugepages)),
          "cudaHostRegister")


def cudaHostUnregister(tensor: torch.Tensor) -> None:
    """Undo cudaHostRegister (worker.py:43-47)."""
    check(_lib.load().fkv_host_unregister(tensor.data_ptr()), "cudaHostUnregister")


def _fill_desc(d: TransferDesc, gpu_ids: torch.Tensor, cpu_ids: torch.Tensor,
               layer_ptrs: torch.Tensor, cpu_tensor: torch.Tensor, gpu_kv_stride_in_bytes: int,
               gpu_block_stride_in_bytes: int, cpu_kv_stride_in_bytes: int,
               cpu_layer_stride_in_bytes: int, cpu_block_stride_in_bytes: int,
               chunk_size_in_bytes: int, start_layer_id: int, transfer_sms: int,
               is_host_to_device: bool, use_ce_transfer: bool, is_mla: bool,
               ce_min_run_bytes: Optional[int], synchronous: bool, gpu_layer_bytes: int,
               cpu_startoff_inside_chunks: int = 0, ce_schedule: Optional[int] = None) -> None:
    _lib.load().fkv_transfer_desc_init(ctypes.byref(d))
    if gpu_ids.numel() != cpu_ids.numel():
        raise RuntimeError("gpu and cpu block id tensors differ in length")
    d.num_blocks = gpu_ids.numel()
    d.start_layer_id = int(start_layer_id)
    d.num_layers = layer_ptrs.numel()
    d.is_host_to_device = int(bool(is_host_to_device))
    d.is_mla = int(bool(is_mla))
    d.transfer_sms = int(transfer_sms)
    d.use_ce_transfer = int(bool(use_ce_transfer))
    d.synchronous = int(bool(synchronous))
    d.gpu_block_ids = gpu_ids.data_ptr()
    d.cpu_block_ids = cpu_ids.data_ptr()
    d.gpu_layer_ptrs = layer_ptrs.data_ptr()
    d.cpu_ptr = cpu_tensor.data_ptr()
    d.gpu_kv_stride_in_bytes = int(gpu_kv_stride_in_bytes)
    d.gpu_block_stride_in_bytes = int(gpu_block_stride_in_bytes)
    d.cpu_kv_stride_in_bytes = int(cpu_kv_stride_in_bytes)
    d.cpu_layer_stride_in_bytes = int(cpu_layer_stride_in_bytes)
    d.cpu_block_stride_in_bytes = int(cpu_block_stride_in_bytes)
    d.cpu_startoff_inside_chunks = int(cpu_startoff_inside_chunks)
    d.chunk_size_in_bytes = int(chunk_size_in_bytes)
    d.cpu_pool_bytes = _nbytes(cpu_tensor)
    d.gpu_layer_bytes = int(gpu_layer_bytes)
    d.ce_min_run_bytes = -1 if ce_min_run_bytes is None else int(ce_min_run_bytes)
    d.ce_schedule = -1 if ce_schedule is None else int(ce_schedule)


def transfer_kv_blocks(gpu_block_id_tensor: torch.Tensor, gpu_layer_ptrs_tensor: torch.Tensor,
                       gpu_kv_stride_in_bytes: int, gpu_block_stride_in_bytes: int,
                       cpu_block_id_tensor: torch.Tensor, cpu_tensor: torch.Tensor,
                       cpu_kv_stride_in_bytes: int, cpu_layer_stride_in_bytes: int,
                       cpu_block_stride_in_bytes: int, chunk_size_in_bytes: int,
                       start_layer_id: int, transfer_sms: int = -1,
                       is_host_to_device: bool = True, use_ce_transfer: bool = False,
                       is_mla: bool = False, *, ce_min_run_bytes: Optional[int] = None,
                       synchronous: bool = True, gpu_layer_bytes: int = 0,
                       ce_schedule: Optional[int] = None) -> None:
    """Move (layer, kv, block) chunks between GPU layers and the host pool
    (bindings.cpp:25-55 -> transfer.cu:63-132) on the current CUDA stream.
    ``gpu_layer_ptrs_tensor`` is an int64 CPU tensor of per-layer device
    addresses, already sliced to the op's layers; ``start_layer_id`` offsets
    the CPU side only."""
    gpu_ids = _host_i64(gpu_block_id_tensor, "gpu_block_id_tensor")
    cpu_ids = _host_i64(cpu_block_id_tensor, "cpu_block_id_tensor")
    ptrs = _host_i64(gpu_layer_ptrs_tensor, "gpu_layer_ptrs_tensor")
    if cpu_tensor.is_cuda:
        raise RuntimeError("cpu_tensor must be a host tensor")
    d = TransferDesc()
    _fill_desc(d, gpu_ids, cpu_ids, ptrs, cpu_tensor, gpu_kv_stride_in_bytes,
               gpu_block_stride_in_bytes, cpu_kv_stride_in_bytes, cpu_layer_stride_in_bytes,
               cpu_block_stride_in_bytes, chunk_size_in_bytes, start_layer_id, transfer_sms,
               is_host_to_device, use_ce_transfer, is_mla, ce_min_run_bytes, synchronous,
               gpu_layer_bytes, ce_schedule=ce_schedule)
    check(_lib.load().fkv_transfer_kv_blocks_ex(ctypes.byref(d), _stream_handle()),
          "transfer_kv_blocks")


class TransferPlan:
    """Validated, coalesced, device-resident form of one transfer, for
    callers that replay the same block lists (``execute`` only launches).
    Arguments as ``transfer_kv_blocks``; the plan keeps its tensors alive."""

    def __init__(self, gpu_block_id_tensor, gpu_layer_ptrs_tensor, gpu_kv_stride_in_bytes,
                 gpu_block_stride_in_bytes, cpu_block_id_tensor, cpu_tensor,
                 cpu_kv_stride_in_bytes, cpu_layer_stride_in_bytes, cpu_block_stride_in_bytes,
                 chunk_size_in_bytes, start_layer_id, transfer_sms=-1, is_host_to_device=True,
                 use_ce_transfer=False, is_mla=False, *, ce_min_run_bytes=None,
                 gpu_layer_bytes=0, cpu_startoff_inside_chunks=0, ce_schedule=None,
                 device: int = -1):
        self._lib = _lib.load()
        self._handle = None
        gpu_ids = _host_i64(gpu_block_id_tensor, "gpu_block_id_tensor")
        cpu_ids = _host_i64(cpu_block_id_tensor, "cpu_block_id_tensor")
        ptrs = _host_i64(gpu_layer_ptrs_tensor, "gpu_layer_ptrs_tensor")
        self._keep = (cpu_tensor,)
        d = TransferDesc()
        _fill_desc(d, gpu_ids, cpu_ids, ptrs, cpu_tensor, gpu_kv_stride_in_bytes,
                   gpu_block_stride_in_bytes, cpu_kv_stride_in_bytes, cpu_layer_stride_in_bytes,
                   cpu_block_stride_in_bytes, chunk_size_in_bytes, start_layer_id, transfer_sms,
                   is_host_to_device, use_ce_transfer, is_mla, ce_min_run_bytes, False,
                   gpu_layer_bytes, cpu_startoff_inside_chunks, ce_schedule)
        h = ctypes.c_void_p()
        check(self._lib.fkv_plan_create(ctypes.byref(d), int(device), ctypes.byref(h)),
              "fkv_plan_create")
        self._handle = h

    def execute(self, stream: Optional[torch.cuda.Stream] = None,
                kernel_events: Optional[tuple] = None) -> None:
        """Launch the plan on ``stream`` (default: current stream).  With
        ``kernel_events=(start, end)`` (torch.cuda.Event, timing enabled)
        the events bracket the SM copy kernel alone.  torch creates an
        event's CUDA handle on its first record(), so each event must have
        been recorded once before it is passed here."""
        s = int(stream.cuda_stream) if stream is not None else _stream_handle()
        if kernel_events is None:
            check(self._lib.fkv_plan_execute(self._handle, s), "fkv_plan_execute")
        else:
            a, b = kernel_events
            if not a.cuda_event or not b.cuda_event:
                raise RuntimeError("kernel_events must have been recorded once (no CUDA handle yet)")
            check(self._lib.fkv_plan_execute_ex(self._handle, s, a.cuda_event, b.cuda_event),
                  "fkv_plan_execute_ex")

    def stats(self) -> dict:
        a, b, c, e = (ctypes.c_int64() for _ in range(4))
        check(self._lib.fkv_plan_stats(self._handle, ctypes.byref(a), ctypes.byref(b),
                                       ctypes.byref(c), ctypes.byref(e)), "fkv_plan_stats")
        return {"sm_chunks": a.value, "ce_copies": b.value, "ce_bytes": c.value,
                "sm_bytes": e.value}

    def close(self) -> None:
        if self._handle is not None:
            self._lib.fkv_plan_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TPTransferThreadGroup:
    """Mirror of flexkv::TPTransferThreadGroup (bindings.cpp:144-158)."""

    def __init__(self, num_gpus: int, gpu_blocks: Sequence[Sequence[torch.Tensor]],
                 cpu_blocks: torch.Tensor, dp_group_id: int):
        self._lib = _lib.load()
        self._handle = None
        if len(gpu_blocks) != num_gpus:
            raise RuntimeError("gpu_blocks must hold one list of layer tensors per TP rank")
        num_layers = len(gpu_blocks[0])
        if any(len(r) != num_layers for r in gpu_blocks):
            raise RuntimeError("every TP rank needs the same number of layer tensors")
        ptrs = torch.tensor([t.data_ptr() for r in gpu_blocks for t in r], dtype=torch.int64)
        devs = torch.tensor([r[0].device.index if r[0].is_cuda else -1 for r in gpu_blocks],
                            dtype=torch.int32)
        self._keep = (gpu_blocks, cpu_blocks, ptrs, devs)
        self.num_gpus = num_gpus
        h = ctypes.c_void_p()
        check(self._lib.fkv_tp_group_create(int(num_gpus), int(dp_group_id), devs.data_ptr(),
                                            ptrs.data_ptr(), int(num_layers),
                                            cpu_blocks.data_ptr(), _nbytes(cpu_blocks),
                                            ctypes.byref(h)), "TPTransferThreadGroup")
        self._handle = h

    def tp_group_transfer(self, gpu_block_id_tensor: torch.Tensor, gpu_kv_stride_in_bytes: int,
                          gpu_block_stride_in_bytes: int, gpu_chunk_size_in_bytes: int,
                          cpu_block_id_tensor: torch.Tensor, cpu_kv_stride_in_bytes: int,
                          cpu_layer_stride_in_bytes: int, cpu_block_stride_in_bytes: int,
                          cpu_chunk_size_in_bytes: int, transfer_sms: int,
                          is_host_to_device: bool, use_ce_transfer: bool, layer_id: int,
                          layer_granularity: int, is_mla: bool) -> None:
        gpu_ids = _host_i64(gpu_block_id_tensor, "gpu_block_id_tensor")
        cpu_ids = _host_i64(cpu_block_id_tensor, "cpu_block_id_tensor")
        if gpu_ids.numel() != cpu_ids.numel():
            raise RuntimeError("gpu and cpu block id tensors differ in length")
        check(self._lib.fkv_tp_group_transfer(
            self._handle, gpu_ids.data_ptr(), cpu_ids.data_ptr(), gpu_ids.numel(),
            int(gpu_kv_stride_in_bytes), int(gpu_block_stride_in_bytes),
            int(gpu_chunk_size_in_bytes), int(cpu_kv_stride_in_bytes),
            int(cpu_layer_stride_in_bytes), int(cpu_block_stride_in_bytes),
            int(cpu_chunk_size_in_bytes), int(transfer_sms), int(bool(is_host_to_device)),
            int(bool(use_ce_transfer)), int(layer_id), int(layer_granularity),
            int(bool(is_mla))), "tp_group_transfer")

    def close(self) -> None:
        if self._handle is not None:
            self._lib.fkv_tp_group_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def get_hash_size() -> int:
    """Size of one block hash in bytes (hash.cpp:15)."""
    return int(_lib.load().fkv_get_hash_size())


class Hasher:
    """Streaming XXH64, seed 0 (cache_utils.h:17-26), computed on the GPU of
    the current device; the state never leaves device memory."""

    def __init__(self) -> None:
        self._lib = _lib.load()
        self._handle = None
        h = ctypes.c_void_p()
        check(self._lib.fkv_hasher_create(-1, ctypes.byref(h)), "Hasher")
        self._handle = h

    def reset(self) -> None:
        check(self._lib.fkv_hasher_reset(self._handle, _stream_handle()), "Hasher.reset")

    def update(self, input, size: Optional[int] = None) -> "Hasher":
        """update(tensor) hashes the tensor's bytes; update(ptr, size) hashes
        ``size`` bytes at address ``ptr`` (host or device)."""
        if isinstance(input, torch.Tensor):
            if size is not None:
                raise TypeError("update(tensor) takes no size")
            t = input.contiguous()
            check(self._lib.fkv_hasher_update(self._handle, t.data_ptr(), _nbytes(t),
                                              _stream_handle()), "Hasher.update")
        else:
            if size is None:
                raise TypeError("update(ptr, size) needs a size")
            check(self._lib.fkv_hasher_update(self._handle, int(input), int(size),
                                              _stream_handle()), "Hasher.update")
        return self

    def digest(self) -> int:
        out = ctypes.c_uint64()
        check(self._lib.fkv_hasher_digest(self._handle, ctypes.byref(out), _stream_handle()),
              "Hasher.digest")
        return int(out.value)

    def close(self) -> None:
        if self._handle is not None:
            self._lib.fkv_hasher_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gen_hashes(hasher: Hasher, token_ids: torch.Tensor, tokens_per_block: int,
               block_hashes: torch.Tensor) -> None:
    """Prefix-chained block hashes (hash.cpp:47-66): block_hashes[b] =
    XXH64 of everything the hasher has consumed through block b.  Writes
    ``block_hashes`` (uint64/int64, host or CUDA) in place."""
    if token_ids.dim() != 1 or block_hashes.dim() != 1:
        raise RuntimeError("token_ids and block_hashes must be 1-D")
    if token_ids.element_size() != 8 or block_hashes.element_size() != 8:
        raise RuntimeError("token_ids and block_hashes must have 8-byte elements")
    if not block_hashes.is_contiguous():
        raise RuntimeError("block_hashes must be contiguous")
    tok = token_ids.contiguous()
    check(hasher._lib.fkv_gen_hashes(hasher._handle, tok.data_ptr(), tok.numel(),
                                     int(tokens_per_block), block_hashes.data_ptr(),
                                     block_hashes.numel(), _stream_handle()), "gen_hashes")


def gen_hashes_batched(token_ids: torch.Tensor, seq_offsets: Sequence[int], tokens_per_block: int,
                       block_hashes: Optional[torch.Tensor] = None) -> torch.Tensor:
    """gen_hashes over many independent sequences at once, each with a fresh
    hasher (one SequenceMeta each, block.py:49-57).  Sequence s is
    token_ids[seq_offsets[s]:seq_offsets[s+1]]; its floor(len/tpb) hashes
    follow those of sequence s-1 in the output.  seq_offsets may be a list,
    a numpy array or a CPU tensor (arrays avoid a per-call conversion)."""
    if isinstance(seq_offsets, torch.Tensor):
        seq_offsets = seq_offsets.detach().cpu().numpy()
    offs_np = np.ascontiguousarray(seq_offsets, dtype=np.int64)
    n = offs_np.size - 1
    total = int((np.diff(offs_np) // tokens_per_block).sum()) if n > 0 else 0
    if block_hashes is None:  # every entry is written
        block_hashes = torch.empty(total, dtype=torch.uint64, device=token_ids.device)
    if block_hashes.numel() < total:
        raise RuntimeError("block_hashes is too small")
    tok = token_ids.contiguous()
    if tok.element_size() != 8:
        raise RuntimeError("token_ids must have 8-byte elements")
    dev = tok.device if tok.is_cuda else None
    ctx = torch.cuda.device(dev) if dev is not None else torch.cuda.device(torch.cuda.current_device())
    with ctx:
        check(_lib.load().fkv_gen_hashes_batched(tok.data_ptr(), offs_np.ctypes.data, n,
                                                 int(tokens_per_block), block_hashes.data_ptr(),
                                                 _stream_handle()), "gen_hashes_batched")
    return block_hashes


class SSDIOCTX:
    """Mirror of flexkv::SSDIOCTX (csrc/transfer_ssd.h:170-242, bound at
    bindings.cpp:141-142): ``SSDIOCTX(ssd_files, num_devices,
    iouring_entries, iouring_flags)`` with ``ssd_files[d]`` the file paths of
    SSD device d (all devices hold as many files as device 0, as the
    reference assumes).  Opens every file read-write.  iouring_entries > 0
    issues requests through io_uring rings of that depth; 0 (or a kernel
    without io_uring) issues them from a thread pool."""

    def __init__(self, ssd_files: Dict[int, List[str]], num_devices: int, iouring_entries: int = 0,
                 iouring_flags: int = 0):
        self._handle = None
        nf = len(ssd_files[0])
        paths = [str(ssd_files[d][f]) for d in range(num_devices) for f in range(nf)]
        arr = (ctypes.c_char_p * len(paths))(*[p.encode() for p in paths])
        h = ctypes.c_void_p()
        check(_lib.load().fkv_ssd_ctx_create(arr, int(num_devices), nf, int(iouring_entries),
                                             int(iouring_flags), ctypes.byref(h)), "SSDIOCTX")
        self._handle = h
        self.num_devices, self.num_files_per_device = int(num_devices), nf

    @property
    def uses_io_uring(self) -> bool:
        return bool(_lib.load().fkv_ssd_ctx_uses_io_uring(self._handle))

    def last_stats(self) -> Tuple[int, int]:
        """(file requests, bytes) of the most recent transfer on this context."""
        n, b = ctypes.c_int64(), ctypes.c_int64()
        check(_lib.load().fkv_ssd_last_stats(self._handle, ctypes.byref(n), ctypes.byref(b)), "last_stats")
        return n.value, b.value

    def close(self) -> None:
        if self._handle:
            _lib.load().fkv_ssd_ctx_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _ssd_ids(t, name: str):
    if isinstance(t, np.ndarray):
        if t.dtype != np.int64:
            raise RuntimeError(f"{name} must be int64")
        return np.ascontiguousarray(t)
    if not isinstance(t, torch.Tensor) or t.dtype != torch.int64:
        raise RuntimeError(f"{name} must be int64")  # TORCH_CHECK, bindings.cpp:66-69
    return t.detach().cpu().contiguous()


def transfer_kv_blocks_ssd(ioctx: SSDIOCTX, cpu_layer_id_list, cpu_tensor_ptr: int, ssd_block_ids,
                           cpu_block_ids, cpu_layer_stride_in_bytes: int, cpu_kv_stride_in_bytes: int,
                           ssd_layer_stride_in_bytes: int, ssd_kv_stride_in_bytes: int,
                           chunk_size_in_bytes: int, block_stride_in_bytes: int, is_read: bool,
                           num_blocks_per_file: int, round_robin: int = 1,
                           num_threads_per_device: int = 16, is_mla: bool = False,
                           cpu_pool_bytes: int = 0) -> None:
    """Drop-in for flexkv.c_ext.transfer_kv_blocks_ssd (bindings.cpp:57-77,
    110-119; same keyword names and defaults).  Layers
    [cpu_layer_id_list[0], cpu_layer_id_list[0] + len(cpu_layer_id_list))
    move between the CPU pool at cpu_tensor_ptr and the SSD files, SSD ->
    CPU when is_read.  Synchronous.  cpu_pool_bytes (not in the reference)
    enables a bounds check of the CPU side."""
    s_ids = _ssd_ids(ssd_block_ids, "ssd_block_ids")
    c_ids = _ssd_ids(cpu_block_ids, "cpu_block_ids")
    if len(s_ids) != len(c_ids):
        raise RuntimeError("ssd_block_ids and cpu_block_ids differ in length")
    layers = cpu_layer_id_list.tolist() if hasattr(cpu_layer_id_list, "tolist") else list(cpu_layer_id_list)
    start = int(layers[0]) if layers else 0
    sp = s_ids.ctypes.data if isinstance(s_ids, np.ndarray) else s_ids.data_ptr()
    cp = c_ids.ctypes.data if isinstance(c_ids, np.ndarray) else c_ids.data_ptr()
    check(_lib.load().fkv_transfer_kv_blocks_ssd(
        ioctx._handle, start, len(layers), ctypes.c_void_p(int(cpu_tensor_ptr)), int(cpu_pool_bytes), sp, cp,
        len(s_ids), int(cpu_layer_stride_in_bytes), int(cpu_kv_stride_in_bytes),
        int(ssd_layer_stride_in_bytes), int(ssd_kv_stride_in_bytes), int(chunk_size_in_bytes),
        int(block_stride_in_bytes), int(bool(is_read)), int(num_blocks_per_file), int(round_robin),
        int(num_threads_per_device), int(bool(is_mla))), "transfer_kv_blocks_ssd")
