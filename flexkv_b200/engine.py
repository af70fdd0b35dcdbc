"""TransferEngine for the GPU<->CPU data plane, over the native engine of
libflexkv_b200 (``fkv_engine_*`` in include/flexkv_b200.h).

Mirrors the surface FlexKV's KVManager and tests use
(flexkv/transfer/transfer_engine.py:42-307): ``start()``,
``submit_transfer_graph(graph)``, ``get_completed_graphs_and_ops(timeout)``
returning ``(graph_id, op_id)`` pairs with ``op_id == -1`` for a finished
graph, and ``shutdown()``.  Graphs are FlexKV ``TransferOpGraph`` objects
(read by duck typing: ``graph_id``, ``_op_map``, each op's ``op_id``,
``transfer_type``, ``src_descriptor`` / ``dst_descriptor``
``.physical_block_ids``, ``layer_id``, ``layer_granularity``,
``predecessors``, ``dp_id``) or the light mirrors defined here.

One native engine per data-parallel group; a group's tensor-parallel ranks
share its host pool (rank i owns byte slice i of every CPU chunk).  Only the
GPU<->CPU op types (H2D, D2H) and VIRTUAL are handled; the SSD and remote
tiers are not part of this package.

Unlike the reference, where a failed op is logged and then reported as
finished (worker.py:166-169), a failure is also kept in ``failed_ops``.
"""
from __future__ import annotations

import ctypes
import itertools
import threading
from dataclasses import dataclass, field
from enum import Enum
from typing import Dict, List, Optional, Sequence, Set, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import FKV_OP_D2H, FKV_OP_DISK2H, FKV_OP_H2D, FKV_OP_H2DISK, FKV_OP_VIRTUAL, EngineConfig, \
    EngineOp, check
from .layout import KVCacheLayout


class TransferType(Enum):
    """Names as flexkv/common/transfer.py:15-28 (the tiers handled here)."""
    H2D = "H2D"
    D2H = "D2H"
    DISK2H = "DISK2H"
    H2DISK = "H2DISK"
    VIRTUAL = "Virtual"


@dataclass
class TransferDescriptor:
    physical_block_ids: torch.Tensor = field(default_factory=lambda: torch.tensor([], dtype=torch.int64))


_op_ids = itertools.count()
_graph_ids = itertools.count()
_id_lock = threading.Lock()


@dataclass
class TransferOp:
    """Light mirror of flexkv.common.transfer.TransferOp."""
    graph_id: int
    transfer_type: TransferType
    layer_id: int = -1
    layer_granularity: int = -1
    src_descriptor: TransferDescriptor = field(default_factory=TransferDescriptor)
    dst_descriptor: TransferDescriptor = field(default_factory=TransferDescriptor)
    predecessors: Set[int] = field(default_factory=set)
    successors: Set[int] = field(default_factory=set)
    dp_id: int = 0
    op_id: int = field(init=False)

    def __post_init__(self):
        if self.transfer_type != TransferType.VIRTUAL and (
                len(self.src_descriptor.physical_block_ids) != len(self.dst_descriptor.physical_block_ids)):
            raise ValueError("src_descriptor and dst_descriptor must have the same number of physical blocks")
        with _id_lock:
            self.op_id = next(_op_ids)


class TransferOpGraph:
    """Light mirror of flexkv.common.transfer.TransferOpGraph."""

    def __init__(self):
        with _id_lock:
            self.graph_id = next(_graph_ids)
        self._op_map: Dict[int, TransferOp] = {}

    def add_transfer_op(self, op: TransferOp) -> None:
        op.graph_id = self.graph_id
        self._op_map[op.op_id] = op

    def add_virtual_op(self, op: TransferOp) -> None:
        op.graph_id = self.graph_id
        op.transfer_type = TransferType.VIRTUAL
        self._op_map[op.op_id] = op

    def add_dependency(self, successor_op_id: int, predecessor_op_id: int) -> None:
        assert successor_op_id in self._op_map and predecessor_op_id in self._op_map
        self._op_map[successor_op_id].predecessors.add(predecessor_op_id)
        self._op_map[predecessor_op_id].successors.add(successor_op_id)

    def bind_to_dp_group(self, dp_id: int) -> None:
        for op in self._op_map.values():
            op.dp_id = dp_id

    @property
    def num_ops(self) -> int:
        return len(self._op_map)


def _type_code(t) -> int:
    name = getattr(t, "name", str(t)).upper()
    if name == "H2D":
        return FKV_OP_H2D
    if name == "D2H":
        return FKV_OP_D2H
    if name == "VIRTUAL":
        return FKV_OP_VIRTUAL
    if name == "DISK2H":
        return FKV_OP_DISK2H
    if name == "H2DISK":
        return FKV_OP_H2DISK
    raise ValueError(f"transfer type {name} is not handled by this engine")


def _ids(desc) -> np.ndarray:
    t = desc.physical_block_ids
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu().numpy()
    return np.ascontiguousarray(t, dtype=np.int64)


# Engines whose bounded shutdown timed out keep running detached; what they
# move (tensors held by the group, an SSD context) is kept alive here.
_DETACHED: list = []


class _GroupEngine:
    """One native engine: the GPUs of one data-parallel group."""

    def __init__(self, gpu_blocks: Sequence[Sequence[torch.Tensor]], cpu_blocks: torch.Tensor,
                 gpu_layout: KVCacheLayout, cpu_layout: KVCacheLayout, itemsize: int,
                 transfer_sms_h2d: int, transfer_sms_d2h: int, use_ce_h2d: bool, use_ce_d2h: bool,
                 staging_bytes: int, ssd=None, streams_per_direction: int = 0):
        self._lib = _lib.load()
        self._handle = None
        nr, nl = len(gpu_blocks), len(gpu_blocks[0])
        per = gpu_layout.div_layer(gpu_layout.num_layer)
        self._ptrs = np.array([t.data_ptr() for r in gpu_blocks for t in r], dtype=np.uint64)
        self._devs = np.array([r[0].device.index for r in gpu_blocks], dtype=np.int32)
        self._keep = (gpu_blocks, cpu_blocks)
        c = EngineConfig()
        self._lib.fkv_engine_config_init(ctypes.byref(c))
        c.num_ranks, c.num_layers = nr, nl
        c.device_ids = self._devs.ctypes.data
        c.gpu_layer_ptrs = self._ptrs.ctypes.data
        c.cpu_ptr = cpu_blocks.data_ptr()
        c.cpu_pool_bytes = cpu_blocks.numel() * cpu_blocks.element_size()
        c.gpu_layer_bytes = per.get_total_elements() * itemsize
        c.gpu_kv_stride_in_bytes = per.get_kv_stride() * itemsize
        c.gpu_block_stride_in_bytes = per.get_block_stride() * itemsize
        c.gpu_chunk_size_in_bytes = per.get_chunk_size() * itemsize
        c.cpu_kv_stride_in_bytes = cpu_layout.get_kv_stride() * itemsize
        c.cpu_layer_stride_in_bytes = cpu_layout.get_layer_stride() * itemsize
        c.cpu_block_stride_in_bytes = cpu_layout.get_block_stride() * itemsize
        c.cpu_chunk_size_in_bytes = cpu_layout.get_chunk_size() * itemsize
        c.is_mla = int(bool(gpu_layout.is_mla))
        c.transfer_sms_h2d, c.transfer_sms_d2h = int(transfer_sms_h2d), int(transfer_sms_d2h)
        c.use_ce_h2d, c.use_ce_d2h = int(bool(use_ce_h2d)), int(bool(use_ce_d2h))
        c.staging_bytes = int(staging_bytes)
        c.streams_per_direction = int(streams_per_direction)
        if ssd is not None:
            ctx, st, per_file, rr, threads = ssd
            c.ssd_ctx = ctx._handle
            c.ssd_layer_stride_in_bytes = st.ssd_layer_stride_in_bytes
            c.ssd_kv_stride_in_bytes = st.ssd_kv_stride_in_bytes
            c.ssd_num_blocks_per_file = int(per_file)
            c.ssd_round_robin = int(rr)
            c.ssd_threads_per_device = int(threads)
        h = ctypes.c_void_p()
        check(self._lib.fkv_engine_create(ctypes.byref(c), ctypes.byref(h)), "TransferEngine")
        self._handle = h

    def submit(self, graph_id: int, ops) -> None:
        arr = (EngineOp * max(len(ops), 1))()
        keep = []
        for i, op in enumerate(ops):
            code = _type_code(op.transfer_type)
            e = arr[i]
            e.op_id = int(op.op_id)
            e.type = code
            if code == FKV_OP_VIRTUAL:
                e.num_blocks = 0
            else:
                src, dst = _ids(op.src_descriptor), _ids(op.dst_descriptor)
                if src.size != dst.size:
                    raise ValueError(f"op {op.op_id}: source and destination block counts differ")
                # H2D: src = CPU ids, dst = GPU ids; D2H the reverse (worker.py:272-281).
                # DISK2H: src = SSD ids, dst = CPU ids; H2DISK the reverse
                # (worker.py:549-556); the SSD ids ride in the gpu-id slot.
                g, c = (dst, src) if code in (FKV_OP_H2D, FKV_OP_H2DISK) else (src, dst)
                keep += [g, c]
                e.num_blocks = g.size
                e.gpu_block_ids = g.ctypes.data
                e.cpu_block_ids = c.ctypes.data
            e.layer_id = int(op.layer_id)
            e.layer_granularity = int(op.layer_granularity)
            preds = np.array(sorted(int(p) for p in getattr(op, "predecessors", ()) or ()), dtype=np.int64)
            keep.append(preds)
            e.num_predecessors = preds.size
            e.predecessors = preds.ctypes.data if preds.size else None
        check(self._lib.fkv_engine_submit_graph(self._handle, int(graph_id), arr, len(ops)),
              "submit_transfer_graph")

    def poll(self, timeout_ms: int, max_n: int = 4096) -> List[Tuple[int, int, int]]:
        g = np.zeros(max_n, dtype=np.int64)
        o = np.zeros(max_n, dtype=np.int64)
        s = np.zeros(max_n, dtype=np.int32)
        n = ctypes.c_int()
        check(self._lib.fkv_engine_poll(self._handle, g.ctypes.data, o.ctypes.data, s.ctypes.data,
                                        max_n, int(timeout_ms), ctypes.byref(n)), "poll")
        return [(int(g[i]), int(o[i]), int(s[i])) for i in range(n.value)]

    def pending(self) -> int:
        return int(self._lib.fkv_engine_pending_ops(self._handle))

    def close(self, timeout_s: Optional[float] = None) -> None:
        if self._handle is not None:
            h, self._handle = self._handle, None
            ms = -1 if timeout_s is None else max(0, int(timeout_s * 1000))
            rc = self._lib.fkv_engine_shutdown(h, ms)
            if rc != 0:
                _DETACHED.append(self)  # its tensors stay alive for the detached engine
            check(rc, "shutdown")


class TransferEngine:
    """GPU<->CPU TransferEngine for ``dp_size`` groups of ``tp_size`` GPUs.

    ``gpu_blocks[g]`` is the list of per-layer KV tensors of global GPU
    ``g = dp_id * tp_size + tp_rank`` (each [kv, num_blocks, tpb, heads/tp,
    head_dim]); ``cpu_blocks`` is the flat host pool with ``cpu_layout``
    (page-locked here if it is not already).  ``gpu_layout`` is the per-rank
    GPU layout (heads already divided for TP).

    SSD tier (optional): ``ssd_files`` (SSD device -> file paths, as
    SSDAllocator makes them), ``ssd_layout`` and ``ssd_num_blocks_per_file``
    enable DISK2H / H2DISK ops, run as CPUSSDDiskTransferWorker does
    (worker.py:482-590) on two engine I/O threads, dependencies honoured
    across the tiers.  ``streams_per_direction`` sizes the per-GPU stream
    pool of each direction (0 = 2)."""

    def __init__(self, gpu_blocks: Sequence[Sequence[torch.Tensor]], cpu_blocks: torch.Tensor,
                 gpu_layout: KVCacheLayout, cpu_layout: KVCacheLayout, tp_size: int = 1,
                 dp_size: int = 1, transfer_sms_h2d: int = -1, transfer_sms_d2h: int = -1,
                 use_ce_transfer_h2d: bool = False, use_ce_transfer_d2h: bool = False,
                 staging_bytes: int = 0, ssd_files: Optional[Dict[int, List[str]]] = None,
                 ssd_layout: Optional[KVCacheLayout] = None, ssd_num_blocks_per_file: int = 0,
                 ssd_iouring_entries: int = 0, ssd_iouring_flags: int = 0,
                 ssd_threads_per_device: int = 32, ssd_round_robin: int = 1,
                 streams_per_direction: int = 0):
        if len(gpu_blocks) != tp_size * dp_size:
            raise ValueError("gpu_blocks needs one list of layer tensors per GPU (dp_size * tp_size)")
        self._cpu = cpu_blocks
        self._registered = False
        if not cpu_blocks.is_pinned():
            from .c_ext import cudaHostRegister
            try:
                cudaHostRegister(cpu_blocks)
                self._registered = True
            except RuntimeError as e:  # registered already by the caller
                if "AlreadyRegistered" not in str(e):
                    raise
        itemsize = cpu_blocks.element_size()
        self._ssd_ctx = None
        ssd = None
        if ssd_files is not None:
            from .c_ext import SSDIOCTX
            from .ssd import SsdStrides
            if ssd_layout is None or ssd_num_blocks_per_file <= 0:
                raise ValueError("the SSD tier needs ssd_layout and ssd_num_blocks_per_file")
            self._ssd_ctx = SSDIOCTX(ssd_files, len(ssd_files), ssd_iouring_entries, ssd_iouring_flags)
            nfiles = sum(len(v) for v in ssd_files.values())
            st = SsdStrides.of(cpu_layout, ssd_layout, nfiles, itemsize)
            ssd = (self._ssd_ctx, st, ssd_num_blocks_per_file, ssd_round_robin, ssd_threads_per_device)
        self._groups = [
            _GroupEngine(gpu_blocks[d * tp_size:(d + 1) * tp_size], cpu_blocks, gpu_layout, cpu_layout,
                         itemsize, transfer_sms_h2d, transfer_sms_d2h, use_ce_transfer_h2d,
                         use_ce_transfer_d2h, staging_bytes, ssd, streams_per_direction)
            for d in range(dp_size)]
        self.failed_ops: Dict[int, int] = {}
        self._running = True

    @classmethod
    def from_handles(cls, gpu_handles, model_config, cache_config, cpu_handle, ssd_handle=None,
                     remote_handle=None) -> "TransferEngine":
        """Build from FlexKV StorageHandles and configs, the arguments of the
        reference constructor (transfer_engine.py:43-49); the SSD handle's
        file list, layout and blocks-per-file configure the SSD tier."""
        if remote_handle is not None:
            raise NotImplementedError("the remote tier is not part of flexkv_b200")
        gpu_blocks = [h.get_tensor_list() for h in gpu_handles]
        g, c = gpu_handles[0].kv_layout, cpu_handle.kv_layout
        from .layout import KVCacheLayoutType
        to = lambda x: KVCacheLayout(KVCacheLayoutType[x.type.name], x.num_layer, x.num_block,
                                     x.tokens_per_block, x.num_head, x.head_size, x.is_mla)
        ssd = {}
        if ssd_handle is not None:
            ssd = dict(ssd_files=ssd_handle.get_file_list(), ssd_layout=to(ssd_handle.kv_layout),
                       ssd_num_blocks_per_file=ssd_handle.num_blocks_per_file,
                       ssd_iouring_entries=getattr(cache_config, "ssd_cache_iouring_entries", 0),
                       ssd_iouring_flags=getattr(cache_config, "ssd_cache_iouring_flags", 0))
        return cls(gpu_blocks, cpu_handle.get_tensor(), to(g), to(c), model_config.tp_size,
                   model_config.dp_size, cache_config.transfer_sms_h2d, cache_config.transfer_sms_d2h,
                   cache_config.use_ce_transfer_h2d, cache_config.use_ce_transfer_d2h, **ssd)

    def start(self) -> None:
        """The engine runs from construction; kept for the reference API."""

    def submit_transfer_graph(self, transfer_graph) -> None:
        ops = list(transfer_graph._op_map.values())
        dp = {int(getattr(op, "dp_id", 0)) for op in ops} or {0}
        if len(dp) != 1:
            raise ValueError("all ops of a graph must belong to one data-parallel group")
        self._groups[dp.pop()].submit(transfer_graph.graph_id, ops)

    def get_completed_graphs_and_ops(self, timeout: Optional[float] = None) -> List[Tuple[int, int]]:
        out: List[Tuple[int, int]] = []
        wait_ms = int((timeout or 0) * 1000)
        for i, g in enumerate(self._groups):
            for gid, oid, st in g.poll(wait_ms if i == 0 else 0):
                if st != 0 and oid >= 0:
                    self.failed_ops[oid] = st
                out.append((gid, oid))
        return out

    def pending_ops(self) -> int:
        return sum(g.pending() for g in self._groups)

    def shutdown(self, timeout: Optional[float] = 60.0) -> None:
        """Drain the submitted ops and release the engine, waiting at most
        ``timeout`` seconds per data-parallel group (None: no limit).  On a
        timeout this raises RuntimeError; that group's engine keeps running
        detached until its ops finish, so the tensors it moves must stay
        alive, and the SSD context (if any) is left open for it."""
        groups, self._groups = self._groups, []
        err = None
        for g in groups:
            try:
                g.close(timeout)
            except RuntimeError as e:
                err = err or e
        if err is not None:
            if getattr(self, "_ssd_ctx", None) is not None:  # still used by the detached engine
                _DETACHED.append(self._ssd_ctx)
                self._ssd_ctx = None
            raise err
        if getattr(self, "_ssd_ctx", None) is not None:  # after the engines: their I/O threads use it
            self._ssd_ctx.close()
            self._ssd_ctx = None
        if self._registered:
            from .c_ext import cudaHostUnregister
            cudaHostUnregister(self._cpu)
            self._registered = False

    def __del__(self):
        try:
            self.shutdown()
        except Exception:
            pass
