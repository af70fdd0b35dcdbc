"""ctypes binding of libflexkv_b200.so (the C ABI in include/flexkv_b200.h).

Loading fails loudly: there is no Python or CPU fallback for any entry point.
Build the library with ``python -m flexkv_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_u64 = ctypes.c_uint64
c_vp = ctypes.c_void_p
c_char_p = ctypes.c_char_p
P_i64 = ctypes.POINTER(ctypes.c_int64)
P_u64 = ctypes.POINTER(ctypes.c_uint64)

FKV_OK = 0
FKV_ERR_INVALID_ARG = 1
FKV_ERR_OUT_OF_RANGE = 2
FKV_ERR_MISALIGNED = 3
FKV_ERR_CUDA = 4
FKV_ERR_UNSUPPORTED = 5
FKV_ERR_TIMEOUT = 6
FKV_ERR_IO = 7


class TransferDesc(ctypes.Structure):
    """Mirror of ``fkv_transfer_desc`` (field order and types must match)."""

    _fields_ = [
        ("num_blocks", c_int),
        ("start_layer_id", c_int),
        ("num_layers", c_int),
        ("is_host_to_device", c_int),
        ("is_mla", c_int),
        ("transfer_sms", c_int),
        ("use_ce_transfer", c_int),
        ("synchronous", c_int),
        ("gpu_block_ids", c_vp),
        ("cpu_block_ids", c_vp),
        ("gpu_layer_ptrs", c_vp),
        ("cpu_ptr", c_vp),
        ("gpu_kv_stride_in_bytes", c_i64),
        ("gpu_block_stride_in_bytes", c_i64),
        ("cpu_kv_stride_in_bytes", c_i64),
        ("cpu_layer_stride_in_bytes", c_i64),
        ("cpu_block_stride_in_bytes", c_i64),
        ("cpu_startoff_inside_chunks", c_i64),
        ("chunk_size_in_bytes", c_i64),
        ("cpu_pool_bytes", c_i64),
        ("gpu_layer_bytes", c_i64),
        ("ce_min_run_bytes", c_i64),
        ("num_ce_streams", c_int),
        ("ce_schedule", c_int),
    ]


class EngineConfig(ctypes.Structure):
    """Mirror of ``fkv_engine_config``."""

    _fields_ = [
        ("num_ranks", c_int),
        ("num_layers", c_int),
        ("device_ids", c_vp),
        ("gpu_layer_ptrs", c_vp),
        ("cpu_ptr", c_vp),
        ("cpu_pool_bytes", c_i64),
        ("gpu_layer_bytes", c_i64),
        ("gpu_kv_stride_in_bytes", c_i64),
        ("gpu_block_stride_in_bytes", c_i64),
        ("gpu_chunk_size_in_bytes", c_i64),
        ("cpu_kv_stride_in_bytes", c_i64),
        ("cpu_layer_stride_in_bytes", c_i64),
        ("cpu_block_stride_in_bytes", c_i64),
        ("cpu_chunk_size_in_bytes", c_i64),
        ("is_mla", c_int),
        ("transfer_sms_h2d", c_int),
        ("transfer_sms_d2h", c_int),
        ("use_ce_h2d", c_int),
        ("use_ce_d2h", c_int),
        ("streams_per_direction", c_int),
        ("staging_bytes", c_i64),
        ("ssd_ctx", c_vp),
        ("ssd_layer_stride_in_bytes", c_i64),
        ("ssd_kv_stride_in_bytes", c_i64),
        ("ssd_num_blocks_per_file", c_int),
        ("ssd_round_robin", c_int),
        ("ssd_threads_per_device", c_int),
        ("ssd_reserved", c_int),
    ]


class EngineOp(ctypes.Structure):
    """Mirror of ``fkv_engine_op``."""

    _fields_ = [
        ("op_id", c_i64),
        ("type", c_int),
        ("num_blocks", c_int),
        ("gpu_block_ids", c_vp),
        ("cpu_block_ids", c_vp),
        ("layer_id", c_int),
        ("layer_granularity", c_int),
        ("num_predecessors", c_int),
        ("reserved", c_int),
        ("predecessors", c_vp),
    ]


FKV_OP_H2D, FKV_OP_D2H, FKV_OP_VIRTUAL, FKV_OP_DISK2H, FKV_OP_H2DISK = 0, 1, 2, 3, 4


class IpcHandle(ctypes.Structure):
    """Mirror of ``fkv_ipc_handle``."""

    _fields_ = [
        ("cuda_handle", ctypes.c_ubyte * 64),
        ("base_addr", c_u64),
        ("alloc_bytes", c_u64),
        ("offset", c_i64),
        ("bytes", c_i64),
        ("device", ctypes.c_int32),
        ("pid", ctypes.c_int32),
    ]

# name -> (restype, argtypes)
_SIGNATURES = {
    "fkv_last_error": (c_char_p, []),
    "fkv_version": (c_char_p, []),
    "fkv_kernel_launch_count": (c_u64, []),
    "fkv_host_register": (c_int, [c_vp, c_i64, c_int]),
    "fkv_host_unregister": (c_int, [c_vp]),
    "fkv_transfer_kv_blocks": (
        c_int,
        [c_int, c_int, c_int, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
         c_i64, c_i64, c_vp, c_int, c_int, c_int, c_int],
    ),
    "fkv_transfer_desc_init": (None, [ctypes.POINTER(TransferDesc)]),
    "fkv_transfer_kv_blocks_ex": (c_int, [ctypes.POINTER(TransferDesc), c_vp]),
    "fkv_plan_create": (c_int, [ctypes.POINTER(TransferDesc), c_int, ctypes.POINTER(c_vp)]),
    "fkv_plan_execute": (c_int, [c_vp, c_vp]),
    "fkv_plan_execute_ex": (c_int, [c_vp, c_vp, c_vp, c_vp]),
    "fkv_plan_stats": (c_int, [c_vp, P_i64, P_i64, P_i64, P_i64]),
    "fkv_plan_destroy": (None, [c_vp]),
    "fkv_coalesce_runs": (c_i64, [c_vp, c_vp, c_i64, c_vp, c_i64]),
    "fkv_tp_group_create": (
        c_int, [c_int, c_int, c_vp, c_vp, c_int, c_vp, c_i64, ctypes.POINTER(c_vp)]),
    "fkv_tp_group_transfer": (
        c_int,
        [c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_int,
         c_int, c_int, c_int, c_int, c_int],
    ),
    "fkv_tp_group_num_gpus": (c_int, [c_vp]),
    "fkv_tp_group_destroy": (None, [c_vp]),
    "fkv_get_hash_size": (c_int, []),
    "fkv_hasher_create": (c_int, [c_int, ctypes.POINTER(c_vp)]),
    "fkv_hasher_destroy": (None, [c_vp]),
    "fkv_hasher_reset": (c_int, [c_vp, c_vp]),
    "fkv_hasher_update": (c_int, [c_vp, c_vp, c_i64, c_vp]),
    "fkv_hasher_update_bounded": (c_int, [c_vp, c_vp, c_i64, c_u64, c_i64, c_vp]),
    "fkv_hasher_digest": (c_int, [c_vp, P_u64, c_vp]),
    "fkv_gen_hashes": (c_int, [c_vp, c_vp, c_i64, c_int, c_vp, c_i64, c_vp]),
    "fkv_gen_hashes_batched": (c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp]),
    "fkv_engine_config_init": (None, [ctypes.POINTER(EngineConfig)]),
    "fkv_engine_create": (c_int, [ctypes.POINTER(EngineConfig), ctypes.POINTER(c_vp)]),
    "fkv_engine_submit_graph": (c_int, [c_vp, c_i64, ctypes.POINTER(EngineOp), c_int]),
    "fkv_engine_poll": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, ctypes.POINTER(c_int)]),
    "fkv_engine_pending_ops": (c_i64, [c_vp]),
    "fkv_engine_destroy": (None, [c_vp]),
    "fkv_engine_shutdown": (c_int, [c_vp, c_int]),
    "fkv_ipc_export": (c_int, [c_vp, c_i64, ctypes.POINTER(IpcHandle)]),
    "fkv_ipc_open": (c_int, [ctypes.POINTER(IpcHandle), c_int, ctypes.POINTER(c_vp)]),
    "fkv_ipc_close": (c_int, [c_vp]),
    "fkv_ipc_open_count": (c_int, []),
    "fkv_ssd_ctx_create": (c_int, [ctypes.POINTER(c_char_p), c_int, c_int, c_int, c_int, ctypes.POINTER(c_vp)]),
    "fkv_ssd_ctx_destroy": (None, [c_vp]),
    "fkv_transfer_kv_blocks_ssd": (
        c_int,
        [c_vp, c_int, c_int, c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
         c_int, c_int, c_int, c_int, c_int],
    ),
    "fkv_ssd_last_stats": (c_int, [c_vp, P_i64, P_i64]),
    "fkv_ssd_ctx_uses_io_uring": (c_int, [c_vp]),
    "fkv_transfer_kv_blocks_noalloc": (
        c_int,
        [c_int, c_int, c_int, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
         c_i64, c_i64, c_i64, c_vp, c_int, c_int, c_int],
    ),
    "fkv_cache_index_create": (c_int, [c_int, c_i64, c_int, ctypes.POINTER(c_vp)]),
    "fkv_cache_index_destroy": (None, [c_vp]),
    "fkv_cache_index_match": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_vp]),
    "fkv_cache_index_put": (
        c_int, [c_vp, c_vp, c_vp, c_int, c_vp, ctypes.POINTER(TransferDesc), c_int, c_int, c_vp, c_vp,
                c_vp, c_vp, c_vp]),
    "fkv_cache_index_put2": (
        c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_vp, ctypes.POINTER(TransferDesc), c_int, c_vp, c_vp, c_vp,
                c_vp, c_vp, c_vp, c_vp]),
    "fkv_cache_index_get": (
        c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_vp, ctypes.POINTER(TransferDesc), c_int, c_vp, c_int, c_vp,
                c_vp, c_vp]),
    "fkv_cache_index_set_ready": (c_int, [c_vp, c_vp, c_i64, c_int, P_i64, c_vp]),
    "fkv_cache_index_remove": (c_int, [c_vp, c_vp, c_i64, c_vp, c_vp]),
    "fkv_cache_index_recycle": (c_int, [c_vp, c_vp, c_i64, c_vp]),
    "fkv_cache_index_take": (c_int, [c_vp, c_i64, c_vp, P_i64, c_vp]),
    "fkv_cache_index_stats": (c_int, [c_vp, c_vp, c_vp]),
}

_lock = threading.Lock()
_lib = None


class FlexKVError(RuntimeError):
    """A non-zero status from libflexkv_b200 (RuntimeError, as the
    reference's pybind layer raises for CUDA failures, bindings.cpp:51-54)."""

    def __init__(self, code: int, where: str, message: str):
        super().__init__(f"{where} failed (status {code}): {message}")
        self.code = code


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with argument types declared."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or os.environ.get("FLEXKV_B200_LIB", LIB_PATH)
        if not os.path.exists(p):
            raise ImportError(
                f"libflexkv_b200.so not found at {p}; build it with `python -m flexkv_b200.build`")
        lib = ctypes.CDLL(p)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int, where: str) -> None:
    if rc != FKV_OK:
        msg = load().fkv_last_error()
        raise FlexKVError(rc, where, msg.decode() if msg else "")


def lib_path() -> str:
    return load()._name
