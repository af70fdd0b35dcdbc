"""Sharing GPU tensors between processes over CUDA IPC.

Mirror of ``TensorSharedHandle`` (flexkv/common/memory_handle.py:17-56):
the inference engine's process wraps each KV-cache tensor in a handle,
pickles it to the process that runs the transfers (KVTPClient.
register_to_server, flexkv/server/client.py:199-215), and that process
calls ``get_tensor()`` to map the same device memory.  The reference goes
through ``torch.multiprocessing.reductions``; this one goes through the C
ABI (``fkv_ipc_export`` / ``fkv_ipc_open`` / ``fkv_ipc_close``), so the
handle is plain data that a process without torch can also consume.

Differences kept small on purpose: the constructor raises ValueError for a
non-CUDA tensor (as the reference does); ``get_tensor()`` returns a
zero-copy view with the original dtype, shape and strides, on the
exporting device ordinal.  The mapping is released when the last tensor
viewing it is freed.
"""
from __future__ import annotations

import ctypes
import os
from typing import Tuple

import torch

from . import _lib

_TYPESTR = "|u1"


class _IpcMemory:
    """Owner of one fkv_ipc_open; exposes the bytes to torch through the
    CUDA array interface and releases the open when torch drops it."""

    def __init__(self, ptr: int, nbytes: int, device: int):
        self.ptr, self.nbytes, self.device = ptr, nbytes, device
        self.__cuda_array_interface__ = {
            "shape": (nbytes,), "typestr": _TYPESTR, "data": (ptr, False), "version": 2}

    def __del__(self):
        if self.ptr:
            _lib.load().fkv_ipc_close(ctypes.c_void_p(self.ptr))
            self.ptr = 0


def _span_bytes(t: torch.Tensor) -> int:
    if t.numel() == 0:
        return 0
    last = sum((n - 1) * s for n, s in zip(t.shape, t.stride()))
    return (last + 1) * t.element_size()


class TensorSharedHandle:
    """Picklable handle to a CUDA tensor's memory for another process."""

    def __init__(self, tensor: torch.Tensor):
        if not tensor.is_cuda:
            raise ValueError("Only support CUDA tensor sharing")
        if any(s < 0 for s in tensor.stride()):
            raise ValueError("tensors with negative strides cannot be shared")
        self.device = tensor.device
        self.dtype = tensor.dtype
        self.shape: Tuple[int, ...] = tuple(tensor.shape)
        self.stride: Tuple[int, ...] = tuple(tensor.stride())
        self.nbytes = _span_bytes(tensor)
        self.exporter_pid = os.getpid()
        self._raw = b""
        if self.nbytes:
            h = _lib.IpcHandle()
            _lib.check(_lib.load().fkv_ipc_export(ctypes.c_void_p(tensor.data_ptr()), self.nbytes,
                                                  ctypes.byref(h)), "fkv_ipc_export")
            self._raw = ctypes.string_at(ctypes.addressof(h), ctypes.sizeof(h))

    def get_tensor(self) -> torch.Tensor:
        dev = self.device.index if self.device.index is not None else 0
        if not self.nbytes:
            return torch.empty(self.shape, dtype=self.dtype, device=f"cuda:{dev}")
        h = _lib.IpcHandle.from_buffer_copy(self._raw)
        ptr = ctypes.c_void_p()
        _lib.check(_lib.load().fkv_ipc_open(ctypes.byref(h), dev, ctypes.byref(ptr)), "fkv_ipc_open")
        mem = _IpcMemory(ptr.value, self.nbytes, dev)
        with torch.cuda.device(dev):
            raw = torch.as_tensor(mem, device=f"cuda:{dev}")
        return raw.view(self.dtype).as_strided(self.shape, self.stride)


def ipc_open_count() -> int:
    """Allocations currently mapped in this process through get_tensor()."""
    return int(_lib.load().fkv_ipc_open_count())
