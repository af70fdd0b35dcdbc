"""GPU-side helpers for the -m gpu tests: put oracle images on the device,
run the transfer through the C ABI (flexkv_b200.c_ext) and through the
reference's own transfer.cu (oracle/_ref), and read results back."""
from __future__ import annotations

import ctypes
from typing import List

import numpy as np
import torch

from flexkv_b200 import c_ext
from kvcase import Case, fill_bytes


class Pools:
    """Device layers + pinned host pool holding copies of host images."""

    def __init__(self, case: Case, gpu_imgs: List[np.ndarray], cpu_img: np.ndarray,
                 device: str = "cuda:0", alloc: str = "separate"):
        """alloc: "separate" (one tensor per layer, placement up to the
        allocator), "contiguous" (one allocation viewed per layer: uniform
        layer stride, which the planner folds), "irregular" (one allocation
        with uneven gaps between layers: never folded)."""
        self.case = case
        self.st = case.strides()
        if alloc == "separate":
            self.layers = [torch.from_numpy(g.copy()).to(device) for g in gpu_imgs]
        else:
            nb = self.st["gpu_layer_bytes"]
            gaps = [0] * len(gpu_imgs) if alloc == "contiguous" else \
                [256 * ((7 * l) % 5 + 1) for l in range(len(gpu_imgs))]
            offs, o = [], 0
            for gp in gaps:
                o += gp
                offs.append(o)
                o += nb
            self._base = torch.empty(o, dtype=torch.uint8, device=device)
            self.layers = []
            for g, off in zip(gpu_imgs, offs):
                v = self._base[off:off + nb]
                v.copy_(torch.from_numpy(g))
                self.layers.append(v)
        self.cpu = torch.from_numpy(cpu_img.copy()).pin_memory()
        self.ptrs = torch.tensor([t.data_ptr() for t in self.layers], dtype=torch.int64)

    def gpu_images(self) -> List[np.ndarray]:
        return [t.cpu().numpy() for t in self.layers]

    def cpu_image(self) -> np.ndarray:
        return self.cpu.numpy()

    def transfer(self, gids: np.ndarray, cids: np.ndarray, h2d: bool, mode: str = "auto",
                 rank: int = 0, transfer_sms: int = -1) -> None:
        case, st = self.case, self.st
        kw = {}
        use_ce = False
        if mode == "sm":
            kw["ce_min_run_bytes"] = 0
        elif mode == "ce":
            use_ce = True
        elif mode == "hybrid":
            kw["ce_min_run_bytes"] = 2 * st["gpu_chunk"]
        off = 0 if case.is_mla else rank * st["gpu_chunk"]
        if off:
            plan = c_ext.TransferPlan(
                torch.from_numpy(gids), self.ptrs, st["gpu_kv"], st["gpu_block"],
                torch.from_numpy(cids), self.cpu, st["cpu_kv"], st["cpu_layer"],
                st["cpu_block"], st["gpu_chunk"], case.layer_id, transfer_sms, h2d, use_ce,
                case.is_mla, cpu_startoff_inside_chunks=off,
                gpu_layer_bytes=st["gpu_layer_bytes"], **kw)
            plan.execute()
            torch.cuda.synchronize()
            plan.close()
            return
        c_ext.transfer_kv_blocks(
            torch.from_numpy(gids), self.ptrs, st["gpu_kv"], st["gpu_block"],
            torch.from_numpy(cids), self.cpu, st["cpu_kv"], st["cpu_layer"], st["cpu_block"],
            st["gpu_chunk"], case.layer_id, transfer_sms, h2d, use_ce, case.is_mla,
            gpu_layer_bytes=st["gpu_layer_bytes"], **kw)

    def reference_transfer(self, gids: np.ndarray, cids: np.ndarray, h2d: bool,
                           use_ce: bool = False, rank: int = 0, transfer_sms: int = 8) -> None:
        """The reference's own transfer.cu on the same buffers (pinned ids and
        pinned layer-pointer table, as its kernel reads them zero-copy)."""
        from oracle import oracle as O
        case, st = self.case, self.st
        g = torch.from_numpy(gids.astype(np.int64)).pin_memory()
        c = torch.from_numpy(cids.astype(np.int64)).pin_memory()
        ptrs = self.ptrs.pin_memory()
        off = 0 if case.is_mla else rank * st["gpu_chunk"]
        stream = torch.cuda.current_stream().cuda_stream
        rc = O.ref_lib().ref_transfer_kv_blocks(
            len(gids), case.layer_id, len(self.layers), g.data_ptr(), ptrs.data_ptr(),
            st["gpu_kv"], st["gpu_block"], c.data_ptr(), self.cpu.data_ptr(), st["cpu_kv"],
            st["cpu_layer"], st["cpu_block"], off, st["gpu_chunk"], stream, transfer_sms,
            int(h2d), int(use_ce), int(case.is_mla))
        assert rc == 0, f"reference transfer.cu returned CUDA error {rc}"
        torch.cuda.synchronize()


def initial_images(case: Case, gpu_seed_base: int = 100, cpu_seed: int = 99):
    st = case.strides()
    gpu = [fill_bytes(st["gpu_layer_bytes"], gpu_seed_base + l) for l in range(case.gran)]
    cpu = fill_bytes(st["cpu_pool_bytes"], cpu_seed)
    return gpu, cpu


def oracle_transfer(case: Case, gpu_imgs, cpu_img, gids, cids, h2d: bool, rank: int = 0):
    from oracle import oracle as O
    st = case.strides()
    off = 0 if case.is_mla else rank * st["gpu_chunk"]
    O.transfer(len(gids), case.layer_id, gids, gpu_imgs, st["gpu_kv"], st["gpu_block"], cids,
               cpu_img, st["cpu_kv"], st["cpu_layer"], st["cpu_block"], off, st["gpu_chunk"],
               h2d, case.is_mla, num_threads=4)
