"""The importing side of the cross-process IPC tests: runs in a spawned
process that maps the parent's KV layers through TensorSharedHandle and
moves blocks with the library (C ABI and TransferEngine), as the transfer
process of a deployment does with the inference engine's cache."""
from __future__ import annotations

import traceback


def child_main(handles, case, gids, cids, cpu_seed, new_cpu_seed, gpu_seed_base, q):
    try:
        import numpy as np
        import torch

        from flexkv_b200 import c_ext
        from flexkv_b200.engine import TransferDescriptor, TransferEngine, TransferOp, TransferOpGraph, \
            TransferType
        from flexkv_b200.memory_handle import ipc_open_count
        from gpu_util import initial_images, oracle_transfer

        st = case.strides()
        layers = [h.get_tensor() for h in handles]
        opened = ipc_open_count()
        # 1. D2H through the C ABI: the imported layers hold the parent's data.
        gpu, cpu = initial_images(case, gpu_seed_base, cpu_seed)
        pool = torch.from_numpy(cpu.copy()).pin_memory()
        ptrs = torch.tensor([t.data_ptr() for t in layers], dtype=torch.int64)
        c_ext.transfer_kv_blocks(torch.from_numpy(gids), ptrs, st["gpu_kv"], st["gpu_block"],
                                 torch.from_numpy(cids), pool, st["cpu_kv"], st["cpu_layer"],
                                 st["cpu_block"], st["gpu_chunk"], 0, -1, False, False, False)
        oracle_transfer(case, gpu, cpu, gids, cids, False)
        d2h_ok = bool(np.array_equal(pool.numpy(), cpu))
        # 2. H2D through the TransferEngine built on the imported tensors:
        #    new host data flows into the parent's cache.
        from flexkv_b200.layout import KVCacheLayout, KVCacheLayoutType
        gl = KVCacheLayout(KVCacheLayoutType.LAYERWISE, case.num_layers, case.gpu_blocks, case.tpb,
                           case.heads, case.head_dim, case.is_mla)
        cl = case.cpu_layout_obj()
        from kvcase import fill_bytes
        pool2 = torch.from_numpy(fill_bytes(st["cpu_pool_bytes"], new_cpu_seed)).pin_memory()
        typed = [t.view(torch.bfloat16).view(gl.kv_shape[1:]) for t in layers]
        eng = TransferEngine([typed], pool2.view(torch.bfloat16), gl, cl, 1, 1)
        g = TransferOpGraph()
        op = TransferOp(graph_id=g.graph_id, transfer_type=TransferType.H2D, layer_id=-1, layer_granularity=-1,
                        src_descriptor=TransferDescriptor(torch.from_numpy(cids)),
                        dst_descriptor=TransferDescriptor(torch.from_numpy(gids)))
        g.add_transfer_op(op)
        eng.submit_transfer_graph(g)
        done, failed = False, []
        import time
        t0 = time.time()
        while not done and time.time() - t0 < 60:
            for gid, oid in eng.get_completed_graphs_and_ops(timeout=0.05):
                done = done or (gid == g.graph_id and oid == -1)
        failed = list(eng.failed_ops)
        eng.shutdown()
        torch.cuda.synchronize()
        del typed, layers
        import gc
        gc.collect()
        q.put(("ok", {"opened": opened, "d2h_ok": d2h_ok, "h2d_done": done, "failed": failed,
                      "open_after_release": ipc_open_count()}))
    except Exception:  # reported to the parent, which fails the test
        q.put(("err", traceback.format_exc()))
