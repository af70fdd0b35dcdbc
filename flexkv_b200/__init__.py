"""flexkv_b200 — B200-native (sm_100a) FlexKV transfer data plane.

``flexkv_b200.c_ext`` mirrors FlexKV's native module ``flexkv.c_ext`` for the
KV-block gather/scatter, the tensor-parallel group, the XXH64 block hashes
and the SSD tier; ``flexkv_b200.engine.TransferEngine`` mirrors FlexKV's
TransferEngine (GPU, CPU and SSD ops with dependencies);
``flexkv_b200.cache_index.CpuCacheIndex`` runs the CPU tier's put path
(block index, block pool, fused put) on the device;
``flexkv_b200.memory_handle.TensorSharedHandle`` shares the inference
engine's GPU KV tensors across processes.  Everything runs in
libflexkv_b200.so (C ABI: include/flexkv_b200.h).
"""
__version__ = "0.1.0"


def lib_path() -> str:
    """Path of the loaded libflexkv_b200.so (loads it; raises if missing)."""
    from . import _lib
    return _lib.lib_path()
