/*
 * TEST INFRASTRUCTURE ONLY — C entry point into the reference's own copy
 * kernel, linhu-nv/FlexKV csrc/transfer.cu (compiled unmodified from the
 * reference tree by oracle/Makefile into oracle/_ref/libref_transfer.so).
 * Used by the -m gpu parity tests as a second oracle and by
 * `bench.py --impl reference` as the reference arm.  As in the reference,
 * the id arrays and the layer-pointer table must be page-locked host
 * memory (the kernel reads them through zero-copy) and the call is
 * synchronous.
 */
#include <cuda_runtime.h>
#include <cstdint>

namespace flexkv {
void transfer_kv_blocks(int num_blocks, int start_layer_id, int num_layers, int64_t *gpu_block_ids,
                        void **gpu_layer_ptrs, int64_t gpu_kv_stride_in_bytes,
                        int64_t gpu_block_stride_in_bytes, int64_t *cpu_block_ids, void *cpu_ptr,
                        int64_t cpu_kv_stride_in_bytes, int64_t cpu_layer_stride_in_bytes,
                        int64_t cpu_block_stride_in_bytes, int64_t cpu_startoff_inside_chunks,
                        int64_t chunk_size_in_bytes, cudaStream_t stream, int transfer_sms,
                        bool is_host_to_device, bool use_ce_transfer, bool is_mla);
}

extern "C" int ref_transfer_kv_blocks(int num_blocks, int start_layer_id, int num_layers,
                                      int64_t *gpu_block_ids, void **gpu_layer_ptrs,
                                      int64_t gpu_kv_stride_in_bytes,
                                      int64_t gpu_block_stride_in_bytes, int64_t *cpu_block_ids,
                                      void *cpu_ptr, int64_t cpu_kv_stride_in_bytes,
                                      int64_t cpu_layer_stride_in_bytes,
                                      int64_t cpu_block_stride_in_bytes,
                                      int64_t cpu_startoff_inside_chunks,
                                      int64_t chunk_size_in_bytes, void *stream, int transfer_sms,
                                      int is_host_to_device, int use_ce_transfer, int is_mla) {
  flexkv::transfer_kv_blocks(num_blocks, start_layer_id, num_layers, gpu_block_ids, gpu_layer_ptrs,
                             gpu_kv_stride_in_bytes, gpu_block_stride_in_bytes, cpu_block_ids,
                             cpu_ptr, cpu_kv_stride_in_bytes, cpu_layer_stride_in_bytes,
                             cpu_block_stride_in_bytes, cpu_startoff_inside_chunks,
                             chunk_size_in_bytes, (cudaStream_t)stream, transfer_sms,
                             is_host_to_device != 0, use_ce_transfer != 0, is_mla != 0);
  return (int)cudaGetLastError();
}
