/*
 * TEST INFRASTRUCTURE ONLY — C entry points into the reference's own SSD
 * tier, linhu-nv/FlexKV csrc/transfer_ssd.cpp and transfer_ssd.h (compiled
 * unmodified from the reference tree by oracle/Makefile into
 * oracle/_ref/libref_ssd.so, with ref_stub_ssd/ standing in for libtorch
 * and liburing).  The CPU tests compare flexkv_b200's SSD tier with it byte
 * for byte.  Contexts are opened with iouring_entries = 0: the reference's
 * thread-pool path (one thread per (device, slice) per call, one
 * pread/pwrite per chunk, transfer_ssd.cpp:119-176, 214-275).
 */
#include <fcntl.h>
#include <unistd.h>

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "transfer_ssd.h"  // uses open/close/posix_fadvise: included after the POSIX headers, as transfer_ssd.cpp does

extern "C" {

/* paths[d * files_per_device + f] = file f of SSD device d.  0 or -1. */
int ref_ssd_ctx_create(const char *const *paths, int num_devices, int files_per_device, void **out) {
  try {
    std::map<int, std::vector<std::string>> files;
    for (int d = 0; d < num_devices; ++d)
      for (int f = 0; f < files_per_device; ++f) files[d].push_back(paths[d * files_per_device + f]);
    *out = new flexkv::SSDIOCTX(files, num_devices, 0, 0);
    return 0;
  } catch (...) {
    return -1;
  }
}

void ref_ssd_ctx_destroy(void *ctx) { delete static_cast<flexkv::SSDIOCTX *>(ctx); }

/* flexkv::transfer_kv_blocks_ssd over layers [start_layer, start_layer +
 * num_layers).  0, or -1 when the reference threw. */
int ref_ssd_transfer(void *ctx, int start_layer, int num_layers, void *cpu_ptr, const int64_t *ssd_block_ids,
                     const int64_t *cpu_block_ids, int64_t num_blocks, int64_t cpu_layer_stride,
                     int64_t cpu_kv_stride, int64_t ssd_layer_stride, int64_t ssd_kv_stride, int64_t chunk,
                     int64_t block_stride, int is_read, int num_blocks_per_file, int round_robin,
                     int threads_per_device, int is_mla) {
  try {
    std::vector<int32_t> layers(num_layers > 0 ? num_layers : 1);
    for (int l = 0; l < num_layers; ++l) layers[l] = start_layer + l;
    torch::Tensor layer_ids(layers.data(), num_layers);
    torch::Tensor ssd_ids(const_cast<int64_t *>(ssd_block_ids), num_blocks);
    torch::Tensor cpu_ids(const_cast<int64_t *>(cpu_block_ids), num_blocks);
    flexkv::transfer_kv_blocks_ssd(*static_cast<flexkv::SSDIOCTX *>(ctx), layer_ids,
                                   reinterpret_cast<int64_t>(cpu_ptr), ssd_ids, cpu_ids, cpu_layer_stride,
                                   cpu_kv_stride, ssd_layer_stride, ssd_kv_stride, chunk, block_stride,
                                   is_read != 0, num_blocks_per_file, round_robin, threads_per_device,
                                   is_mla != 0);
    return 0;
  } catch (...) {
    return -1;
  }
}

}  // extern "C"
