// Tensor-parallel transfer group: one persistent host thread and one CUDA
// stream per TP rank, replacing flexkv::TPTransferThreadGroup
// (csrc/tp_transfer_thread_group.cpp:23-109), which spawns and joins a new
// std::thread per rank on every call.
//
// Rank i moves its head slice: its GPU chunk (gpu_chunk bytes, its own
// KV-head range) lands at byte offset i*gpu_chunk inside each CPU chunk of
// the shared host pool (offset 0 for MLA, where every rank holds the whole
// latent vector) — tp_transfer_thread_group.cpp:79-80.  Rank i's layer
// pointers are row i of the rank-major [num_gpus][num_layers] table.
// Divergence: the reference indexes that table with a row length of
// layer_granularity (:70,77), which equals the intended num_layers only for
// full-layer ops; this group always uses num_layers.
#include <cuda_runtime.h>

#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "fkv_common.h"

struct fkv_tp_group {
  int num_gpus = 0;
  int dp_group_id = 0;
  int num_layers = 0;
  std::vector<int> devices;
  std::vector<void *> layer_ptrs;  // [num_gpus * num_layers]
  void *cpu_ptr = nullptr;
  int64_t cpu_pool_bytes = 0;

  std::vector<std::thread> threads;
  std::vector<cudaStream_t> streams;
  std::mutex call_mu;  // one transfer at a time: concurrent callers take turns
  std::mutex mu;
  std::condition_variable cv_job, cv_done;
  uint64_t job_seq = 0;
  int pending = 0;
  int ready = 0;
  bool stop = false;
  fkv_transfer_desc job{};            // rank-independent part of the job
  int64_t gpu_chunk = 0;
  int layer_id = 0;
  std::vector<int> rc;
  std::vector<std::string> msg;
};

namespace {

void rank_main(fkv_tp_group *g, int rank) {
  int init_rc = FKV_OK;
  std::string init_msg;
  cudaStream_t stream = nullptr;
  cudaError_t e = cudaSetDevice(g->devices[rank]);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    init_rc = FKV_ERR_CUDA;
    init_msg = std::string("rank ") + std::to_string(rank) + " init: " + cudaGetErrorString(e);
  }
  {
    std::lock_guard<std::mutex> lk(g->mu);
    g->streams[rank] = stream;
    g->rc[rank] = init_rc;
    g->msg[rank] = init_msg;
    g->ready++;
  }
  g->cv_done.notify_all();

  uint64_t seen = 0;
  for (;;) {
    fkv_transfer_desc d;
    {
      std::unique_lock<std::mutex> lk(g->mu);
      g->cv_job.wait(lk, [&] { return g->stop || g->job_seq != seen; });
      if (g->stop) break;
      seen = g->job_seq;
      d = g->job;
    }
    int rc = init_rc;
    std::string m = init_msg;
    if (rc == FKV_OK) {
      d.gpu_layer_ptrs = g->layer_ptrs.data() + (size_t)rank * g->num_layers + g->layer_id;
      d.cpu_startoff_inside_chunks = d.is_mla ? 0 : (int64_t)rank * g->gpu_chunk;
      d.chunk_size_in_bytes = g->gpu_chunk;
      d.synchronous = 1;
      rc = fkv_transfer_kv_blocks_ex(&d, stream);
      if (rc != FKV_OK) m = std::string("rank ") + std::to_string(rank) + ": " + fkv_last_error();
    }
    {
      std::lock_guard<std::mutex> lk(g->mu);
      g->rc[rank] = rc;
      g->msg[rank] = m;
      g->pending--;
    }
    g->cv_done.notify_all();
  }
  if (stream) cudaStreamDestroy(stream);
}

}  // namespace

extern "C" {

int fkv_tp_group_create(int num_gpus, int dp_group_id, const int *device_ids,
                        void *const *gpu_layer_ptrs, int num_layers, void *cpu_ptr,
                        int64_t cpu_pool_bytes, fkv_tp_group **out) {
  fkv::clear_error();
  if (!out) return fkv::fail(FKV_ERR_INVALID_ARG, "null output");
  *out = nullptr;
  if (num_gpus <= 0 || num_layers <= 0 || !gpu_layer_ptrs || !cpu_ptr)
    return fkv::fail(FKV_ERR_INVALID_ARG, "tp group needs num_gpus>0, num_layers>0, layer pointers and a cpu pool");
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess) return fkv::fail_cuda(e, "cudaGetDeviceCount");
  auto *g = new fkv_tp_group();
  g->num_gpus = num_gpus;
  g->dp_group_id = dp_group_id;
  g->num_layers = num_layers;
  g->cpu_ptr = cpu_ptr;
  g->cpu_pool_bytes = cpu_pool_bytes;
  g->layer_ptrs.assign(gpu_layer_ptrs, gpu_layer_ptrs + (size_t)num_gpus * num_layers);
  for (int i = 0; i < num_gpus; ++i) {
    int dev = device_ids ? device_ids[i] : dp_group_id * num_gpus + i;
    if (dev < 0 || dev >= ndev) {
      delete g;
      return fkv::fail(FKV_ERR_INVALID_ARG, "tp rank " + std::to_string(i) + " maps to missing device " + std::to_string(dev));
    }
    g->devices.push_back(dev);
  }
  g->streams.assign(num_gpus, nullptr);
  g->rc.assign(num_gpus, FKV_OK);
  g->msg.assign(num_gpus, "");
  for (int i = 0; i < num_gpus; ++i) g->threads.emplace_back(rank_main, g, i);
  {
    std::unique_lock<std::mutex> lk(g->mu);
    g->cv_done.wait(lk, [&] { return g->ready == num_gpus; });
  }
  for (int i = 0; i < num_gpus; ++i) {
    if (g->rc[i] != FKV_OK) {
      std::string m = g->msg[i];
      fkv_tp_group_destroy(g);
      return fkv::fail(FKV_ERR_CUDA, "tp group init failed: " + m);
    }
  }
  *out = g;
  return FKV_OK;
}

int fkv_tp_group_transfer(fkv_tp_group *g, const int64_t *gpu_block_ids,
                          const int64_t *cpu_block_ids, int num_blocks,
                          int64_t gpu_kv_stride_in_bytes, int64_t gpu_block_stride_in_bytes,
                          int64_t gpu_chunk_size_in_bytes, int64_t cpu_kv_stride_in_bytes,
                          int64_t cpu_layer_stride_in_bytes, int64_t cpu_block_stride_in_bytes,
                          int64_t cpu_chunk_size_in_bytes, int transfer_sms,
                          int is_host_to_device, int use_ce_transfer, int layer_id,
                          int layer_granularity, int is_mla) {
  fkv::clear_error();
  if (!g) return fkv::fail(FKV_ERR_INVALID_ARG, "null tp group");
  if (layer_id < 0 || layer_granularity < 0 || layer_id + layer_granularity > g->num_layers)
    return fkv::fail(FKV_ERR_INVALID_ARG, "layer range [layer_id, layer_id+layer_granularity) exceeds the group's layers");
  if (gpu_chunk_size_in_bytes < 0 || cpu_chunk_size_in_bytes < 0)
    return fkv::fail(FKV_ERR_INVALID_ARG, "negative chunk size");
  if (!is_mla && (int64_t)g->num_gpus * gpu_chunk_size_in_bytes > cpu_chunk_size_in_bytes)
    return fkv::fail(FKV_ERR_INVALID_ARG, "num_gpus * gpu_chunk exceeds cpu_chunk: rank slices would overflow the cpu chunk");
  if (num_blocks <= 0 || layer_granularity == 0) return FKV_OK;

  std::lock_guard<std::mutex> call(g->call_mu);
  fkv_transfer_desc d;
  fkv_transfer_desc_init(&d);
  d.num_blocks = num_blocks;
  d.start_layer_id = layer_id;  // CPU layer offset, as the reference passes it (:83)
  d.num_layers = layer_granularity;
  d.is_host_to_device = is_host_to_device;
  d.is_mla = is_mla;
  d.transfer_sms = transfer_sms;
  d.use_ce_transfer = use_ce_transfer;
  d.gpu_block_ids = gpu_block_ids;
  d.cpu_block_ids = cpu_block_ids;
  d.cpu_ptr = g->cpu_ptr;
  d.gpu_kv_stride_in_bytes = gpu_kv_stride_in_bytes;
  d.gpu_block_stride_in_bytes = gpu_block_stride_in_bytes;
  d.cpu_kv_stride_in_bytes = cpu_kv_stride_in_bytes;
  d.cpu_layer_stride_in_bytes = cpu_layer_stride_in_bytes;
  d.cpu_block_stride_in_bytes = cpu_block_stride_in_bytes;
  d.cpu_pool_bytes = g->cpu_pool_bytes;
  {
    std::unique_lock<std::mutex> lk(g->mu);
    g->job = d;
    g->gpu_chunk = gpu_chunk_size_in_bytes;
    g->layer_id = layer_id;
    g->pending = g->num_gpus;
    g->job_seq++;
  }
  g->cv_job.notify_all();
  std::string err;
  int err_code = FKV_OK;
  {
    std::unique_lock<std::mutex> lk(g->mu);
    g->cv_done.wait(lk, [&] { return g->pending == 0; });
    for (int i = 0; i < g->num_gpus; ++i)
      if (g->rc[i] != FKV_OK && err_code == FKV_OK) {
        err_code = g->rc[i];
        err = g->msg[i];
      }
  }
  if (err_code != FKV_OK) return fkv::fail(err_code, "tp_group_transfer failed: " + err);
  return FKV_OK;
}

int fkv_tp_group_num_gpus(const fkv_tp_group *g) { return g ? g->num_gpus : 0; }

void fkv_tp_group_destroy(fkv_tp_group *g) {
  if (!g) return;
  {
    std::lock_guard<std::mutex> lk(g->mu);
    g->stop = true;
  }
  g->cv_job.notify_all();
  for (auto &t : g->threads)
    if (t.joinable()) t.join();
  delete g;
}

}  // extern "C"
