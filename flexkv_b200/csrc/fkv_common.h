// Shared host-side plumbing of libflexkv_b200: error reporting, launch
// accounting and the per-thread, per-device resources (side streams, events,
// pinned staging) that the transfer and hash entry points reuse.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/flexkv_b200.h"

namespace fkv {

// Thread-local last error; set by fail() and returned through fkv_last_error.
void set_error(const std::string &msg);
void clear_error();
const char *last_error();

// Record a failure and return its code (for `return fail(...)` chains).
int fail(int code, const std::string &msg);
int fail_cuda(cudaError_t e, const char *what);

// Count of kernels launched by this library (all threads).
extern std::atomic<uint64_t> g_kernel_launches;
inline void note_launch(uint64_t n = 1) { g_kernel_launches.fetch_add(n, std::memory_order_relaxed); }

#define FKV_CUDA(call)                                     \
  do {                                                     \
    cudaError_t fkv_e_ = (call);                           \
    if (fkv_e_ != cudaSuccess) return ::fkv::fail_cuda(fkv_e_, #call); \
  } while (0)

// Resources owned by one host thread on one device.  Created lazily, never
// freed before process exit (CUDA teardown order at exit is unspecified).
struct ThreadDeviceCtx {
  int device = -1;
  int num_sms = 0;
  std::vector<cudaStream_t> side_streams;  // copy-engine streams
  std::vector<cudaEvent_t> join_events;    // one per side stream
  cudaEvent_t fork_event = nullptr;
  // Pinned staging for small uploads (plan tables, hash state): a ring of
  // slots used in turn, each freed by an event recorded after the upload
  // that read it, so up to kStagingSlots asynchronous calls (on any mix of
  // streams) are in flight before a call waits for an old upload.
  static constexpr int kStagingSlots = 8;
  struct StagingSlot {
    char *buf = nullptr;
    size_t cap = 0;
    cudaEvent_t free = nullptr;  // recorded after the upload that read this slot
    bool pending = false;
  };
  StagingSlot staging[kStagingSlots];
  int staging_next = 0;  // slot the next acquire takes
  int staging_cur = -1;  // slot handed out by the last acquire, until its release
};

// Context of the calling thread for `device` (current device if -1).
int get_ctx(int device, ThreadDeviceCtx **out);
// Stream-ordered scratch from a library-owned memory pool of `device` that
// keeps its memory cached (release threshold = max), so per-call
// allocations never remap physical memory after a synchronize.
int scratch_alloc(int device, size_t bytes, cudaStream_t s, void **out);
int scratch_free(void *p, cudaStream_t s);
// Host-phase timing to stderr when FKV_PROFILE=1 (diagnostics only).
bool profiling();
double now_us();
// Ensure `n` side streams exist in ctx.
int ensure_side_streams(ThreadDeviceCtx *ctx, int n);
// Pinned staging buffer of at least `bytes`, safe to overwrite now (the
// next slot of the thread's ring; waits only if that slot's last upload has
// not run yet).
int acquire_staging(ThreadDeviceCtx *ctx, size_t bytes, char **out);
// Mark that an async copy on `stream` reads the buffer the last
// acquire_staging returned.
int release_staging(ThreadDeviceCtx *ctx, cudaStream_t stream);

// Plan and enqueue one transfer on `s` without synchronizing (transfer.cu).
// An op whose SM part fits the kernel's parameters (up to 128 blocks and 96
// layers) carries its id table there.  Otherwise the table is staged in
// `ext_stage` (page-locked host memory of ext_cap bytes that the caller
// keeps untouched until `s` passes this point), or in the thread's own
// staging ring when ext_stage is null.
int transfer_enqueue(const fkv_transfer_desc &d, cudaStream_t s, char *ext_stage, size_t ext_cap);
// Upper bound of the staging bytes transfer_enqueue needs for `d`.
size_t transfer_stage_bytes(const fkv_transfer_desc &d);
// Enqueue the SM copy kernel over device-resident id lists (capacity n_max)
// whose length an earlier kernel on `s` writes to *n_dev.  `d` gives the
// layout and direction; its id arrays and num_blocks are not used.  The
// producer of the lists guarantees the GPU ids are in range; cpu ids are at
// most max_cpu_id, checked here against d.cpu_pool_bytes when that is set.
// layer_granularity > 0 splits the layers into groups of that many (it must
// divide them), copied one launch per group in order; group_events[g]
// (optional cudaEvent_t handles) is recorded after group g.
int transfer_enqueue_device_ids(const fkv_transfer_desc &d, const int64_t *gpu_ids_dev,
                                const int64_t *cpu_ids_dev, const int64_t *n_dev, int64_t n_max,
                                int64_t max_cpu_id, cudaStream_t s, int layer_granularity = 0,
                                void *const *group_events = nullptr);
// The checks transfer_enqueue_device_ids makes before it launches, alone:
// callers that change state before the copy run them first.
int transfer_check_device_ids(const fkv_transfer_desc &d, int64_t n_max, int64_t max_cpu_id);

// Classify a pointer: 1 = device memory (or managed), 0 = host.
int pointer_is_device(const void *p, int *is_device, int *device);
// Base and size of the device allocation that contains p (driver
// cuMemGetAddressRange, looked up through the runtime so the library needs
// no -lcuda).  False if p is not inside a device allocation.
bool alloc_range(const void *p, uint64_t *base, size_t *size);

}  // namespace fkv
