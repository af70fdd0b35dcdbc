// CUDA-IPC export and import of device memory ranges: the registration
// boundary between the inference engine's process, which owns the paged GPU
// KV cache, and the process that runs the transfers.  Replaces
// TensorSharedHandle (flexkv/common/memory_handle.py:17-56), which rides on
// torch.multiprocessing.reductions and so needs torch on both sides.
//
// A legacy CUDA IPC handle names a whole allocation, and a process may map
// an allocation only once; KV tensors are often views into one larger
// allocation (a caching-allocator segment, or one tensor sliced per layer).
// So a handle carries the allocation's identity plus the range's offset,
// and this process keeps one mapping per allocation with a reference count.
#include <unistd.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "fkv_common.h"

namespace fkv {
namespace {

struct Mapping {
  uint64_t base = 0;   // address in this process
  uint64_t bytes = 0;  // allocation size
  int refs = 0;
  int device = -1;
  bool local = false;  // exported by this process: nothing to unmap
  std::string key;
};

std::mutex g_mu;
std::map<std::string, uint64_t> g_by_key;  // handle identity -> base here
std::map<uint64_t, Mapping> g_by_base;     // base here -> mapping

std::string key_of(const fkv_ipc_handle &h) {
  std::string k(reinterpret_cast<const char *>(h.cuda_handle), sizeof(h.cuda_handle));
  k.append(reinterpret_cast<const char *>(&h.pid), sizeof(h.pid));
  k.append(reinterpret_cast<const char *>(&h.base_addr), sizeof(h.base_addr));
  return k;
}

struct DeviceSwitch {
  int prev = -1;
  bool switched = false;
  cudaError_t enter(int dev) {
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return e;
    if (prev != dev) {
      e = cudaSetDevice(dev);
      if (e != cudaSuccess) return e;
      switched = true;
    }
    return cudaSuccess;
  }
  ~DeviceSwitch() {
    if (switched) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace fkv

using namespace fkv;

extern "C" {

int fkv_ipc_export(const void *dev_ptr, int64_t bytes, fkv_ipc_handle *out) {
  clear_error();
  if (!out || !dev_ptr || bytes < 0) return fail(FKV_ERR_INVALID_ARG, "ipc export: null pointer or negative size");
  std::memset(out, 0, sizeof(*out));
  int is_dev = 0, dev = -1;
  pointer_is_device(dev_ptr, &is_dev, &dev);
  if (!is_dev || dev < 0) return fail(FKV_ERR_INVALID_ARG, "ipc export: pointer is not device memory");
  uint64_t base = 0;
  size_t size = 0;
  if (!alloc_range(dev_ptr, &base, &size))
    return fail(FKV_ERR_INVALID_ARG, "ipc export: pointer lies in no device allocation");
  const uint64_t p = (uint64_t)(uintptr_t)dev_ptr;
  if (p + (uint64_t)bytes > base + size) return fail(FKV_ERR_INVALID_ARG, "ipc export: range runs past its allocation");
  DeviceSwitch g;
  FKV_CUDA(g.enter(dev));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(FKV_ERR_CUDA, std::string("ipc export: cudaIpcGetMemHandle failed (") + cudaGetErrorString(e) +
                                  "); only cudaMalloc-style allocations can be exported, not virtual-memory "
                                  "ones such as torch expandable segments");
  }
  static_assert(sizeof(h) == sizeof(out->cuda_handle), "IPC handle size");
  std::memcpy(out->cuda_handle, &h, sizeof(h));
  out->base_addr = base;
  out->alloc_bytes = size;
  out->offset = (int64_t)(p - base);
  out->bytes = bytes;
  out->device = dev;
  out->pid = (int32_t)getpid();
  return FKV_OK;
}

int fkv_ipc_open(const fkv_ipc_handle *h, int device, void **out_ptr) {
  clear_error();
  if (!h || !out_ptr) return fail(FKV_ERR_INVALID_ARG, "ipc open: null handle or output");
  *out_ptr = nullptr;
  if (h->offset < 0 || h->bytes < 0 || (uint64_t)h->offset + (uint64_t)h->bytes > h->alloc_bytes)
    return fail(FKV_ERR_INVALID_ARG, "ipc open: range lies outside the exported allocation");
  const int dev = device < 0 ? h->device : device;
  const std::string key = key_of(*h);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_by_key.find(key);
  if (it != g_by_key.end()) {
    Mapping &m = g_by_base[it->second];
    ++m.refs;
    *out_ptr = reinterpret_cast<void *>(m.base + (uint64_t)h->offset);
    return FKV_OK;
  }
  Mapping m;
  m.bytes = h->alloc_bytes;
  m.device = dev;
  m.key = key;
  m.refs = 1;
  if (h->pid == (int32_t)getpid()) {
    // The exporter's own address is valid here (CUDA refuses to open a
    // process's own handle); the exporter keeps the memory alive.
    m.base = h->base_addr;
    m.local = true;
  } else {
    DeviceSwitch g;
    FKV_CUDA(g.enter(dev));
    cudaIpcMemHandle_t ch;
    std::memcpy(&ch, h->cuda_handle, sizeof(ch));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, ch, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(FKV_ERR_CUDA, std::string("ipc open: cudaIpcOpenMemHandle failed (") + cudaGetErrorString(e) + ")");
    }
    m.base = (uint64_t)(uintptr_t)p;
  }
  g_by_key[key] = m.base;
  *out_ptr = reinterpret_cast<void *>(m.base + (uint64_t)h->offset);
  g_by_base[m.base] = std::move(m);
  return FKV_OK;
}

int fkv_ipc_close(void *ptr) {
  clear_error();
  const uint64_t p = (uint64_t)(uintptr_t)ptr;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_by_base.upper_bound(p);
  if (it == g_by_base.begin()) return fail(FKV_ERR_INVALID_ARG, "ipc close: pointer lies in no opened range");
  --it;
  Mapping &m = it->second;
  if (p >= m.base + (m.bytes ? m.bytes : 1)) return fail(FKV_ERR_INVALID_ARG, "ipc close: pointer lies in no opened range");
  if (--m.refs > 0) return FKV_OK;
  int rc = FKV_OK;
  if (!m.local) {
    DeviceSwitch g;
    cudaError_t e = g.enter(m.device);
    if (e == cudaSuccess) e = cudaIpcCloseMemHandle(reinterpret_cast<void *>(m.base));
    if (e != cudaSuccess) rc = fail_cuda(e, "cudaIpcCloseMemHandle");
  }
  g_by_key.erase(m.key);
  g_by_base.erase(it);
  return rc;
}

int fkv_ipc_open_count(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  return (int)g_by_base.size();
}

}  // extern "C"
