// Host plumbing shared by every entry point of libflexkv_b200.
#include "fkv_common.h"

#include <sys/mman.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>

namespace fkv {

std::atomic<uint64_t> g_kernel_launches{0};

namespace {
thread_local std::string t_error;
thread_local std::map<int, std::unique_ptr<ThreadDeviceCtx>> t_ctx;
}  // namespace

void set_error(const std::string &msg) { t_error = msg; }
void clear_error() { t_error.clear(); }
const char *last_error() { return t_error.c_str(); }

int fail(int code, const std::string &msg) {
  set_error(msg);
  return code;
}

int fail_cuda(cudaError_t e, const char *what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                  cudaGetErrorString(e) + ")";
  set_error(m);
  return FKV_ERR_CUDA;
}

int get_ctx(int device, ThreadDeviceCtx **out) {
  if (device < 0) FKV_CUDA(cudaGetDevice(&device));
  auto it = t_ctx.find(device);
  if (it != t_ctx.end()) {
    *out = it->second.get();
    return FKV_OK;
  }
  auto ctx = std::make_unique<ThreadDeviceCtx>();
  ctx->device = device;
  FKV_CUDA(cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device));
  int prev = -1;
  FKV_CUDA(cudaGetDevice(&prev));
  if (prev != device) FKV_CUDA(cudaSetDevice(device));
  cudaError_t e = cudaEventCreateWithFlags(&ctx->fork_event, cudaEventDisableTiming);
  for (int i = 0; e == cudaSuccess && i < ThreadDeviceCtx::kStagingSlots; ++i)
    e = cudaEventCreateWithFlags(&ctx->staging[i].free, cudaEventDisableTiming);
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaEventCreateWithFlags");
  *out = ctx.get();
  t_ctx.emplace(device, std::move(ctx));
  return FKV_OK;
}

int ensure_side_streams(ThreadDeviceCtx *ctx, int n) {
  if ((int)ctx->side_streams.size() >= n) return FKV_OK;
  int prev = -1;
  FKV_CUDA(cudaGetDevice(&prev));
  if (prev != ctx->device) FKV_CUDA(cudaSetDevice(ctx->device));
  int rc = FKV_OK;
  while ((int)ctx->side_streams.size() < n) {
    cudaStream_t s;
    cudaEvent_t ev;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) { rc = fail_cuda(e, "cudaStreamCreateWithFlags"); break; }
    e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e != cudaSuccess) { rc = fail_cuda(e, "cudaEventCreateWithFlags"); break; }
    ctx->side_streams.push_back(s);
    ctx->join_events.push_back(ev);
  }
  if (prev != ctx->device) cudaSetDevice(prev);
  return rc;
}

int acquire_staging(ThreadDeviceCtx *ctx, size_t bytes, char **out) {
  const int i = ctx->staging_next;
  ThreadDeviceCtx::StagingSlot &sl = ctx->staging[i];
  if (sl.pending) {
    FKV_CUDA(cudaEventSynchronize(sl.free));
    sl.pending = false;
  }
  if (bytes > sl.cap) {
    if (sl.buf) FKV_CUDA(cudaFreeHost(sl.buf));
    sl.buf = nullptr;
    sl.cap = 0;
    size_t cap = 4096;
    while (cap < bytes) cap <<= 1;
    FKV_CUDA(cudaHostAlloc((void **)&sl.buf, cap, cudaHostAllocPortable));
    sl.cap = cap;
  }
  ctx->staging_cur = i;
  *out = sl.buf;
  return FKV_OK;
}

int release_staging(ThreadDeviceCtx *ctx, cudaStream_t stream) {
  const int i = ctx->staging_cur;
  if (i < 0) return fail(FKV_ERR_INVALID_ARG, "release_staging without acquire_staging");
  ThreadDeviceCtx::StagingSlot &sl = ctx->staging[i];
  FKV_CUDA(cudaEventRecord(sl.free, stream));
  sl.pending = true;
  ctx->staging_cur = -1;
  ctx->staging_next = (i + 1) % ThreadDeviceCtx::kStagingSlots;
  return FKV_OK;
}

namespace {
std::mutex g_pool_mu;
cudaMemPool_t g_pools[64] = {nullptr};
}  // namespace

int scratch_alloc(int device, size_t bytes, cudaStream_t s, void **out) {
  if (device < 0) FKV_CUDA(cudaGetDevice(&device));
  if (device >= 64)  // one pool per device ordinal below 64; never alias another device's pool
    return fail(FKV_ERR_INVALID_ARG, "device ordinal " + std::to_string(device) + " is outside [0, 64)");
  cudaMemPool_t pool;
  {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    pool = g_pools[device];
    if (!pool) {
      cudaMemPoolProps props;
      std::memset(&props, 0, sizeof(props));
      props.allocType = cudaMemAllocationTypePinned;
      props.handleTypes = cudaMemHandleTypeNone;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = device;
      FKV_CUDA(cudaMemPoolCreate(&pool, &props));
      uint64_t keep = UINT64_MAX;
      FKV_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
      g_pools[device] = pool;
    }
  }
  FKV_CUDA(cudaMallocFromPoolAsync(out, bytes < 256 ? 256 : bytes, pool, s));
  return FKV_OK;
}

int scratch_free(void *p, cudaStream_t s) {
  if (p) FKV_CUDA(cudaFreeAsync(p, s));
  return FKV_OK;
}

bool profiling() {
  static const bool on = [] {
    const char *e = std::getenv("FKV_PROFILE");
    return e && *e == '1';
  }();
  return on;
}

double now_us() {
  return std::chrono::duration<double, std::micro>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

int pointer_is_device(const void *p, int *is_device, int *device) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();  // unregistered host pointer on old runtimes
    *is_device = 0;
    *device = -1;
    return FKV_OK;
  }
  *is_device = (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged);
  *device = attr.device;
  return FKV_OK;
}

bool alloc_range(const void *p, uint64_t *base, size_t *size) {
  using GetRange = int (*)(unsigned long long *, size_t *, unsigned long long);
  static GetRange fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return (GetRange) nullptr;
    }
    return reinterpret_cast<GetRange>(f);
  }();
  if (!fn) return false;
  unsigned long long b = 0;
  size_t n = 0;
  if (fn(&b, &n, (unsigned long long)(uintptr_t)p) != 0) return false;
  *base = b;
  *size = n;
  return true;
}

}  // namespace fkv

extern "C" {

const char *fkv_last_error(void) { return fkv::last_error(); }

const char *fkv_version(void) { return "flexkv_b200 0.1.0 (sm_100a)"; }

uint64_t fkv_kernel_launch_count(void) {
  return fkv::g_kernel_launches.load(std::memory_order_relaxed);
}

int fkv_host_register(void *ptr, int64_t bytes, int advise_hugepages) {
  fkv::clear_error();
  if (ptr == nullptr || bytes <= 0)
    return fkv::fail(FKV_ERR_INVALID_ARG, "fkv_host_register: null pointer or non-positive size");
  if (advise_hugepages) {
    // Best effort: only helps for pages not yet touched.
    uintptr_t a = (uintptr_t)ptr, page = 4096;
    uintptr_t lo = (a + page - 1) & ~(page - 1);
    uintptr_t hi = (a + (uintptr_t)bytes) & ~(page - 1);
    if (hi > lo) madvise((void *)lo, hi - lo, MADV_HUGEPAGE);
  }
  cudaError_t e = cudaHostRegister(ptr, (size_t)bytes,
                                   cudaHostRegisterPortable | cudaHostRegisterMapped);
  if (e != cudaSuccess) return fkv::fail_cuda(e, "cudaHostRegister");
  return FKV_OK;
}

int fkv_host_unregister(void *ptr) {
  fkv::clear_error();
  cudaError_t e = cudaHostUnregister(ptr);
  if (e != cudaSuccess) return fkv::fail_cuda(e, "cudaHostUnregister");
  return FKV_OK;
}

}  // extern "C"
