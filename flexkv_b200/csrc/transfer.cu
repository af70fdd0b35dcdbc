// KV-block gather/scatter between a paged GPU KV cache and a page-locked
// host pool — the B200 data plane that replaces flexkv::transfer_kv_blocks
// (csrc/transfer.cu:26-132 of linhu-nv/FlexKV).
//
// Work split (decided on the host, per call):
//   * runs of blocks whose GPU and CPU ids both advance by one are
//     coalesced; a run whose per-(layer,kv) span reaches ce_min_run_bytes
//     becomes one (1-D or 2-D) cudaMemcpyAsync on a side stream, so the copy
//     engines move it with large PCIe requests;
//   * every other chunk goes to kv_copy_kernel: a persistent grid sized by
//     the SM budget, one warp per (layer, kv, block) chunk, 16-byte
//     vector loads/stores with UNROLL loads in flight per lane, reading or
//     writing the host pool through its mapped (zero-copy) address.
//   The caller's stream forks to the side streams and joins back, so the
//   whole transfer is ordered on the caller's stream like the reference.
//
// Address arithmetic is the reference's (transfer.cu:39-50, 84-93): byte
// strides truncated to int64 units, start_layer_id offsets the CPU side
// only, and the copied size is 16*floor(chunk/16).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "fkv_common.h"

namespace fkv {
namespace {

constexpr int kThreads = 256;          // 8 warps per CTA
// Defaults from interleaved A/B runs on one B200 (Llama-3-8B shape,
// 2048-block batches with half the blocks in joint runs; DeepSeek-V3 MLA
// batches; Qwen2-7B-shaped scattered 16 KiB chunks; each direction alone and
// both in flight together):
//  * SM budget (transfer_sms == -1): 8 SMs for a synchronous call, 16 for an
//    asynchronous one or a plan.  Two SMs already fill the link on their
//    own.  While copy-engine runs share the link, fewer SMs leave it more of
//    the copy engines' larger requests: alone, H2D moves 51.3 GB/s with 8
//    against 50.6 with 16.  With the other direction in flight 16 SMs are
//    faster (73.5-74.5 against 71.9-72.9 GB/s for both directions).  A
//    synchronous call is the only transfer its thread has in flight (the
//    pattern of FlexKV's worker); asynchronous calls and plans usually share
//    the link with the other direction.
//  * Copy-engine threshold per (layer,kv) row of a run: 1 MiB; 256 KiB for
//    H2D when the caller asks for 4 SMs or fewer (the only budget where the
//    smaller runs pay off); 512 KiB, 2 MiB and serial schedules are slower.
//  * 16 loads in flight per lane (UNROLL): one pass moves 8 KiB per warp, a
//    16 KiB chunk takes two passes instead of four (scattered 16 KiB chunks,
//    both directions in flight: +4 %; 32 KiB chunks: within noise).
constexpr int kDefaultSmsSync = 8;
constexpr int kDefaultSmsAsync = 16;
constexpr int kDefaultSms = kDefaultSmsSync;  // device-side id lists (synchronous put/get paths)
constexpr int kFewSms = 4;
constexpr int kDefaultUnroll = 16;
constexpr int64_t kDefaultCeMinRunBytes = 1ll << 20;
constexpr int64_t kDefaultCeMinRunBytesFewSms = 256ll << 10;
constexpr int64_t kDefaultCeMinRunBytesFolded = 128ll << 10;
constexpr int kDefaultCeStreams = 2;
constexpr int kMaxCeStreams = 8;
constexpr int kDefaultCeSchedule = 0;  // copy engines concurrent with the SM kernel

struct CopyParams {
  const int64_t *gpu_ids;     // device [n]
  const int64_t *cpu_ids;     // device [n]
  char *const *layer_ptrs;    // device [num_layers]
  char *cpu_base;             // device-visible host address of layer start_layer_id, + startoff
  int64_t gpu_kv_stride;
  int64_t gpu_block_stride;
  int64_t cpu_layer_stride;
  int64_t cpu_kv_stride;
  int64_t cpu_block_stride;
  int64_t n_vec;              // 16-byte vectors per chunk
  uint32_t n;                 // blocks
  uint32_t per_layer;         // kv_dim * n
  uint32_t num_chunks;        // num_layers * kv_dim * n
};

// Coherent (not .nc) load on purpose: with .nc the assembler may legally
// sink each store between the loads (the data is declared read-only), which
// leaves one load per lane in flight instead of UNROLL — fatal for reads
// that cross PCIe with microsecond latency.  PF256 adds the L2 256-byte
// prefetch-size hint (a tuning variant for reads of host memory).
template <bool PF256>
__device__ __forceinline__ uint4 ld_stream(const uint4 *p) {
  uint4 r;
  if (PF256) {
    asm volatile("ld.global.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
  } else {
    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
  }
  return r;
}

__device__ __forceinline__ void st_stream(uint4 *p, const uint4 &v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// One warp copies one chunk: lane l moves vectors l, l+32, ...; each pass
// keeps UNROLL 16-byte loads in flight per lane (UNROLL*512 bytes per warp).
template <int UNROLL, bool PF256>
__device__ __forceinline__ void copy_chunk(const uint4 *__restrict__ src,
                                           uint4 *__restrict__ dst,
                                           int64_t n_vec, int lane) {
  constexpr int64_t kStep = 32 * UNROLL;
  int64_t base = 0;
  for (; base + kStep <= n_vec; base += kStep) {
    uint4 r[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) r[u] = ld_stream<PF256>(src + base + u * 32 + lane);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) st_stream(dst + base + u * 32 + lane, r[u]);
  }
  // Remainder: fewer than 32*UNROLL vectors.
  for (int64_t v = base + lane; v < n_vec; v += 32) st_stream(dst + v, ld_stream<PF256>(src + v));
}

// Table entries of chunk c: its block ids and its layer's GPU pointer.
struct ChunkRef {
  int64_t g, h;
  char *layer;
};

__device__ __forceinline__ ChunkRef chunk_ref(const CopyParams &p, uint32_t c) {
  const uint32_t layer = c / p.per_layer;
  const uint32_t rem = c - layer * p.per_layer;
  const uint32_t i = rem - (rem / p.n) * p.n;
  return {p.gpu_ids[i], p.cpu_ids[i], p.layer_ptrs[layer]};
}

// Each warp walks its chunks with the next chunk's table entries loaded
// before the current chunk's copy starts: the copy's loads and stores are
// volatile asm (compiler barriers), so without this order every chunk
// would begin with a dependent round trip to the id and pointer tables.
template <bool H2D, int UNROLL, bool PF256>
__device__ __forceinline__ void copy_body(const CopyParams &p) {
  const int lane = threadIdx.x & 31;
  const uint32_t warp = (blockIdx.x * kThreads + threadIdx.x) >> 5;
  const uint32_t nwarps = (gridDim.x * kThreads) >> 5;
  uint32_t c = warp;
  if (c >= p.num_chunks) return;
  ChunkRef cur = chunk_ref(p, c);
  for (; c < p.num_chunks; c += nwarps) {
    const uint32_t nxt_c = c + nwarps;
    const ChunkRef nxt = nxt_c < p.num_chunks ? chunk_ref(p, nxt_c) : cur;
    const uint32_t layer = c / p.per_layer;
    const uint32_t kv = (c - layer * p.per_layer) / p.n;
    char *gpu = cur.layer + kv * p.gpu_kv_stride + cur.g * p.gpu_block_stride;
    char *cpu = p.cpu_base + layer * p.cpu_layer_stride + kv * p.cpu_kv_stride +
                cur.h * p.cpu_block_stride;
    const uint4 *src = reinterpret_cast<const uint4 *>(H2D ? cpu : gpu);
    uint4 *dst = reinterpret_cast<uint4 *>(H2D ? gpu : cpu);
    copy_chunk<UNROLL, PF256>(src, dst, p.n_vec, lane);
    cur = nxt;
  }
}

template <bool H2D, int UNROLL, bool PF256>
__global__ void __launch_bounds__(kThreads) kv_copy_kernel(const CopyParams p) {
  copy_body<H2D, UNROLL, PF256>(p);
}

// The same copy over id lists whose length a preceding kernel on the stream
// wrote to *n_dev (clamped to n_max, the capacity of the lists): the fused
// put path decides on the device which blocks move.
template <bool H2D>
__global__ void __launch_bounds__(kThreads) kv_copy_devn_kernel(CopyParams p, const int64_t *n_dev,
                                                                uint32_t kv_dim, uint32_t num_layers,
                                                                uint32_t n_max) {
  const int64_t nd = *n_dev;
  const uint32_t n = nd <= 0 ? 0u : (nd >= (int64_t)n_max ? n_max : (uint32_t)nd);
  if (n == 0) return;
  p.n = n;
  p.per_layer = kv_dim * n;
  p.num_chunks = num_layers * p.per_layer;
  copy_body<H2D, kDefaultUnroll, false>(p);
}

// Small ops carry their id table inside the kernel's parameters instead of a
// device buffer: no scratch allocation and no table upload before the
// kernel can start (a per-call cost of a few to ten microseconds that
// matters for ops of a few blocks).  The parameters are __grid_constant__,
// so the copy reads the arrays in place through their generic addresses.
// Capacity: kInlineMaxBlocks blocks on the SM path and kInlineMaxLayers
// layers; the whole struct stays under the classic 4 KiB parameter limit.
constexpr int kInlineMaxBlocks = 128;
constexpr int kInlineMaxLayers = 96;

struct InlineCopyParams {
  CopyParams p;  // its table pointers are replaced by the arrays below
  int64_t layer_ptrs[kInlineMaxLayers];
  int64_t gpu_ids[kInlineMaxBlocks];
  int64_t cpu_ids[kInlineMaxBlocks];
};
static_assert(sizeof(InlineCopyParams) <= 4000, "inline copy parameters must fit the 4 KiB limit");

template <bool H2D>
__global__ void __launch_bounds__(kThreads) kv_copy_inline_kernel(const __grid_constant__ InlineCopyParams q) {
  CopyParams p = q.p;
  p.layer_ptrs = reinterpret_cast<char *const *>(q.layer_ptrs);
  p.gpu_ids = q.gpu_ids;
  p.cpu_ids = q.cpu_ids;
  copy_body<H2D, kDefaultUnroll, false>(p);
}

struct CeCopy {
  char *dst;
  const char *src;
  size_t width, height, dpitch, spitch;  // height==1 -> 1-D copy
};

int env_int(const char *name, int dflt) {
  const char *s = std::getenv(name);
  return (s && *s) ? std::atoi(s) : dflt;
}
int64_t env_i64(const char *name, int64_t dflt) {
  const char *s = std::getenv(name);
  return (s && *s) ? std::atoll(s) : dflt;
}

// Kernel variants: index = unroll_idx (0:4, 1:8, 2:16) + 3 * pf256.
constexpr int kNumVariants = 6;

template <bool H2D>
const void *kernel_ptr(int variant) {
  switch (variant) {
    case 0: return (const void *)kv_copy_kernel<H2D, 4, false>;
    case 1: return (const void *)kv_copy_kernel<H2D, 8, false>;
    case 2: return (const void *)kv_copy_kernel<H2D, 16, false>;
    case 3: return (const void *)kv_copy_kernel<H2D, 4, true>;
    case 4: return (const void *)kv_copy_kernel<H2D, 8, true>;
    default: return (const void *)kv_copy_kernel<H2D, 16, true>;
  }
}

int variant_index(int unroll, int pf256) {
  const int u = unroll >= 16 ? 2 : (unroll >= 8 ? 1 : 0);
  return u + (pf256 ? 3 : 0);
}

// Per-device caches below hold this many devices; a larger ordinal is
// refused rather than aliased onto another device's entry.
constexpr int kMaxDevices = 64;

int check_device(int device) {
  if (device < 0 || device >= kMaxDevices)
    return fail(FKV_ERR_INVALID_ARG, "device ordinal " + std::to_string(device) + " is outside [0, 64)");
  return FKV_OK;
}

// Occupancy (CTAs per SM) of each kernel variant, cached per device.
struct OccCache {
  std::mutex mu;
  int max_pitch[kMaxDevices] = {0};
  int occ[kMaxDevices][2][kNumVariants] = {{{0}}};
};
OccCache g_occ;

int ctas_per_sm(int device, bool h2d, int variant, int *out) {
  if (int rc = check_device(device)) return rc;
  std::lock_guard<std::mutex> lk(g_occ.mu);
  const int d = device;
  int &v = g_occ.occ[d][h2d ? 1 : 0][variant];
  if (v == 0) {
    const void *k = h2d ? kernel_ptr<true>(variant) : kernel_ptr<false>(variant);
    int n = 0;
    FKV_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kThreads, 0));
    v = std::max(n, 1);
  }
  *out = v;
  return FKV_OK;
}

int max_pitch(int device, int *out) {
  if (int rc = check_device(device)) return rc;
  std::lock_guard<std::mutex> lk(g_occ.mu);
  const int d = device;
  if (g_occ.max_pitch[d] == 0) {
    int mp = 0;
    FKV_CUDA(cudaDeviceGetAttribute(&mp, cudaDevAttrMaxPitch, device));
    g_occ.max_pitch[d] = mp > 0 ? mp : 1;
  }
  *out = g_occ.max_pitch[d];
  return FKV_OK;
}

// Whether a and b lie in one device allocation.  A 2-D copy may not span
// allocations even when they happen to be adjacent in the address space.
bool same_allocation(const void *a, const void *b) {
  uint64_t base_a = 0, base_b = 0;
  size_t size_a = 0, size_b = 0;
  if (!alloc_range(a, &base_a, &size_a) || !alloc_range(b, &base_b, &size_b)) return false;
  return base_a == base_b;
}

}  // namespace
}  // namespace fkv

struct fkv_plan {
  int device = -1;
  bool h2d = true;
  int grid = 0;
  int unroll_idx = 1;
  fkv::CopyParams params{};
  char *dev_buf = nullptr;       // layer ptrs + ids (cudaMalloc, plan-owned)
  std::vector<fkv::CeCopy> ce;
  int num_ce_streams = 0;
  int ce_schedule = 0;
  int64_t sm_chunks = 0, ce_bytes = 0, sm_bytes = 0;
};

namespace fkv {
namespace {

// Everything the host learns from the descriptor before any device work.
struct HostPlan {
  bool h2d = true;
  int kv_dim = 2;
  int num_layers = 0;
  int64_t copy_bytes = 0;
  int64_t gkv = 0, gbs = 0, cls = 0, ckv = 0, cbs = 0;
  int64_t base_off = 0;          // start_layer*cls + startoff
  char *cpu_dev_base = nullptr;  // device view of cpu_ptr + base_off
  const char *cpu_host_base = nullptr;
  std::vector<int64_t> sm_gpu, sm_cpu;  // blocks for the SM kernel
  std::vector<CeCopy> ce;
  int64_t ce_bytes = 0;
  int grid = 0;
  int unroll_idx = 1;
  int num_ce_streams = 0;
  int ce_schedule = 0;
  bool layer_folded = false;
};

inline int64_t trunc8(int64_t b) { return (b / 8) * 8; }  // transfer.cu:86-93

// Argument checks that need no CUDA call.
int validate_desc(const fkv_transfer_desc &d) {
  if (d.num_blocks < 0 || d.num_layers < 0)
    return fail(FKV_ERR_INVALID_ARG, "num_blocks and num_layers must be non-negative");
  if (d.chunk_size_in_bytes < 0)
    return fail(FKV_ERR_INVALID_ARG, "chunk_size_in_bytes must be non-negative");
  if (d.gpu_kv_stride_in_bytes < 0 || d.gpu_block_stride_in_bytes < 0 ||
      d.cpu_kv_stride_in_bytes < 0 || d.cpu_layer_stride_in_bytes < 0 ||
      d.cpu_block_stride_in_bytes < 0 || d.cpu_startoff_inside_chunks < 0 ||
      d.start_layer_id < 0)
    return fail(FKV_ERR_INVALID_ARG, "strides, start offset and start_layer_id must be non-negative");
  return FKV_OK;
}

// Checks of the layout every copy path shares: int64-unit strides, the
// page-locked host pool and its device view, 16-byte alignment of every
// chunk base and GPU layer pointer.  n = blocks the op may move.  Fills the
// stride and base fields of hp.
int layout_checks(const fkv_transfer_desc &d, int64_t n, HostPlan &hp) {
  hp.gkv = trunc8(d.gpu_kv_stride_in_bytes);
  hp.gbs = trunc8(d.gpu_block_stride_in_bytes);
  hp.cls = trunc8(d.cpu_layer_stride_in_bytes);
  hp.ckv = trunc8(d.cpu_kv_stride_in_bytes);
  hp.cbs = trunc8(d.cpu_block_stride_in_bytes);
  const int64_t startoff = trunc8(d.cpu_startoff_inside_chunks);
  const int64_t L = d.num_layers, KV = hp.kv_dim;
  if ((uint64_t)L * KV * n >= (1ull << 31))
    return fail(FKV_ERR_INVALID_ARG, "num_layers*kv_dim*num_blocks must stay below 2^31; split the op");

  // The host pool must be page-locked so the device can address it.
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, d.cpu_ptr);
  if (e != cudaSuccess || attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr) {
    cudaGetLastError();
    return fail(FKV_ERR_INVALID_ARG,
                "cpu_ptr is not page-locked host memory (allocate it pinned or cudaHostRegister it)");
  }
  const int64_t base_off = (int64_t)d.start_layer_id * hp.cls + startoff;
  hp.cpu_host_base = (const char *)d.cpu_ptr + base_off;
  hp.cpu_dev_base = (char *)attr.devicePointer + base_off;

  // Alignment of every chunk start (the vector path needs 16 bytes).
  if (((uintptr_t)hp.cpu_dev_base & 15) || ((uintptr_t)hp.cpu_host_base & 15))
    return fail(FKV_ERR_MISALIGNED, "cpu chunk base (cpu_ptr + start_layer*layer_stride + startoff) is not 16-byte aligned");
  if (L > 1 && (hp.cls & 15))
    return fail(FKV_ERR_MISALIGNED, "cpu_layer_stride_in_bytes is not a multiple of 16");
  if (KV > 1 && ((hp.ckv & 15) || (hp.gkv & 15)))
    return fail(FKV_ERR_MISALIGNED, "kv strides are not multiples of 16");
  for (int64_t l = 0; l < L; ++l) {
    if (d.gpu_layer_ptrs[l] == nullptr)
      return fail(FKV_ERR_INVALID_ARG, "null gpu layer pointer at index " + std::to_string(l));
    if ((uintptr_t)d.gpu_layer_ptrs[l] & 15)
      return fail(FKV_ERR_MISALIGNED, "gpu layer pointer " + std::to_string(l) + " is not 16-byte aligned");
  }
  hp.base_off = base_off;
  return FKV_OK;
}

int build_host_plan(const fkv_transfer_desc &d, int device, HostPlan &hp) {
  if (int rc = validate_desc(d)) return rc;
  hp.h2d = d.is_host_to_device != 0;
  hp.kv_dim = d.is_mla ? 1 : 2;
  hp.num_layers = d.num_layers;
  hp.copy_bytes = (d.chunk_size_in_bytes / 16) * 16;  // transfer.cu:35 floor to float4
  if (d.num_blocks == 0 || d.num_layers == 0 || hp.copy_bytes == 0) return FKV_OK;
  if (!d.gpu_block_ids || !d.cpu_block_ids || !d.gpu_layer_ptrs || !d.cpu_ptr)
    return fail(FKV_ERR_INVALID_ARG, "null id array, layer pointer table or cpu pointer");
  const int64_t L = d.num_layers, KV = hp.kv_dim, n = d.num_blocks;
  if (int rc = layout_checks(d, n, hp)) return rc;
  const int64_t base_off = hp.base_off;

  // Per-id checks: range, alignment, pool bounds (reference truncates ids
  // to int, transfer.cu:41-42, so ids must fit in [0, 2^31)).
  const int64_t cpu_extent_fixed = base_off + (L - 1) * hp.cls + (KV - 1) * hp.ckv + hp.copy_bytes;
  const int64_t gpu_extent_fixed = (KV - 1) * hp.gkv + hp.copy_bytes;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t g = d.gpu_block_ids[i], c = d.cpu_block_ids[i];
    if (g < 0 || c < 0 || g >= (1ll << 31) || c >= (1ll << 31))
      return fail(FKV_ERR_OUT_OF_RANGE, "block id out of [0, 2^31) at index " + std::to_string(i));
    if (((g * hp.gbs) & 15) || ((c * hp.cbs) & 15))
      return fail(FKV_ERR_MISALIGNED, "block stride times id is not 16-byte aligned at index " + std::to_string(i));
    if (d.cpu_pool_bytes > 0 && c * hp.cbs + cpu_extent_fixed > d.cpu_pool_bytes)
      return fail(FKV_ERR_OUT_OF_RANGE, "cpu block id " + std::to_string(c) + " at index " +
                                            std::to_string(i) + " addresses past the cpu pool");
    if (d.gpu_layer_bytes > 0 && g * hp.gbs + gpu_extent_fixed > d.gpu_layer_bytes)
      return fail(FKV_ERR_OUT_OF_RANGE, "gpu block id " + std::to_string(g) + " at index " +
                                            std::to_string(i) + " addresses past the gpu layer");
  }

  // Split into copy-engine runs and SM chunks.
  const bool ce_all = d.use_ce_transfer != 0;
  const int64_t thr_user = d.ce_min_run_bytes >= 0 ? d.ce_min_run_bytes : env_i64("FKV_CE_MIN_RUN_BYTES", -1);
  // The SM budget asked for (-1: the default, decided after the split).
  // Order: the caller's transfer_sms, FKV_TRANSFER_SMS_H2D / _D2H, FKV_TRANSFER_SMS, the default.
  const int sms_dir = env_int(hp.h2d ? "FKV_TRANSFER_SMS_H2D" : "FKV_TRANSFER_SMS_D2H", -1);
  const int sms_req = d.transfer_sms > 0 ? d.transfer_sms
                                         : (sms_dir > 0 ? sms_dir : env_int("FKV_TRANSFER_SMS", -1));
  // The lower H2D threshold pays only while few SMs share the link with the
  // copy engines (at the default 8 SMs the 1 MiB threshold is faster).
  const int64_t thr = (hp.h2d && sms_req > 0 && sms_req <= kFewSms) ? kDefaultCeMinRunBytesFewSms
                                                                    : kDefaultCeMinRunBytes;
  const int64_t thr_folded = kDefaultCeMinRunBytesFolded;
  int mp = 0;
  if (int rc = max_pitch(device, &mp)) return rc;
  const size_t cb = (size_t)hp.copy_bytes;
  const bool contig = (hp.gbs == hp.copy_bytes && hp.cbs == hp.copy_bytes);
  auto pitch_ok = [&](int64_t p) { return p >= hp.copy_bytes && p <= mp; };
  // Layer folding.  When the GPU layer tensors sit at one uniform stride
  // equal to kv_dim * gpu_kv_stride (one allocation viewed per layer) and the
  // CPU layer stride equals kv_dim * cpu_kv_stride (true of both host
  // layouts), the (layer, kv) chunks of a block are L*kv_dim rows of one
  // pitch on each side, so a single 2-D copy moves a block -- or a run of
  // blocks contiguous on both sides -- through every layer at once.
  bool fold = false;
  int64_t fold_gp = 0, fold_cp = 0;
  const int64_t rows = L * KV;
  if (L > 1) {
    const char *p0 = (const char *)d.gpu_layer_ptrs[0];
    const int64_t sg = (int64_t)((const char *)d.gpu_layer_ptrs[1] - p0);
    bool uniform = sg > 0;
    for (int64_t l = 2; uniform && l < L; ++l)
      uniform = ((const char *)d.gpu_layer_ptrs[l] - p0) == l * sg;
    // The whole folded extent must sit in one allocation.
    if (uniform) uniform = same_allocation(d.gpu_layer_ptrs[0], (const char *)d.gpu_layer_ptrs[L - 1] + (KV - 1) * hp.gkv);
    if (uniform) {
      fold_gp = KV > 1 ? hp.gkv : sg;
      fold_cp = KV > 1 ? hp.ckv : hp.cls;
      fold = (KV == 1 || (sg == KV * hp.gkv && hp.cls == KV * hp.ckv)) && pitch_ok(fold_gp) &&
             pitch_ok(fold_cp);
    }
  }
  hp.layer_folded = fold;
  auto emit = [&](char *g, char *c, size_t w, size_t h, size_t gp, size_t cp) {
    CeCopy x;
    x.width = w;
    x.height = h;
    if (hp.h2d) { x.dst = g; x.src = c; x.dpitch = gp; x.spitch = cp; }
    else        { x.dst = c; x.src = g; x.dpitch = cp; x.spitch = gp; }
    hp.ce.push_back(x);
    hp.ce_bytes += (int64_t)(w * h);
  };
  hp.sm_gpu.reserve(n);
  hp.sm_cpu.reserve(n);
  int64_t i = 0;
  while (i < n) {
    int64_t r = 1;
    const int64_t g0 = d.gpu_block_ids[i], c0 = d.cpu_block_ids[i];
    while (i + r < n && d.gpu_block_ids[i + r] == g0 + r && d.cpu_block_ids[i + r] == c0 + r) ++r;
    const int64_t span = r * hp.copy_bytes;
    const bool fold_run = fold && contig && fold_gp >= span && fold_cp >= span;
    // A run goes to the copy engines when its row (one layer and kv half)
    // is wide enough; a run that folds across all layers becomes a single
    // descriptor, so a narrower row already pays off.
    const int64_t row_thr = thr_user >= 0 ? thr_user : (fold_run ? thr_folded : thr);
    const bool to_ce = ce_all || (row_thr > 0 && span >= row_thr);
    if (to_ce && (fold_run || (fold && ce_all))) {
      char *g = (char *)d.gpu_layer_ptrs[0] + g0 * hp.gbs;
      char *c = (char *)hp.cpu_host_base + c0 * hp.cbs;
      if (fold_run) {
        emit(g, c, (size_t)span, (size_t)rows, (size_t)fold_gp, (size_t)fold_cp);
      } else {
        for (int64_t k = 0; k < r; ++k)
          emit(g + k * hp.gbs, c + k * hp.cbs, cb, (size_t)rows, (size_t)fold_gp, (size_t)fold_cp);
      }
      i += r;
      continue;
    }
    if (!to_ce) {
      for (int64_t k = 0; k < r; ++k) {
        hp.sm_gpu.push_back(g0 + k);
        hp.sm_cpu.push_back(c0 + k);
      }
      i += r;
      continue;
    }
    for (int64_t l = 0; l < L; ++l) {
      char *gl = (char *)d.gpu_layer_ptrs[l] + g0 * hp.gbs;
      char *cl = (char *)hp.cpu_host_base + l * hp.cls + c0 * hp.cbs;
      if (contig && (KV == 1 || (hp.gkv >= span && hp.ckv >= span && hp.gkv <= mp && hp.ckv <= mp))) {
        // The run is contiguous on both sides: one row per kv half.
        emit(gl, cl, (size_t)span, (size_t)KV, (size_t)hp.gkv, (size_t)hp.ckv);
      } else if (r == 1 && KV > 1 && pitch_ok(hp.gkv) && pitch_ok(hp.ckv)) {
        emit(gl, cl, cb, (size_t)KV, (size_t)hp.gkv, (size_t)hp.ckv);
      } else {
        for (int64_t kv = 0; kv < KV; ++kv) {
          char *g = gl + kv * hp.gkv, *c = cl + kv * hp.ckv;
          if (contig) {
            emit(g, c, (size_t)span, 1, 0, 0);
          } else if (pitch_ok(hp.gbs) && pitch_ok(hp.cbs)) {
            emit(g, c, cb, (size_t)r, (size_t)hp.gbs, (size_t)hp.cbs);
          } else {
            for (int64_t k = 0; k < r; ++k) emit(g + k * hp.gbs, c + k * hp.cbs, cb, 1, 0, 0);
          }
        }
      }
    }
    i += r;
  }

  // SM budget -> persistent grid.
  if (!hp.sm_gpu.empty()) {
    ThreadDeviceCtx *ctx = nullptr;
    if (int rc = get_ctx(device, &ctx)) return rc;
    int sms = sms_req > 0 ? sms_req : (d.synchronous ? kDefaultSmsSync : kDefaultSmsAsync);
    sms = std::min(sms, ctx->num_sms);
    hp.unroll_idx = variant_index(env_int("FKV_UNROLL", kDefaultUnroll), env_int("FKV_LD_PF256", 0));
    int occ = 1;
    if (int rc = ctas_per_sm(device, hp.h2d, hp.unroll_idx, &occ)) return rc;
    const int64_t chunks = L * KV * (int64_t)hp.sm_gpu.size();
    const int64_t warps_per_cta = kThreads / 32;
    int64_t grid = (int64_t)sms * occ;
    grid = std::min<int64_t>(grid, (chunks + warps_per_cta - 1) / warps_per_cta);
    hp.grid = (int)std::max<int64_t>(grid, 1);
  }
  hp.num_ce_streams = d.num_ce_streams > 0 ? d.num_ce_streams : env_int("FKV_CE_STREAMS", kDefaultCeStreams);
  hp.num_ce_streams = std::max(1, std::min(hp.num_ce_streams, kMaxCeStreams));
  hp.ce_schedule = d.ce_schedule >= 0 ? d.ce_schedule : env_int("FKV_CE_SCHEDULE", kDefaultCeSchedule);
  if (hp.ce_schedule < 0 || hp.ce_schedule > 2)
    return fail(FKV_ERR_INVALID_ARG, "ce_schedule must be -1 (default), 0, 1 or 2");
  return FKV_OK;
}

// Device table layout: [layer_ptrs L][gpu_ids n][cpu_ids n] (int64 words).
size_t table_bytes(const HostPlan &hp) {
  return 8 * ((size_t)hp.num_layers + 2 * hp.sm_gpu.size());
}

void fill_table(const HostPlan &hp, const fkv_transfer_desc &d, int64_t *t) {
  const size_t L = hp.num_layers, n = hp.sm_gpu.size();
  for (size_t l = 0; l < L; ++l) t[l] = (int64_t)(uintptr_t)d.gpu_layer_ptrs[l];
  std::memcpy(t + L, hp.sm_gpu.data(), n * 8);
  std::memcpy(t + L + n, hp.sm_cpu.data(), n * 8);
}

CopyParams make_params(const HostPlan &hp, char *dev_table) {
  CopyParams p{};
  const size_t L = hp.num_layers, n = hp.sm_gpu.size();
  int64_t *t = reinterpret_cast<int64_t *>(dev_table);
  if (t) {
    p.layer_ptrs = reinterpret_cast<char *const *>(t);
    p.gpu_ids = t + L;
    p.cpu_ids = t + L + n;
  }
  p.cpu_base = hp.cpu_dev_base;
  p.gpu_kv_stride = hp.gkv;
  p.gpu_block_stride = hp.gbs;
  p.cpu_layer_stride = hp.cls;
  p.cpu_kv_stride = hp.ckv;
  p.cpu_block_stride = hp.cbs;
  p.n_vec = hp.copy_bytes / 16;
  p.n = (uint32_t)n;
  p.per_layer = (uint32_t)(hp.kv_dim * n);
  p.num_chunks = (uint32_t)(L * hp.kv_dim * n);
  return p;
}

int launch_copy(bool h2d, int variant, int grid, const CopyParams &p, cudaStream_t s) {
  const void *k = h2d ? kernel_ptr<true>(variant) : kernel_ptr<false>(variant);
  void *args[] = {const_cast<CopyParams *>(&p)};
  FKV_CUDA(cudaLaunchKernel(k, dim3(grid), dim3(kThreads), args, 0, s));
  note_launch();
  return FKV_OK;
}

int launch_inline_copy(bool h2d, int grid, const InlineCopyParams &q, cudaStream_t s) {
  const void *k = h2d ? (const void *)kv_copy_inline_kernel<true> : (const void *)kv_copy_inline_kernel<false>;
  void *args[] = {const_cast<InlineCopyParams *>(&q)};
  FKV_CUDA(cudaLaunchKernel(k, dim3(grid), dim3(kThreads), args, 0, s));
  note_launch();
  return FKV_OK;
}

// Whether the SM part of a host plan can carry its table in the kernel's
// parameters (the default kernel variant only).
// FKV_INLINE_TABLE=0 turns the path off (the table then goes through a
// device buffer like larger ops).
bool inline_table_fits(const HostPlan &hp) {
  static const bool enabled = env_int("FKV_INLINE_TABLE", 1) != 0;
  return enabled && hp.num_layers <= kInlineMaxLayers && (int64_t)hp.sm_gpu.size() <= kInlineMaxBlocks &&
         hp.unroll_idx == variant_index(kDefaultUnroll, 0);
}

void fill_inline(const HostPlan &hp, const fkv_transfer_desc &d, InlineCopyParams &q) {
  std::memset(&q, 0, sizeof(q));
  q.p = make_params(hp, nullptr);
  q.p.layer_ptrs = nullptr;  // the kernel points these at the arrays below
  q.p.gpu_ids = nullptr;
  q.p.cpu_ids = nullptr;
  const size_t L = hp.num_layers, n = hp.sm_gpu.size();
  for (size_t l = 0; l < L; ++l) q.layer_ptrs[l] = (int64_t)(uintptr_t)d.gpu_layer_ptrs[l];
  std::memcpy(q.gpu_ids, hp.sm_gpu.data(), n * 8);
  std::memcpy(q.cpu_ids, hp.sm_cpu.data(), n * 8);
}

// Fork the side streams from `s`, enqueue the copy-engine descriptors on
// them (contiguous slices per stream keep each engine's accesses
// sequential) and, when `join`, make `s` wait for all of them.
// Each direction has its own side streams (lane 0 = H2D, lane 1 = D2H, up
// to kMaxCeStreams each), so an H2D transfer and a D2H transfer in flight
// together never queue their copy-engine work behind each other.
int fork_ce(ThreadDeviceCtx *ctx, const std::vector<CeCopy> &ce, int nstreams, bool h2d,
            cudaStream_t s) {
  const int base = h2d ? 0 : kMaxCeStreams;
  if (int rc = ensure_side_streams(ctx, base + nstreams)) return rc;
  FKV_CUDA(cudaEventRecord(ctx->fork_event, s));
  for (int k = 0; k < nstreams; ++k)
    FKV_CUDA(cudaStreamWaitEvent(ctx->side_streams[base + k], ctx->fork_event, 0));
  const cudaMemcpyKind kind = h2d ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost;
  const size_t per = (ce.size() + nstreams - 1) / nstreams;
  for (size_t j = 0; j < ce.size(); ++j) {
    const CeCopy &x = ce[j];
    cudaStream_t ss = ctx->side_streams[base + std::min<size_t>(j / per, nstreams - 1)];
    if (x.height <= 1) {
      FKV_CUDA(cudaMemcpyAsync(x.dst, x.src, x.width, kind, ss));
    } else {
      FKV_CUDA(cudaMemcpy2DAsync(x.dst, x.dpitch, x.src, x.spitch, x.width, x.height, kind, ss));
    }
  }
  return FKV_OK;
}

int join_ce(ThreadDeviceCtx *ctx, int nstreams, bool h2d, cudaStream_t s) {
  const int base = h2d ? 0 : kMaxCeStreams;
  for (int k = 0; k < nstreams; ++k) {
    FKV_CUDA(cudaEventRecord(ctx->join_events[base + k], ctx->side_streams[base + k]));
    FKV_CUDA(cudaStreamWaitEvent(s, ctx->join_events[base + k], 0));
  }
  return FKV_OK;
}

// Enqueue one transfer on `s`: the SM kernel (bracketed by the optional
// events) and the copy-engine descriptors, ordered by `schedule`:
//   0 — concurrent: copy engines on side streams forked from `s`, joined back;
//   1 — copy engines first (on side streams, joined), then the kernel;
//   2 — the kernel first, then the copy engines.
// A serial order keeps the two kinds of host-link traffic apart.
int enqueue_transfer(ThreadDeviceCtx *ctx, bool h2d, int variant, int grid, const CopyParams *p,
                     bool has_sm, const std::vector<CeCopy> &ce, int nstreams, int schedule,
                     cudaStream_t s, cudaEvent_t ev_start, cudaEvent_t ev_end,
                     const InlineCopyParams *iq = nullptr) {
  auto kernel = [&]() -> int {
    if (ev_start) FKV_CUDA(cudaEventRecord(ev_start, s));
    if (has_sm) {
      if (iq) {
        if (int rc = launch_inline_copy(h2d, grid, *iq, s)) return rc;
      } else if (int rc = launch_copy(h2d, variant, grid, *p, s)) {
        return rc;
      }
    }
    if (ev_end) FKV_CUDA(cudaEventRecord(ev_end, s));
    return FKV_OK;
  };
  if (ce.empty()) return kernel();
  if (schedule == 0) {  // fork before the kernel so both run together
    if (int rc = fork_ce(ctx, ce, nstreams, h2d, s)) return rc;
    if (int rc = kernel()) return rc;
    return join_ce(ctx, nstreams, h2d, s);
  }
  if (schedule == 1) {
    if (int rc = fork_ce(ctx, ce, nstreams, h2d, s)) return rc;
    if (int rc = join_ce(ctx, nstreams, h2d, s)) return rc;
    return kernel();
  }
  if (int rc = kernel()) return rc;
  if (int rc = fork_ce(ctx, ce, nstreams, h2d, s)) return rc;
  return join_ce(ctx, nstreams, h2d, s);
}

int current_device(int *dev) {
  FKV_CUDA(cudaGetDevice(dev));
  return FKV_OK;
}

}  // namespace
}  // namespace fkv

namespace fkv {

size_t transfer_stage_bytes(const fkv_transfer_desc &d) {
  return 8 * ((size_t)std::max(d.num_layers, 0) + 2 * (size_t)std::max(d.num_blocks, 0));
}

int transfer_enqueue(const fkv_transfer_desc &d, cudaStream_t s, char *ext_stage, size_t ext_cap) {
  if (int rc = validate_desc(d)) return rc;
  if (d.num_blocks == 0 || d.num_layers == 0 || d.chunk_size_in_bytes < 16) return FKV_OK;
  int device = 0;
  if (int rc = current_device(&device)) return rc;
  HostPlan hp;
  if (int rc = build_host_plan(d, device, hp)) return rc;
  ThreadDeviceCtx *ctx = nullptr;
  if (int rc = get_ctx(device, &ctx)) return rc;
  char *dev_table = nullptr;
  CopyParams p{};
  if (!hp.sm_gpu.empty() && inline_table_fits(hp)) {
    // Small op: the table rides in the kernel's parameters (no allocation, no
    // upload); a caller's staging slice, if given, simply goes unused.
    InlineCopyParams q;
    fill_inline(hp, d, q);
    return enqueue_transfer(ctx, hp.h2d, hp.unroll_idx, hp.grid, nullptr, true, hp.ce, hp.num_ce_streams,
                            hp.ce_schedule, s, nullptr, nullptr, &q);
  }
  if (!hp.sm_gpu.empty()) {
    const size_t tb = table_bytes(hp);
    char *stage = ext_stage;
    if (stage != nullptr) {
      if (tb > ext_cap) return fail(FKV_ERR_INVALID_ARG, "staging slice too small for the id table");
    } else if (int rc = acquire_staging(ctx, tb, &stage)) {
      return rc;
    }
    fill_table(hp, d, reinterpret_cast<int64_t *>(stage));
    if (int rc = scratch_alloc(device, tb, s, (void **)&dev_table)) return rc;
    cudaError_t e = cudaMemcpyAsync(dev_table, stage, tb, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
      scratch_free(dev_table, s);
      return fail_cuda(e, "cudaMemcpyAsync(plan table)");
    }
    if (ext_stage == nullptr)
      if (int rc = release_staging(ctx, s)) return rc;
    p = make_params(hp, dev_table);
  }
  int rc = enqueue_transfer(ctx, hp.h2d, hp.unroll_idx, hp.grid, &p, !hp.sm_gpu.empty(), hp.ce,
                            hp.num_ce_streams, hp.ce_schedule, s, nullptr, nullptr);
  if (dev_table) {
    int rf = scratch_free(dev_table, s);
    if (rc == FKV_OK) rc = rf;
  }
  return rc;
}

namespace {
// The host-side checks of a device-id-list copy (see transfer_check_device_ids).
int device_ids_plan(const fkv_transfer_desc &d, int64_t n_max, int64_t max_cpu_id, HostPlan &hp) {
  if (int rc = validate_desc(d)) return rc;
  hp.h2d = d.is_host_to_device != 0;
  hp.kv_dim = d.is_mla ? 1 : 2;
  hp.num_layers = d.num_layers;
  hp.copy_bytes = (d.chunk_size_in_bytes / 16) * 16;
  if (n_max <= 0 || d.num_layers == 0 || d.chunk_size_in_bytes < 16) return FKV_OK;
  if (!d.gpu_layer_ptrs || !d.cpu_ptr)
    return fail(FKV_ERR_INVALID_ARG, "null layer pointer table or cpu pointer");
  if (int rc = layout_checks(d, n_max, hp)) return rc;
  // Every id the lists can hold must be 16-byte aligned and, when the pool
  // sizes are given, inside them (the ids are produced on the device).
  if ((hp.cbs & 15) || (hp.gbs & 15))
    return fail(FKV_ERR_MISALIGNED, "block strides must be multiples of 16 bytes for device-side id lists");
  const int64_t L = d.num_layers, KV = hp.kv_dim;
  if (d.cpu_pool_bytes > 0 &&
      max_cpu_id * hp.cbs + hp.base_off + (L - 1) * hp.cls + (KV - 1) * hp.ckv + hp.copy_bytes > d.cpu_pool_bytes)
    return fail(FKV_ERR_OUT_OF_RANGE, "cpu block id " + std::to_string(max_cpu_id) + " addresses past the cpu pool");
  return FKV_OK;
}
}  // namespace

int transfer_check_device_ids(const fkv_transfer_desc &d, int64_t n_max, int64_t max_cpu_id) {
  HostPlan hp;
  return device_ids_plan(d, n_max, max_cpu_id, hp);
}

int transfer_enqueue_device_ids(const fkv_transfer_desc &d, const int64_t *gpu_ids_dev,
                                const int64_t *cpu_ids_dev, const int64_t *n_dev, int64_t n_max,
                                int64_t max_cpu_id, cudaStream_t s, int layer_granularity,
                                void *const *group_events) {
  HostPlan hp;
  if (int rc = device_ids_plan(d, n_max, max_cpu_id, hp)) return rc;
  if (n_max <= 0 || d.num_layers == 0 || d.chunk_size_in_bytes < 16) return FKV_OK;
  if (!gpu_ids_dev || !cpu_ids_dev || !n_dev) return fail(FKV_ERR_INVALID_ARG, "null id list");
  int device = 0;
  if (int rc = current_device(&device)) return rc;
  const int64_t L = d.num_layers, KV = hp.kv_dim;
  ThreadDeviceCtx *ctx = nullptr;
  if (int rc = get_ctx(device, &ctx)) return rc;
  const void *k = hp.h2d ? (const void *)kv_copy_devn_kernel<true> : (const void *)kv_copy_devn_kernel<false>;
  if (int rc = check_device(device)) return rc;
  static int occ_cache[kMaxDevices][2] = {{0}};  // CTAs per SM, per device and direction
  int occ = 0;
  {
    std::lock_guard<std::mutex> lk(g_occ.mu);
    occ = occ_cache[device][hp.h2d ? 1 : 0];
  }
  if (occ == 0) {
    FKV_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kThreads, 0));
    occ = std::max(occ, 1);
    std::lock_guard<std::mutex> lk(g_occ.mu);
    occ_cache[device][hp.h2d ? 1 : 0] = occ;
  }
  int sms = d.transfer_sms > 0 ? d.transfer_sms : env_int("FKV_TRANSFER_SMS", kDefaultSms);
  sms = std::min(sms, ctx->num_sms);
  const int64_t G = layer_granularity > 0 ? layer_granularity : L;
  if (L % G != 0) return fail(FKV_ERR_INVALID_ARG, "layer_granularity must divide the number of layers");
  const int64_t warps_per_cta = kThreads / 32;
  int64_t grid = std::min<int64_t>((int64_t)sms * std::max(occ, 1), (G * KV * n_max + warps_per_cta - 1) / warps_per_cta);
  grid = std::max<int64_t>(grid, 1);
  // Layer pointer table: staged once, uploaded on s, freed on s after the kernels.
  const size_t tb = 8 * (size_t)L;
  char *stage = nullptr;
  if (int rc = acquire_staging(ctx, tb, &stage)) return rc;
  for (int64_t l = 0; l < L; ++l) reinterpret_cast<int64_t *>(stage)[l] = (int64_t)(uintptr_t)d.gpu_layer_ptrs[l];
  char *dev_table = nullptr;
  if (int rc = scratch_alloc(device, tb, s, (void **)&dev_table)) return rc;
  cudaError_t e = cudaMemcpyAsync(dev_table, stage, tb, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) {
    scratch_free(dev_table, s);
    return fail_cuda(e, "cudaMemcpyAsync(layer table)");
  }
  if (int rc = release_staging(ctx, s)) return rc;
  // One launch per group of G layers, in order; group_events[g] (optional)
  // is recorded after group g.
  int rc = FKV_OK;
  for (int64_t g0 = 0; g0 < L && rc == FKV_OK; g0 += G) {
    CopyParams p{};
    p.layer_ptrs = reinterpret_cast<char *const *>(dev_table) + g0;
    p.gpu_ids = gpu_ids_dev;
    p.cpu_ids = cpu_ids_dev;
    p.cpu_base = hp.cpu_dev_base + g0 * hp.cls;
    p.gpu_kv_stride = hp.gkv;
    p.gpu_block_stride = hp.gbs;
    p.cpu_layer_stride = hp.cls;
    p.cpu_kv_stride = hp.ckv;
    p.cpu_block_stride = hp.cbs;
    p.n_vec = hp.copy_bytes / 16;
    const uint32_t kvd = (uint32_t)KV, nl = (uint32_t)G, nm = (uint32_t)n_max;
    void *args[] = {&p, const_cast<int64_t **>(&n_dev), (void *)&kvd, (void *)&nl, (void *)&nm};
    e = cudaLaunchKernel(k, dim3((unsigned)grid), dim3(kThreads), args, 0, s);
    if (e != cudaSuccess) {
      rc = fail_cuda(e, "cudaLaunchKernel(kv_copy_devn_kernel)");
      break;
    }
    note_launch();
    if (group_events && group_events[g0 / G]) {
      e = cudaEventRecord((cudaEvent_t)group_events[g0 / G], s);
      if (e != cudaSuccess) rc = fail_cuda(e, "cudaEventRecord(layer group)");
    }
  }
  int rf = scratch_free(dev_table, s);
  return rc != FKV_OK ? rc : rf;
}

}  // namespace fkv

using namespace fkv;

extern "C" {

void fkv_transfer_desc_init(fkv_transfer_desc *d) {
  std::memset(d, 0, sizeof(*d));
  d->transfer_sms = -1;
  d->synchronous = 1;
  d->ce_min_run_bytes = -1;
  d->num_ce_streams = 0;
  d->ce_schedule = -1;
  d->is_host_to_device = 1;
}

int64_t fkv_coalesce_runs(const int64_t *g, const int64_t *c, int64_t n, int64_t *out,
                          int64_t max_runs) {
  int64_t runs = 0, i = 0;
  while (i < n) {
    int64_t r = 1;
    while (i + r < n && g[i + r] == g[i] + r && c[i + r] == c[i] + r) ++r;
    if (runs >= max_runs) return -1;
    out[3 * runs] = g[i];
    out[3 * runs + 1] = c[i];
    out[3 * runs + 2] = r;
    ++runs;
    i += r;
  }
  return runs;
}

int fkv_transfer_kv_blocks_ex(const fkv_transfer_desc *d, void *stream_) {
  clear_error();
  if (!d) return fail(FKV_ERR_INVALID_ARG, "null descriptor");
  cudaStream_t s = (cudaStream_t)stream_;
  const double tstart = profiling() ? now_us() : 0;
  if (int rc = transfer_enqueue(*d, s, nullptr, 0)) return rc;
  const double t1 = profiling() ? now_us() : 0;
  if (d->synchronous) FKV_CUDA(cudaStreamSynchronize(s));  // transfer.cu:131
  if (profiling())
    std::fprintf(stderr, "[fkv] transfer %s n=%d: plan+enqueue %.1fus sync %.1fus\n",
                 d->is_host_to_device ? "h2d" : "d2h", d->num_blocks, t1 - tstart, now_us() - t1);
  return FKV_OK;
}

int fkv_transfer_kv_blocks(int num_blocks, int start_layer_id, int num_layers,
                           const int64_t *gpu_block_ids, void *const *gpu_layer_ptrs,
                           int64_t gpu_kv_stride_in_bytes, int64_t gpu_block_stride_in_bytes,
                           const int64_t *cpu_block_ids, void *cpu_ptr,
                           int64_t cpu_kv_stride_in_bytes, int64_t cpu_layer_stride_in_bytes,
                           int64_t cpu_block_stride_in_bytes, int64_t cpu_startoff_inside_chunks,
                           int64_t chunk_size_in_bytes, void *stream, int transfer_sms,
                           int is_host_to_device, int use_ce_transfer, int is_mla) {
  fkv_transfer_desc d;
  fkv_transfer_desc_init(&d);
  d.num_blocks = num_blocks;
  d.start_layer_id = start_layer_id;
  d.num_layers = num_layers;
  d.gpu_block_ids = gpu_block_ids;
  d.gpu_layer_ptrs = gpu_layer_ptrs;
  d.gpu_kv_stride_in_bytes = gpu_kv_stride_in_bytes;
  d.gpu_block_stride_in_bytes = gpu_block_stride_in_bytes;
  d.cpu_block_ids = cpu_block_ids;
  d.cpu_ptr = cpu_ptr;
  d.cpu_kv_stride_in_bytes = cpu_kv_stride_in_bytes;
  d.cpu_layer_stride_in_bytes = cpu_layer_stride_in_bytes;
  d.cpu_block_stride_in_bytes = cpu_block_stride_in_bytes;
  d.cpu_startoff_inside_chunks = cpu_startoff_inside_chunks;
  d.chunk_size_in_bytes = chunk_size_in_bytes;
  d.transfer_sms = transfer_sms;
  d.is_host_to_device = is_host_to_device;
  d.use_ce_transfer = use_ce_transfer;
  d.is_mla = is_mla;
  return fkv_transfer_kv_blocks_ex(&d, stream);
}

int fkv_plan_create(const fkv_transfer_desc *d, int device, fkv_plan **out) {
  clear_error();
  if (!d || !out) return fail(FKV_ERR_INVALID_ARG, "null descriptor or output");
  *out = nullptr;
  if (int rc = validate_desc(*d)) return rc;
  int prev = 0;
  if (int rc = current_device(&prev)) return rc;
  if (device < 0) device = prev;
  if (device != prev) FKV_CUDA(cudaSetDevice(device));
  HostPlan hp;
  int rc = build_host_plan(*d, device, hp);
  fkv_plan *p = nullptr;
  if (rc == FKV_OK) {
    p = new fkv_plan();
    p->device = device;
    p->h2d = hp.h2d;
    p->grid = hp.grid;
    p->unroll_idx = hp.unroll_idx;
    p->ce = std::move(hp.ce);
    p->num_ce_streams = hp.num_ce_streams;
    p->ce_schedule = hp.ce_schedule;
    p->ce_bytes = hp.ce_bytes;
    p->sm_chunks = (int64_t)hp.num_layers * hp.kv_dim * (int64_t)hp.sm_gpu.size();
    p->sm_bytes = p->sm_chunks * hp.copy_bytes;
    if (!hp.sm_gpu.empty()) {
      const size_t tb = table_bytes(hp);
      std::vector<int64_t> host(tb / 8);
      fill_table(hp, *d, host.data());
      cudaError_t e = cudaMalloc((void **)&p->dev_buf, tb);
      if (e == cudaSuccess) e = cudaMemcpy(p->dev_buf, host.data(), tb, cudaMemcpyHostToDevice);
      if (e != cudaSuccess) {
        rc = fail_cuda(e, "plan table upload");
      } else {
        p->params = make_params(hp, p->dev_buf);
      }
    }
    if (rc != FKV_OK) {
      if (p->dev_buf) cudaFree(p->dev_buf);
      delete p;
      p = nullptr;
    }
  }
  if (device != prev) cudaSetDevice(prev);
  *out = p;
  return rc;
}

int fkv_plan_execute_ex(fkv_plan *p, void *stream_, void *ev_start, void *ev_end) {
  clear_error();
  if (!p) return fail(FKV_ERR_INVALID_ARG, "null plan");
  cudaStream_t s = (cudaStream_t)stream_;
  int prev = 0;
  if (int rc = current_device(&prev)) return rc;
  if (prev != p->device) FKV_CUDA(cudaSetDevice(p->device));
  ThreadDeviceCtx *ctx = nullptr;
  int rc = get_ctx(p->device, &ctx);
  if (rc == FKV_OK)
    rc = enqueue_transfer(ctx, p->h2d, p->unroll_idx, p->grid, &p->params, p->sm_chunks > 0, p->ce,
                          p->num_ce_streams, p->ce_schedule, s, (cudaEvent_t)ev_start,
                          (cudaEvent_t)ev_end);
  if (prev != p->device) cudaSetDevice(prev);
  return rc;
}

int fkv_plan_execute(fkv_plan *p, void *stream_) {
  return fkv_plan_execute_ex(p, stream_, nullptr, nullptr);
}

int fkv_plan_stats(const fkv_plan *p, int64_t *sm_chunks, int64_t *ce_copies, int64_t *ce_bytes,
                   int64_t *sm_bytes) {
  if (!p) return fail(FKV_ERR_INVALID_ARG, "null plan");
  if (sm_chunks) *sm_chunks = p->sm_chunks;
  if (ce_copies) *ce_copies = (int64_t)p->ce.size();
  if (ce_bytes) *ce_bytes = p->ce_bytes;
  if (sm_bytes) *sm_bytes = p->sm_bytes;
  return FKV_OK;
}

void fkv_plan_destroy(fkv_plan *p) {
  if (!p) return;
  if (p->dev_buf) cudaFree(p->dev_buf);
  delete p;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of fkv_transfer_kv_blocks.
//
// Some callers cannot allocate device memory at the moment they move KV
// blocks: an engine that hands the whole GPU to its own caching allocator
// and forbids outside cudaMalloc, a host thread running under a strict
// memory budget, or code that must not trigger the implicit
// synchronization an allocation can cause.  This entry point keeps its
// scratch (the layer-pointer table and the two block-id arrays the copy
// kernel reads) in the file-scope device array below instead of the
// library's memory pool, and never calls an allocating CUDA routine.
//
// Limits: at most kNoAllocMaxLayers layers and kNoAllocMaxBlocks blocks per
// call (132 KiB of device memory, held by every GPU that loads this library
// until the process exits).  Only the SM copy kernel is used (no copy
// engines, no side streams).  Every call shares the one array and
// overwrites the part it uses; the call is synchronous, so calls made one
// after another are safe, while calls that overlap on the GPU (from several
// host threads or streams at once) race on the array.  The first call on a
// device resolves the array's device address with cudaGetSymbolAddress
// (with that device current); make that first call before any stream
// capture.
// ---------------------------------------------------------------------------
namespace fkv {
namespace {

constexpr int kNoAllocMaxLayers = 512;
constexpr int kNoAllocMaxBlocks = 8192;
constexpr int kNoAllocWords = kNoAllocMaxLayers + 2 * kNoAllocMaxBlocks;

static __device__ __align__(256) int64_t g_noalloc_table[kNoAllocWords];

// Device address of g_noalloc_table per device, resolved once per device.
std::mutex g_noalloc_mu;
int64_t *g_noalloc_addr[kMaxDevices] = {nullptr};

int noalloc_table(int device, int64_t **out) {
  if (int rc = check_device(device)) return rc;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  int64_t *&p = g_noalloc_addr[device];
  if (p == nullptr) {
    void *addr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_table);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(g_noalloc_table)");
    p = static_cast<int64_t *>(addr);
  }
  *out = p;
  return FKV_OK;
}

}  // namespace
}  // namespace fkv

extern "C" int fkv_transfer_kv_blocks_noalloc(
    int num_blocks, int start_layer_id, int num_layers, const int64_t *gpu_block_ids,
    void *const *gpu_layer_ptrs, int64_t gpu_kv_stride_in_bytes, int64_t gpu_block_stride_in_bytes,
    const int64_t *cpu_block_ids, void *cpu_ptr, int64_t cpu_kv_stride_in_bytes,
    int64_t cpu_layer_stride_in_bytes, int64_t cpu_block_stride_in_bytes,
    int64_t cpu_startoff_inside_chunks, int64_t chunk_size_in_bytes, int64_t cpu_pool_bytes,
    int64_t gpu_layer_bytes, void *stream_, int transfer_sms, int is_host_to_device, int is_mla) {
  clear_error();
  if (num_blocks > kNoAllocMaxBlocks)
    return fail(FKV_ERR_INVALID_ARG, "fkv_transfer_kv_blocks_noalloc: num_blocks exceeds the limit of 8192");
  if (num_layers > kNoAllocMaxLayers)
    return fail(FKV_ERR_INVALID_ARG, "fkv_transfer_kv_blocks_noalloc: num_layers exceeds the limit of 512");
  if (num_blocks < 0 || num_layers < 0 || chunk_size_in_bytes < 0 || start_layer_id < 0 ||
      gpu_kv_stride_in_bytes < 0 || gpu_block_stride_in_bytes < 0 || cpu_kv_stride_in_bytes < 0 ||
      cpu_layer_stride_in_bytes < 0 || cpu_block_stride_in_bytes < 0 ||
      cpu_startoff_inside_chunks < 0)
    return fail(FKV_ERR_INVALID_ARG, "fkv_transfer_kv_blocks_noalloc: negative size, stride or offset");
  const int64_t copy_bytes = (chunk_size_in_bytes / 16) * 16;  // transfer.cu:35
  if (num_blocks == 0 || num_layers == 0 || copy_bytes == 0) return FKV_OK;
  if (!gpu_block_ids || !cpu_block_ids || !gpu_layer_ptrs || !cpu_ptr)
    return fail(FKV_ERR_INVALID_ARG, "fkv_transfer_kv_blocks_noalloc: null id array, layer table or cpu pointer");
  cudaStream_t s = (cudaStream_t)stream_;
  int device = 0;
  FKV_CUDA(cudaGetDevice(&device));
  int64_t *table = nullptr;
  if (int rc = noalloc_table(device, &table)) return rc;

  const int kv_dim = is_mla ? 1 : 2;
  const int64_t gkv = trunc8(gpu_kv_stride_in_bytes), gbs = trunc8(gpu_block_stride_in_bytes);
  const int64_t cls = trunc8(cpu_layer_stride_in_bytes), ckv = trunc8(cpu_kv_stride_in_bytes);
  const int64_t cbs = trunc8(cpu_block_stride_in_bytes);
  const int64_t base_off = (int64_t)start_layer_id * cls + trunc8(cpu_startoff_inside_chunks);
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, cpu_ptr);
  if (e != cudaSuccess || attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr) {
    cudaGetLastError();
    return fail(FKV_ERR_INVALID_ARG, "fkv_transfer_kv_blocks_noalloc: cpu_ptr is not page-locked host memory");
  }
  char *cpu_dev_base = (char *)attr.devicePointer + base_off;
  if (((uintptr_t)cpu_dev_base & 15) || (num_layers > 1 && (cls & 15)) ||
      (kv_dim > 1 && ((ckv & 15) || (gkv & 15))))
    return fail(FKV_ERR_MISALIGNED, "fkv_transfer_kv_blocks_noalloc: cpu base or strides not 16-byte aligned");
  for (int l = 0; l < num_layers; ++l)
    if (gpu_layer_ptrs[l] == nullptr || ((uintptr_t)gpu_layer_ptrs[l] & 15))
      return fail(FKV_ERR_MISALIGNED, "fkv_transfer_kv_blocks_noalloc: null or misaligned gpu layer pointer");
  const int64_t cpu_fixed = base_off + (int64_t)(num_layers - 1) * cls + (kv_dim - 1) * ckv + copy_bytes;
  const int64_t gpu_fixed = (kv_dim - 1) * gkv + copy_bytes;
  for (int i = 0; i < num_blocks; ++i) {
    const int64_t g = gpu_block_ids[i], c = cpu_block_ids[i];
    if (g < 0 || c < 0 || g >= (1ll << 31) || c >= (1ll << 31))
      return fail(FKV_ERR_OUT_OF_RANGE, "fkv_transfer_kv_blocks_noalloc: block id out of [0, 2^31)");
    if (((g * gbs) & 15) || ((c * cbs) & 15))
      return fail(FKV_ERR_MISALIGNED, "fkv_transfer_kv_blocks_noalloc: block stride times id is not 16-byte aligned");
    if (cpu_pool_bytes > 0 && c * cbs + cpu_fixed > cpu_pool_bytes)
      return fail(FKV_ERR_OUT_OF_RANGE, "fkv_transfer_kv_blocks_noalloc: cpu block id addresses past the cpu pool");
    if (gpu_layer_bytes > 0 && g * gbs + gpu_fixed > gpu_layer_bytes)
      return fail(FKV_ERR_OUT_OF_RANGE, "fkv_transfer_kv_blocks_noalloc: gpu block id addresses past the gpu layer");
  }

  // Table layout as in the pooled path: [layer ptrs L][gpu ids n][cpu ids n].
  static_assert(sizeof(void *) == sizeof(int64_t), "64-bit pointers expected");
  FKV_CUDA(cudaMemcpyAsync(table, gpu_layer_ptrs, (size_t)num_layers * 8, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemcpyAsync(table + num_layers, gpu_block_ids, (size_t)num_blocks * 8,
                           cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemcpyAsync(table + num_layers + num_blocks, cpu_block_ids, (size_t)num_blocks * 8,
                           cudaMemcpyHostToDevice, s));

  CopyParams p{};
  p.layer_ptrs = reinterpret_cast<char *const *>(table);
  p.gpu_ids = table + num_layers;
  p.cpu_ids = table + num_layers + num_blocks;
  p.cpu_base = cpu_dev_base;
  p.gpu_kv_stride = gkv;
  p.gpu_block_stride = gbs;
  p.cpu_layer_stride = cls;
  p.cpu_kv_stride = ckv;
  p.cpu_block_stride = cbs;
  p.n_vec = copy_bytes / 16;
  p.n = (uint32_t)num_blocks;
  p.per_layer = (uint32_t)(kv_dim * num_blocks);
  p.num_chunks = (uint32_t)(num_layers * kv_dim * num_blocks);

  int num_sms = 0;
  FKV_CUDA(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device));
  int sms = transfer_sms > 0 ? std::min(transfer_sms, num_sms) : std::min(kDefaultSms, num_sms);
  const bool h2d = is_host_to_device != 0;
  const int variant = variant_index(kDefaultUnroll, 0);
  int occ = 1;
  if (int rc = ctas_per_sm(device, h2d, variant, &occ)) return rc;
  const int64_t warps_per_cta = kThreads / 32;
  int64_t grid = std::min<int64_t>((int64_t)sms * occ, ((int64_t)p.num_chunks + warps_per_cta - 1) / warps_per_cta);
  if (int rc = launch_copy(h2d, variant, (int)std::max<int64_t>(grid, 1), p, s)) return rc;
  FKV_CUDA(cudaStreamSynchronize(s));  // the shared table is free again on return
  return FKV_OK;
}
