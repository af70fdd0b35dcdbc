// CPU-tier block index, block pool and fused put path on the device — the
// B200 replacement for the put side of FlexKV's cache engine:
//   GlobalCacheEngine.put / _put_impl_local   flexkv/cache/cache_engine.py:550-615, 787-902
//   RadixTreeIndex match_prefix / insert / set_ready   flexkv/cache/radixtree.py:143-316
//   Mempool allocate_blocks / recycle_blocks          flexkv/cache/mempool.py:28-55
//
// Block hashes are prefix-chained (block j's hash covers tokens
// [0,(j+1)*tpb)), so every cached prefix is present block by block and the
// tree walk of match_prefix reduces to "the leading blocks whose hash is
// present".  The index is therefore an open-addressing table in HBM keyed by
// the 64-bit block hash (value: pool block id, flag: ready); a batch of
// requests is matched with one probe per block instead of a pointer walk per
// request on the host.
//
// A put batch runs as one stream of kernels, with no host round trip:
//   hash (xxh_batched_kernel) -> lookup (index + a batch-local table that
//   gives equal hashes one slot) -> decide (one warp walks the requests in
//   order: matched prefix, pool allocation, id lists) -> insert (not ready)
//   -> D2H copy of the blocks decided (kv_copy_devn_kernel) -> mark ready.
// The decide step is the only sequential one: request r sees the blocks that
// requests < r of the same batch inserted, exactly as consecutive puts do.
//
// Differences from the reference, all outside its normal operation:
//   * no eviction on the device: when the pool is short, a put comes back
//     empty, as the reference's does when take() finds nothing evictable.
//     Eviction is the caller's: fkv_cache_index_remove + _recycle;
//   * the two largest 64-bit values are the table's empty/deleted markers;
//     a block whose hash equals one of them fails the call (probability
//     2^-63 per block) instead of being cached;
//   * a hash collision between different prefixes (probability ~2^-64 per
//     pair) fails the call; the tree would keep both in separate branches.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "fkv_common.h"

namespace fkv {
namespace {

constexpr uint64_t kEmpty = ~0ull;     // never-used slot
constexpr uint64_t kTomb = ~0ull - 1;  // removed entry (reusable by inserts)
constexpr uint32_t kReadyBit = 1u;

// Device state words.
enum : int {
  kNumFree = 0,  // Mempool._num_free
  kListLen,      // len(Mempool._free_ids)
  kOffset,       // Mempool._free_ids_offset
  kLive,         // entries in the table
  kTombs,        // deleted slots
  kErr,          // first error (ErrCode), 0 = none
  kErrArg,       // the index or id that caused it
  kStateWords
};
enum ErrCode : int64_t { kErrNone = 0, kErrFull = 1, kErrReserved = 2, kErrCollision = 3, kErrRecycleFree = 4 };

// put outcome per request (res[3r+2])
enum : int64_t { kPutEmpty = 0, kPutDone = 1, kPutNoSpace = 2, kPutSourceNotReady = 3 };

struct Table {
  uint64_t *keys;
  int64_t *vals;
  uint32_t *flags;
  uint64_t mask;  // slots - 1
  int shift;      // 64 - log2(slots)
};

__device__ __forceinline__ uint64_t home(uint64_t key, int shift) {
  return (key * 0x9E3779B97F4A7C15ull) >> shift;  // Fibonacci hashing
}

__device__ __forceinline__ void set_error(int64_t *state, int64_t code, int64_t arg) {
  if (atomicCAS(reinterpret_cast<unsigned long long *>(state + kErr), 0ull, (unsigned long long)code) == 0ull)
    state[kErrArg] = arg;
}

// Slot holding key, or -1.  Probes stop at an empty slot; every probe loop
// is bounded by the table size.
__device__ __forceinline__ int64_t find(const Table &t, uint64_t key) {
  if (key >= kTomb) return -1;
  uint64_t s = home(key, t.shift);
  for (uint64_t p = 0; p <= t.mask; ++p) {
    const uint64_t k = t.keys[s];
    if (k == key) return (int64_t)s;
    if (k == kEmpty) return -1;
    s = (s + 1) & t.mask;
  }
  return -1;
}

// Insert a key that the caller knows is absent and that no other thread of
// the launch inserts.  Returns the slot, or -1 (table full) / -2 (present).
__device__ __forceinline__ int64_t insert_absent(const Table &t, uint64_t key, int64_t val, uint32_t fl,
                                                 bool *reused_tomb) {
  uint64_t s = home(key, t.shift);
  for (uint64_t p = 0; p <= t.mask; ++p) {
    uint64_t k = t.keys[s];
    if (k == key) return -2;
    if (k == kEmpty || k == kTomb) {
      const uint64_t was = atomicCAS(reinterpret_cast<unsigned long long *>(t.keys + s),
                                     (unsigned long long)k, (unsigned long long)key);
      if (was == k) {
        t.vals[s] = val;
        t.flags[s] = fl;
        *reused_tomb = (k == kTomb);
        return (int64_t)s;
      }
      if (was == key) return -2;
    }
    s = (s + 1) & t.mask;
  }
  return -1;
}

__global__ void init_pool_kernel(uint8_t *free_mask, int64_t mask_bytes, int64_t *free_ids, int64_t n,
                                 int64_t *state) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < mask_bytes; i += stride) {
    free_mask[i] = i < n ? 1 : 0;
    if (i < n) free_ids[i] = i;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    state[kNumFree] = n;
    state[kListLen] = n;
    for (int w = kOffset; w < kStateWords; ++w) state[w] = 0;
  }
}

// Per block of the batch: present in the index before this call, and its
// slot in the batch-local table (one slot per distinct hash).
__global__ void put_lookup_kernel(Table t, const uint64_t *hashes, int64_t nb, uint8_t *before,
                                  uint64_t *lkeys, uint64_t lmask, int lshift, int32_t *lslot,
                                  int64_t *state) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nb; i += stride) {
    const uint64_t key = hashes[i];
    if (key >= kTomb) {
      set_error(state, kErrReserved, i);
      before[i] = 0;
      lslot[i] = -1;
      continue;
    }
    before[i] = find(t, key) >= 0 ? 1 : 0;
    uint64_t s = home(key, lshift);
    int32_t got = -1;
    for (uint64_t p = 0; p <= lmask; ++p) {
      uint64_t k = lkeys[s];
      if (k == kEmpty) {
        k = atomicCAS(reinterpret_cast<unsigned long long *>(lkeys + s), (unsigned long long)kEmpty,
                      (unsigned long long)key);
        if (k == kEmpty) k = key;
      }
      if (k == key) {
        got = (int32_t)s;
        break;
      }
      s = (s + 1) & lmask;
    }
    lslot[i] = got;
  }
}

// Mempool._update_free_ids (mempool.py:53-55) by one warp: the free ids in
// ascending order.  Each lane tests 16 mask bytes per pass (mask_bytes is a
// multiple of 512, padding bytes are 0).
__device__ int64_t rebuild_free_ids(const uint8_t *mask, int64_t mask_bytes, int64_t *ids, int lane) {
  int64_t total = 0;
  for (int64_t base = 0; base < mask_bytes; base += 512) {
    const uint4 v = reinterpret_cast<const uint4 *>(mask + base)[lane];
    const int c = __popc(v.x) + __popc(v.y) + __popc(v.z) + __popc(v.w);  // bytes are 0 or 1
    int incl = c;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    int64_t at = total + incl - c;
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 16; ++q)
      if ((w[q >> 2] >> (8 * (q & 3))) & 0xffu) ids[at++] = base + 16 * lane + q;
    total += __shfl_sync(0xffffffffu, incl, 31);
  }
  __syncwarp();
  return total;
}

// The put decisions, one warp, requests in order (cache_engine.py:787-902,
// CPU tier): matched prefix m (leading blocks present before this call or
// inserted by an earlier put of the batch), k = n - m blocks to move,
// take(k) without eviction, and on success the id lists of the copy and of
// the inserts.  res[3r] = skipped blocks, res[3r+1] = moved blocks,
// res[3r+2] = outcome.
__global__ void __launch_bounds__(32) put_decide_kernel(
    int num_req, const int64_t *blk_off, const uint8_t *before, const int32_t *lslot, int32_t *ins_req,
    const int64_t *gpu_ids, uint8_t *free_mask, int64_t mask_bytes, int64_t *free_ids, int64_t *state,
    int64_t *res, int64_t *cpu_out, int64_t *d2h_gpu, int64_t *d2h_cpu, int64_t *new_blk, int64_t *count,
    const int64_t *done) {
  const int lane = threadIdx.x;
  if (*done) return;  // put_decide_fast_kernel decided the batch
  if (state[kErr] != kErrNone) {  // an earlier step failed: change nothing
    if (lane == 0) *count = 0;
    return;
  }
  int64_t num_free = state[kNumFree], list_len = state[kListLen], offset = state[kOffset];
  int64_t cnt = 0;
  for (int r = 0; r < num_req; ++r) {
    const int64_t o = blk_off[r], n = blk_off[r + 1] - o;
    int64_t m = n;
    for (int64_t jb = 0; jb < n; jb += 32) {
      const int64_t j = jb + lane;
      bool miss = false;
      if (j < n) {
        const int32_t sl = lslot[o + j];
        miss = !(before[o + j] || (sl >= 0 && ins_req[sl] < r));
      }
      const unsigned b = __ballot_sync(0xffffffffu, miss);
      if (b) {
        m = jb + __ffs(b) - 1;
        break;
      }
    }
    const int64_t k = n - m;
    int64_t *rr = res + 3 * (int64_t)r;
    if (k == 0) {
      if (lane == 0) { rr[0] = 0; rr[1] = 0; rr[2] = kPutEmpty; }
      continue;
    }
    int64_t a = k < num_free ? k : num_free;  // take(strict=False), nothing evicted
    if (a > list_len - offset) {               // mempool.py:37-38
      list_len = rebuild_free_ids(free_mask, mask_bytes, free_ids, lane);
      offset = 0;
    }
    if (a > list_len - offset) a = list_len - offset;  // never reads past the snapshot
    if (a < k) {
      // allocate(a) then recycle the same ids (cache_engine.py:862-867):
      // the mask and count end unchanged, the snapshot offset moves on.
      offset += a;
      if (lane == 0) { rr[0] = 0; rr[1] = 0; rr[2] = kPutNoSpace; }
      continue;
    }
    for (int64_t t = lane; t < k; t += 32) {
      const int64_t i = o + m + t, c = free_ids[offset + t];
      free_mask[c] = 0;
      cpu_out[i] = c;
      d2h_gpu[cnt + t] = gpu_ids[i];
      d2h_cpu[cnt + t] = c;
      new_blk[cnt + t] = i;
      const int32_t sl = lslot[i];
      if (sl >= 0) ins_req[sl] = r;
    }
    offset += k;
    num_free -= k;
    cnt += k;
    if (lane == 0) { rr[0] = m; rr[1] = k; rr[2] = kPutDone; }
    __syncwarp();  // ins_req and mask writes visible to every lane for the next request
  }
  if (lane == 0) {
    state[kNumFree] = num_free;
    state[kListLen] = list_len;
    state[kOffset] = offset;
    *count = cnt;
  }
}

// The same decisions in parallel, for the common case: when the batch's
// new blocks all fit both the free count and what is left of the pool's id
// snapshot, no request comes back empty and no snapshot refresh happens, so
// a block is present for request r exactly when the index held it before
// the call or an earlier request of the batch holds it (first_req, the
// smallest request index per distinct hash), and ids are taken from the
// snapshot in request order (a prefix sum of the counts).  One CTA; each
// thread a contiguous run of requests.  Sets *done = 1 when it decided;
// otherwise it changes nothing but res and first_req, and the one-warp walk
// decides.
constexpr int kDecideThreads = 1024;
__global__ void __launch_bounds__(kDecideThreads) put_decide_fast_kernel(
    int num_req, const int64_t *blk_off, const uint8_t *before, const int32_t *lslot, int32_t *first_req,
    const int64_t *gpu_ids, uint8_t *free_mask, const int64_t *free_ids, int64_t *state, int64_t *res,
    int64_t *cpu_out, int64_t *d2h_gpu, int64_t *d2h_cpu, int64_t *new_blk, int64_t *count, int64_t *done) {
  __shared__ int64_t sums[kDecideThreads];
  const int t = threadIdx.x;
  if (state[kErr] != kErrNone) {  // an earlier step failed: change nothing
    if (t == 0) {
      *count = 0;
      *done = 1;
    }
    return;
  }
  const int per = (num_req + kDecideThreads - 1) / kDecideThreads;
  const int r0 = min(num_req, t * per), r1 = min(num_req, r0 + per);
  for (int r = r0; r < r1; ++r)
    for (int64_t i = blk_off[r]; i < blk_off[r + 1]; ++i) {
      const int32_t sl = lslot[i];
      if (sl >= 0) atomicMin(first_req + sl, r);
    }
  __syncthreads();
  int64_t mine = 0;
  for (int r = r0; r < r1; ++r) {
    const int64_t o = blk_off[r], n = blk_off[r + 1] - o;
    int64_t m = n;
    for (int64_t j = 0; j < n; ++j) {
      const int32_t sl = lslot[o + j];
      if (!(before[o + j] || (sl >= 0 && first_req[sl] < r))) {
        m = j;
        break;
      }
    }
    res[3 * (int64_t)r] = m;
    res[3 * (int64_t)r + 1] = n - m;
    mine += n - m;
  }
  sums[t] = mine;
  __syncthreads();
  for (int d = 1; d < kDecideThreads; d <<= 1) {  // inclusive scan (Hillis-Steele)
    const int64_t add = t >= d ? sums[t - d] : 0;
    __syncthreads();
    sums[t] += add;
    __syncthreads();
  }
  const int64_t total = sums[kDecideThreads - 1];
  const int64_t num_free = state[kNumFree], list_len = state[kListLen], offset = state[kOffset];
  if (total > num_free || total > list_len - offset) {  // the walk decides
    if (t == 0) *done = 0;
    return;
  }
  int64_t at = sums[t] - mine;
  for (int r = r0; r < r1; ++r) {
    const int64_t o = blk_off[r], m = res[3 * (int64_t)r], k = res[3 * (int64_t)r + 1];
    if (k == 0) {
      res[3 * (int64_t)r] = 0;
      res[3 * (int64_t)r + 2] = kPutEmpty;
      continue;
    }
    for (int64_t q = 0; q < k; ++q) {
      const int64_t i = o + m + q, c = free_ids[offset + at + q];
      free_mask[c] = 0;
      cpu_out[i] = c;
      d2h_gpu[at + q] = gpu_ids[i];
      d2h_cpu[at + q] = c;
      new_blk[at + q] = i;
    }
    res[3 * (int64_t)r + 2] = kPutDone;
    at += k;
  }
  __syncthreads();
  if (t == 0) {
    state[kNumFree] = num_free - total;
    state[kOffset] = offset + total;
    *count = total;
    *done = 1;
  }
}

// Per block: present in a tier's index before the call, the pool block it
// holds there (-1 if absent) and whether that block is ready.
__global__ void tier_lookup_kernel(Table t, const uint64_t *hashes, int64_t nb, uint8_t *present, int64_t *phys,
                                   uint8_t *ready) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nb; i += stride) {
    const int64_t s = find(t, hashes[i]);
    present[i] = s >= 0 ? 1 : 0;
    if (phys) phys[i] = s >= 0 ? t.vals[s] : -1;
    if (ready) ready[i] = (s >= 0 && (t.flags[s] & kReadyBit)) ? 1 : 0;
  }
}

// One tier's pool in the two-tier decide step.
struct PoolRef {
  uint8_t *mask;
  int64_t mask_bytes;
  int64_t *free_ids;
  int64_t *state;
};

// The two-tier put decisions (cache_engine.py:787-902 with the SSD tier on),
// one warp, requests in order.  Per request: m_c / m_s leading blocks
// present in the CPU / SSD tier (before the call, or inserted there by an
// earlier request of the batch); k = n - m_c blocks go D2H into new CPU
// blocks; f2 = n - m_s blocks go CPU -> SSD into new SSD blocks (the block's
// CPU copy: new for j >= m_c, the cached one below); both takes must succeed
// or the request comes back empty with both allocations given back
// (cache_engine.py:838-852).  When the SSD tier is behind the CPU tier
// (m_s < m_c, only after a caller evicted from the SSD tier alone), a block
// below m_c goes to the SSD tier from its cached CPU block; if one of those
// cached blocks is not ready (its own D2H may still be in flight), the
// request is refused: it comes back empty and allocates nothing.
// res[4r..4r+3] = skipped, moved D2H, moved to SSD, outcome.
__global__ void __launch_bounds__(32) put2_decide_kernel(
    int num_req, const int64_t *blk_off, const uint8_t *before_c, const uint8_t *before_s, const int64_t *phys_c,
    const uint8_t *ready_c, const int32_t *lslot, int32_t *ins_c, int32_t *ins_s, int64_t *slot_cpu, const int64_t *gpu_ids, PoolRef pc,
    PoolRef ps, int64_t *res, int64_t *cpu_out, int64_t *ssd_out, int64_t *d2h_gpu, int64_t *d2h_cpu,
    int64_t *new_c, int64_t *new_s, int64_t *counts) {
  const int lane = threadIdx.x;
  if (pc.state[kErr] != kErrNone || ps.state[kErr] != kErrNone) {  // an earlier step failed
    if (lane == 0) counts[0] = counts[1] = 0;
    return;
  }
  int64_t free_c = pc.state[kNumFree], len_c = pc.state[kListLen], off_c = pc.state[kOffset];
  int64_t free_s = ps.state[kNumFree], len_s = ps.state[kListLen], off_s = ps.state[kOffset];
  int64_t cnt_c = 0, cnt_s = 0;
  for (int r = 0; r < num_req; ++r) {
    const int64_t o = blk_off[r], n = blk_off[r + 1] - o;
    int64_t m_c = n, m_s = n;
    bool found_c = false, found_s = false;
    for (int64_t jb = 0; jb < n && !(found_c && found_s); jb += 32) {
      const int64_t j = jb + lane;
      bool miss_c = false, miss_s = false;
      if (j < n) {
        const int32_t sl = lslot[o + j];
        miss_c = !(before_c[o + j] || (sl >= 0 && ins_c[sl] < r));
        miss_s = !(before_s[o + j] || (sl >= 0 && ins_s[sl] < r));
      }
      const unsigned bc = __ballot_sync(0xffffffffu, miss_c);
      const unsigned bs = __ballot_sync(0xffffffffu, miss_s);
      if (!found_c && bc) { m_c = jb + __ffs(bc) - 1; found_c = true; }
      if (!found_s && bs) { m_s = jb + __ffs(bs) - 1; found_s = true; }
    }
    const int64_t k = n - m_c, f2 = n - m_s;
    int64_t *rr = res + 4 * (int64_t)r;
    if (k == 0) {  // the CPU tier holds every block: nothing moves (cache_engine.py:819-820)
      if (lane == 0) { rr[0] = 0; rr[1] = 0; rr[2] = 0; rr[3] = kPutEmpty; }
      continue;
    }
    bool unready = false;  // an H2DISK source cached before the call but not ready
    for (int64_t jb = m_s; jb < m_c && !unready; jb += 32) {
      const int64_t j = jb + lane;
      const bool bad = j < m_c && before_c[o + j] && !ready_c[o + j];
      unready = __ballot_sync(0xffffffffu, bad) != 0u;
    }
    if (unready) {
      if (lane == 0) { rr[0] = 0; rr[1] = 0; rr[2] = 0; rr[3] = kPutSourceNotReady; }
      continue;
    }
    int64_t a = k < free_c ? k : free_c;
    if (a > len_c - off_c) {
      len_c = rebuild_free_ids(pc.mask, pc.mask_bytes, pc.free_ids, lane);
      off_c = 0;
    }
    if (a > len_c - off_c) a = len_c - off_c;
    int64_t b = f2 < free_s ? f2 : free_s;
    if (b > len_s - off_s) {
      len_s = rebuild_free_ids(ps.mask, ps.mask_bytes, ps.free_ids, lane);
      off_s = 0;
    }
    if (b > len_s - off_s) b = len_s - off_s;
    if (a < k || b < f2) {  // allocate then recycle both: masks and counts unchanged
      off_c += a;
      off_s += b;
      if (lane == 0) { rr[0] = 0; rr[1] = 0; rr[2] = 0; rr[3] = kPutNoSpace; }
      continue;
    }
    for (int64_t t = lane; t < k; t += 32) {
      const int64_t i = o + m_c + t, c = pc.free_ids[off_c + t];
      pc.mask[c] = 0;
      cpu_out[i] = c;
      d2h_gpu[cnt_c + t] = gpu_ids[i];
      d2h_cpu[cnt_c + t] = c;
      new_c[cnt_c + t] = i;
      const int32_t sl = lslot[i];
      if (sl >= 0) {
        ins_c[sl] = r;
        slot_cpu[sl] = c;
      }
    }
    __syncwarp();
    for (int64_t t = lane; t < f2; t += 32) {
      const int64_t j = m_s + t, i = o + j, sid = ps.free_ids[off_s + t];
      ps.mask[sid] = 0;
      ssd_out[i] = sid;
      if (j < m_c) {  // already on the CPU tier: its cached block is the H2DISK source
        const int32_t sl = lslot[i];
        cpu_out[i] = before_c[i] ? phys_c[i] : (sl >= 0 ? slot_cpu[sl] : -1);
      }
      new_s[cnt_s + t] = i;
      const int32_t sl = lslot[i];
      if (sl >= 0) ins_s[sl] = r;
    }
    off_c += k;
    free_c -= k;
    cnt_c += k;
    off_s += f2;
    free_s -= f2;
    cnt_s += f2;
    if (lane == 0) { rr[0] = m_c; rr[1] = k; rr[2] = f2; rr[3] = kPutDone; }
    __syncwarp();
  }
  if (lane == 0) {
    pc.state[kNumFree] = free_c;
    pc.state[kListLen] = len_c;
    pc.state[kOffset] = off_c;
    ps.state[kNumFree] = free_s;
    ps.state[kListLen] = len_s;
    ps.state[kOffset] = off_s;
    counts[0] = cnt_c;
    counts[1] = cnt_s;
  }
}

// Insert the decided blocks, not ready (radixtree.py:202-256 with
// is_ready=False, as _put_impl_local does).
__global__ void put_insert_kernel(Table t, const uint64_t *hashes, const int64_t *new_blk, const int64_t *cpu_out,
                                  const int64_t *count, int64_t *new_slot, int64_t *state) {
  const int64_t n = *count;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t reused = 0, added = 0;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n; q += stride) {
    const int64_t i = new_blk[q];
    bool tomb = false;
    const int64_t s = insert_absent(t, hashes[i], cpu_out[i], 0u, &tomb);
    new_slot[q] = s;
    if (s >= 0) {
      ++added;
      reused += tomb ? 1 : 0;
    } else {
      set_error(state, s == -1 ? kErrFull : kErrCollision, i);
    }
  }
  if (added) atomicAdd(reinterpret_cast<unsigned long long *>(state + kLive), (unsigned long long)added);
  if (reused) atomicAdd(reinterpret_cast<unsigned long long *>(state + kTombs), (unsigned long long)(-reused));
}

// The put callback's set_ready (cache_engine.py:83-85, 904-910) once the
// copy before it on the stream is done.
__global__ void mark_slots_ready_kernel(Table t, const int64_t *slots, const int64_t *count) {
  const int64_t n = *count;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n; q += stride) {
    const int64_t s = slots[q];
    if (s >= 0) t.flags[s] |= kReadyBit;
  }
}

// match_prefix for a batch (radixtree.py:143-195), one warp per request:
// matched = leading blocks present; ready = matched blocks marked ready;
// phys[j] = pool block of block j for j < matched, -1 after.
__global__ void match_kernel(Table t, const uint64_t *hashes, const int64_t *blk_off, int num_req,
                             int64_t *res, int64_t *phys) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < num_req; r += warps) {
    const int64_t o = blk_off[r], n = blk_off[r + 1] - o;
    int64_t matched = n, ready = 0;
    bool done = false;
    for (int64_t jb = 0; jb < n && !done; jb += 32) {
      const int64_t j = jb + lane;
      int64_t s = -1;
      if (j < n) s = find(t, hashes[o + j]);
      const unsigned miss = __ballot_sync(0xffffffffu, j < n && s < 0);
      const int64_t lim = miss ? (int64_t)(__ffs(miss) - 1) : 32;  // present lanes before the first miss
      const bool in = j < n && lane < lim;
      if (j < n) phys[o + j] = in ? t.vals[s] : -1;
      ready += __popc(__ballot_sync(0xffffffffu, in && (t.flags[s] & kReadyBit)));
      if (miss) {
        matched = jb + lim;
        done = true;
      }
    }
    // blocks after the first miss of a later pass were never visited
    for (int64_t j = (matched / 32 + 1) * 32 + lane; j < n; j += 32) phys[o + j] = -1;
    if (lane == 0) {
      res[2 * (int64_t)r] = matched;
      res[2 * (int64_t)r + 1] = ready;
    }
  }
}

// The get decisions (cache_engine.py:412-548, CPU tier), after
// match_kernel: request r reads physical_blocks[:num_ready][start_r:n_r]
// (the reference takes the first num_ready matched blocks) into its leading
// GPU blocks.  Gets change neither the index nor the pool, so requests are
// independent: one CTA of kGetThreads threads, each thread a contiguous
// run of requests; the per-thread block counts are scanned in shared
// memory to place every request's entries in the copy lists.
constexpr int kGetThreads = 1024;
__global__ void __launch_bounds__(kGetThreads) get_lists_kernel(
    int num_req, const int64_t *blk_off, const int64_t *starts, const int64_t *goff, const int64_t *match_res,
    const int64_t *phys, const int64_t *gpu_ids, int64_t *h2d_gpu, int64_t *h2d_cpu, int64_t *cpu_out,
    int64_t *moved, int64_t *count) {
  __shared__ int64_t sums[kGetThreads];
  const int t = threadIdx.x;
  const int per = (num_req + kGetThreads - 1) / kGetThreads;
  const int r0 = t * per, r1 = min(num_req, r0 + per);
  int64_t mine = 0;
  for (int r = r0; r < r1; ++r) {
    const int64_t o = blk_off[r], n = blk_off[r + 1] - o, bs = starts[r];
    const int64_t ready = match_res[2 * (int64_t)r + 1];
    int64_t f = (ready < n ? ready : n) - bs;
    if (f < 0 || n == 0) f = 0;
    moved[r] = f;
    mine += f;
  }
  sums[t] = mine;
  __syncthreads();
  for (int d = 1; d < kGetThreads; d <<= 1) {  // inclusive scan (Hillis-Steele)
    const int64_t add = t >= d ? sums[t - d] : 0;
    __syncthreads();
    sums[t] += add;
    __syncthreads();
  }
  int64_t at = sums[t] - mine;  // exclusive prefix
  for (int r = r0; r < r1; ++r) {
    const int64_t o = blk_off[r], bs = starts[r], f = moved[r], go = goff[r];
    for (int64_t q = 0; q < f; ++q) {
      const int64_t c = phys[o + bs + q];
      h2d_gpu[at + q] = gpu_ids[go + q];
      h2d_cpu[at + q] = c;
      cpu_out[go + q] = c;
    }
    at += f;
  }
  if (t == kGetThreads - 1) *count = sums[t];
}

// Flag changes by hash (set_ready for a batch of blocks): ready or not.
__global__ void set_flags_kernel(Table t, const uint64_t *hashes, int64_t n, int ready, int64_t *found) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t f = 0;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n; q += stride) {
    const int64_t s = find(t, hashes[q]);
    if (s < 0) continue;
    if (ready) atomicOr(t.flags + s, kReadyBit);
    else atomicAnd(t.flags + s, ~kReadyBit);
    ++f;
  }
  if (f) atomicAdd(reinterpret_cast<unsigned long long *>(found), (unsigned long long)f);
}

// Remove entries by hash (the caller's eviction); out[q] = the pool block the
// entry held, or -1 when absent (or removed by an earlier duplicate).
__global__ void remove_kernel(Table t, const uint64_t *hashes, int64_t n, int64_t *out, int64_t *state) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t removed = 0;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n; q += stride) {
    const uint64_t key = hashes[q];
    const int64_t s = find(t, key);
    int64_t v = -1;
    if (s >= 0) {
      const int64_t held = t.vals[s];
      if (atomicCAS(reinterpret_cast<unsigned long long *>(t.keys + s), (unsigned long long)key,
                    (unsigned long long)kTomb) == key) {
        v = held;
        t.flags[s] = 0;
        ++removed;
      }
    }
    out[q] = v;
  }
  if (removed) {
    atomicAdd(reinterpret_cast<unsigned long long *>(state + kLive), (unsigned long long)(-removed));
    atomicAdd(reinterpret_cast<unsigned long long *>(state + kTombs), (unsigned long long)removed);
  }
}

// recycle_blocks (mempool.py:44-51): first check that no id is free...
__global__ void recycle_check_kernel(const uint8_t *free_mask, const int64_t *ids, int64_t n, int64_t *state) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n; q += stride)
    if (free_mask[ids[q]]) set_error(state, kErrRecycleFree, ids[q]);
}
// ...then free them all (the host refused repeated ids).
__global__ void recycle_apply_kernel(uint8_t *free_mask, const int64_t *ids, int64_t n, int64_t *state) {
  if (state[kErr] != kErrNone) return;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < n; q += stride) free_mask[ids[q]] = 1;
  if (blockIdx.x == 0 && threadIdx.x == 0) state[kNumFree] += n;
}

// CacheEngine.take(n, strict=False) without eviction: allocate
// min(n, num_free) ids (mempool.py:28-42).  One warp.
__global__ void __launch_bounds__(32) take_kernel(int64_t want, uint8_t *free_mask, int64_t mask_bytes,
                                                  int64_t *free_ids, int64_t *state, int64_t *out,
                                                  int64_t *got) {
  const int lane = threadIdx.x;
  int64_t num_free = state[kNumFree], list_len = state[kListLen], offset = state[kOffset];
  int64_t a = want < num_free ? want : num_free;
  if (a > list_len - offset) {
    list_len = rebuild_free_ids(free_mask, mask_bytes, free_ids, lane);
    offset = 0;
  }
  if (a > list_len - offset) a = list_len - offset;  // never reads past the snapshot
  for (int64_t t = lane; t < a; t += 32) {
    const int64_t c = free_ids[offset + t];
    free_mask[c] = 0;
    out[t] = c;
  }
  __syncwarp();
  if (lane == 0) {
    state[kNumFree] = num_free - a;
    state[kListLen] = list_len;
    state[kOffset] = offset + a;
    *got = a;
  }
}

// Ready entries (total_ready_blocks); live entries are counted in state.
__global__ void count_ready_kernel(Table t, int64_t *out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t c = 0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s <= (int64_t)t.mask; s += stride)
    c += (t.keys[s] < kTomb && (t.flags[s] & kReadyBit)) ? 1 : 0;
  c = __reduce_add_sync(0xffffffffu, (unsigned)c);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(reinterpret_cast<unsigned long long *>(out), (unsigned long long)c);
}

// Re-insert the live entries of `from` into the empty table `to` (drops
// the deleted slots once they make up a quarter of the table).
__global__ void rehash_kernel(Table from, Table to, int64_t *state) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s <= (int64_t)from.mask; s += stride) {
    const uint64_t k = from.keys[s];
    if (k >= kTomb) continue;
    bool tomb = false;
    if (insert_absent(to, k, from.vals[s], from.flags[s], &tomb) < 0) set_error(state, kErrFull, s);
  }
}

int grid_for(int64_t n, int threads = 256) {
  const int64_t g = (n + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 8));
}

uint64_t pow2_at_least(uint64_t x) {
  uint64_t p = 64;
  while (p < x) p <<= 1;
  return p;
}

int log2u(uint64_t p) {
  int l = 0;
  while ((1ull << l) < p) ++l;
  return l;
}

std::string err_message(int64_t code, int64_t arg) {
  switch (code) {
    case kErrFull: return "block index table is full";
    case kErrReserved: return "block " + std::to_string(arg) + " hashes to a value reserved by the index (2^64-1 or 2^64-2)";
    case kErrCollision: return "block " + std::to_string(arg) + ": its hash is already cached for a different prefix (hash collision)";
    case kErrRecycleFree: return "cannot recycle block " + std::to_string(arg) + ": it is already free";
    default: return "block index error " + std::to_string(code);
  }
}

}  // namespace
}  // namespace fkv

using namespace fkv;

struct fkv_cache_index {
  int device = -1;
  int tpb = 0;
  int64_t num_blocks = 0;
  uint64_t slots = 0;
  uint64_t *keys = nullptr;
  int64_t *vals = nullptr;
  uint32_t *flags = nullptr;
  uint8_t *free_mask = nullptr;
  int64_t mask_bytes = 0;
  int64_t *free_ids = nullptr;
  int64_t *state = nullptr;      // device [kStateWords]
  char *pin = nullptr;           // page-locked bounce for uploads and results
  size_t pin_cap = 0;
  cudaEvent_t decided = nullptr; // after a put's / get's results reached the bounce
  std::mutex mu;

  Table table() const {
    return Table{keys, vals, flags, slots - 1, 64 - log2u(slots)};
  }
};

namespace {

int ensure_pin(fkv_cache_index *ci, size_t bytes) {
  if (bytes <= ci->pin_cap) return FKV_OK;
  if (ci->pin) cudaFreeHost(ci->pin);
  ci->pin = nullptr;
  ci->pin_cap = 0;
  size_t cap = 1 << 16;
  while (cap < bytes) cap <<= 1;
  FKV_CUDA(cudaHostAlloc((void **)&ci->pin, cap, cudaHostAllocPortable));
  ci->pin_cap = cap;
  return FKV_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Device scratch carved into 16-byte aligned pieces, freed on the stream.
struct Scratch {
  char *base = nullptr;
  cudaStream_t s = nullptr;
  ~Scratch() {
    if (base) scratch_free(base, s);
  }
};
size_t al16(size_t x) { return (x + 15) & ~size_t(15); }

// Read the state words and the first error after a synchronize.
int read_state(fkv_cache_index *ci, cudaStream_t s, int64_t *st) {
  if (int rc = ensure_pin(ci, 8 * kStateWords)) return rc;
  FKV_CUDA(cudaMemcpyAsync(ci->pin, ci->state, 8 * kStateWords, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  std::memcpy(st, ci->pin, 8 * kStateWords);
  return FKV_OK;
}

// Fail with the recorded device error (and clear it so the index stays
// usable: every step that mutates state checks the word first).
int take_device_error(fkv_cache_index *ci, cudaStream_t s, const int64_t *st) {
  if (st[kErr] == kErrNone) return FKV_OK;
  const int code = st[kErr] == kErrRecycleFree ? FKV_ERR_INVALID_ARG : FKV_ERR_UNSUPPORTED;
  const std::string msg = err_message(st[kErr], st[kErrArg]);
  FKV_CUDA(cudaMemsetAsync(ci->state + kErr, 0, 16, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  return fail(code, msg);
}

// Block offsets of a batch from its token offsets (floor(len/tpb) blocks per
// sequence, SequenceMeta.num_blocks, flexkv/common/block.py:27-29).
int batch_offsets(const int64_t *seq_offsets, int num_seqs, int tpb, std::vector<int64_t> &blk) {
  blk.assign((size_t)num_seqs + 1, 0);
  for (int i = 0; i < num_seqs; ++i) {
    const int64_t a = seq_offsets[i], b = seq_offsets[i + 1];
    if (a < 0 || b < a) return fail(FKV_ERR_INVALID_ARG, "seq_offsets must be non-decreasing and non-negative");
    blk[i + 1] = blk[i] + (b - a) / tpb;
  }
  return FKV_OK;
}

// Hash a batch into hashes_dev (tokens may be host or device memory).
int hash_batch(fkv_cache_index *ci, const int64_t *token_ids, const int64_t *seq_offsets, int num_seqs,
               uint64_t *hashes_dev, cudaStream_t s, Scratch &tok_scratch) {
  const int64_t total_tokens = seq_offsets[num_seqs];
  int is_dev = 0, dev = -1;
  pointer_is_device(token_ids, &is_dev, &dev);
  const int64_t *tok = token_ids;
  if (!is_dev) {
    const size_t tb = 8 * (size_t)total_tokens;
    if (int rc = ensure_pin(ci, tb)) return rc;
    std::memcpy(ci->pin, token_ids, tb);
    tok_scratch.s = s;
    if (int rc = scratch_alloc(ci->device, tb, s, (void **)&tok_scratch.base)) return rc;
    FKV_CUDA(cudaMemcpyAsync(tok_scratch.base, ci->pin, tb, cudaMemcpyHostToDevice, s));
    tok = reinterpret_cast<const int64_t *>(tok_scratch.base);
  }
  if (int rc = fkv_gen_hashes_batched(tok, seq_offsets, num_seqs, ci->tpb, hashes_dev, s)) return rc;
  // the page-locked bounce is reused by the caller: wait for the upload
  if (!is_dev) FKV_CUDA(cudaStreamSynchronize(s));
  return FKV_OK;
}

int compact_if_needed(fkv_cache_index *ci, cudaStream_t s) {
  int64_t st[kStateWords];
  if (int rc = read_state(ci, s, st)) return rc;
  if ((uint64_t)st[kTombs] * 4 < ci->slots) return FKV_OK;
  Table from = ci->table();
  uint64_t *keys = nullptr;
  int64_t *vals = nullptr;
  uint32_t *flags = nullptr;
  FKV_CUDA(cudaMalloc(&keys, 8 * ci->slots));
  cudaError_t e = cudaMalloc(&vals, 8 * ci->slots);
  if (e == cudaSuccess) e = cudaMalloc(&flags, 4 * ci->slots);
  if (e != cudaSuccess) {
    cudaFree(keys);
    cudaFree(vals);
    return fail_cuda(e, "cudaMalloc(block index)");
  }
  Table to{keys, vals, flags, ci->slots - 1, from.shift};
  FKV_CUDA(cudaMemsetAsync(keys, 0xff, 8 * ci->slots, s));
  FKV_CUDA(cudaMemsetAsync(flags, 0, 4 * ci->slots, s));
  rehash_kernel<<<grid_for((int64_t)ci->slots), 256, 0, s>>>(from, to, ci->state);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  FKV_CUDA(cudaMemsetAsync(ci->state + kTombs, 0, 8, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  cudaFree(ci->keys);
  cudaFree(ci->vals);
  cudaFree(ci->flags);
  ci->keys = keys;
  ci->vals = vals;
  ci->flags = flags;
  if (int rc = read_state(ci, s, st)) return rc;
  return take_device_error(ci, s, st);
}

}  // namespace

extern "C" {

int fkv_cache_index_create(int device, int64_t num_total_blocks, int tokens_per_block, fkv_cache_index **out) {
  clear_error();
  if (!out) return fail(FKV_ERR_INVALID_ARG, "null output");
  *out = nullptr;
  if (num_total_blocks <= 0 || num_total_blocks >= (1ll << 31))
    return fail(FKV_ERR_INVALID_ARG, "num_total_blocks must be in [1, 2^31)");
  if (tokens_per_block <= 0) return fail(FKV_ERR_INVALID_ARG, "tokens_per_block must be positive");
  if (device < 0) FKV_CUDA(cudaGetDevice(&device));
  DeviceGuard g(device);
  auto *ci = new fkv_cache_index();
  ci->device = device;
  ci->tpb = tokens_per_block;
  ci->num_blocks = num_total_blocks;
  ci->slots = pow2_at_least(2 * (uint64_t)num_total_blocks);
  ci->mask_bytes = (num_total_blocks + 511) / 512 * 512;
  cudaError_t e = cudaMalloc(&ci->keys, 8 * ci->slots);
  if (e == cudaSuccess) e = cudaMalloc(&ci->vals, 8 * ci->slots);
  if (e == cudaSuccess) e = cudaMalloc(&ci->flags, 4 * ci->slots);
  if (e == cudaSuccess) e = cudaMalloc(&ci->free_mask, ci->mask_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&ci->free_ids, 8 * num_total_blocks);
  if (e == cudaSuccess) e = cudaMalloc(&ci->state, 8 * kStateWords);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ci->decided, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaMemset(ci->keys, 0xff, 8 * ci->slots);
  if (e == cudaSuccess) e = cudaMemset(ci->flags, 0, 4 * ci->slots);
  if (e == cudaSuccess) {
    init_pool_kernel<<<grid_for(ci->mask_bytes), 256>>>(ci->free_mask, ci->mask_bytes, ci->free_ids,
                                                         num_total_blocks, ci->state);
    e = cudaGetLastError();
    note_launch();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    fkv_cache_index_destroy(ci);
    return fail_cuda(e, "fkv_cache_index_create");
  }
  *out = ci;
  return FKV_OK;
}

void fkv_cache_index_destroy(fkv_cache_index *ci) {
  if (!ci) return;
  {
    DeviceGuard g(ci->device);
    cudaFree(ci->keys);
    cudaFree(ci->vals);
    cudaFree(ci->flags);
    cudaFree(ci->free_mask);
    cudaFree(ci->free_ids);
    cudaFree(ci->state);
    if (ci->decided) cudaEventDestroy(ci->decided);
    if (ci->pin) cudaFreeHost(ci->pin);
  }
  delete ci;
}

int fkv_cache_index_match(fkv_cache_index *ci, const int64_t *token_ids, const int64_t *seq_offsets,
                          int num_seqs, int64_t *num_matched, int64_t *num_ready, int64_t *physical_blocks,
                          void *stream) {
  clear_error();
  if (!ci) return fail(FKV_ERR_INVALID_ARG, "null index");
  if (num_seqs < 0 || (num_seqs > 0 && (!seq_offsets || !num_matched || !num_ready)))
    return fail(FKV_ERR_INVALID_ARG, "bad batch description");
  if (num_seqs == 0) return FKV_OK;
  std::lock_guard<std::mutex> lk(ci->mu);
  DeviceGuard g(ci->device);
  cudaStream_t s = (cudaStream_t)stream;
  std::vector<int64_t> blk;
  if (int rc = batch_offsets(seq_offsets, num_seqs, ci->tpb, blk)) return rc;
  const int64_t nb = blk[num_seqs];
  if (nb == 0) {
    for (int r = 0; r < num_seqs; ++r) num_matched[r] = num_ready[r] = 0;
    return FKV_OK;
  }
  if (!token_ids) return fail(FKV_ERR_INVALID_ARG, "null token ids");
  const size_t o_hash = 0, o_off = al16(o_hash + 8 * nb), o_res = al16(o_off + 8 * (num_seqs + 1)),
               o_phys = al16(o_res + 16 * (size_t)num_seqs), total = al16(o_phys + 8 * nb);
  Scratch sc, tok;
  sc.s = s;
  if (int rc = scratch_alloc(ci->device, total, s, (void **)&sc.base)) return rc;
  uint64_t *hashes = reinterpret_cast<uint64_t *>(sc.base + o_hash);
  int64_t *d_off = reinterpret_cast<int64_t *>(sc.base + o_off);
  int64_t *d_res = reinterpret_cast<int64_t *>(sc.base + o_res);
  int64_t *d_phys = reinterpret_cast<int64_t *>(sc.base + o_phys);
  if (int rc = hash_batch(ci, token_ids, seq_offsets, num_seqs, hashes, s, tok)) return rc;
  if (int rc = ensure_pin(ci, std::max<size_t>(8 * (num_seqs + 1), 16 * (size_t)num_seqs + 8 * nb))) return rc;
  std::memcpy(ci->pin, blk.data(), 8 * (num_seqs + 1));
  FKV_CUDA(cudaMemcpyAsync(d_off, ci->pin, 8 * (num_seqs + 1), cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaStreamSynchronize(s));  // the bounce is reused for the results
  match_kernel<<<grid_for(32ll * num_seqs), 256, 0, s>>>(ci->table(), hashes, d_off, num_seqs, d_res, d_phys);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  FKV_CUDA(cudaMemcpyAsync(ci->pin, d_res, 16 * (size_t)num_seqs, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(ci->pin + 16 * (size_t)num_seqs, d_phys, 8 * nb, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  const int64_t *res = reinterpret_cast<const int64_t *>(ci->pin);
  for (int r = 0; r < num_seqs; ++r) {
    num_matched[r] = res[2 * r];
    num_ready[r] = res[2 * r + 1];
  }
  if (physical_blocks) std::memcpy(physical_blocks, ci->pin + 16 * (size_t)num_seqs, 8 * nb);
  return FKV_OK;
}

int fkv_cache_index_put(fkv_cache_index *ci, const int64_t *token_ids, const int64_t *seq_offsets, int num_seqs,
                        const int64_t *gpu_block_ids, const fkv_transfer_desc *layout, int mark_ready,
                        int synchronous, int64_t *num_skipped, int64_t *num_transferred,
                        int64_t *cpu_block_ids, uint64_t *block_hashes, void *stream) {
  clear_error();
  if (!ci || !layout) return fail(FKV_ERR_INVALID_ARG, "null index or layout");
  if (num_seqs < 0 || (num_seqs > 0 && (!seq_offsets || !num_skipped || !num_transferred)))
    return fail(FKV_ERR_INVALID_ARG, "bad batch description");
  if (num_seqs == 0) return FKV_OK;
  std::lock_guard<std::mutex> lk(ci->mu);
  DeviceGuard g(ci->device);
  cudaStream_t s = (cudaStream_t)stream;
  std::vector<int64_t> blk;
  if (int rc = batch_offsets(seq_offsets, num_seqs, ci->tpb, blk)) return rc;
  const int64_t nb = blk[num_seqs];
  for (int r = 0; r < num_seqs; ++r) num_skipped[r] = num_transferred[r] = 0;
  if (nb == 0) return FKV_OK;
  if (!token_ids || !gpu_block_ids) return fail(FKV_ERR_INVALID_ARG, "null token ids or gpu block ids");
  if (nb >= (1ll << 29)) return fail(FKV_ERR_INVALID_ARG, "too many blocks in one batch (limit 2^29)");
  if (layout->is_host_to_device) return fail(FKV_ERR_INVALID_ARG, "the put path copies device to host");
  // The copy's layout is checked before any state changes.
  if (int rc = transfer_check_device_ids(*layout, nb, ci->num_blocks - 1)) return rc;

  // GPU ids: on the host for the checks the copy kernel does not make.
  std::vector<int64_t> gids((size_t)nb);
  int gdev = 0, gd = -1;
  pointer_is_device(gpu_block_ids, &gdev, &gd);
  if (gdev) FKV_CUDA(cudaMemcpy(gids.data(), gpu_block_ids, 8 * nb, cudaMemcpyDeviceToHost));
  else std::memcpy(gids.data(), gpu_block_ids, 8 * nb);
  const int64_t gbs = (layout->gpu_block_stride_in_bytes / 8) * 8;
  const int64_t gkv = (layout->gpu_kv_stride_in_bytes / 8) * 8;
  const int64_t copy_bytes = (layout->chunk_size_in_bytes / 16) * 16;
  const int64_t gpu_extent = (layout->is_mla ? 0 : gkv) + copy_bytes;
  for (int64_t i = 0; i < nb; ++i) {
    const int64_t gi = gids[i];
    if (gi < 0 || gi >= (1ll << 31))
      return fail(FKV_ERR_OUT_OF_RANGE, "gpu block id out of [0, 2^31) at index " + std::to_string(i));
    if (layout->gpu_layer_bytes > 0 && gi * gbs + gpu_extent > layout->gpu_layer_bytes)
      return fail(FKV_ERR_OUT_OF_RANGE, "gpu block id " + std::to_string(gi) + " at index " +
                                            std::to_string(i) + " addresses past the gpu layer");
  }

  // Device scratch.
  const uint64_t lslots = pow2_at_least(2 * (uint64_t)nb);
  size_t off = 0;
  auto carve = [&](size_t bytes) { const size_t at = off; off = al16(off + bytes); return at; };
  const size_t o_hash = carve(8 * nb), o_before = carve(nb), o_lslot = carve(4 * nb),
               o_lkeys = carve(8 * lslots), o_ins = carve(4 * lslots), o_off = carve(8 * (num_seqs + 1)),
               o_gid = carve(8 * nb), o_res = carve(24 * (size_t)num_seqs), o_cpu = carve(8 * nb),
               o_d2hg = carve(8 * nb), o_d2hc = carve(8 * nb), o_new = carve(8 * nb), o_slot = carve(8 * nb),
               o_cnt = carve(16), o_first = carve(4 * lslots);
  Scratch sc, tok;
  sc.s = s;
  if (int rc = scratch_alloc(ci->device, off, s, (void **)&sc.base)) return rc;
  char *b = sc.base;
  uint64_t *hashes = reinterpret_cast<uint64_t *>(b + o_hash);
  int64_t *d_cnt = reinterpret_cast<int64_t *>(b + o_cnt);
  if (int rc = hash_batch(ci, token_ids, seq_offsets, num_seqs, hashes, s, tok)) return rc;

  // Upload block offsets and GPU ids through the bounce buffer.
  const size_t up_off = 8 * (num_seqs + 1), up = up_off + 8 * nb;
  const size_t down_res = 24 * (size_t)num_seqs, down = down_res + 16 * nb + 8 * kStateWords;
  if (int rc = ensure_pin(ci, std::max(up, down))) return rc;
  std::memcpy(ci->pin, blk.data(), up_off);
  std::memcpy(ci->pin + up_off, gids.data(), 8 * nb);
  FKV_CUDA(cudaMemcpyAsync(b + o_off, ci->pin, up_off, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemcpyAsync(b + o_gid, ci->pin + up_off, 8 * nb, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemsetAsync(b + o_lkeys, 0xff, 8 * lslots, s));
  FKV_CUDA(cudaMemsetAsync(b + o_ins, 0x7f, 4 * lslots, s));  // 0x7f7f7f7f: after every request
  FKV_CUDA(cudaMemsetAsync(b + o_first, 0x7f, 4 * lslots, s));
  FKV_CUDA(cudaMemsetAsync(b + o_cpu, 0xff, 8 * nb, s));      // -1: not moved
  FKV_CUDA(cudaMemsetAsync(d_cnt, 0, 16, s));  // d_cnt[0] = count, d_cnt[1] = decided by the parallel kernel

  const Table t = ci->table();
  put_lookup_kernel<<<grid_for(nb), 256, 0, s>>>(t, hashes, nb, reinterpret_cast<uint8_t *>(b + o_before),
                                                  reinterpret_cast<uint64_t *>(b + o_lkeys), lslots - 1,
                                                  64 - log2u(lslots), reinterpret_cast<int32_t *>(b + o_lslot),
                                                  ci->state);
  FKV_CUDA(cudaGetLastError());
  put_decide_fast_kernel<<<1, kDecideThreads, 0, s>>>(
      num_seqs, reinterpret_cast<int64_t *>(b + o_off), reinterpret_cast<uint8_t *>(b + o_before),
      reinterpret_cast<int32_t *>(b + o_lslot), reinterpret_cast<int32_t *>(b + o_first),
      reinterpret_cast<int64_t *>(b + o_gid), ci->free_mask, ci->free_ids, ci->state,
      reinterpret_cast<int64_t *>(b + o_res), reinterpret_cast<int64_t *>(b + o_cpu),
      reinterpret_cast<int64_t *>(b + o_d2hg), reinterpret_cast<int64_t *>(b + o_d2hc),
      reinterpret_cast<int64_t *>(b + o_new), d_cnt, d_cnt + 1);
  FKV_CUDA(cudaGetLastError());
  put_decide_kernel<<<1, 32, 0, s>>>(num_seqs, reinterpret_cast<int64_t *>(b + o_off),
                                     reinterpret_cast<uint8_t *>(b + o_before),
                                     reinterpret_cast<int32_t *>(b + o_lslot), reinterpret_cast<int32_t *>(b + o_ins),
                                     reinterpret_cast<int64_t *>(b + o_gid), ci->free_mask, ci->mask_bytes,
                                     ci->free_ids, ci->state, reinterpret_cast<int64_t *>(b + o_res),
                                     reinterpret_cast<int64_t *>(b + o_cpu), reinterpret_cast<int64_t *>(b + o_d2hg),
                                     reinterpret_cast<int64_t *>(b + o_d2hc), reinterpret_cast<int64_t *>(b + o_new),
                                     d_cnt, d_cnt + 1);
  FKV_CUDA(cudaGetLastError());
  put_insert_kernel<<<grid_for(nb), 256, 0, s>>>(t, hashes, reinterpret_cast<int64_t *>(b + o_new),
                                                  reinterpret_cast<int64_t *>(b + o_cpu), d_cnt,
                                                  reinterpret_cast<int64_t *>(b + o_slot), ci->state);
  FKV_CUDA(cudaGetLastError());
  note_launch(4);
  // The decisions go back before the copy, so an asynchronous caller gets
  // them as soon as they exist (the reference's put returns its graph and
  // mask before the transfer runs).
  FKV_CUDA(cudaMemcpyAsync(ci->pin, b + o_res, down_res, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(ci->pin + down_res, b + o_cpu, 8 * nb, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(ci->pin + down_res + 8 * nb, hashes, 8 * nb, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(ci->pin + down_res + 16 * nb, ci->state, 8 * kStateWords, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaEventRecord(ci->decided, s));
  fkv_transfer_desc d = *layout;
  d.is_host_to_device = 0;
  if (int rc = transfer_enqueue_device_ids(d, reinterpret_cast<int64_t *>(b + o_d2hg),
                                           reinterpret_cast<int64_t *>(b + o_d2hc), d_cnt, nb,
                                           ci->num_blocks - 1, s))
    return rc;
  if (mark_ready) {
    mark_slots_ready_kernel<<<grid_for(nb), 256, 0, s>>>(t, reinterpret_cast<int64_t *>(b + o_slot), d_cnt);
    FKV_CUDA(cudaGetLastError());
    note_launch();
  }
  if (synchronous) FKV_CUDA(cudaStreamSynchronize(s));
  else FKV_CUDA(cudaEventSynchronize(ci->decided));
  int64_t st[kStateWords];
  std::memcpy(st, ci->pin + down_res + 16 * nb, 8 * kStateWords);
  if (int rc = take_device_error(ci, s, st)) return rc;
  const int64_t *res = reinterpret_cast<const int64_t *>(ci->pin);
  for (int r = 0; r < num_seqs; ++r) {
    num_skipped[r] = res[3 * r];
    num_transferred[r] = res[3 * r + 1];
  }
  if (cpu_block_ids) std::memcpy(cpu_block_ids, ci->pin + down_res, 8 * nb);
  if (block_hashes) std::memcpy(block_hashes, ci->pin + down_res + 8 * nb, 8 * nb);
  return FKV_OK;
}

int fkv_cache_index_put2(fkv_cache_index *cpu, fkv_cache_index *ssd, const int64_t *token_ids,
                         const int64_t *seq_offsets, int num_seqs, const int64_t *gpu_block_ids,
                         const fkv_transfer_desc *layout, int mark_ready, int64_t *num_skipped,
                         int64_t *num_transferred, int64_t *num_to_ssd, int64_t *cpu_block_ids,
                         int64_t *ssd_block_ids, uint64_t *block_hashes, void *stream) {
  clear_error();
  if (!cpu || !ssd || !layout || cpu == ssd) return fail(FKV_ERR_INVALID_ARG, "need two distinct indexes and a layout");
  if (cpu->device != ssd->device || cpu->tpb != ssd->tpb)
    return fail(FKV_ERR_INVALID_ARG, "the CPU and SSD indexes must share the device and tokens_per_block");
  if (num_seqs < 0 || (num_seqs > 0 && (!seq_offsets || !num_skipped || !num_transferred || !num_to_ssd)))
    return fail(FKV_ERR_INVALID_ARG, "bad batch description");
  if (num_seqs == 0) return FKV_OK;
  std::scoped_lock lk(cpu->mu, ssd->mu);
  DeviceGuard g(cpu->device);
  cudaStream_t s = (cudaStream_t)stream;
  std::vector<int64_t> blk;
  if (int rc = batch_offsets(seq_offsets, num_seqs, cpu->tpb, blk)) return rc;
  const int64_t nb = blk[num_seqs];
  for (int r = 0; r < num_seqs; ++r) num_skipped[r] = num_transferred[r] = num_to_ssd[r] = 0;
  if (nb == 0) return FKV_OK;
  if (!token_ids || !gpu_block_ids) return fail(FKV_ERR_INVALID_ARG, "null token ids or gpu block ids");
  if (nb >= (1ll << 29)) return fail(FKV_ERR_INVALID_ARG, "too many blocks in one batch (limit 2^29)");
  if (layout->is_host_to_device) return fail(FKV_ERR_INVALID_ARG, "the put path copies device to host");
  if (int rc = transfer_check_device_ids(*layout, nb, cpu->num_blocks - 1)) return rc;
  std::vector<int64_t> gids((size_t)nb);
  int gdev = 0, gd = -1;
  pointer_is_device(gpu_block_ids, &gdev, &gd);
  if (gdev) FKV_CUDA(cudaMemcpy(gids.data(), gpu_block_ids, 8 * nb, cudaMemcpyDeviceToHost));
  else std::memcpy(gids.data(), gpu_block_ids, 8 * nb);
  const int64_t gbs = (layout->gpu_block_stride_in_bytes / 8) * 8;
  const int64_t gkv = (layout->gpu_kv_stride_in_bytes / 8) * 8;
  const int64_t gpu_extent = (layout->is_mla ? 0 : gkv) + (layout->chunk_size_in_bytes / 16) * 16;
  for (int64_t i = 0; i < nb; ++i) {
    const int64_t gi = gids[i];
    if (gi < 0 || gi >= (1ll << 31))
      return fail(FKV_ERR_OUT_OF_RANGE, "gpu block id out of [0, 2^31) at index " + std::to_string(i));
    if (layout->gpu_layer_bytes > 0 && gi * gbs + gpu_extent > layout->gpu_layer_bytes)
      return fail(FKV_ERR_OUT_OF_RANGE, "gpu block id " + std::to_string(gi) + " at index " +
                                            std::to_string(i) + " addresses past the gpu layer");
  }
  const uint64_t lslots = pow2_at_least(2 * (uint64_t)nb);
  size_t off = 0;
  auto carve = [&](size_t bytes) { const size_t at = off; off = al16(off + bytes); return at; };
  const size_t o_hash = carve(8 * nb), o_bc = carve(nb), o_bs = carve(nb), o_phys = carve(8 * nb),
               o_rdy = carve(nb), o_lslot = carve(4 * nb), o_lkeys = carve(8 * lslots), o_insc = carve(4 * lslots),
               o_inss = carve(4 * lslots), o_scpu = carve(8 * lslots), o_off = carve(8 * (num_seqs + 1)),
               o_gid = carve(8 * nb), o_res = carve(32 * (size_t)num_seqs), o_cpu = carve(8 * nb),
               o_ssd = carve(8 * nb), o_d2hg = carve(8 * nb), o_d2hc = carve(8 * nb), o_newc = carve(8 * nb),
               o_news = carve(8 * nb), o_slotc = carve(8 * nb), o_slots = carve(8 * nb), o_cnt = carve(16);
  Scratch sc, tok;
  sc.s = s;
  if (int rc = scratch_alloc(cpu->device, off, s, (void **)&sc.base)) return rc;
  char *b = sc.base;
  auto I64 = [&](size_t o) { return reinterpret_cast<int64_t *>(b + o); };
  uint64_t *hashes = reinterpret_cast<uint64_t *>(b + o_hash);
  int64_t *counts = I64(o_cnt);
  if (int rc = hash_batch(cpu, token_ids, seq_offsets, num_seqs, hashes, s, tok)) return rc;
  const size_t up_off = 8 * (num_seqs + 1);
  const size_t down_res = 32 * (size_t)num_seqs, down = down_res + 24 * nb + 16 * kStateWords;
  if (int rc = ensure_pin(cpu, std::max(up_off + 8 * nb, down))) return rc;
  std::memcpy(cpu->pin, blk.data(), up_off);
  std::memcpy(cpu->pin + up_off, gids.data(), 8 * nb);
  FKV_CUDA(cudaMemcpyAsync(b + o_off, cpu->pin, up_off, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemcpyAsync(b + o_gid, cpu->pin + up_off, 8 * nb, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemsetAsync(b + o_lkeys, 0xff, 8 * lslots, s));
  FKV_CUDA(cudaMemsetAsync(b + o_insc, 0x7f, 4 * lslots, s));
  FKV_CUDA(cudaMemsetAsync(b + o_inss, 0x7f, 4 * lslots, s));
  FKV_CUDA(cudaMemsetAsync(b + o_cpu, 0xff, 8 * nb, s));
  FKV_CUDA(cudaMemsetAsync(b + o_ssd, 0xff, 8 * nb, s));
  FKV_CUDA(cudaMemsetAsync(counts, 0, 16, s));
  const Table tc = cpu->table(), ts = ssd->table();
  put_lookup_kernel<<<grid_for(nb), 256, 0, s>>>(tc, hashes, nb, reinterpret_cast<uint8_t *>(b + o_bc),
                                                  reinterpret_cast<uint64_t *>(b + o_lkeys), lslots - 1,
                                                  64 - log2u(lslots), reinterpret_cast<int32_t *>(b + o_lslot),
                                                  cpu->state);
  FKV_CUDA(cudaGetLastError());
  tier_lookup_kernel<<<grid_for(nb), 256, 0, s>>>(tc, hashes, nb, reinterpret_cast<uint8_t *>(b + o_bc), I64(o_phys),
                                                   reinterpret_cast<uint8_t *>(b + o_rdy));
  FKV_CUDA(cudaGetLastError());
  tier_lookup_kernel<<<grid_for(nb), 256, 0, s>>>(ts, hashes, nb, reinterpret_cast<uint8_t *>(b + o_bs), nullptr,
                                                   nullptr);
  FKV_CUDA(cudaGetLastError());
  const PoolRef pc{cpu->free_mask, cpu->mask_bytes, cpu->free_ids, cpu->state};
  const PoolRef ps{ssd->free_mask, ssd->mask_bytes, ssd->free_ids, ssd->state};
  put2_decide_kernel<<<1, 32, 0, s>>>(num_seqs, I64(o_off), reinterpret_cast<uint8_t *>(b + o_bc),
                                      reinterpret_cast<uint8_t *>(b + o_bs), I64(o_phys),
                                      reinterpret_cast<uint8_t *>(b + o_rdy), reinterpret_cast<int32_t *>(b + o_lslot), reinterpret_cast<int32_t *>(b + o_insc),
                                      reinterpret_cast<int32_t *>(b + o_inss), I64(o_scpu), I64(o_gid), pc, ps,
                                      I64(o_res), I64(o_cpu), I64(o_ssd), I64(o_d2hg), I64(o_d2hc), I64(o_newc),
                                      I64(o_news), counts);
  FKV_CUDA(cudaGetLastError());
  put_insert_kernel<<<grid_for(nb), 256, 0, s>>>(tc, hashes, I64(o_newc), I64(o_cpu), counts, I64(o_slotc), cpu->state);
  FKV_CUDA(cudaGetLastError());
  put_insert_kernel<<<grid_for(nb), 256, 0, s>>>(ts, hashes, I64(o_news), I64(o_ssd), counts + 1, I64(o_slots),
                                                  ssd->state);
  FKV_CUDA(cudaGetLastError());
  note_launch(6);
  char *pin = cpu->pin;
  FKV_CUDA(cudaMemcpyAsync(pin, b + o_res, down_res, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(pin + down_res, b + o_cpu, 8 * nb, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(pin + down_res + 8 * nb, b + o_ssd, 8 * nb, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(pin + down_res + 16 * nb, hashes, 8 * nb, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(pin + down_res + 24 * nb, cpu->state, 8 * kStateWords, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(pin + down_res + 24 * nb + 8 * kStateWords, ssd->state, 8 * kStateWords,
                           cudaMemcpyDeviceToHost, s));
  fkv_transfer_desc d = *layout;
  d.is_host_to_device = 0;
  if (int rc = transfer_enqueue_device_ids(d, I64(o_d2hg), I64(o_d2hc), counts, nb, cpu->num_blocks - 1, s))
    return rc;
  if (mark_ready) {
    mark_slots_ready_kernel<<<grid_for(nb), 256, 0, s>>>(tc, I64(o_slotc), counts);
    FKV_CUDA(cudaGetLastError());
    note_launch();
  }
  FKV_CUDA(cudaStreamSynchronize(s));
  int64_t st_c[kStateWords], st_s[kStateWords];
  std::memcpy(st_c, pin + down_res + 24 * nb, 8 * kStateWords);
  std::memcpy(st_s, pin + down_res + 24 * nb + 8 * kStateWords, 8 * kStateWords);
  if (int rc = take_device_error(cpu, s, st_c)) return rc;
  if (int rc = take_device_error(ssd, s, st_s)) return rc;
  const int64_t *res = reinterpret_cast<const int64_t *>(pin);
  for (int r = 0; r < num_seqs; ++r) {
    num_skipped[r] = res[4 * r];
    num_transferred[r] = res[4 * r + 1];
    num_to_ssd[r] = res[4 * r + 2];
  }
  if (cpu_block_ids) std::memcpy(cpu_block_ids, pin + down_res, 8 * nb);
  if (ssd_block_ids) std::memcpy(ssd_block_ids, pin + down_res + 8 * nb, 8 * nb);
  if (block_hashes) std::memcpy(block_hashes, pin + down_res + 16 * nb, 8 * nb);
  return FKV_OK;
}

int fkv_cache_index_get(fkv_cache_index *ci, const int64_t *token_ids, const int64_t *seq_offsets, int num_seqs,
                        const int64_t *block_starts, const int64_t *gpu_block_ids, const fkv_transfer_desc *layout,
                        int layer_granularity, void *const *group_events, int synchronous,
                        int64_t *num_transferred, int64_t *cpu_block_ids, void *stream) {
  clear_error();
  if (!ci || !layout) return fail(FKV_ERR_INVALID_ARG, "null index or layout");
  if (num_seqs < 0 || (num_seqs > 0 && (!seq_offsets || !num_transferred)))
    return fail(FKV_ERR_INVALID_ARG, "bad batch description");
  if (num_seqs == 0) return FKV_OK;
  std::lock_guard<std::mutex> lk(ci->mu);
  DeviceGuard g(ci->device);
  cudaStream_t s = (cudaStream_t)stream;
  std::vector<int64_t> blk;
  if (int rc = batch_offsets(seq_offsets, num_seqs, ci->tpb, blk)) return rc;
  const int64_t nb = blk[num_seqs];
  for (int r = 0; r < num_seqs; ++r) num_transferred[r] = 0;
  // GPU entries: request r brings n_r - start_r GPU blocks (the mask's range).
  std::vector<int64_t> starts((size_t)num_seqs, 0), goff((size_t)num_seqs + 1, 0);
  for (int r = 0; r < num_seqs; ++r) {
    const int64_t n = blk[r + 1] - blk[r];
    const int64_t bs = block_starts ? block_starts[r] : 0;
    if (n > 0 && (bs < 0 || bs >= n))
      return fail(FKV_ERR_INVALID_ARG, "block_starts[" + std::to_string(r) + "] must lie in [0, blocks)");
    starts[r] = n > 0 ? bs : 0;
    goff[r + 1] = goff[r] + (n - starts[r]);
  }
  const int64_t ng = goff[num_seqs];
  if (nb == 0) return FKV_OK;
  if (!token_ids || !gpu_block_ids) return fail(FKV_ERR_INVALID_ARG, "null token ids or gpu block ids");
  if (nb >= (1ll << 29)) return fail(FKV_ERR_INVALID_ARG, "too many blocks in one batch (limit 2^29)");
  if (!layout->is_host_to_device) return fail(FKV_ERR_INVALID_ARG, "the get path copies host to device");
  const int L = layout->num_layers;
  const int G = layer_granularity > 0 ? layer_granularity : L;
  if (L > 0 && (G > L || L % G != 0))  // transfer_pattern.py:377
    return fail(FKV_ERR_INVALID_ARG, "layer_granularity must divide the number of layers");
  if (int rc = transfer_check_device_ids(*layout, ng, ci->num_blocks - 1)) return rc;
  std::vector<int64_t> gids((size_t)ng);
  int gdev = 0, gd = -1;
  pointer_is_device(gpu_block_ids, &gdev, &gd);
  if (gdev) FKV_CUDA(cudaMemcpy(gids.data(), gpu_block_ids, 8 * ng, cudaMemcpyDeviceToHost));
  else std::memcpy(gids.data(), gpu_block_ids, 8 * ng);
  const int64_t gbs = (layout->gpu_block_stride_in_bytes / 8) * 8;
  const int64_t gkv = (layout->gpu_kv_stride_in_bytes / 8) * 8;
  const int64_t gpu_extent = (layout->is_mla ? 0 : gkv) + (layout->chunk_size_in_bytes / 16) * 16;
  for (int64_t i = 0; i < ng; ++i) {
    const int64_t gi = gids[i];
    if (gi < 0 || gi >= (1ll << 31))
      return fail(FKV_ERR_OUT_OF_RANGE, "gpu block id out of [0, 2^31) at index " + std::to_string(i));
    if (layout->gpu_layer_bytes > 0 && gi * gbs + gpu_extent > layout->gpu_layer_bytes)
      return fail(FKV_ERR_OUT_OF_RANGE, "gpu block id " + std::to_string(gi) + " at index " +
                                            std::to_string(i) + " addresses past the gpu layer");
  }
  size_t off = 0;
  auto carve = [&](size_t bytes) { const size_t at = off; off = al16(off + bytes); return at; };
  const size_t R1 = (size_t)num_seqs + 1;
  const size_t o_hash = carve(8 * nb), o_off = carve(8 * R1), o_start = carve(8 * num_seqs), o_goff = carve(8 * R1),
               o_res = carve(16 * (size_t)num_seqs), o_phys = carve(8 * nb), o_gid = carve(8 * ng + 8),
               o_h2dg = carve(8 * ng + 8), o_h2dc = carve(8 * ng + 8), o_cpu = carve(8 * ng + 8),
               o_moved = carve(8 * num_seqs), o_cnt = carve(16);
  Scratch sc, tok;
  sc.s = s;
  if (int rc = scratch_alloc(ci->device, off, s, (void **)&sc.base)) return rc;
  char *b = sc.base;
  uint64_t *hashes = reinterpret_cast<uint64_t *>(b + o_hash);
  int64_t *d_cnt = reinterpret_cast<int64_t *>(b + o_cnt);
  if (int rc = hash_batch(ci, token_ids, seq_offsets, num_seqs, hashes, s, tok)) return rc;
  const size_t up = 8 * (R1 + num_seqs + R1 + ng);
  const size_t down = 8 * (size_t)num_seqs + 8 * ng;
  if (int rc = ensure_pin(ci, std::max(up, down))) return rc;
  int64_t *pin = reinterpret_cast<int64_t *>(ci->pin);
  std::memcpy(pin, blk.data(), 8 * R1);
  std::memcpy(pin + R1, starts.data(), 8 * num_seqs);
  std::memcpy(pin + R1 + num_seqs, goff.data(), 8 * R1);
  std::memcpy(pin + 2 * R1 + num_seqs, gids.data(), 8 * ng);
  FKV_CUDA(cudaMemcpyAsync(b + o_off, pin, 8 * R1, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemcpyAsync(b + o_start, pin + R1, 8 * num_seqs, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemcpyAsync(b + o_goff, pin + R1 + num_seqs, 8 * R1, cudaMemcpyHostToDevice, s));
  if (ng) FKV_CUDA(cudaMemcpyAsync(b + o_gid, pin + 2 * R1 + num_seqs, 8 * ng, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemsetAsync(b + o_cpu, 0xff, 8 * ng + 8, s));  // -1: not read
  FKV_CUDA(cudaMemsetAsync(d_cnt, 0, 16, s));
  const int64_t *d_off = reinterpret_cast<int64_t *>(b + o_off);
  int64_t *d_res = reinterpret_cast<int64_t *>(b + o_res);
  int64_t *d_phys = reinterpret_cast<int64_t *>(b + o_phys);
  match_kernel<<<grid_for(32ll * num_seqs), 256, 0, s>>>(ci->table(), hashes, d_off, num_seqs, d_res, d_phys);
  FKV_CUDA(cudaGetLastError());
  get_lists_kernel<<<1, kGetThreads, 0, s>>>(num_seqs, d_off, reinterpret_cast<int64_t *>(b + o_start),
                                    reinterpret_cast<int64_t *>(b + o_goff), d_res, d_phys,
                                    reinterpret_cast<int64_t *>(b + o_gid), reinterpret_cast<int64_t *>(b + o_h2dg),
                                    reinterpret_cast<int64_t *>(b + o_h2dc), reinterpret_cast<int64_t *>(b + o_cpu),
                                    reinterpret_cast<int64_t *>(b + o_moved), d_cnt);
  FKV_CUDA(cudaGetLastError());
  note_launch(2);
  FKV_CUDA(cudaMemcpyAsync(pin, b + o_moved, 8 * num_seqs, cudaMemcpyDeviceToHost, s));
  if (ng) FKV_CUDA(cudaMemcpyAsync(pin + num_seqs, b + o_cpu, 8 * ng, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaEventRecord(ci->decided, s));
  // One copy per layer group, in order (convert_read_graph_to_layer_wise_graph,
  // transfer_pattern.py:370-428: group i after group i-1); the caller's event
  // for group i marks its layers as loaded (wait_at_layer_group).
  {
    fkv_transfer_desc d = *layout;
    d.is_host_to_device = 1;
    if (ng > 0) {
      if (int rc = transfer_enqueue_device_ids(d, reinterpret_cast<int64_t *>(b + o_h2dg),
                                               reinterpret_cast<int64_t *>(b + o_h2dc), d_cnt, ng,
                                               ci->num_blocks - 1, s, G, group_events))
        return rc;
    } else if (group_events) {
      for (int g0 = 0; g0 < L; g0 += G)
        if (group_events[g0 / G]) FKV_CUDA(cudaEventRecord((cudaEvent_t)group_events[g0 / G], s));
    }
  }
  if (synchronous) FKV_CUDA(cudaStreamSynchronize(s));
  else FKV_CUDA(cudaEventSynchronize(ci->decided));
  std::memcpy(num_transferred, pin, 8 * num_seqs);
  if (cpu_block_ids && ng) std::memcpy(cpu_block_ids, pin + num_seqs, 8 * ng);
  return FKV_OK;
}

int fkv_cache_index_set_ready(fkv_cache_index *ci, const uint64_t *block_hashes, int64_t n, int ready,
                              int64_t *num_found, void *stream) {
  clear_error();
  if (!ci || n < 0 || (n > 0 && !block_hashes)) return fail(FKV_ERR_INVALID_ARG, "bad arguments");
  if (num_found) *num_found = 0;
  if (n == 0) return FKV_OK;
  std::lock_guard<std::mutex> lk(ci->mu);
  DeviceGuard g(ci->device);
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc;
  sc.s = s;
  if (int rc = scratch_alloc(ci->device, al16(8 * n) + 16, s, (void **)&sc.base)) return rc;
  if (int rc = ensure_pin(ci, 8 * n)) return rc;
  std::memcpy(ci->pin, block_hashes, 8 * n);
  int64_t *found = reinterpret_cast<int64_t *>(sc.base + al16(8 * n));
  FKV_CUDA(cudaMemcpyAsync(sc.base, ci->pin, 8 * n, cudaMemcpyHostToDevice, s));
  FKV_CUDA(cudaMemsetAsync(found, 0, 8, s));
  set_flags_kernel<<<grid_for(n), 256, 0, s>>>(ci->table(), reinterpret_cast<uint64_t *>(sc.base), n, ready, found);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  FKV_CUDA(cudaMemcpyAsync(ci->pin, found, 8, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  if (num_found) std::memcpy(num_found, ci->pin, 8);
  return FKV_OK;
}

int fkv_cache_index_remove(fkv_cache_index *ci, const uint64_t *block_hashes, int64_t n, int64_t *removed_blocks,
                           void *stream) {
  clear_error();
  if (!ci || n < 0 || (n > 0 && !block_hashes)) return fail(FKV_ERR_INVALID_ARG, "bad arguments");
  if (n == 0) return FKV_OK;
  std::lock_guard<std::mutex> lk(ci->mu);
  DeviceGuard g(ci->device);
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc;
  sc.s = s;
  if (int rc = scratch_alloc(ci->device, 2 * al16(8 * n), s, (void **)&sc.base)) return rc;
  if (int rc = ensure_pin(ci, 8 * n)) return rc;
  std::memcpy(ci->pin, block_hashes, 8 * n);
  int64_t *out = reinterpret_cast<int64_t *>(sc.base + al16(8 * n));
  FKV_CUDA(cudaMemcpyAsync(sc.base, ci->pin, 8 * n, cudaMemcpyHostToDevice, s));
  remove_kernel<<<grid_for(n), 256, 0, s>>>(ci->table(), reinterpret_cast<uint64_t *>(sc.base), n, out, ci->state);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  FKV_CUDA(cudaMemcpyAsync(ci->pin, out, 8 * n, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  if (removed_blocks) std::memcpy(removed_blocks, ci->pin, 8 * n);
  return compact_if_needed(ci, s);
}

int fkv_cache_index_recycle(fkv_cache_index *ci, const int64_t *block_ids, int64_t n, void *stream) {
  clear_error();
  if (!ci || n < 0 || (n > 0 && !block_ids)) return fail(FKV_ERR_INVALID_ARG, "bad arguments");
  if (n == 0) return FKV_OK;
  for (int64_t q = 0; q < n; ++q)
    if (block_ids[q] < 0 || block_ids[q] >= ci->num_blocks)
      return fail(FKV_ERR_OUT_OF_RANGE, "block id " + std::to_string(block_ids[q]) + " is outside the pool");
  {
    // The reference counts a repeated id twice (mempool.py:50) and its free
    // count then drifts from the mask; a repeat is refused here instead.
    std::vector<int64_t> sorted(block_ids, block_ids + n);
    std::sort(sorted.begin(), sorted.end());
    for (int64_t q = 1; q < n; ++q)
      if (sorted[q] == sorted[q - 1])
        return fail(FKV_ERR_INVALID_ARG, "block id " + std::to_string(sorted[q]) + " appears twice in one recycle");
  }
  std::lock_guard<std::mutex> lk(ci->mu);
  DeviceGuard g(ci->device);
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc;
  sc.s = s;
  if (int rc = scratch_alloc(ci->device, 8 * n, s, (void **)&sc.base)) return rc;
  if (int rc = ensure_pin(ci, 8 * n)) return rc;
  std::memcpy(ci->pin, block_ids, 8 * n);
  const int64_t *ids = reinterpret_cast<const int64_t *>(sc.base);
  FKV_CUDA(cudaMemcpyAsync(sc.base, ci->pin, 8 * n, cudaMemcpyHostToDevice, s));
  recycle_check_kernel<<<grid_for(n), 256, 0, s>>>(ci->free_mask, ids, n, ci->state);
  recycle_apply_kernel<<<grid_for(n), 256, 0, s>>>(ci->free_mask, ids, n, ci->state);
  FKV_CUDA(cudaGetLastError());
  note_launch(2);
  int64_t st[kStateWords];
  if (int rc = read_state(ci, s, st)) return rc;
  return take_device_error(ci, s, st);
}

int fkv_cache_index_take(fkv_cache_index *ci, int64_t num, int64_t *block_ids, int64_t *num_taken, void *stream) {
  clear_error();
  if (!ci || num < 0 || (num > 0 && !block_ids) || !num_taken) return fail(FKV_ERR_INVALID_ARG, "bad arguments");
  *num_taken = 0;
  if (num == 0) return FKV_OK;
  std::lock_guard<std::mutex> lk(ci->mu);
  DeviceGuard g(ci->device);
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t cap = std::min<int64_t>(num, ci->num_blocks);
  Scratch sc;
  sc.s = s;
  if (int rc = scratch_alloc(ci->device, al16(8 * cap) + 16, s, (void **)&sc.base)) return rc;
  int64_t *got = reinterpret_cast<int64_t *>(sc.base + al16(8 * cap));
  take_kernel<<<1, 32, 0, s>>>(cap, ci->free_mask, ci->mask_bytes, ci->free_ids, ci->state,
                               reinterpret_cast<int64_t *>(sc.base), got);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  if (int rc = ensure_pin(ci, 8 * cap + 8)) return rc;
  FKV_CUDA(cudaMemcpyAsync(ci->pin, got, 8, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(ci->pin + 8, sc.base, 8 * cap, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  std::memcpy(num_taken, ci->pin, 8);
  std::memcpy(block_ids, ci->pin + 8, 8 * (size_t)*num_taken);
  return FKV_OK;
}

int fkv_cache_index_stats(fkv_cache_index *ci, int64_t *out, void *stream) {
  clear_error();
  if (!ci || !out) return fail(FKV_ERR_INVALID_ARG, "bad arguments");
  std::lock_guard<std::mutex> lk(ci->mu);
  DeviceGuard g(ci->device);
  cudaStream_t s = (cudaStream_t)stream;
  Scratch sc;
  sc.s = s;
  if (int rc = scratch_alloc(ci->device, 16, s, (void **)&sc.base)) return rc;
  FKV_CUDA(cudaMemsetAsync(sc.base, 0, 8, s));
  count_ready_kernel<<<grid_for((int64_t)ci->slots), 256, 0, s>>>(ci->table(), reinterpret_cast<int64_t *>(sc.base));
  FKV_CUDA(cudaGetLastError());
  note_launch();
  if (int rc = ensure_pin(ci, 8 * (kStateWords + 1))) return rc;
  FKV_CUDA(cudaMemcpyAsync(ci->pin, ci->state, 8 * kStateWords, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaMemcpyAsync(ci->pin + 8 * kStateWords, sc.base, 8, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  const int64_t *st = reinterpret_cast<const int64_t *>(ci->pin);
  out[0] = st[kNumFree];
  out[1] = st[kLive];
  out[2] = st[kStateWords];  // ready entries
  out[3] = st[kListLen];
  out[4] = st[kOffset];
  out[5] = st[kTombs];
  out[6] = (int64_t)ci->slots;
  return FKV_OK;
}

}  // extern "C"
