// XXH64 (seed 0) block hashing on the GPU — replaces flexkv::Hasher and
// flexkv::gen_hashes (csrc/hash.cpp:15-66, csrc/cache_utils.h:10-28), which
// wrap the xxHash library's streaming XXH64 on the CPU.
//
// The algorithm is the public XXH64 specification (Yann Collet, "xxHash
// fast digest algorithm", XXH64 section): four 64-bit lanes consume 32-byte
// stripes with round(acc, x) = rotl(acc + x*P2, 31) * P1; the digest merges
// the lanes (or starts from seed+P5 below 32 bytes), adds the total length,
// folds the <32-byte tail and avalanches.
//
// gen_hashes semantics (hash.cpp:61-65): the hasher is updated block by
// block and digest() is taken after each, so block b's hash is the XXH64 of
// the whole running prefix.  The lane chain is strictly sequential along a
// sequence, so one sequence is hashed by
//   xxh_chain_kernel    — one warp; lanes 0..3 run the four XXH64 lanes
//                         while the whole warp streams the next token tile
//                         into shared memory with cp.async and forms each
//                         tile's x*P2 products for them; the lane values
//                         at every block boundary go to a scratch array;
//   xxh_finalize_kernel — one thread per block: merge + tail + avalanche,
//                         fully parallel across the grid.
// Independent sequences (fkv_gen_hashes_batched) run one 4-lane quad each
// and finalize in-quad, so a batch needs no scratch at all.
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "fkv_common.h"

namespace fkv {
namespace {

constexpr uint64_t P1 = 0x9E3779B185EBCA87ull;
constexpr uint64_t P2 = 0xC2B2AE3D27D4EB4Full;
constexpr uint64_t P3 = 0x165667B19E3779F9ull;
constexpr uint64_t P4 = 0x85EBCA77C2B2AE63ull;
constexpr uint64_t P5 = 0x27D4EB2F165667C5ull;

// Streaming state; layout shared by every kernel here.  mem holds the
// memsize (< 32) bytes not yet consumed as a stripe.
struct XxhState {
  uint64_t total_len;
  uint64_t v[4];
  uint64_t mem[4];
  uint32_t memsize;
  uint32_t pad;
};

__host__ __device__ __forceinline__ uint64_t rotl64(uint64_t x, int r) {
  return (x << r) | (x >> (64 - r));
}
__host__ __device__ __forceinline__ uint64_t xround(uint64_t acc, uint64_t in) {
  acc += in * P2;
  acc = rotl64(acc, 31);
  return acc * P1;
}
__device__ __forceinline__ uint64_t merge_round(uint64_t acc, uint64_t val) {
  val = xround(0, val);
  acc ^= val;
  return acc * P1 + P4;
}
__device__ __forceinline__ uint64_t avalanche(uint64_t h) {
  h ^= h >> 33;
  h *= P2;
  h ^= h >> 29;
  h *= P3;
  h ^= h >> 32;
  return h;
}

// Byte p of the stream "mem[0..memsize) ++ data[0..)".
__device__ __forceinline__ uint8_t stream_byte(const XxhState &s, const uint8_t *data, int64_t p) {
  if (p < (int64_t)s.memsize) return reinterpret_cast<const uint8_t *>(s.mem)[p];
  return data[p - s.memsize];
}
// Little-endian n-byte word of the stream at p (n <= 8).
__device__ __forceinline__ uint64_t stream_word(const XxhState &s, const uint8_t *data, int64_t p, int n) {
  const int64_t m = s.memsize;
  const int64_t q = p - m;
  if (n == 8 && q >= 0 && ((reinterpret_cast<uintptr_t>(data) + q) & 7) == 0)
    return *reinterpret_cast<const uint64_t *>(data + q);
  uint64_t w = 0;
  for (int b = 0; b < n; ++b) w |= (uint64_t)stream_byte(s, data, p + b) << (8 * b);
  return w;
}

// Digest of a state whose lanes are v, given the total length and the tail
// bytes stream[tail_pos, tail_pos + tail_len).
__device__ __forceinline__ uint64_t finalize(const uint64_t (&v)[4], uint64_t total_len, const XxhState &s0,
                             const uint8_t *data, int64_t tail_pos, int tail_len) {
  uint64_t h;
  if (total_len >= 32) {
    h = rotl64(v[0], 1) + rotl64(v[1], 7) + rotl64(v[2], 12) + rotl64(v[3], 18);
    h = merge_round(h, v[0]);
    h = merge_round(h, v[1]);
    h = merge_round(h, v[2]);
    h = merge_round(h, v[3]);
  } else {
    h = v[2] + P5;  // lane 3 still holds the seed below 32 bytes
  }
  h += total_len;
  int64_t p = tail_pos;
  int left = tail_len;
  while (left >= 8) {
    const uint64_t k1 = xround(0, stream_word(s0, data, p, 8));
    h ^= k1;
    h = rotl64(h, 27) * P1 + P4;
    p += 8;
    left -= 8;
  }
  if (left >= 4) {
    h ^= (stream_word(s0, data, p, 4) & 0xFFFFFFFFull) * P1;
    h = rotl64(h, 23) * P2 + P3;
    p += 4;
    left -= 4;
  }
  while (left > 0) {
    h ^= (uint64_t)stream_byte(s0, data, p) * P5;
    h = rotl64(h, 11) * P1;
    ++p;
    --left;
  }
  return avalanche(h);
}

__global__ void xxh_reset_kernel(XxhState *s) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    s->total_len = 0;
    s->v[0] = P1 + P2;  // seed 0
    s->v[1] = P2;
    s->v[2] = 0;
    s->v[3] = 0 - P1;
    for (int i = 0; i < 4; ++i) s->mem[i] = 0;
    s->memsize = 0;
    s->pad = 0;
  }
}

__global__ void xxh_digest_kernel(const XxhState *s, uint64_t *out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const XxhState st = *s;
    *out = finalize(st.v, st.total_len, st, nullptr, 0, (int)st.memsize);
  }
}

constexpr int kTileWords = 1024;  // 8 KiB of stream per shared-memory tile

__device__ __forceinline__ void cp_async8(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Stage stream words [w0, w0+kTileWords) into buf (words beyond the stream
// are left untouched and never read).  Fast path only: memsize % 8 == 0 and
// data 8-byte aligned, so stream word w is mem[w] or data64[w - memsize/8].
__device__ __forceinline__ void stage_tile(uint64_t *buf, const XxhState &s, const uint64_t *data64,
                                           int64_t w0, int64_t n_words, int lane) {
  const int64_t m8 = s.memsize / 8;
  for (int k = lane; k < kTileWords; k += 32) {
    const int64_t w = w0 + k;
    if (w >= n_words) break;
    if (w < m8) buf[k] = s.mem[w];
    else cp_async8(&buf[k], data64 + (w - m8));
  }
  cp_async_commit();
}

// Fused-round path: two warps.  The producer warp reads each tile of 256
// stripes (8 KiB of tokens) with coalesced loads and writes its x*P2
// products into a shared ring slot, transposed: row j holds lane j's
// products, word j of stripe s at index s + 1, with index 0 and index kt + 1
// zero.  With the one-slot offset the addends of a group of 8 stripes
// (indices 8g+2 .. 8g+9) are four aligned 16-byte pairs.  The row stride
// (268 words) keeps the four chain lanes' reads conflict-free and leaves
// room for their reads one group past the tile end (index <= 8*32 + 9).
// Lanes 0..3 of the chain warp run only the rounds and write block
// snapshots into a shared slot; the producer copies those to global
// memory once the chain has released the slot.  Two slots suffice: a
// tile's loads and products take a fraction of its chain time.
constexpr int kProdStride = 268;
constexpr int kProdSlot = 4 * kProdStride;  // words per product slot
constexpr int kSnapSlot = 4 * 256;          // words per snapshot slot (up to 256 blocks)
constexpr int kRawWords = 2 * kTileWords;   // single-warp paths: two raw tiles
constexpr int kFusedWords = 2 * kProdSlot + 2 * kSnapSlot;
constexpr int kChainSmemWords = kFusedWords > kRawWords ? kFusedWords : kRawWords;
constexpr uint32_t P1L = (uint32_t)P1;
constexpr uint32_t P1H = (uint32_t)(P1 >> 32);
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // a hand-off wait gives up after 2 s

__device__ __forceinline__ uint64_t mad_wide_u32(uint32_t a, uint32_t b, uint64_t c) {
  uint64_t d;
  asm("mad.wide.u32 %0, %1, %2, %3;" : "=l"(d) : "r"(a), "r"(b), "l"(c));
  return d;
}

// One XXH64 round on a lane value that already holds its stripe input,
// a = v + x*P2, kept as 32-bit halves:  a <- rotl(a, 31) * P1 + next,
// where next is the following stripe's x*P2.  The rotation is two funnel
// shifts; the low half of the 64-bit multiply and the following round's
// add are one widening multiply-add; the high half adds the two 32-bit
// cross products.  The dependent path is shift -> multiply-add -> add,
// against add -> add-with-carry -> shift -> multiply -> ... for the plain
// 64-bit form.
__device__ __forceinline__ void fused_round(uint32_t &lo, uint32_t &hi, uint64_t next) {
  const uint32_t rl = __funnelshift_l(hi, lo, 31);  // low half of rotl(a, 31)
  const uint32_t rh = __funnelshift_l(lo, hi, 31);  // high half
  const uint64_t w = mad_wide_u32(rl, P1L, next);
  lo = (uint32_t)w;
  hi = (uint32_t)(w >> 32) + rh * P1L + rl * P1H;
}

__device__ __forceinline__ uint64_t join64(uint32_t lo, uint32_t hi) {
  return ((uint64_t)hi << 32) | lo;
}

__device__ __forceinline__ void load_group(const uint64_t *p, uint64_t (&x)[8]) {
  const ulonglong2 *q = reinterpret_cast<const ulonglong2 *>(p);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const ulonglong2 t = q[k];
    x[2 * k] = t.x;
    x[2 * k + 1] = t.y;
  }
}

// Eight rounds; x[u] is the addend folded in by stripe u's round (the next
// stripe's product).  A block's snapshot is the held value minus the
// addend already folded in, computed off the chain, stored to sn (stride 4
// words per block).
template <int SPB, bool SNAP>
__device__ __forceinline__ void group_rounds(const uint64_t (&x)[8], uint32_t &lo, uint32_t &hi,
                                             uint64_t *sn) {
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    fused_round(lo, hi, x[u]);
    if (SNAP && u % SPB == SPB - 1) sn[(u / SPB) * 4] = join64(lo, hi) - x[u];
  }
}

// One chain lane over one tile of kt stripes (tile and block boundaries
// coincide: SPB divides the 256 stripes of a tile and kt is a multiple of
// SPB).  pj is the lane's product row; sn is the lane's column of the
// tile's snapshot slot (block k of the tile at sn[4k]).  Groups of 8
// stripes run from registers loaded one group ahead, in two alternating
// buffers; the stripes of a last partial group run block by block.  The
// tile's final round folds in the zero at index kt + 1, so v leaves exact.
template <int SPB, bool SNAP>
__device__ __forceinline__ void chain_tile_fused(const uint64_t *pj, int kt, uint64_t &v, uint64_t *sn) {
  static_assert(SPB == 1 || SPB == 2 || SPB == 4 || SPB == 8, "blocks must tile a group of 8 stripes");
  static_assert(8 * 32 + 9 < kProdStride, "product row too short for the pipeline");
  const uint64_t a = v + pj[1];
  uint32_t lo = (uint32_t)a, hi = (uint32_t)(a >> 32);
  const int ng = kt / 8;
  uint64_t A[8], B[8];
  load_group(pj + 2, A);
  int g = 0;
  for (; g + 2 <= ng; g += 2) {
    load_group(pj + 8 * g + 10, B);
    group_rounds<SPB, SNAP>(A, lo, hi, sn + 4 * (8 * g / SPB));
    load_group(pj + 8 * g + 18, A);
    group_rounds<SPB, SNAP>(B, lo, hi, sn + 4 * (8 * (g + 1) / SPB));
  }
  if (g < ng) {
    group_rounds<SPB, SNAP>(A, lo, hi, sn + 4 * (8 * g / SPB));
    ++g;
  }
  for (int st = 8 * g; st < kt; st += SPB) {
#pragma unroll
    for (int t = 0; t < SPB; ++t) fused_round(lo, hi, pj[st + t + 2]);
    if (SNAP) sn[4 * (st / SPB)] = join64(lo, hi) - pj[st + SPB + 1];
  }
  v = join64(lo, hi);
}

// Producer warp: products of one tile of kt stripes whose words start at
// src, into product slot pr.  16-byte loads when src is 16-byte aligned,
// 8-byte loads otherwise; eight loads in flight per lane.
__device__ __forceinline__ void produce_tile(const uint64_t *src, int kt, uint64_t *pr, int lane,
                                             bool al16) {
  const int nw = 4 * kt;
  if (al16) {
    const ulonglong2 *s2 = reinterpret_cast<const ulonglong2 *>(src);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ulonglong2 x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = lane + 32 * (8 * h + i);  // words 2q, 2q+1: stripe q/2, lanes 2(q&1), +1
        if (2 * q < nw) x[i] = __ldg(s2 + q);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = lane + 32 * (8 * h + i);
        if (2 * q < nw) {
          const int at = 2 * (q & 1) * kProdStride + (q >> 1) + 1;
          pr[at] = x[i].x * P2;
          pr[at + kProdStride] = x[i].y * P2;
        }
      }
    }
  } else {
#pragma unroll 1
    for (int h = 0; h < 4; ++h) {
      uint64_t x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int w = lane + 32 * (8 * h + i);
        if (w < nw) x[i] = __ldg(src + w);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int w = lane + 32 * (8 * h + i);
        if (w < nw) pr[(w & 3) * kProdStride + (w >> 2) + 1] = x[i] * P2;
      }
    }
  }
  if (kt < 256 && lane < 4) pr[lane * kProdStride + kt + 1] = 0;
}

__device__ __forceinline__ unsigned smem_u32(const void *p) {
  return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(b))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for the phase of the given parity to complete; false (and the
// caller's error word set) if it does not within limit_ns.
__device__ __noinline__ bool mbar_wait(uint64_t *b, uint32_t parity, volatile int *err, uint64_t limit_ns) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(b, parity)) {
    if (global_ns() - t0 > limit_ns) {
      *err = FKV_ERR_TIMEOUT;
      return false;
    }
  }
  return true;
}

// The two-warp chain over K stripes of aligned data.  Returns false on a
// timed-out hand-off (error word set).  Every hand-off wait gives up after
// limit_ns.  max_tiles >= 0 makes the producer stop after that many tiles
// (a diagnostic that lets the chain warp's wait run out); -1 = all tiles.
template <int SPB, bool SNAP>
__device__ bool chain_fused(const uint64_t *data64, bool al16, int64_t K, uint64_t *smem, uint64_t *bars,
                            int warp, int lane, uint64_t &v, uint64_t *snaps, volatile int *err,
                            uint64_t limit_ns, int64_t max_tiles) {
  uint64_t *prod = smem;                   // [2][kProdSlot]
  uint64_t *snap = smem + 2 * kProdSlot;   // [2][kSnapSlot]
  uint64_t *full = bars, *empty = bars + 2;
  const int64_t T = (K + 255) / 256;
  constexpr int kBlocksPerTile = 256 / SPB;
  auto tile_stripes = [&](int64_t t) { return (int)(K - 256 * t < 256 ? K - 256 * t : 256); };
  if (warp == 1) {
    for (int64_t t = 0; t < T; ++t) {
      if (max_tiles >= 0 && t >= max_tiles) return true;  // stopped on purpose: the chain's wait runs out
      const int sl = (int)(t & 1);
      if (t >= 2) {  // slot sl held tile t-2 (a full tile): wait for the chain, drain its snapshots
        if (!mbar_wait(&empty[sl], (uint32_t)(((t >> 1) - 1) & 1), err, limit_ns)) return false;
        if (SNAP) {
          uint64_t *dst = snaps + 4 * (t - 2) * kBlocksPerTile;
          for (int k = lane; k < 4 * kBlocksPerTile; k += 32) dst[k] = snap[sl * kSnapSlot + k];
        }
      }
      produce_tile(data64 + 1024 * t, tile_stripes(t), prod + sl * kProdSlot, lane, al16);
      mbar_arrive(&full[sl]);
    }
    for (int64_t t = T >= 2 ? T - 2 : 0; t < T; ++t) {  // the last one or two tiles
      const int sl = (int)(t & 1);
      if (!mbar_wait(&empty[sl], (uint32_t)((t >> 1) & 1), err, limit_ns)) return false;
      if (SNAP) {
        uint64_t *dst = snaps + 4 * t * kBlocksPerTile;
        const int n = 4 * (tile_stripes(t) / SPB);
        for (int k = lane; k < n; k += 32) dst[k] = snap[sl * kSnapSlot + k];
      }
    }
  } else if (lane < 4) {
    for (int64_t t = 0; t < T; ++t) {
      const int sl = (int)(t & 1);
      if (!mbar_wait(&full[sl], (uint32_t)((t >> 1) & 1), err, limit_ns)) return false;
      chain_tile_fused<SPB, SNAP>(prod + sl * kProdSlot + lane * kProdStride, tile_stripes(t), v,
                                  snap + sl * kSnapSlot + lane);
      mbar_arrive(&empty[sl]);
    }
  }
  return true;
}

// Same for any stripes-per-block count, with a per-stripe block counter.
__device__ __forceinline__ void chain_tile_generic(const uint64_t *buf, int kt, int j, int lane,
                                                   uint64_t &v, uint64_t *snaps, int64_t &next_b,
                                                   int64_t spb) {
  int64_t in_block = 0;
  for (int i = 0; i < kt; ++i) {
    v = rotl64(v + buf[4 * i + j] * P2, 31) * P1;
    if (++in_block == spb) {
      if (snaps != nullptr && lane < 4) snaps[next_b * 4 + j] = v;
      ++next_b;
      in_block = 0;
    }
  }
}

// Sequential lane chain over stream stripes [0, K) where the stream is
// mem ++ data[0, len); writes lane snapshots for nb block boundaries (block
// b ends at stream byte memsize + bb*(b+1)) and the successor state.
// Launch: 1 block of 64 threads.  With nothing buffered, 8-byte aligned
// data and blocks of 1, 2, 4 or 8 whole stripes (every gen_hashes call
// with tpb a multiple of 4 tokens, and every update of aligned data) the
// two warps run the fused path; otherwise warp 0 runs alone.  err is a
// host-visible word set to FKV_ERR_TIMEOUT if a hand-off wait ran out
// (each gives up after limit_ns); max_tiles caps the producer (see
// chain_fused), -1 in every product call.
__global__ void __launch_bounds__(64) xxh_chain_kernel(const XxhState *in, XxhState *out,
                                                       const uint8_t *data, int64_t len,
                                                       int64_t bb, int64_t nb, uint64_t *snaps,
                                                       int *err, uint64_t limit_ns, int64_t max_tiles) {
  __shared__ __align__(16) uint64_t smem[kChainSmemWords];
  __shared__ __align__(8) uint64_t bars[4];  // full[2], empty[2]
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const XxhState s = *in;
  const int j = lane & 3;
  uint64_t v = s.v[j];
  const int64_t stream_len = (int64_t)s.memsize + len;
  const int64_t K = stream_len / 32;  // stripes consumed by this call
  int64_t next_b = 0;
  auto boundary_stripes = [&](int64_t b) -> int64_t { return ((int64_t)s.memsize + bb * (b + 1)) / 32; };
  const bool data_aligned = (reinterpret_cast<uintptr_t>(data) & 7) == 0;
  const bool aligned_blocks = s.memsize == 0 && data_aligned && (snaps == nullptr || bb % 32 == 0);
  const int64_t spb = snaps ? bb / 32 : 1;  // stripes per block (1 when no snapshots)
  const bool fused = aligned_blocks && (spb == 1 || spb == 2 || spb == 4 || spb == 8);
  if (fused) {
    for (int i = threadIdx.x; i < 2 * kProdSlot; i += blockDim.x) smem[i] = 0;  // index 0 and the pad stay zero
    if (threadIdx.x == 0) {
      mbar_init(&bars[0], 32);
      mbar_init(&bars[1], 32);
      mbar_init(&bars[2], 4);
      mbar_init(&bars[3], 4);
    }
    __syncthreads();
    const uint64_t *data64 = reinterpret_cast<const uint64_t *>(data);
    const bool al16 = (reinterpret_cast<uintptr_t>(data) & 15) == 0;
    volatile int *e = err;
    bool ok;
    if (snaps == nullptr) ok = chain_fused<1, false>(data64, al16, K, smem, bars, warp, lane, v, snaps, e, limit_ns, max_tiles);
    else if (spb == 1) ok = chain_fused<1, true>(data64, al16, K, smem, bars, warp, lane, v, snaps, e, limit_ns, max_tiles);
    else if (spb == 2) ok = chain_fused<2, true>(data64, al16, K, smem, bars, warp, lane, v, snaps, e, limit_ns, max_tiles);
    else if (spb == 4) ok = chain_fused<4, true>(data64, al16, K, smem, bars, warp, lane, v, snaps, e, limit_ns, max_tiles);
    else ok = chain_fused<8, true>(data64, al16, K, smem, bars, warp, lane, v, snaps, e, limit_ns, max_tiles);
    if (!ok || warp != 0) return;
  } else {
    if (warp != 0) return;
    uint64_t(*tiles)[kTileWords] = reinterpret_cast<uint64_t(*)[kTileWords]>(smem);
    // Boundaries reached before any stripe of this call.
    while (snaps && next_b < nb && boundary_stripes(next_b) == 0) {
      if (lane < 4) snaps[next_b * 4 + j] = v;
      ++next_b;
    }
    const bool fast = (s.memsize % 8 == 0) && data_aligned;
    if (aligned_blocks) {  // blocks of whole stripes, other than 1, 2, 4 or 8 of them
      const uint64_t *data64 = reinterpret_cast<const uint64_t *>(data);
      const int64_t n_words = 4 * K;
      int cur = 0;
      if (K > 0) stage_tile(tiles[0], s, data64, 0, n_words, lane);
      for (int64_t t0 = 0; t0 < n_words; t0 += kTileWords) {
        if (t0 + kTileWords < n_words) stage_tile(tiles[cur ^ 1], s, data64, t0 + kTileWords, n_words, lane);
        else cp_async_commit();
        cp_async_wait_1();
        __syncwarp();
        const int64_t k_tile_end = (t0 + kTileWords) / 4;
        const int kt = (int)((K < k_tile_end ? K : k_tile_end) - t0 / 4);
        chain_tile_generic(tiles[cur], kt, j, lane, v, snaps, next_b, spb);
        __syncwarp();
        cur ^= 1;
      }
    } else if (fast) {
      const uint64_t *data64 = reinterpret_cast<const uint64_t *>(data);
      const int64_t n_words = 4 * K;  // only whole stripes are read here
      int cur = 0;
      if (K > 0) stage_tile(tiles[0], s, data64, 0, n_words, lane);
      for (int64_t t0 = 0; t0 < n_words; t0 += kTileWords) {
        // Prefetch the next tile, then wait for the current one.
        if (t0 + kTileWords < n_words) stage_tile(tiles[cur ^ 1], s, data64, t0 + kTileWords, n_words, lane);
        else cp_async_commit();
        cp_async_wait_1();
        __syncwarp();
        const uint64_t *buf = tiles[cur];
        const int64_t k_begin = t0 / 4;
        const int64_t k_tile_end = (t0 + kTileWords) / 4;
        const int64_t k_end = K < k_tile_end ? K : k_tile_end;
        int64_t nbk = (snaps && next_b < nb) ? boundary_stripes(next_b) : INT64_MAX;
        for (int64_t k = k_begin; k < k_end; ++k) {
          v = xround(v, buf[4 * (k - k_begin) + j]);
          if (k + 1 == nbk) {
            do {
              if (lane < 4) snaps[next_b * 4 + j] = v;
              ++next_b;
              nbk = (next_b < nb) ? boundary_stripes(next_b) : INT64_MAX;
            } while (k + 1 == nbk);
          }
        }
        __syncwarp();
        cur ^= 1;
      }
    } else {
      int64_t nbk = (snaps && next_b < nb) ? boundary_stripes(next_b) : INT64_MAX;
      for (int64_t k = 0; k < K; ++k) {
        v = xround(v, stream_word(s, data, 32 * k + 8 * j, 8));
        if (k + 1 == nbk) {
          do {
            if (lane < 4) snaps[next_b * 4 + j] = v;
            ++next_b;
            nbk = (next_b < nb) ? boundary_stripes(next_b) : INT64_MAX;
          } while (k + 1 == nbk);
        }
      }
    }
  }
  if (lane < 4) out->v[j] = v;
  if (lane == 0) {
    out->total_len = s.total_len + (uint64_t)len;
    const int rest = (int)(stream_len - 32 * K);
    uint64_t m[4] = {0, 0, 0, 0};
    for (int b = 0; b < rest; ++b)
      m[b >> 3] |= (uint64_t)stream_byte(s, data, 32 * K + b) << (8 * (b & 7));
    for (int i = 0; i < 4; ++i) out->mem[i] = m[i];
    out->memsize = (uint32_t)rest;
    out->pad = 0;
  }
}

// Digest of block b of a gen_hashes call from its lane snapshot.
__global__ void xxh_finalize_kernel(const XxhState *in, const uint8_t *data, int64_t bb,
                                    int64_t nb, const uint64_t *snaps, uint64_t *out) {
  const XxhState s = *in;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb;
       b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t Lb = (int64_t)s.memsize + bb * (b + 1);
    const int64_t sb = Lb / 32;
    uint64_t v[4];
    const uint4 *sp = reinterpret_cast<const uint4 *>(snaps + 4 * b);
    const uint4 a = sp[0], c = sp[1];
    v[0] = ((uint64_t)a.y << 32) | a.x;
    v[1] = ((uint64_t)a.w << 32) | a.z;
    v[2] = ((uint64_t)c.y << 32) | c.x;
    v[3] = ((uint64_t)c.w << 32) | c.z;
    const uint64_t total = s.total_len + (uint64_t)(bb * (b + 1));
    out[b] = finalize(v, total, s, data, 32 * sb, (int)(Lb - 32 * sb));
  }
}

// Independent fresh-seed sequences, one 4-lane quad each; each quad
// finalizes its own blocks (lane 0 gathers the four lanes by shuffle).
// token words are int64 (8-byte aligned); tpb tokens per block.
__global__ void __launch_bounds__(256) xxh_batched_kernel(const int64_t *tokens,
                                                          const int64_t *seq_tok_off,
                                                          const int64_t *seq_blk_off,
                                                          int num_seqs, int tpb, uint64_t *out) {
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int q = gtid >> 2;
  const int j = threadIdx.x & 3;
  const unsigned quad_mask = 0xFu << (threadIdx.x & 28);
  const bool active = q < num_seqs;
  // Whole quads are either active or not; inactive quads exit together.
  if (!active) return;
  const int64_t t0 = seq_tok_off[q];
  const int64_t nblk = seq_blk_off[q + 1] - seq_blk_off[q];
  const int64_t o0 = seq_blk_off[q];
  const uint64_t *w = reinterpret_cast<const uint64_t *>(tokens + t0);
  uint64_t v = j == 0 ? P1 + P2 : (j == 1 ? P2 : (j == 2 ? 0 : 0 - P1));
  const int64_t bb = 8ll * tpb;  // bytes per block
  int64_t k = 0;                 // stripes consumed
  for (int64_t b = 0; b < nblk; ++b) {
    const int64_t Lb = bb * (b + 1);
    const int64_t sb = Lb / 32;
    for (; k + 4 <= sb; k += 4) {  // four independent loads in flight, then four rounds
      const uint64_t x0 = w[4 * k + j] * P2, x1 = w[4 * k + 4 + j] * P2;
      const uint64_t x2 = w[4 * k + 8 + j] * P2, x3 = w[4 * k + 12 + j] * P2;
      v = rotl64(v + x0, 31) * P1;
      v = rotl64(v + x1, 31) * P1;
      v = rotl64(v + x2, 31) * P1;
      v = rotl64(v + x3, 31) * P1;
    }
    for (; k < sb; ++k) v = xround(v, w[4 * k + j]);
    const uint64_t v0 = __shfl_sync(quad_mask, v, 0, 4);
    const uint64_t v1 = __shfl_sync(quad_mask, v, 1, 4);
    const uint64_t v2 = __shfl_sync(quad_mask, v, 2, 4);
    const uint64_t v3 = __shfl_sync(quad_mask, v, 3, 4);
    if (j == 0) {
      uint64_t h;
      if (Lb >= 32) {
        h = rotl64(v0, 1) + rotl64(v1, 7) + rotl64(v2, 12) + rotl64(v3, 18);
        h = merge_round(h, v0);
        h = merge_round(h, v1);
        h = merge_round(h, v2);
        h = merge_round(h, v3);
      } else {
        h = v2 + P5;
      }
      h += (uint64_t)Lb;
      int64_t p = 32 * sb;  // tail: whole 8-byte words (token bytes)
      for (; p + 8 <= Lb; p += 8) {
        h ^= xround(0, w[p / 8]);
        h = rotl64(h, 27) * P1 + P4;
      }
      out[o0 + b] = avalanche(h);
    }
  }
}

struct DevBuf {
  void *p = nullptr;
  cudaStream_t s = nullptr;
  ~DevBuf() {
    if (p) scratch_free(p, s);
  }
};

}  // namespace
}  // namespace fkv

struct fkv_hasher {
  int device = 0;
  fkv::XxhState *states = nullptr;  // device [2]; `cur` is live
  int cur = 0;
  uint64_t *digest_dev = nullptr;
  uint64_t *digest_host = nullptr;  // pinned
  int *err_host = nullptr;          // pinned, mapped: written by the chain kernel on a timed-out wait
  int *err_dev = nullptr;           // device address of err_host
};

using namespace fkv;

namespace {

struct DeviceGuard {
  int prev = -1;
  bool switched = false;
  int enter(int dev) {
    FKV_CUDA(cudaGetDevice(&prev));
    if (prev != dev) {
      FKV_CUDA(cudaSetDevice(dev));
      switched = true;
    }
    return FKV_OK;
  }
  ~DeviceGuard() {
    if (switched) cudaSetDevice(prev);
  }
};

// Device view of `bytes` at p: p itself if it is device memory of `device`,
// else a stream-ordered copy into `tmp`.
int device_view(const void *p, int64_t bytes, int device, cudaStream_t s, DevBuf &tmp,
                const void **out, bool *was_host) {
  int is_dev = 0, dev = -1;
  pointer_is_device(p, &is_dev, &dev);
  *was_host = !is_dev;
  if (is_dev) {
    if (dev != device) return fail(FKV_ERR_INVALID_ARG, "device buffer lives on another device than the hasher");
    *out = p;
    return FKV_OK;
  }
  tmp.s = s;
  if (int rc = scratch_alloc(device, (size_t)std::max<int64_t>(bytes, 16), s, &tmp.p)) return rc;
  if (bytes > 0) FKV_CUDA(cudaMemcpyAsync(tmp.p, p, (size_t)bytes, cudaMemcpyHostToDevice, s));
  *out = tmp.p;
  return FKV_OK;
}

int run_chain(fkv_hasher *h, const uint8_t *data_dev, int64_t len, int64_t bb, int64_t nb,
              uint64_t *snaps, cudaStream_t s, uint64_t limit_ns = kWaitLimitNs, int64_t max_tiles = -1) {
  XxhState *in = h->states + h->cur;
  XxhState *out = h->states + (h->cur ^ 1);
  xxh_chain_kernel<<<1, 64, 0, s>>>(in, out, data_dev, len, bb, nb, snaps, h->err_dev, limit_ns, max_tiles);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  return FKV_OK;
}

// After a synchronize: report (once) a chain hand-off wait that ran out.
int check_chain(fkv_hasher *h) {
  if (*h->err_host == 0) return FKV_OK;
  const int code = *h->err_host;
  *h->err_host = 0;
  return fail(code, "hash chain kernel: a producer/consumer hand-off wait timed out; the update did not complete");
}

}  // namespace

extern "C" {

int fkv_get_hash_size(void) { return 8; }

int fkv_hasher_create(int device, fkv_hasher **out) {
  clear_error();
  if (!out) return fail(FKV_ERR_INVALID_ARG, "null output");
  *out = nullptr;
  if (device < 0) FKV_CUDA(cudaGetDevice(&device));
  DeviceGuard g;
  if (int rc = g.enter(device)) return rc;
  auto *h = new fkv_hasher();
  h->device = device;
  cudaError_t e = cudaMalloc((void **)&h->states, 2 * sizeof(XxhState));
  if (e == cudaSuccess) e = cudaMalloc((void **)&h->digest_dev, 8);
  if (e == cudaSuccess) e = cudaHostAlloc((void **)&h->digest_host, 8, cudaHostAllocPortable);
  if (e == cudaSuccess) e = cudaHostAlloc((void **)&h->err_host, 4, cudaHostAllocPortable | cudaHostAllocMapped);
  if (e == cudaSuccess) {
    *h->err_host = 0;
    e = cudaHostGetDevicePointer((void **)&h->err_dev, h->err_host, 0);
  }
  if (e != cudaSuccess) {
    fkv_hasher_destroy(h);
    return fail_cuda(e, "hasher allocation");
  }
  xxh_reset_kernel<<<1, 32>>>(h->states);
  note_launch();
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    fkv_hasher_destroy(h);
    return fail_cuda(e, "hasher reset");
  }
  *out = h;
  return FKV_OK;
}

void fkv_hasher_destroy(fkv_hasher *h) {
  if (!h) return;
  if (h->states) cudaFree(h->states);
  if (h->digest_dev) cudaFree(h->digest_dev);
  if (h->digest_host) cudaFreeHost(h->digest_host);
  if (h->err_host) cudaFreeHost(h->err_host);
  delete h;
}

int fkv_hasher_reset(fkv_hasher *h, void *stream) {
  clear_error();
  if (!h) return fail(FKV_ERR_INVALID_ARG, "null hasher");
  DeviceGuard g;
  if (int rc = g.enter(h->device)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  xxh_reset_kernel<<<1, 32, 0, s>>>(h->states + h->cur);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  return FKV_OK;
}

int fkv_hasher_update(fkv_hasher *h, const void *data, int64_t size, void *stream) {
  clear_error();
  if (!h) return fail(FKV_ERR_INVALID_ARG, "null hasher");
  if (size < 0 || (size > 0 && !data)) return fail(FKV_ERR_INVALID_ARG, "bad update buffer");
  if (size == 0) return FKV_OK;
  DeviceGuard g;
  if (int rc = g.enter(h->device)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  DevBuf tmp;
  const void *dv = nullptr;
  bool was_host = false;
  if (int rc = device_view(data, size, h->device, s, tmp, &dv, &was_host)) return rc;
  if (int rc = run_chain(h, (const uint8_t *)dv, size, 0, 0, nullptr, s)) return rc;
  h->cur ^= 1;
  if (was_host) {
    FKV_CUDA(cudaStreamSynchronize(s));
    return check_chain(h);
  }
  return FKV_OK;
}

int fkv_hasher_update_bounded(fkv_hasher *h, const void *data, int64_t size, uint64_t wait_limit_ns,
                              int64_t producer_tiles, void *stream) {
  clear_error();
  if (!h) return fail(FKV_ERR_INVALID_ARG, "null hasher");
  if (size < 0 || (size > 0 && !data)) return fail(FKV_ERR_INVALID_ARG, "bad update buffer");
  if (wait_limit_ns == 0 || wait_limit_ns > kWaitLimitNs)
    return fail(FKV_ERR_INVALID_ARG, "wait_limit_ns must lie in (0, 2 s]");
  if (producer_tiles < -1) return fail(FKV_ERR_INVALID_ARG, "producer_tiles must be -1 or non-negative");
  if (size == 0) return FKV_OK;
  DeviceGuard g;
  if (int rc = g.enter(h->device)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  DevBuf tmp;
  const void *dv = nullptr;
  bool was_host = false;
  if (int rc = device_view(data, size, h->device, s, tmp, &dv, &was_host)) return rc;
  if (int rc = run_chain(h, (const uint8_t *)dv, size, 0, 0, nullptr, s, wait_limit_ns, producer_tiles)) return rc;
  FKV_CUDA(cudaStreamSynchronize(s));
  if (int rc = check_chain(h)) return rc;  // timed out: the state before the call stays live
  h->cur ^= 1;
  return FKV_OK;
}

int fkv_hasher_digest(fkv_hasher *h, uint64_t *out, void *stream) {
  clear_error();
  if (!h || !out) return fail(FKV_ERR_INVALID_ARG, "null hasher or output");
  DeviceGuard g;
  if (int rc = g.enter(h->device)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  xxh_digest_kernel<<<1, 32, 0, s>>>(h->states + h->cur, h->digest_dev);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  FKV_CUDA(cudaMemcpyAsync(h->digest_host, h->digest_dev, 8, cudaMemcpyDeviceToHost, s));
  FKV_CUDA(cudaStreamSynchronize(s));
  if (int rc = check_chain(h)) return rc;
  *out = *h->digest_host;
  return FKV_OK;
}

int fkv_gen_hashes(fkv_hasher *h, const int64_t *token_ids, int64_t num_tokens,
                   int tokens_per_block, uint64_t *block_hashes, int64_t num_blocks,
                   void *stream) {
  clear_error();
  if (!h) return fail(FKV_ERR_INVALID_ARG, "null hasher");
  if (tokens_per_block <= 0) return fail(FKV_ERR_INVALID_ARG, "tokens_per_block must be positive");
  if (num_tokens < 0 || num_blocks < 0) return fail(FKV_ERR_INVALID_ARG, "negative size");
  if (num_tokens / tokens_per_block != num_blocks)  // hash.cpp:51 assert
    return fail(FKV_ERR_INVALID_ARG, "num_blocks must equal num_tokens / tokens_per_block");
  if (num_blocks == 0) return FKV_OK;
  if (!token_ids || !block_hashes) return fail(FKV_ERR_INVALID_ARG, "null token or output buffer");
  DeviceGuard g;
  if (int rc = g.enter(h->device)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t bb = 8ll * tokens_per_block;
  const int64_t len = bb * num_blocks;  // only whole blocks are hashed (hash.cpp:61)
  DevBuf tok_tmp, out_tmp, snaps;
  const void *tok_dev = nullptr;
  bool tok_host = false;
  if (int rc = device_view(token_ids, len, h->device, s, tok_tmp, &tok_dev, &tok_host)) return rc;
  int out_is_dev = 0, out_dev = -1;
  pointer_is_device(block_hashes, &out_is_dev, &out_dev);
  if (out_is_dev && out_dev != h->device)
    return fail(FKV_ERR_INVALID_ARG, "block_hashes lives on another device than the hasher");
  uint64_t *out_dev_ptr = block_hashes;
  if (!out_is_dev) {
    out_tmp.s = s;
    if (int rc = scratch_alloc(h->device, (size_t)num_blocks * 8, s, &out_tmp.p)) return rc;
    out_dev_ptr = (uint64_t *)out_tmp.p;
  }
  snaps.s = s;
  if (int rc = scratch_alloc(h->device, (size_t)num_blocks * 32, s, &snaps.p)) return rc;
  XxhState *in = h->states + h->cur;
  if (int rc = run_chain(h, (const uint8_t *)tok_dev, len, bb, num_blocks, (uint64_t *)snaps.p, s)) return rc;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((num_blocks + threads - 1) / threads, 148 * 8);
  xxh_finalize_kernel<<<(int)blocks, threads, 0, s>>>(in, (const uint8_t *)tok_dev, bb, num_blocks,
                                                      (const uint64_t *)snaps.p, out_dev_ptr);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  h->cur ^= 1;
  if (!out_is_dev)
    FKV_CUDA(cudaMemcpyAsync(block_hashes, out_dev_ptr, (size_t)num_blocks * 8, cudaMemcpyDeviceToHost, s));
  if (!out_is_dev || tok_host) {
    FKV_CUDA(cudaStreamSynchronize(s));
    return check_chain(h);
  }
  return FKV_OK;
}

int fkv_gen_hashes_batched(const int64_t *token_ids, const int64_t *seq_offsets, int num_seqs,
                           int tokens_per_block, uint64_t *block_hashes, void *stream) {
  clear_error();
  if (num_seqs < 0 || tokens_per_block <= 0 || (num_seqs > 0 && !seq_offsets))
    return fail(FKV_ERR_INVALID_ARG, "bad batch description");
  if (num_seqs == 0) return FKV_OK;
  cudaStream_t s = (cudaStream_t)stream;
  std::vector<int64_t> table(2 * (size_t)(num_seqs + 1));
  int64_t *tok_off = table.data();
  int64_t *blk_off = table.data() + num_seqs + 1;
  blk_off[0] = 0;
  for (int i = 0; i < num_seqs; ++i) {
    const int64_t a = seq_offsets[i], b = seq_offsets[i + 1];
    if (a < 0 || b < a) return fail(FKV_ERR_INVALID_ARG, "seq_offsets must be non-decreasing and non-negative");
    tok_off[i] = a;
    blk_off[i + 1] = blk_off[i] + (b - a) / tokens_per_block;
  }
  tok_off[num_seqs] = seq_offsets[num_seqs];
  const int64_t total_blocks = blk_off[num_seqs];
  const int64_t total_tokens = seq_offsets[num_seqs];
  if (total_blocks == 0) return FKV_OK;
  if (!token_ids || !block_hashes) return fail(FKV_ERR_INVALID_ARG, "null token or output buffer");
  int device = 0;
  FKV_CUDA(cudaGetDevice(&device));
  DevBuf tok_tmp, out_tmp, tab;
  const void *tok_dev = nullptr;
  bool tok_host = false;
  if (int rc = device_view(token_ids, total_tokens * 8, device, s, tok_tmp, &tok_dev, &tok_host)) return rc;
  int out_is_dev = 0, out_dev = -1;
  pointer_is_device(block_hashes, &out_is_dev, &out_dev);
  uint64_t *out_dev_ptr = block_hashes;
  if (!out_is_dev) {
    out_tmp.s = s;
    if (int rc = scratch_alloc(device, (size_t)total_blocks * 8, s, &out_tmp.p)) return rc;
    out_dev_ptr = (uint64_t *)out_tmp.p;
  }
  ThreadDeviceCtx *ctx = nullptr;
  if (int rc = get_ctx(device, &ctx)) return rc;
  char *stage = nullptr;
  const size_t tb = table.size() * 8;
  if (int rc = acquire_staging(ctx, tb, &stage)) return rc;
  std::memcpy(stage, table.data(), tb);
  tab.s = s;
  if (int rc = scratch_alloc(device, tb, s, &tab.p)) return rc;
  FKV_CUDA(cudaMemcpyAsync(tab.p, stage, tb, cudaMemcpyHostToDevice, s));
  if (int rc = release_staging(ctx, s)) return rc;
  const int64_t *d_tok_off = (const int64_t *)tab.p;
  const int64_t *d_blk_off = d_tok_off + num_seqs + 1;
  const int threads = 256;
  const int blocks = (int)((4ll * num_seqs + threads - 1) / threads);
  xxh_batched_kernel<<<blocks, threads, 0, s>>>((const int64_t *)tok_dev, d_tok_off, d_blk_off,
                                                 num_seqs, tokens_per_block, out_dev_ptr);
  FKV_CUDA(cudaGetLastError());
  note_launch();
  if (!out_is_dev)
    FKV_CUDA(cudaMemcpyAsync(block_hashes, out_dev_ptr, (size_t)total_blocks * 8, cudaMemcpyDeviceToHost, s));
  if (!out_is_dev || tok_host) FKV_CUDA(cudaStreamSynchronize(s));
  return FKV_OK;
}

}  // extern "C"
