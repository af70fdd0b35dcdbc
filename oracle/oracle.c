/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle of flexkv_b200.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs may load this library, and only as the checker or
 * the CPU baseline; the product path (flexkv_b200) never links or calls it.
 *
 * 1. oracle_transfer_kv_blocks: restatement of the reference copy kernel
 *    (linhu-nv/FlexKV csrc/transfer.cu:26-61, launcher :63-132) on host
 *    "images" of the GPU layers: same int64-unit stride truncation
 *    (:84-93), same int truncation of block ids (:41-42), same CPU-only
 *    start_layer_id offset (:45), same floor-16-byte chunk copy (:35,55-59),
 *    same chunk enumeration order layer -> kv -> block (:39-42).  The TP
 *    rank offset of tp_transfer_thread_group.cpp:79-80 is the caller's
 *    cpu_startoff argument.  Chunks are copied in enumeration order (a
 *    sequential order for what the GPU kernel races on: duplicate
 *    destinations).
 * 2. XXH64 (seed 0) from the public xxHash specification, streaming
 *    (XXH64_reset/update/digest as used by csrc/hash.cpp:17-45) and the
 *    prefix-chained gen_hashes of csrc/hash.cpp:47-66.
 *
 * 3. oracle_ssd_transfer: restatement of the reference's SSD tier without
 *    io_uring (csrc/transfer_ssd.cpp:17-32 device/file remapping,
 *    :133-176 one pread/pwrite per (block, layer) K chunk then V chunk,
 *    :182-287 num_threads_per_device threads created per call per device
 *    over contiguous block ranges, O_DIRECT descriptors for reads when the
 *    chunk is a multiple of 4 KiB, transfer_ssd.h:196-242).  It is the
 *    reference-style baseline the bench times beside the SSD tier, and a
 *    second checker of its bytes.
 *
 * Parity of (2) is pinned against the python `xxhash` package and the
 * system libxxhash.so.0 in tests/test_oracle.py and tests/golden/.
 */
#define _GNU_SOURCE
#include <fcntl.h>
#include <unistd.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* 1. transfer                                                         */
/* ------------------------------------------------------------------ */

typedef struct {
  int num_blocks, start_layer_id, num_layers, kv_dim, is_h2d;
  const int64_t *gpu_block_ids, *cpu_block_ids;
  char *const *gpu_layer_ptrs;
  int64_t gkv, gbs, ckv, cls, cbs, startoff, copy_int64;
  char *cpu_ptr;
  int64_t chunk_begin, chunk_end;
} oracle_job;

static void *oracle_worker(void *arg) {
  const oracle_job *j = (const oracle_job *)arg;
  const int64_t per_layer = (int64_t)j->num_blocks * j->kv_dim;
  for (int64_t c = j->chunk_begin; c < j->chunk_end; ++c) {
    /* transfer.cu:39-42 */
    int layer_idx = (int)(c / per_layer);
    int kv_idx = (int)((c % per_layer) / j->num_blocks);
    int gpu_block_idx = (int)j->gpu_block_ids[c % j->num_blocks];
    int cpu_block_idx = (int)j->cpu_block_ids[c % j->num_blocks];
    /* transfer.cu:44-50, in int64 units */
    int64_t *cpu_chunk = (int64_t *)j->cpu_ptr + (int64_t)(layer_idx + j->start_layer_id) * j->cls +
                         (int64_t)kv_idx * j->ckv + (int64_t)cpu_block_idx * j->cbs + j->startoff;
    int64_t *gpu_chunk = (int64_t *)j->gpu_layer_ptrs[layer_idx] + (int64_t)kv_idx * j->gkv +
                         (int64_t)gpu_block_idx * j->gbs;
    int64_t *src = j->is_h2d ? cpu_chunk : gpu_chunk;
    int64_t *dst = j->is_h2d ? gpu_chunk : cpu_chunk;
    /* transfer.cu:35: copy_size * sizeof(int64_t) / sizeof(float4) float4s */
    int64_t n16 = j->copy_int64 * 8 / 16;
    memmove(dst, src, (size_t)(n16 * 16));
  }
  return NULL;
}

int oracle_transfer_kv_blocks(int num_blocks, int start_layer_id, int num_layers,
                              const int64_t *gpu_block_ids, char *const *gpu_layer_ptrs,
                              int64_t gpu_kv_stride_in_bytes, int64_t gpu_block_stride_in_bytes,
                              const int64_t *cpu_block_ids, char *cpu_ptr,
                              int64_t cpu_kv_stride_in_bytes, int64_t cpu_layer_stride_in_bytes,
                              int64_t cpu_block_stride_in_bytes,
                              int64_t cpu_startoff_inside_chunks, int64_t chunk_size_in_bytes,
                              int is_host_to_device, int is_mla, int num_threads) {
  oracle_job base;
  memset(&base, 0, sizeof(base));
  base.num_blocks = num_blocks;
  base.start_layer_id = start_layer_id;
  base.num_layers = num_layers;
  base.kv_dim = is_mla ? 1 : 2;
  base.is_h2d = is_host_to_device;
  base.gpu_block_ids = gpu_block_ids;
  base.cpu_block_ids = cpu_block_ids;
  base.gpu_layer_ptrs = gpu_layer_ptrs;
  /* transfer.cu:86-93 */
  base.gkv = gpu_kv_stride_in_bytes / 8;
  base.gbs = gpu_block_stride_in_bytes / 8;
  base.ckv = cpu_kv_stride_in_bytes / 8;
  base.cls = cpu_layer_stride_in_bytes / 8;
  base.cbs = cpu_block_stride_in_bytes / 8;
  base.startoff = cpu_startoff_inside_chunks / 8;
  base.copy_int64 = chunk_size_in_bytes / 8;
  base.cpu_ptr = cpu_ptr;
  int64_t num_chunks = (int64_t)num_layers * base.kv_dim * num_blocks;
  if (num_blocks <= 0 || num_chunks <= 0) return 0;
  if (num_threads <= 1 || num_chunks < 2 * num_threads) {
    base.chunk_begin = 0;
    base.chunk_end = num_chunks;
    oracle_worker(&base);
    return 0;
  }
  if (num_threads > 256) num_threads = 256;
  pthread_t th[256];
  oracle_job jobs[256];
  for (int t = 0; t < num_threads; ++t) {
    jobs[t] = base;
    jobs[t].chunk_begin = num_chunks * t / num_threads;
    jobs[t].chunk_end = num_chunks * (t + 1) / num_threads;
    pthread_create(&th[t], NULL, oracle_worker, &jobs[t]);
  }
  for (int t = 0; t < num_threads; ++t) pthread_join(th[t], NULL);
  return 0;
}

/* ------------------------------------------------------------------ */
/* 2. XXH64                                                            */
/* ------------------------------------------------------------------ */

#define XP1 0x9E3779B185EBCA87ull
#define XP2 0xC2B2AE3D27D4EB4Full
#define XP3 0x165667B19E3779F9ull
#define XP4 0x85EBCA77C2B2AE63ull
#define XP5 0x27D4EB2F165667C5ull

typedef struct {
  uint64_t total_len;
  uint64_t v[4];
  uint8_t mem[32];
  uint32_t memsize;
} oracle_xxh64_state;

static uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
static uint64_t rd64(const uint8_t *p) {
  uint64_t v = 0;
  for (int i = 0; i < 8; ++i) v |= (uint64_t)p[i] << (8 * i);
  return v;
}
static uint64_t rd32(const uint8_t *p) {
  uint64_t v = 0;
  for (int i = 0; i < 4; ++i) v |= (uint64_t)p[i] << (8 * i);
  return v;
}
static uint64_t xround(uint64_t acc, uint64_t in) {
  acc += in * XP2;
  acc = rotl(acc, 31);
  return acc * XP1;
}
static uint64_t xmerge(uint64_t acc, uint64_t val) {
  acc ^= xround(0, val);
  return acc * XP1 + XP4;
}

size_t oracle_xxh64_state_size(void) { return sizeof(oracle_xxh64_state); }

void oracle_xxh64_reset(oracle_xxh64_state *s, uint64_t seed) {
  memset(s, 0, sizeof(*s));
  s->v[0] = seed + XP1 + XP2;
  s->v[1] = seed + XP2;
  s->v[2] = seed;
  s->v[3] = seed - XP1;
}

void oracle_xxh64_update(oracle_xxh64_state *s, const void *input, size_t len) {
  const uint8_t *p = (const uint8_t *)input;
  s->total_len += len;
  if (s->memsize + len < 32) {
    memcpy(s->mem + s->memsize, p, len);
    s->memsize += (uint32_t)len;
    return;
  }
  if (s->memsize) {
    size_t fill = 32 - s->memsize;
    memcpy(s->mem + s->memsize, p, fill);
    for (int i = 0; i < 4; ++i) s->v[i] = xround(s->v[i], rd64(s->mem + 8 * i));
    p += fill;
    len -= fill;
    s->memsize = 0;
  }
  while (len >= 32) {
    for (int i = 0; i < 4; ++i) s->v[i] = xround(s->v[i], rd64(p + 8 * i));
    p += 32;
    len -= 32;
  }
  if (len) {
    memcpy(s->mem, p, len);
    s->memsize = (uint32_t)len;
  }
}

uint64_t oracle_xxh64_digest(const oracle_xxh64_state *s) {
  uint64_t h;
  if (s->total_len >= 32) {
    h = rotl(s->v[0], 1) + rotl(s->v[1], 7) + rotl(s->v[2], 12) + rotl(s->v[3], 18);
    for (int i = 0; i < 4; ++i) h = xmerge(h, s->v[i]);
  } else {
    h = s->v[2] + XP5;
  }
  h += s->total_len;
  const uint8_t *p = s->mem;
  size_t left = s->memsize;
  while (left >= 8) {
    h ^= xround(0, rd64(p));
    h = rotl(h, 27) * XP1 + XP4;
    p += 8;
    left -= 8;
  }
  if (left >= 4) {
    h ^= rd32(p) * XP1;
    h = rotl(h, 23) * XP2 + XP3;
    p += 4;
    left -= 4;
  }
  while (left) {
    h ^= (uint64_t)(*p) * XP5;
    h = rotl(h, 11) * XP1;
    ++p;
    --left;
  }
  h ^= h >> 33;
  h *= XP2;
  h ^= h >> 29;
  h *= XP3;
  h ^= h >> 32;
  return h;
}

uint64_t oracle_xxh64(const void *input, size_t len, uint64_t seed) {
  oracle_xxh64_state s;
  oracle_xxh64_reset(&s, seed);
  oracle_xxh64_update(&s, input, len);
  return oracle_xxh64_digest(&s);
}

/* hash.cpp:47-66: one update per block, digest after each (no reset). */
void oracle_gen_hashes(oracle_xxh64_state *s, const int64_t *token_ids, int tokens_per_block,
                       uint64_t *block_hashes, int64_t num_blocks) {
  for (int64_t i = 0; i < num_blocks; ++i) {
    oracle_xxh64_update(s, token_ids + i * tokens_per_block, (size_t)tokens_per_block * 8);
    block_hashes[i] = oracle_xxh64_digest(s);
  }
}

/* Batched form: a fresh seed-0 state per sequence (block.py:49-57 builds
 * one Hasher per SequenceMeta). */
void oracle_gen_hashes_batched(const int64_t *token_ids, const int64_t *seq_offsets, int num_seqs,
                               int tokens_per_block, uint64_t *block_hashes) {
  int64_t o = 0;
  for (int q = 0; q < num_seqs; ++q) {
    oracle_xxh64_state s;
    oracle_xxh64_reset(&s, 0);
    int64_t nb = (seq_offsets[q + 1] - seq_offsets[q]) / tokens_per_block;
    oracle_gen_hashes(&s, token_ids + seq_offsets[q], tokens_per_block, block_hashes + o, nb);
    o += nb;
  }
}

/* The same over num_threads threads, each taking a contiguous range of
 * sequences (one hasher per sequence, as the reference creates per
 * SequenceMeta): the n-core CPU baseline of the batched hash. */
typedef struct {
  const int64_t *tokens, *offs;
  int q0, q1, tpb;
  uint64_t *out;
  int64_t o0;
} oracle_hash_job;

static void *oracle_hash_worker(void *arg) {
  oracle_hash_job *j = (oracle_hash_job *)arg;
  int64_t o = j->o0;
  for (int q = j->q0; q < j->q1; ++q) {
    oracle_xxh64_state s;
    oracle_xxh64_reset(&s, 0);
    int64_t nb = (j->offs[q + 1] - j->offs[q]) / j->tpb;
    oracle_gen_hashes(&s, j->tokens + j->offs[q], j->tpb, j->out + o, nb);
    o += nb;
  }
  return NULL;
}

void oracle_gen_hashes_batched_mt(const int64_t *token_ids, const int64_t *seq_offsets, int num_seqs,
                                  int tokens_per_block, uint64_t *block_hashes, int num_threads) {
  if (num_threads < 1) num_threads = 1;
  if (num_threads > num_seqs) num_threads = num_seqs > 0 ? num_seqs : 1;
  pthread_t *th = (pthread_t *)calloc((size_t)num_threads, sizeof(pthread_t));
  oracle_hash_job *jobs = (oracle_hash_job *)calloc((size_t)num_threads, sizeof(oracle_hash_job));
  char *started = (char *)calloc((size_t)num_threads, 1);
  int64_t o = 0;
  int q = 0;
  for (int t = 0; t < num_threads; ++t) {
    const int q1 = (int)((int64_t)num_seqs * (t + 1) / num_threads);
    jobs[t] = (oracle_hash_job){token_ids, seq_offsets, q, q1, tokens_per_block, block_hashes, o};
    for (int k = q; k < q1; ++k) o += (seq_offsets[k + 1] - seq_offsets[k]) / tokens_per_block;
    q = q1;
    started[t] = pthread_create(&th[t], NULL, oracle_hash_worker, &jobs[t]) == 0;
    if (!started[t]) oracle_hash_worker(&jobs[t]);
  }
  for (int t = 0; t < num_threads; ++t)
    if (started[t]) pthread_join(th[t], NULL);
  free(started);
  free(jobs);
  free(th);
}


/* ------------------------------------------------------------------ */
/* 3. SSD tier (reference-style loop)                                  */
/* ------------------------------------------------------------------ */

typedef struct {
  const int *fds; /* this device's files */
  int files_per_device;
  const int *cpu_ids, *ssd_in_dev;
  int begin, end, start_layer, end_layer, is_read, is_mla;
  char *cpu;
  int64_t cls, sls, ckv, skv, chunk, bstride;
  int rc;
} oracle_ssd_job;

static void *oracle_ssd_worker(void *arg) {
  oracle_ssd_job *j = (oracle_ssd_job *)arg;
  for (int i = j->begin; i < j->end; ++i) {
    int s = j->ssd_in_dev[i];
    const int fd = j->fds[s % j->files_per_device];
    s /= j->files_per_device;
    for (int l = j->start_layer; l < j->end_layer; ++l) {
      for (int k = 0; k < (j->is_mla ? 1 : 2); ++k) {
        const int64_t so = (int64_t)s * j->bstride + l * j->sls + k * j->skv;
        char *cp = j->cpu + (int64_t)j->cpu_ids[i] * j->bstride + l * j->cls + k * j->ckv;
        const ssize_t n = j->is_read ? pread(fd, cp, (size_t)j->chunk, so) : pwrite(fd, cp, (size_t)j->chunk, so);
        if (n != j->chunk) {
          j->rc = 1;
          return NULL;
        }
      }
    }
  }
  return NULL;
}

/* fds_buf / fds_direct: [num_devices * files_per_device] descriptors opened
 * by the caller (buffered, and with O_DIRECT).  Returns 0, or 1 on a
 * failed or short request. */
int oracle_ssd_transfer(const int *fds_buf, const int *fds_direct, int num_devices, int files_per_device,
                        int start_layer, int num_layers, char *cpu, const int64_t *ssd_ids,
                        const int64_t *cpu_ids, int num_blocks, int64_t cpu_layer_stride,
                        int64_t cpu_kv_stride, int64_t ssd_layer_stride, int64_t ssd_kv_stride,
                        int64_t chunk, int64_t block_stride, int is_read, int round_robin,
                        int threads_per_device, int is_mla) {
  const int direct = is_read && chunk % 4096 == 0;
  const int *fds = direct ? fds_direct : fds_buf;
  int *cpu_part = (int *)malloc(sizeof(int) * (size_t)(num_blocks > 0 ? num_blocks : 1) * num_devices);
  int *ssd_part = (int *)malloc(sizeof(int) * (size_t)(num_blocks > 0 ? num_blocks : 1) * num_devices);
  int *count = (int *)calloc((size_t)num_devices, sizeof(int));
  for (int i = 0; i < num_blocks; ++i) {
    const int64_t sid = ssd_ids[i];
    const int d = (int)((sid / round_robin) % num_devices);
    const int in_dev = (int)(((sid / round_robin) / num_devices) * round_robin + sid % round_robin);
    cpu_part[d * num_blocks + count[d]] = (int)cpu_ids[i];
    ssd_part[d * num_blocks + count[d]] = in_dev;
    ++count[d];
  }
  const int nt = num_devices * threads_per_device;
  pthread_t *th = (pthread_t *)calloc((size_t)nt, sizeof(pthread_t));
  oracle_ssd_job *jobs = (oracle_ssd_job *)calloc((size_t)nt, sizeof(oracle_ssd_job));
  char *started = (char *)calloc((size_t)nt, 1);
  for (int d = 0; d < num_devices; ++d) {
    const int per = (count[d] + threads_per_device - 1) / threads_per_device;
    for (int t = 0; t < threads_per_device; ++t) {
      const int b = t * per, e = b + per < count[d] ? b + per : count[d];
      if (b >= e) continue;
      oracle_ssd_job *j = &jobs[d * threads_per_device + t];
      j->fds = fds + d * files_per_device;
      j->files_per_device = files_per_device;
      j->cpu_ids = cpu_part + d * num_blocks;
      j->ssd_in_dev = ssd_part + d * num_blocks;
      j->begin = b;
      j->end = e;
      j->start_layer = start_layer;
      j->end_layer = start_layer + num_layers;
      j->is_read = is_read;
      j->is_mla = is_mla;
      j->cpu = cpu;
      j->cls = cpu_layer_stride;
      j->sls = ssd_layer_stride;
      j->ckv = cpu_kv_stride;
      j->skv = ssd_kv_stride;
      j->chunk = chunk;
      j->bstride = block_stride;
      started[d * threads_per_device + t] = pthread_create(&th[d * threads_per_device + t], NULL,
                                                           oracle_ssd_worker, j) == 0;
      if (!started[d * threads_per_device + t]) oracle_ssd_worker(j);
    }
  }
  int rc = 0;
  for (int i = 0; i < nt; ++i) {
    if (started[i]) pthread_join(th[i], NULL);
    rc |= jobs[i].rc;
  }
  free(started);
  free(jobs);
  free(th);
  free(count);
  free(ssd_part);
  free(cpu_part);
  return rc;
}
