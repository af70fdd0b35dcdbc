/*
 * A caller of the flexkv_b200 C ABI with no Python and no torch: what a
 * native binding (pybind11, cgo, JNI, ...) sees.  Built by
 * tests/test_c_abi.py with plain gcc against include/flexkv_b200.h.
 *
 *   c_abi_demo <token_count> <tokens_per_block>
 *
 * 1. KV round trip: 4 layers of [2, 64 blocks, 16 tokens, 2 heads, 64 dims]
 *    bf16 in device memory, a page-locked LAYERWISE host pool of 128 blocks;
 *    D2H of 24 block pairs, zero those GPU blocks, H2D back, compare every
 *    byte of the layers with the original.
 * 2. Block hashes: gen_hashes over token ids 0..token_count-1 (int64) from
 *    host memory; prints the digests, one per line, for the caller to check.
 * 3. CPU-tier cache index: put two 5-block sequences that share 3 blocks
 *    (the second skips the shared prefix), match both, then get the first
 *    into other GPU blocks and compare those bytes with its source blocks.
 * Exit status 0 on success; any failure prints fkv_last_error().
 */
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "flexkv_b200.h"

#define CHECK(x)                                                             \
  do {                                                                       \
    int rc_ = (x);                                                           \
    if (rc_ != 0) {                                                          \
      fprintf(stderr, "%s failed (%d): %s\n", #x, rc_, fkv_last_error());    \
      return 1;                                                              \
    }                                                                        \
  } while (0)
#define CUDA(x)                                                              \
  do {                                                                       \
    cudaError_t e_ = (x);                                                    \
    if (e_ != cudaSuccess) {                                                 \
      fprintf(stderr, "%s failed: %s\n", #x, cudaGetErrorString(e_));        \
      return 1;                                                              \
    }                                                                        \
  } while (0)

int main(int argc, char **argv) {
  const int64_t n_tok = argc > 1 ? atoll(argv[1]) : 256;
  const int tpb = argc > 2 ? atoi(argv[2]) : 16;
  enum { L = 4, KV = 2, NG = 64, NC = 128, N = 24 };
  const int64_t chunk = 16 * 2 * 64 * 2;               /* tpb * heads * dim * bf16 */
  const int64_t layer_bytes = (int64_t)KV * NG * chunk;
  const int64_t pool_bytes = (int64_t)L * KV * NC * chunk;

  /* device layers with a byte pattern, and their host copies */
  void *layers[L];
  unsigned char *orig = (unsigned char *)malloc((size_t)(L * layer_bytes));
  for (int64_t i = 0; i < L * layer_bytes; ++i) orig[i] = (unsigned char)((i * 2654435761u) >> 13);
  for (int l = 0; l < L; ++l) {
    CUDA(cudaMalloc(&layers[l], (size_t)layer_bytes));
    CUDA(cudaMemcpy(layers[l], orig + l * layer_bytes, (size_t)layer_bytes, cudaMemcpyHostToDevice));
  }
  void *pool = NULL;
  CUDA(cudaHostAlloc(&pool, (size_t)pool_bytes, cudaHostAllocPortable | cudaHostAllocMapped));
  memset(pool, 0, (size_t)pool_bytes);

  int64_t gids[N], cids[N];
  for (int i = 0; i < N; ++i) {
    gids[i] = (i * 37 + 5) % NG;  /* distinct: 37 is coprime with 64 */
    cids[i] = (i * 53 + 11) % NC; /* distinct: 53 is coprime with 128 */
  }
  /* LAYERWISE host strides: layer kv*NC*chunk, kv NC*chunk, block chunk;
   * GPU per-layer strides: kv NG*chunk, block chunk. */
  CHECK(fkv_transfer_kv_blocks(N, 0, L, gids, (void *const *)layers, NG * chunk, chunk, cids, pool,
                               NC * chunk, KV * NC * chunk, chunk, 0, chunk, NULL, -1, 0, 0, 0));
  for (int l = 0; l < L; ++l)
    for (int k = 0; k < KV; ++k)
      for (int i = 0; i < N; ++i)
        CUDA(cudaMemset((char *)layers[l] + k * NG * chunk + gids[i] * chunk, 0, (size_t)chunk));
  CHECK(fkv_transfer_kv_blocks(N, 0, L, gids, (void *const *)layers, NG * chunk, chunk, cids, pool,
                               NC * chunk, KV * NC * chunk, chunk, 0, chunk, NULL, -1, 1, 0, 0));
  unsigned char *back = (unsigned char *)malloc((size_t)layer_bytes);
  for (int l = 0; l < L; ++l) {
    CUDA(cudaMemcpy(back, layers[l], (size_t)layer_bytes, cudaMemcpyDeviceToHost));
    if (memcmp(back, orig + l * layer_bytes, (size_t)layer_bytes) != 0) {
      fprintf(stderr, "layer %d differs after the round trip\n", l);
      return 1;
    }
  }

  /* block hashes from host buffers */
  int64_t *tok = (int64_t *)malloc((size_t)n_tok * 8);
  for (int64_t i = 0; i < n_tok; ++i) tok[i] = i;
  const int64_t nb = n_tok / tpb;
  uint64_t *hashes = (uint64_t *)calloc((size_t)(nb > 0 ? nb : 1), 8);
  fkv_hasher *h = NULL;
  CHECK(fkv_hasher_create(-1, &h));
  CHECK(fkv_gen_hashes(h, tok, n_tok, tpb, hashes, nb, NULL));
  fkv_hasher_destroy(h);
  for (int64_t b = 0; b < nb; ++b) printf("%llu\n", (unsigned long long)hashes[b]);

  /* CPU-tier cache index: put, match, get */
  {
    enum { TPB = 16, NB = 5 };
    int64_t seq[2 * NB * TPB];
    for (int i = 0; i < NB * TPB; ++i) seq[i] = 1000 + i;                       /* A */
    for (int i = 0; i < NB * TPB; ++i) seq[NB * TPB + i] = i < 3 * TPB ? 1000 + i : 5000 + i; /* B */
    const int64_t offs[3] = {0, NB * TPB, 2 * NB * TPB};
    int64_t put_gpu[2 * NB], skipped[2], moved[2], cpu_of[2 * NB];
    for (int i = 0; i < NB; ++i) { put_gpu[i] = i; put_gpu[NB + i] = 10 + i; }
    fkv_transfer_desc d;
    fkv_transfer_desc_init(&d);
    d.num_layers = L;
    d.gpu_layer_ptrs = (void *const *)layers;
    d.cpu_ptr = pool;
    d.gpu_kv_stride_in_bytes = NG * chunk;
    d.gpu_block_stride_in_bytes = chunk;
    d.cpu_kv_stride_in_bytes = NC * chunk;
    d.cpu_layer_stride_in_bytes = KV * NC * chunk;
    d.cpu_block_stride_in_bytes = chunk;
    d.chunk_size_in_bytes = chunk;
    d.cpu_pool_bytes = pool_bytes;
    d.gpu_layer_bytes = layer_bytes;
    fkv_cache_index *ci = NULL;
    CHECK(fkv_cache_index_create(-1, NC, TPB, &ci));
    d.is_host_to_device = 0;
    CHECK(fkv_cache_index_put(ci, seq, offs, 2, put_gpu, &d, 1, 1, skipped, moved, cpu_of, NULL, NULL));
    if (skipped[0] != 0 || moved[0] != NB || skipped[1] != 3 || moved[1] != 2) {
      fprintf(stderr, "put: skipped %lld/%lld moved %lld/%lld\n", (long long)skipped[0], (long long)skipped[1],
              (long long)moved[0], (long long)moved[1]);
      return 1;
    }
    int64_t matched[2], ready[2];
    CHECK(fkv_cache_index_match(ci, seq, offs, 2, matched, ready, NULL, NULL));
    if (matched[0] != NB || matched[1] != NB || ready[0] != NB || ready[1] != NB) {
      fprintf(stderr, "match: %lld/%lld ready %lld/%lld\n", (long long)matched[0], (long long)matched[1],
              (long long)ready[0], (long long)ready[1]);
      return 1;
    }
    int64_t get_gpu[NB], got[1];
    for (int i = 0; i < NB; ++i) get_gpu[i] = 20 + i;
    d.is_host_to_device = 1;
    CHECK(fkv_cache_index_get(ci, seq, offs, 1, NULL, get_gpu, &d, 0, NULL, 1, got, NULL, NULL));
    if (got[0] != NB) {
      fprintf(stderr, "get: %lld blocks\n", (long long)got[0]);
      return 1;
    }
    for (int l = 0; l < L; ++l) {
      CUDA(cudaMemcpy(back, layers[l], (size_t)layer_bytes, cudaMemcpyDeviceToHost));
      for (int k = 0; k < KV; ++k)
        for (int i = 0; i < NB; ++i)
          if (memcmp(back + k * NG * chunk + (20 + i) * chunk, orig + l * layer_bytes + k * NG * chunk + i * chunk,
                     (size_t)chunk) != 0) {
            fprintf(stderr, "get: layer %d kv %d block %d differs\n", l, k, 20 + i);
            return 1;
          }
    }
    int64_t st[7];
    CHECK(fkv_cache_index_stats(ci, st, NULL));
    if (st[0] != NC - 7 || st[1] != 7 || st[2] != 7) {
      fprintf(stderr, "stats: free %lld cached %lld ready %lld\n", (long long)st[0], (long long)st[1],
              (long long)st[2]);
      return 1;
    }
    fkv_cache_index_destroy(ci);
  }

  for (int l = 0; l < L; ++l) cudaFree(layers[l]);
  cudaFreeHost(pool);
  free(orig);
  free(back);
  free(tok);
  free(hashes);
  return 0;
}
