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

  for (int l = 0; l < L; ++l) cudaFree(layers[l]);
  cudaFreeHost(pool);
  free(orig);
  free(back);
  free(tok);
  free(hashes);
  return 0;
}
