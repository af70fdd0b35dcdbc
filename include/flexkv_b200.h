/*
 * flexkv_b200 — C ABI of the B200-native FlexKV transfer data plane.
 *
 * Plain pointers, sizes and status codes; no torch types.  Every entry
 * point returns FKV_OK (0) or a positive FKV_ERR_* code; the message of the
 * last failure on the calling thread is returned by fkv_last_error().
 *
 * Reference interfaces replaced (paths inside linhu-nv/FlexKV):
 *   fkv_transfer_kv_blocks      <- flexkv::transfer_kv_blocks
 *                                  csrc/transfer.cuh:23-30, csrc/transfer.cu:63-132
 *                                  (called through csrc/bindings.cpp:25-55)
 *   fkv_tp_group_*              <- flexkv::TPTransferThreadGroup
 *                                  csrc/tp_transfer_thread_group.h:30-57,
 *                                  csrc/tp_transfer_thread_group.cpp:23-109
 *   fkv_hasher_*, fkv_gen_hashes, fkv_get_hash_size
 *                               <- flexkv::Hasher / gen_hashes / get_hash_size
 *                                  csrc/cache_utils.h:10-28, csrc/hash.cpp:15-66
 *   fkv_host_register           <- cudaHostRegister helper, flexkv/transfer/worker.py:35-47
 *
 * Byte-layout contract (identical to the reference kernel, transfer.cu:39-59):
 *   for layer l in [0,L), kv in [0,kv_dim), i in [0,N):
 *     cpu = cpu_ptr + (l+start_layer_id)*cpu_layer_stride + kv*cpu_kv_stride
 *                   + cpu_block_ids[i]*cpu_block_stride + cpu_startoff
 *     gpu = gpu_layer_ptrs[l] + kv*gpu_kv_stride + gpu_block_ids[i]*gpu_block_stride
 *     copy 16*floor(chunk/16) bytes, direction by is_host_to_device.
 *   Strides and the start offset are truncated to multiples of 8 bytes, as
 *   the reference's int64-unit conversion does (transfer.cu:84-93).
 */
#ifndef FLEXKV_B200_H_
#define FLEXKV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define FKV_OK 0
#define FKV_ERR_INVALID_ARG 1  /* bad shape/size/flag combination           */
#define FKV_ERR_OUT_OF_RANGE 2 /* a block id addresses outside a pool       */
#define FKV_ERR_MISALIGNED 3   /* a chunk address is not 16-byte aligned    */
#define FKV_ERR_CUDA 4         /* a CUDA runtime call failed                */
#define FKV_ERR_UNSUPPORTED 5  /* feature not provided by this build        */
#define FKV_ERR_TIMEOUT 6      /* a bounded wait ran out                    */
#define FKV_ERR_IO 7           /* a file operation failed or came up short  */

/* Message of the last failure on this thread ("" if none). */
const char *fkv_last_error(void);
/* Library version string. */
const char *fkv_version(void);
/* Number of CUDA kernels this library launched so far (all threads). */
uint64_t fkv_kernel_launch_count(void);

/* ---- host pool registration (worker.py:35-47) -------------------------- */
/* Page-lock [ptr, ptr+bytes) for zero-copy device access (Portable|Mapped).
 * advise_hugepages != 0 first asks the kernel for transparent huge pages on
 * the range (only effective before the pages are first touched). */
int fkv_host_register(void *ptr, int64_t bytes, int advise_hugepages);
int fkv_host_unregister(void *ptr);

/* ---- KV block gather/scatter ------------------------------------------ */

/* Drop-in for flexkv::transfer_kv_blocks (transfer.cu:63-132).
 * gpu_block_ids / cpu_block_ids / gpu_layer_ptrs are HOST arrays (pinned or
 * pageable); cpu_ptr is a page-locked host pool; stream is a cudaStream_t
 * (NULL = legacy default stream).  transfer_sms = -1 picks the default SM
 * budget.  use_ce_transfer != 0 routes every chunk through the copy engines
 * (coalesced into runs); otherwise long contiguous runs go to the copy
 * engines and the rest to the SM copy kernel.  Synchronous on return, like
 * the reference (transfer.cu:131).  Unlike the reference it validates
 * alignment and (when the pool sizes are known, see _ex) bounds on the host
 * and returns an error instead of faulting. */
int fkv_transfer_kv_blocks(int num_blocks, int start_layer_id, int num_layers,
                           const int64_t *gpu_block_ids,
                           void *const *gpu_layer_ptrs,
                           int64_t gpu_kv_stride_in_bytes,
                           int64_t gpu_block_stride_in_bytes,
                           const int64_t *cpu_block_ids, void *cpu_ptr,
                           int64_t cpu_kv_stride_in_bytes,
                           int64_t cpu_layer_stride_in_bytes,
                           int64_t cpu_block_stride_in_bytes,
                           int64_t cpu_startoff_inside_chunks,
                           int64_t chunk_size_in_bytes, void *stream,
                           int transfer_sms, int is_host_to_device,
                           int use_ce_transfer, int is_mla);

/* Allocation-free variant of fkv_transfer_kv_blocks, with no counterpart in
 * the reference.  For callers that cannot allocate device memory while they
 * move KV blocks (an engine whose caching allocator owns the GPU, a thread
 * under a strict memory budget): the copy kernel's scratch (layer-pointer
 * table and block-id arrays) lives in a 132 KiB file-scope device array
 * that every GPU loading this library holds until exit, instead of the
 * library's memory pool.  At most 8192 blocks and 512 layers per call
 * (larger requests return FKV_ERR_INVALID_ARG); SM copy kernel only.
 * Synchronous.  All calls share the one array, so calls that overlap on the
 * GPU (several threads or streams at once) race.  The first call on a
 * device resolves the array's address (cudaGetSymbolAddress with that
 * device current); make it before any stream capture.  cpu_pool_bytes /
 * gpu_layer_bytes > 0 enable the bounds checks. */
int fkv_transfer_kv_blocks_noalloc(int num_blocks, int start_layer_id, int num_layers,
                                   const int64_t *gpu_block_ids,
                                   void *const *gpu_layer_ptrs,
                                   int64_t gpu_kv_stride_in_bytes,
                                   int64_t gpu_block_stride_in_bytes,
                                   const int64_t *cpu_block_ids, void *cpu_ptr,
                                   int64_t cpu_kv_stride_in_bytes,
                                   int64_t cpu_layer_stride_in_bytes,
                                   int64_t cpu_block_stride_in_bytes,
                                   int64_t cpu_startoff_inside_chunks,
                                   int64_t chunk_size_in_bytes, int64_t cpu_pool_bytes,
                                   int64_t gpu_layer_bytes, void *stream,
                                   int transfer_sms, int is_host_to_device, int is_mla);

/* Full descriptor of one transfer (superset of the reference arguments). */
typedef struct fkv_transfer_desc {
  int num_blocks;
  int start_layer_id;
  int num_layers;
  int is_host_to_device;
  int is_mla;
  int transfer_sms;       /* SMs for the copy kernel; -1 = default: 8 for a
                             synchronous call, 16 for an asynchronous one or
                             a plan (measured A/B: fewer SMs leave the copy
                             engines more of the link while one direction
                             runs alone; 16 keep both directions fuller)  */
  int use_ce_transfer;    /* 1 = copy engines only                         */
  int synchronous;        /* 1 = stream-synchronize before returning       */
  const int64_t *gpu_block_ids;
  const int64_t *cpu_block_ids;
  void *const *gpu_layer_ptrs;
  void *cpu_ptr;
  int64_t gpu_kv_stride_in_bytes;
  int64_t gpu_block_stride_in_bytes;
  int64_t cpu_kv_stride_in_bytes;
  int64_t cpu_layer_stride_in_bytes;
  int64_t cpu_block_stride_in_bytes;
  int64_t cpu_startoff_inside_chunks;
  int64_t chunk_size_in_bytes;
  int64_t cpu_pool_bytes;    /* >0: bounds-check every CPU chunk           */
  int64_t gpu_layer_bytes;   /* >0: bounds-check every GPU chunk per layer */
  int64_t ce_min_run_bytes;  /* <0 default (1 MiB; 256 KiB for H2D when
                                transfer_sms is 1-4; 128 KiB for a run that
                                folds into one descriptor across all
                                layers); 0 = SM kernel only; else runs whose
                                per-(layer,kv) row reaches this many bytes
                                go to the copy engines.  Folding: when the
                                GPU layers sit at one uniform stride (one
                                allocation viewed per layer), a run
                                contiguous on both sides is one 2-D copy
                                through every layer.                      */
  int num_ce_streams;        /* <=0 default                               */
  int ce_schedule;           /* -1 default; 0 copy engines concurrent with
                                the SM kernel; 1 copy engines first; 2 SM
                                kernel first                              */
} fkv_transfer_desc;

/* Zero-fill *d and set the defaults (transfer_sms=-1, synchronous=1,
 * ce_min_run_bytes=-1, num_ce_streams=0, ce_schedule=-1). */
void fkv_transfer_desc_init(fkv_transfer_desc *d);

int fkv_transfer_kv_blocks_ex(const fkv_transfer_desc *d, void *stream);

/* Two-phase form: plan once (validate, coalesce runs, upload ids to the
 * device), execute many times.  Execute is asynchronous on the stream and
 * launches the SM kernel plus the copy-engine copies of the plan. */
typedef struct fkv_plan fkv_plan;
int fkv_plan_create(const fkv_transfer_desc *d, int device, fkv_plan **out);
int fkv_plan_execute(fkv_plan *plan, void *stream);
/* As fkv_plan_execute; when non-NULL, the cudaEvent_t handles are recorded
 * on `stream` immediately before and after the SM copy kernel (both at the
 * same point when the plan has no SM chunks), so the kernel can be timed
 * apart from the overlapping copy-engine work. */
int fkv_plan_execute_ex(fkv_plan *plan, void *stream, void *kernel_start_event,
                        void *kernel_end_event);
/* Number of SM-kernel chunks and copy-engine copies in the plan. */
int fkv_plan_stats(const fkv_plan *plan, int64_t *sm_chunks,
                   int64_t *ce_copies, int64_t *ce_bytes, int64_t *sm_bytes);
void fkv_plan_destroy(fkv_plan *plan);

/* Host-side run coalescing (pure host logic, no CUDA): writes up to
 * max_runs triples (gpu_start, cpu_start, length) of maximal runs where
 * both ids advance by one, returns the run count (or -1 when max_runs is
 * too small). */
int64_t fkv_coalesce_runs(const int64_t *gpu_block_ids,
                          const int64_t *cpu_block_ids, int64_t num_blocks,
                          int64_t *runs_out, int64_t max_runs);

/* ---- tensor-parallel group (tp_transfer_thread_group.cpp) -------------- */
typedef struct fkv_tp_group fkv_tp_group;

/* gpu_layer_ptrs is rank-major [num_gpus][num_layers]; device_ids[i] is the
 * CUDA device of rank i (the reference uses dp_group_id*num_gpus+i,
 * tp_transfer_thread_group.cpp:41,81).  One persistent host thread and one
 * stream per rank. cpu_pool_bytes > 0 enables CPU bounds checks. */
int fkv_tp_group_create(int num_gpus, int dp_group_id, const int *device_ids,
                        void *const *gpu_layer_ptrs, int num_layers,
                        void *cpu_ptr, int64_t cpu_pool_bytes,
                        fkv_tp_group **out);
/* Same arguments as TPTransferThreadGroup::tp_group_transfer
 * (tp_transfer_thread_group.cpp:48-59).  Rank i moves its gpu_chunk bytes to
 * CPU offset i*gpu_chunk inside each CPU chunk (0 for MLA).  Layer pointers
 * of rank i are gpu_layer_ptrs[i*num_layers + layer_id + l]. */
int fkv_tp_group_transfer(fkv_tp_group *g, const int64_t *gpu_block_ids,
                          const int64_t *cpu_block_ids, int num_blocks,
                          int64_t gpu_kv_stride_in_bytes,
                          int64_t gpu_block_stride_in_bytes,
                          int64_t gpu_chunk_size_in_bytes,
                          int64_t cpu_kv_stride_in_bytes,
                          int64_t cpu_layer_stride_in_bytes,
                          int64_t cpu_block_stride_in_bytes,
                          int64_t cpu_chunk_size_in_bytes, int transfer_sms,
                          int is_host_to_device, int use_ce_transfer,
                          int layer_id, int layer_granularity, int is_mla);
int fkv_tp_group_num_gpus(const fkv_tp_group *g);
void fkv_tp_group_destroy(fkv_tp_group *g);

/* ---- transfer engine (TransferEngine data plane) ------------------------
 * Replaces the GPU<->CPU part of flexkv/transfer/transfer_engine.py:197-307
 * and its worker processes (flexkv/transfer/worker.py:144-177, 259-480):
 * one engine per data-parallel group (one GPU, or the GPUs of a TP group).
 * A graph's ops are enqueued at once; a dependency is an event wait on the
 * GPU; H2D and D2H ops use separate streams per GPU; id tables are staged
 * in an engine-owned pinned ring; completions are polled as (graph_id,
 * op_id) pairs with op_id = -1 for a finished graph.  Independent ops of
 * one direction alternate over a small stream pool, so consecutive small
 * ops overlap their tails.  With an SSD context
 * the engine also runs DISK2H / H2DISK ops (CPUSSDDiskTransferWorker,
 * worker.py:482-590) on two engine-owned I/O threads, one per direction:
 * such an op starts once its predecessors have completed, and a GPU op
 * that follows one is enqueued once it has completed. */
#define FKV_OP_H2D 0
#define FKV_OP_D2H 1
#define FKV_OP_VIRTUAL 2 /* no data; completes when its predecessors do */
#define FKV_OP_DISK2H 3  /* SSD -> cpu pool (needs the config's ssd_ctx)  */
#define FKV_OP_H2DISK 4  /* cpu pool -> SSD                                */

typedef struct fkv_engine fkv_engine;
typedef struct fkv_ssd_ctx fkv_ssd_ctx; /* SSD tier context, declared below */

typedef struct fkv_engine_config {
  int num_ranks;                /* GPUs of the group (TP ranks)              */
  int num_layers;
  const int *device_ids;        /* [num_ranks]; NULL = 0..num_ranks-1        */
  void *const *gpu_layer_ptrs;  /* rank-major [num_ranks][num_layers]        */
  void *cpu_ptr;                /* page-locked host pool shared by the ranks */
  int64_t cpu_pool_bytes;       /* >0: bounds-check CPU chunks               */
  int64_t gpu_layer_bytes;      /* >0: bounds-check GPU chunks               */
  int64_t gpu_kv_stride_in_bytes;
  int64_t gpu_block_stride_in_bytes;
  int64_t gpu_chunk_size_in_bytes;
  int64_t cpu_kv_stride_in_bytes;
  int64_t cpu_layer_stride_in_bytes;
  int64_t cpu_block_stride_in_bytes;
  int64_t cpu_chunk_size_in_bytes;
  int is_mla;
  int transfer_sms_h2d;         /* -1 = default                              */
  int transfer_sms_d2h;
  int use_ce_h2d;               /* copy engines only, per direction          */
  int use_ce_d2h;
  int streams_per_direction;    /* stream pool per direction per GPU; <= 0 = 2 */
  int64_t staging_bytes;        /* pinned id-table ring; <= 0 = 32 MiB       */
  /* SSD tier (optional; ssd_ctx NULL = no DISK2H / H2DISK ops).  Chunk and
   * block stride are the cpu pool's, as CPUSSDDiskTransferWorker passes
   * them (worker.py:514-520); the ctx stays owned by the caller. */
  fkv_ssd_ctx *ssd_ctx;
  int64_t ssd_layer_stride_in_bytes;
  int64_t ssd_kv_stride_in_bytes;
  int ssd_num_blocks_per_file;
  int ssd_round_robin;          /* <= 0 = 1                                  */
  int ssd_threads_per_device;   /* <= 0 = 32 (worker.py:573)                 */
  int ssd_reserved;
} fkv_engine_config;

typedef struct fkv_engine_op {
  int64_t op_id;
  int type;                     /* FKV_OP_*                                  */
  int num_blocks;
  const int64_t *gpu_block_ids; /* host arrays, copied at submission; the
                                   SSD block ids for DISK2H / H2DISK         */
  const int64_t *cpu_block_ids;
  int layer_id;                 /* first layer; -1 = 0 (worker.py:318-321)   */
  int layer_granularity;        /* layers; -1 = all remaining                */
  int num_predecessors;
  int reserved;
  const int64_t *predecessors;  /* op ids of the same graph                  */
} fkv_engine_op;

/* Zero-fill and set defaults (num_ranks=1, transfer_sms_*=-1). */
void fkv_engine_config_init(fkv_engine_config *c);
int fkv_engine_create(const fkv_engine_config *c, fkv_engine **out);
/* Queue a graph; returns once its ops are copied (non-blocking). */
int fkv_engine_submit_graph(fkv_engine *e, int64_t graph_id, const fkv_engine_op *ops,
                            int n_ops);
/* Up to max completions (graph_id, op_id, status); waits up to timeout_ms
 * (0 = poll) for the first one. */
int fkv_engine_poll(fkv_engine *e, int64_t *graph_ids, int64_t *op_ids, int *statuses,
                    int max, int timeout_ms, int *n_out);
/* Ops submitted and not yet reported complete. */
int64_t fkv_engine_pending_ops(fkv_engine *e);
/* Finish the ops already submitted, then release the engine. */
void fkv_engine_destroy(fkv_engine *e);
/* fkv_engine_destroy with a bound (the reference's worker shutdown joins
 * for 5 s and then terminates, worker.py:190-202): waits at most timeout_ms
 * (< 0: no limit) for the submitted ops to drain.  FKV_ERR_TIMEOUT if they
 * did not: the engine keeps running detached until they finish, stays
 * allocated, and must not be used again (its buffers must stay valid). */
int fkv_engine_shutdown(fkv_engine *e, int timeout_ms);

/* ---- XXH64 block hashing (hash.cpp) ------------------------------------ */
typedef struct fkv_hasher fkv_hasher;

/* sizeof(XXH64 digest) = 8 (hash.cpp:15). */
int fkv_get_hash_size(void);

/* A streaming XXH64 (seed 0) whose state lives in device memory of
 * `device`; all mixing arithmetic runs in CUDA kernels. */
int fkv_hasher_create(int device, fkv_hasher **out);
void fkv_hasher_destroy(fkv_hasher *h);
int fkv_hasher_reset(fkv_hasher *h, void *stream);
/* data may be host or device memory; returns after the state is updated. */
int fkv_hasher_update(fkv_hasher *h, const void *data, int64_t size,
                      void *stream);
/* Diagnostic form of fkv_hasher_update (no counterpart in the reference):
 * every producer/consumer hand-off wait of the two-warp chain kernel gives
 * up after wait_limit_ns (at most 2 s, the limit of every other call), and
 * producer_tiles >= 0 makes the producer warp stop after that many 8 KiB
 * tiles (-1: all).  With fewer tiles than the data holds, the chain warp's
 * wait runs out and the call returns FKV_ERR_TIMEOUT; the kernel returns
 * cleanly, the hasher keeps the state it had before the call and the CUDA
 * context stays usable.  Synchronous.  Used by the tests of the bounded
 * waits; the data must be device memory, 8-byte aligned, for the two-warp
 * path (other data takes the one-warp path, which has no hand-off). */
int fkv_hasher_update_bounded(fkv_hasher *h, const void *data, int64_t size,
                              uint64_t wait_limit_ns, int64_t producer_tiles,
                              void *stream);
int fkv_hasher_digest(fkv_hasher *h, uint64_t *out, void *stream);

/* gen_hashes (hash.cpp:47-66): for block b, update the hasher with tokens
 * [b*tpb,(b+1)*tpb) (int64) and store digest() — the XXH64 of the running
 * prefix — into block_hashes[b].  token_ids / block_hashes may each be
 * host or device memory.  The hasher keeps the state after the last block.
 * num_blocks must equal num_tokens / tokens_per_block. */
int fkv_gen_hashes(fkv_hasher *h, const int64_t *token_ids, int64_t num_tokens,
                   int tokens_per_block, uint64_t *block_hashes,
                   int64_t num_blocks, void *stream);

/* Batched gen_hashes over independent sequences, each with a fresh seed-0
 * hasher: sequence s owns tokens [seq_offsets[s], seq_offsets[s+1]) and
 * writes floor(len_s/tpb) digests starting at block_hashes[block_offset_s],
 * block_offset_s being the running sum of the previous sequences' counts.
 * seq_offsets is a host array of num_seqs+1 entries; token_ids and
 * block_hashes may be host or device memory. */
int fkv_gen_hashes_batched(const int64_t *token_ids,
                           const int64_t *seq_offsets, int num_seqs,
                           int tokens_per_block, uint64_t *block_hashes,
                           void *stream);

/* ------------------------------------------------------------------------
 * CUDA-IPC registration boundary.  The inference engine's process owns the
 * paged GPU KV cache; the process running the transfers maps it.  Replaces
 * TensorSharedHandle (flexkv/common/memory_handle.py:17-56, used by
 * KVTPClient.register_to_server, flexkv/server/client.py:199-215), which
 * goes through torch.multiprocessing.reductions; this handle is a plain
 * struct that a process with or without torch can produce and consume.
 *
 * Only memory from cudaMalloc-style allocations can be exported (torch's
 * default caching allocator); virtual-memory allocations (torch
 * expandable segments) fail with FKV_ERR_CUDA and a message saying so.
 * ---------------------------------------------------------------------- */
typedef struct fkv_ipc_handle {
  unsigned char cuda_handle[64]; /* cudaIpcMemHandle_t of the allocation     */
  uint64_t base_addr;            /* allocation base in the exporting process  */
  uint64_t alloc_bytes;          /* allocation size                            */
  int64_t offset;                /* range start - allocation base              */
  int64_t bytes;                 /* range length                               */
  int32_t device;                /* exporting device ordinal                   */
  int32_t pid;                   /* exporting process id                       */
} fkv_ipc_handle;

/* Describe [dev_ptr, dev_ptr + bytes) for another process.  Does not
 * allocate or copy; the exporter keeps the memory alive while any importer
 * uses it. */
int fkv_ipc_export(const void *dev_ptr, int64_t bytes, fkv_ipc_handle *out);

/* Map the range described by h into this process and return its address.
 * Opens of ranges of one allocation share one mapping (reference counted).
 * device = -1 maps on h->device; another ordinal maps through peer access.
 * In the exporting process itself the original address is returned. */
int fkv_ipc_open(const fkv_ipc_handle *h, int device, void **out_ptr);

/* Release one open of the mapping containing ptr; the last release unmaps.
 * FKV_ERR_INVALID_ARG if ptr lies in no range opened here. */
int fkv_ipc_close(void *ptr);

/* Number of allocations currently mapped through fkv_ipc_open. */
int fkv_ipc_open_count(void);

/* ------------------------------------------------------------------------
 * SSD tier: CPU pool <-> SSD files.  Replaces SSDIOCTX and
 * transfer_kv_blocks_ssd (csrc/transfer_ssd.h:170-264,
 * csrc/transfer_ssd.cpp:17-287, bound at csrc/bindings.cpp:57-77,110-119,
 * 141-142) with the same on-disk format: SSD block s is on device
 * d = (s/rr) % D at in-device index i = ((s/rr)/D)*rr + s%rr, in file i % F
 * at file block i / F; chunk (layer l, kv k) at file byte
 * (i/F)*block_stride + l*ssd_layer_stride + k*ssd_kv_stride.
 * ---------------------------------------------------------------------- */
/* paths[d * files_per_device + f] is file f of device d; every file is
 * opened read-write (buffered, plus O_DIRECT where the filesystem allows).
 * iouring_entries > 0 issues requests through io_uring rings of that depth
 * (one per direction; iouring_flags go to io_uring_setup), as the
 * reference's optional io_uring path does; 0, or a ring that cannot be set
 * up, issues them from a thread pool. */
int fkv_ssd_ctx_create(const char *const *paths, int num_devices,
                       int files_per_device, int iouring_entries,
                       int iouring_flags, fkv_ssd_ctx **out);
void fkv_ssd_ctx_destroy(fkv_ssd_ctx *ctx);

/* Move layers [start_layer, start_layer + num_layers) of each block pair
 * (is_read: SSD -> CPU, else CPU -> SSD).  Synchronous: returns when every
 * byte is in place.  cpu_pool_bytes > 0 bounds-checks the CPU side (the
 * reference does no check; 0 keeps that).  num_threads_per_device requests
 * run in parallel per device.  num_blocks_per_file is accepted and, as in
 * the reference, not used.  Ids must lie in [0, 2^31). */
int fkv_transfer_kv_blocks_ssd(fkv_ssd_ctx *ctx, int start_layer, int num_layers,
                               void *cpu_ptr, int64_t cpu_pool_bytes,
                               const int64_t *ssd_block_ids,
                               const int64_t *cpu_block_ids, int64_t num_blocks,
                               int64_t cpu_layer_stride_in_bytes,
                               int64_t cpu_kv_stride_in_bytes,
                               int64_t ssd_layer_stride_in_bytes,
                               int64_t ssd_kv_stride_in_bytes,
                               int64_t chunk_size_in_bytes,
                               int64_t block_stride_in_bytes, int is_read,
                               int num_blocks_per_file, int round_robin,
                               int num_threads_per_device, int is_mla);

/* 1 if the context issues requests through io_uring, 0 for the thread pool. */
int fkv_ssd_ctx_uses_io_uring(const fkv_ssd_ctx *ctx);

/* File requests and bytes of the context's most recent transfer (chunks
 * adjacent in both the file and the pool are merged into one request). */
int fkv_ssd_last_stats(const fkv_ssd_ctx *ctx, int64_t *num_ios, int64_t *bytes);

/* ------------------------------------------------------------------------
 * Put and get paths of the CPU tier on the device: block index, block pool,
 * the fused put (hash -> match -> allocate -> insert -> D2H copy -> ready in
 * one stream of kernels) and the fused get (hash -> match -> H2D copy).
 * Replaces, for the CPU tier:
 *   GlobalCacheEngine.put / _put_impl_local  flexkv/cache/cache_engine.py:550-615, 787-902
 *   GlobalCacheEngine.get / _get_impl_local  cache_engine.py:150-219, 412-548 (SSD off)
 *   CacheEngine.match / insert / take / cleanup / recycle   cache_engine.py:63-107
 *   RadixTreeIndex.match_prefix / insert / set_ready         flexkv/cache/radixtree.py:143-316
 *   Mempool.allocate_blocks / recycle_blocks                 flexkv/cache/mempool.py:28-55
 * A batch is num_seqs token sequences, sequence s owning tokens
 * [seq_offsets[s], seq_offsets[s+1]) of token_ids (int64, host or device;
 * seq_offsets on the host) and floor(len_s / tokens_per_block) blocks at
 * block offset blk_s (running sum of the previous sequences' blocks).  The
 * requests of a batch take effect in order, as consecutive puts do.  Every
 * call returns with its work done on `stream`, except the copies of a put
 * or get called with synchronous = 0: those return once the decisions (the
 * outputs) are known, with the copy -- and the put's ready marks -- still
 * running on `stream`, as the reference's put/get return before their
 * transfer graphs run.  The caller then waits on `stream` (an event recorded
 * after the call) before it reuses the copied GPU blocks or pool blocks.
 *
 * Not done on the device: eviction.  When the pool is short a put comes back
 * empty, as the reference's does when take() finds nothing evictable; the
 * caller evicts with fkv_cache_index_remove + fkv_cache_index_recycle. */
typedef struct fkv_cache_index fkv_cache_index;

/* An empty index over a pool of num_total_blocks blocks (ids handed out in
 * the reference Mempool's order). */
int fkv_cache_index_create(int device, int64_t num_total_blocks, int tokens_per_block,
                           fkv_cache_index **out);
void fkv_cache_index_destroy(fkv_cache_index *ci);

/* match_prefix of each sequence: num_matched[s] leading blocks cached,
 * num_ready[s] of them ready; physical_blocks (optional, one entry per block
 * of the batch) gets the pool block of every matched block and -1 after. */
int fkv_cache_index_match(fkv_cache_index *ci, const int64_t *token_ids, const int64_t *seq_offsets,
                          int num_seqs, int64_t *num_matched, int64_t *num_ready,
                          int64_t *physical_blocks, void *stream);

/* put of each sequence (CPU tier): skip the matched prefix, take pool blocks
 * for the rest, insert them not ready, copy those GPU blocks to them, then
 * (mark_ready != 0) mark them ready, as the put callback does.
 * gpu_block_ids: one GPU block per block of the batch (host or device; the
 * reference derives them from the slot mapping).  layout: the D2H copy's
 * layout as for fkv_transfer_kv_blocks_ex (layer pointers, strides, cpu
 * pointer, chunk size, is_mla, transfer_sms, cpu_pool_bytes,
 * gpu_layer_bytes); its id arrays, num_blocks and direction are not used.
 * Out: num_skipped[s] / num_transferred[s] (both 0 for an empty put, which
 * includes a put the pool could not hold); cpu_block_ids (optional, per
 * block: the pool block it was copied to, -1 if not copied); block_hashes
 * (optional, per block). */
int fkv_cache_index_put(fkv_cache_index *ci, const int64_t *token_ids, const int64_t *seq_offsets,
                        int num_seqs, const int64_t *gpu_block_ids, const fkv_transfer_desc *layout,
                        int mark_ready, int synchronous, int64_t *num_skipped,
                        int64_t *num_transferred, int64_t *cpu_block_ids, uint64_t *block_hashes,
                        void *stream);

/* put of each sequence with the SSD tier on (cache_engine.py:787-902):
 * `cpu` and `ssd` are the two tiers' indexes (same device and
 * tokens_per_block).  Per sequence: m_c / m_s leading blocks cached in the
 * CPU / SSD tier; the n - m_c others are copied D2H into new CPU blocks
 * (inserted, ready after the copy when mark_ready); the n - m_s blocks the
 * SSD tier lacks get new SSD blocks (inserted, not ready).  Both takes must
 * succeed, else the put is empty and gives both allocations back.  When a
 * caller's eviction left the SSD tier behind the CPU tier (m_s < m_c), the
 * SSD copy of a block below m_c comes from its cached CPU block; if such a
 * block is not ready yet, the put is refused (empty, nothing allocated).
 * Out: num_skipped (m_c), num_transferred (D2H blocks), num_to_ssd (SSD
 * blocks); per block of the batch: cpu_block_ids, ssd_block_ids,
 * block_hashes.  cpu_block_ids[i] differs from fkv_cache_index_put's: it is
 * the new CPU block for a block copied D2H, the cached CPU block for a block
 * below m_c that the SSD tier lacks (the H2DISK source, nothing is copied
 * into it), and -1 for every other block (cached in both tiers, or in an
 * empty put).  ssd_block_ids[i] is the block's new SSD block, else -1.
 * The caller then writes each
 * (cpu_block_ids[i] -> ssd_block_ids[i]) pair to the SSD tier
 * (fkv_transfer_kv_blocks_ssd) and marks those blocks ready in `ssd`
 * (fkv_cache_index_set_ready), the H2DISK op and callback of the reference's
 * put graph.  Synchronous. */
int fkv_cache_index_put2(fkv_cache_index *cpu, fkv_cache_index *ssd, const int64_t *token_ids,
                         const int64_t *seq_offsets, int num_seqs, const int64_t *gpu_block_ids,
                         const fkv_transfer_desc *layout, int mark_ready, int64_t *num_skipped,
                         int64_t *num_transferred, int64_t *num_to_ssd, int64_t *cpu_block_ids,
                         int64_t *ssd_block_ids, uint64_t *block_hashes, void *stream);

/* get of each sequence (CPU tier, cache_engine.py:150-219, 412-548, SSD
 * off): the mask selects full blocks [block_starts[s], n_s) (block_starts
 * NULL: all from 0); of the sequence's first num_ready matched blocks, those
 * in that range are read into its leading GPU blocks.  gpu_block_ids: per
 * sequence n_s - block_starts[s] GPU blocks (the reference's slot mapping of
 * the masked blocks), concatenated.  layout: the H2D copy's layout (as for
 * fkv_cache_index_put).  Out: num_transferred[s] blocks read (the return
 * mask covers blocks [block_starts[s], +num_transferred[s])); cpu_block_ids
 * (optional, one per GPU entry): the pool block read into it, -1 if none.
 * The index and the pool do not change.  layer_granularity > 0 copies the
 * layers in groups of that many, in order (it must divide the number of
 * layers, as convert_read_graph_to_layer_wise_graph requires,
 * transfer_pattern.py:370-428); group_events (optional, one cudaEvent_t per
 * group) are recorded on `stream` after each group, for the caller's
 * wait_at_layer_group (kvmanager.py:480). */
int fkv_cache_index_get(fkv_cache_index *ci, const int64_t *token_ids, const int64_t *seq_offsets,
                        int num_seqs, const int64_t *block_starts, const int64_t *gpu_block_ids,
                        const fkv_transfer_desc *layout, int layer_granularity,
                        void *const *group_events, int synchronous, int64_t *num_transferred,
                        int64_t *cpu_block_ids, void *stream);

/* Mark cached blocks ready (ready != 0) or not, by block hash (host array);
 * *num_found = how many were cached. */
int fkv_cache_index_set_ready(fkv_cache_index *ci, const uint64_t *block_hashes, int64_t n, int ready,
                              int64_t *num_found, void *stream);

/* Drop cached blocks by hash (the caller's eviction); removed_blocks[q] =
 * the pool block block q held, -1 if it was not cached.  The blocks stay
 * allocated until fkv_cache_index_recycle. */
int fkv_cache_index_remove(fkv_cache_index *ci, const uint64_t *block_hashes, int64_t n,
                           int64_t *removed_blocks, void *stream);

/* Mempool.recycle_blocks: return blocks to the pool; FKV_ERR_INVALID_ARG if
 * one is already free (nothing changes) or appears twice. */
int fkv_cache_index_recycle(fkv_cache_index *ci, const int64_t *block_ids, int64_t n, void *stream);

/* CacheEngine.take(num, strict=False) with nothing to evict: allocate
 * min(num, free) blocks into block_ids; *num_taken = how many. */
int fkv_cache_index_take(fkv_cache_index *ci, int64_t num, int64_t *block_ids, int64_t *num_taken,
                         void *stream);

/* out[0..6] = free blocks, cached blocks, ready blocks, pool snapshot
 * length, snapshot offset, deleted table slots, table slots. */
int fkv_cache_index_stats(fkv_cache_index *ci, int64_t *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* FLEXKV_B200_H_ */
