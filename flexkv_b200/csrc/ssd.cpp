// CPU pool <-> SSD block transfers: the SSD tier of FlexKV
// (csrc/transfer_ssd.cpp:17-287, csrc/transfer_ssd.h:170-264).
//
// On-disk format (kept exactly, so caches written by either side read back
// on the other): SSD block id s lives on device d = (s / rr) % D at
// in-device index i = ((s / rr) / D) * rr + s % rr (transfer_ssd.cpp:17-32),
// in file i % F of that device at file block b = i / F (:50-52); chunk
// (layer l, kv k) of it sits at file byte b*block_stride + l*ssd_layer_stride
// + k*ssd_kv_stride, and its CPU twin at cpu_block*block_stride +
// l*cpu_layer_stride + k*cpu_kv_stride (:56-60).  Layers are absolute:
// [start_layer, start_layer + num_layers) on both sides.
//
// What differs from the reference is how the bytes move:
//   * chunks adjacent on both sides are merged into one I/O (a whole
//     BLOCKWISE block, or a run of consecutive blocks of one LAYERWISE
//     layer), instead of one pread/pwrite per chunk;
//   * a persistent per-context thread pool issues them (the reference
//     creates its threads on every call);
//   * O_DIRECT reads (chunk a multiple of 4 KiB, the reference's rule) are
//     used only where the buffer and offset are 4 KiB aligned too; other
//     reads fall back to the buffered descriptor instead of failing;
//   * partial reads and writes are resumed; a short read (end of file) or
//     an I/O error fails the call with the file and offset in the message.
// With iouring_entries > 0 (the reference's optional io_uring path,
// transfer_ssd.h:9-168) requests go through io_uring instead, one ring per
// direction, driven by the kernel interface directly (no liburing): up to
// iouring_entries requests in flight from the calling thread.  When the
// ring cannot be set up, the thread pool serves, as the reference falls
// back to its threads.
#include <fcntl.h>
#include <linux/io_uring.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <sys/uio.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "fkv_common.h"

namespace {

constexpr int64_t kDirectAlign = 4096;
constexpr int64_t kMaxSegBytes = 8ll << 20;  // split longer runs so threads share them

// One batch of jobs on the shared pool; the caller waits for its own batch.
struct Batch {
  std::mutex mu;
  std::condition_variable cv;
  int remaining = 0;
  int rc = FKV_OK;
  std::string error;
};

class IoPool {
 public:
  ~IoPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto &t : th_) t.join();
  }
  void ensure(int n) {
    std::lock_guard<std::mutex> lk(mu_);
    while ((int)th_.size() < n) th_.emplace_back([this] { loop(); });
  }
  // Run every job (each returns FKV_OK or fills err); first failure wins.
  int run(std::vector<std::function<int(std::string &)>> &jobs, std::string &err) {
    if (jobs.empty()) return FKV_OK;
    auto b = std::make_shared<Batch>();
    b->remaining = (int)jobs.size();
    {
      std::lock_guard<std::mutex> lk(mu_);
      for (auto &j : jobs) q_.push_back({b, std::move(j)});
    }
    cv_.notify_all();
    std::unique_lock<std::mutex> lk(b->mu);
    b->cv.wait(lk, [&] { return b->remaining == 0; });
    err = b->error;
    return b->rc;
  }

 private:
  struct Item {
    std::shared_ptr<Batch> batch;
    std::function<int(std::string &)> fn;
  };
  void loop() {
    for (;;) {
      Item it;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || !q_.empty(); });
        if (stop_ && q_.empty()) return;
        it = std::move(q_.front());
        q_.pop_front();
      }
      std::string e;
      const int rc = it.fn(e);
      std::lock_guard<std::mutex> lk(it.batch->mu);
      if (rc != FKV_OK && it.batch->rc == FKV_OK) {
        it.batch->rc = rc;
        it.batch->error = e;
      }
      if (--it.batch->remaining == 0) it.batch->cv.notify_all();
    }
  }
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Item> q_;
  std::vector<std::thread> th_;
  bool stop_ = false;
};

struct Seg {
  int file;  // index d * F + f
  int64_t off;
  char *cpu;
  int64_t len;
};

// One file request for the ring path.
struct Req {
  int fd;
  int file;
  char *buf;
  int64_t len;
  int64_t off;
};

// A minimal io_uring: READV / WRITEV submissions from one thread at a time.
class IoRing {
 public:
  ~IoRing() {
    if (sqes_) munmap(sqes_, sqes_sz_);
    if (cq_ptr_ && cq_ptr_ != sq_ptr_) munmap(cq_ptr_, cq_sz_);
    if (sq_ptr_) munmap(sq_ptr_, sq_sz_);
    if (fd_ >= 0) close(fd_);
  }
  bool init(unsigned entries, unsigned flags) {
    io_uring_params p;
    std::memset(&p, 0, sizeof(p));
    p.flags = flags;
    fd_ = (int)syscall(__NR_io_uring_setup, entries, &p);
    if (fd_ < 0) return false;
    sq_sz_ = p.sq_off.array + p.sq_entries * sizeof(unsigned);
    cq_sz_ = p.cq_off.cqes + p.cq_entries * sizeof(io_uring_cqe);
    const bool single = (p.features & IORING_FEAT_SINGLE_MMAP) != 0;
    if (single) sq_sz_ = cq_sz_ = std::max(sq_sz_, cq_sz_);
    sq_ptr_ = mmap(nullptr, sq_sz_, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd_, IORING_OFF_SQ_RING);
    if (sq_ptr_ == MAP_FAILED) {
      sq_ptr_ = nullptr;
      return false;
    }
    cq_ptr_ = single ? sq_ptr_
                     : mmap(nullptr, cq_sz_, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd_,
                            IORING_OFF_CQ_RING);
    if (cq_ptr_ == MAP_FAILED) {
      cq_ptr_ = nullptr;
      return false;
    }
    sqes_sz_ = p.sq_entries * sizeof(io_uring_sqe);
    void *q = mmap(nullptr, sqes_sz_, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd_, IORING_OFF_SQES);
    if (q == MAP_FAILED) return false;
    sqes_ = static_cast<io_uring_sqe *>(q);
    char *sq = static_cast<char *>(sq_ptr_), *cq = static_cast<char *>(cq_ptr_);
    sq_head_ = reinterpret_cast<unsigned *>(sq + p.sq_off.head);
    sq_tail_ = reinterpret_cast<unsigned *>(sq + p.sq_off.tail);
    sq_mask_ = *reinterpret_cast<unsigned *>(sq + p.sq_off.ring_mask);
    sq_array_ = reinterpret_cast<unsigned *>(sq + p.sq_off.array);
    cq_head_ = reinterpret_cast<unsigned *>(cq + p.cq_off.head);
    cq_tail_ = reinterpret_cast<unsigned *>(cq + p.cq_off.tail);
    cq_mask_ = *reinterpret_cast<unsigned *>(cq + p.cq_off.ring_mask);
    cqes_ = reinterpret_cast<io_uring_cqe *>(cq + p.cq_off.cqes);
    depth_ = p.sq_entries;
    return true;
  }
  // Move every request; partial transfers are resubmitted for the rest.
  // On a failure no new requests start, the ones in flight are reaped, and
  // the first error is returned.
  int run(const std::vector<Req> &reqs, bool read, const std::vector<std::string> &paths, std::string &err) {
    std::lock_guard<std::mutex> lk(mu_);
    struct Slot {
      Req r;
      iovec iov;
    };
    std::vector<Slot> slots(depth_);
    std::vector<unsigned> free_slots(depth_);
    for (unsigned k = 0; k < depth_; ++k) free_slots[k] = depth_ - 1 - k;
    std::deque<Req> pending(reqs.begin(), reqs.end());
    unsigned inflight = 0;
    int rc = FKV_OK;
    int enter_failures = 0;  // consecutive io_uring_enter failures other than interrupts
    while ((rc == FKV_OK && !pending.empty()) || inflight > 0) {
      unsigned tail = *sq_tail_;
      unsigned added = 0;
      while (rc == FKV_OK && !pending.empty() && !free_slots.empty()) {
        const unsigned k = free_slots.back();
        free_slots.pop_back();
        Slot &sl = slots[k];
        sl.r = pending.front();
        pending.pop_front();
        sl.iov.iov_base = sl.r.buf;
        sl.iov.iov_len = (size_t)sl.r.len;
        const unsigned idx = tail & sq_mask_;
        io_uring_sqe *e = &sqes_[idx];
        std::memset(e, 0, sizeof(*e));
        e->opcode = read ? IORING_OP_READV : IORING_OP_WRITEV;
        e->fd = sl.r.fd;
        e->off = (uint64_t)sl.r.off;
        e->addr = (uint64_t)(uintptr_t)&sl.iov;
        e->len = 1;
        e->user_data = k;
        sq_array_[idx] = idx;
        ++tail;
        ++added;
      }
      __atomic_store_n(sq_tail_, tail, __ATOMIC_RELEASE);
      inflight += added;  // every queued entry completes once the kernel consumes it
      // Submit everything the kernel has not consumed yet (an interrupted
      // call may leave entries behind) and wait for at least one completion.
      const unsigned unsub = tail - __atomic_load_n(sq_head_, __ATOMIC_ACQUIRE);
      const int got = (int)syscall(__NR_io_uring_enter, fd_, unsub, inflight > 0 ? 1 : 0,
                                   IORING_ENTER_GETEVENTS, nullptr, 0);
      if (got < 0 && errno != EINTR && errno != EAGAIN && errno != EBUSY) {
        if (rc == FKV_OK) {
          rc = FKV_ERR_IO;
          err = std::string("io_uring_enter failed: ") + std::strerror(errno);
        }
        // Entries the kernel never took will not complete: stop counting
        // them.  Those it took complete and are reaped below; a ring that
        // keeps failing is given up after a few tries.
        const unsigned left = tail - __atomic_load_n(sq_head_, __ATOMIC_ACQUIRE);
        inflight -= std::min(inflight, left);
        if (++enter_failures >= 4) break;
      } else if (got >= 0) {
        enter_failures = 0;
      }
      unsigned head = *cq_head_;
      const unsigned ctail = __atomic_load_n(cq_tail_, __ATOMIC_ACQUIRE);
      for (; head != ctail; ++head) {
        const io_uring_cqe &c = cqes_[head & cq_mask_];
        const unsigned k = (unsigned)c.user_data;
        Req r = slots[k].r;
        free_slots.push_back(k);
        --inflight;
        if (c.res < 0) {
          if (c.res == -EINTR || c.res == -EAGAIN) {
            pending.push_front(r);
          } else if (rc == FKV_OK) {
            rc = FKV_ERR_IO;
            err = std::string(read ? "read" : "write") + " of " + std::to_string(r.len) + " bytes at offset " +
                  std::to_string(r.off) + " in " + paths[r.file] + " failed: " + std::strerror(-c.res);
          }
        } else if (c.res == 0 && r.len > 0) {
          if (rc == FKV_OK) {
            rc = FKV_ERR_IO;
            err = "short read at offset " + std::to_string(r.off) + " in " + paths[r.file] +
                  " (past the end of the file)";
          }
        } else if (c.res < r.len) {
          r.buf += c.res;
          r.off += c.res;
          r.len -= c.res;
          pending.push_front(r);
        }
      }
      __atomic_store_n(cq_head_, head, __ATOMIC_RELEASE);
    }
    return rc;
  }

 private:
  int fd_ = -1;
  void *sq_ptr_ = nullptr, *cq_ptr_ = nullptr;
  size_t sq_sz_ = 0, cq_sz_ = 0, sqes_sz_ = 0;
  io_uring_sqe *sqes_ = nullptr;
  io_uring_cqe *cqes_ = nullptr;
  unsigned *sq_head_ = nullptr, *sq_tail_ = nullptr, *sq_array_ = nullptr, *cq_head_ = nullptr,
           *cq_tail_ = nullptr;
  unsigned sq_mask_ = 0, cq_mask_ = 0, depth_ = 0;
  std::mutex mu_;
};

int io_all(int fd, char *p, int64_t len, int64_t off, bool read, std::string &err, const std::string &path) {
  while (len > 0) {
    const ssize_t n = read ? pread(fd, p, (size_t)len, (off_t)off) : pwrite(fd, p, (size_t)len, (off_t)off);
    if (n < 0) {
      if (errno == EINTR) continue;
      err = std::string(read ? "read" : "write") + " of " + std::to_string(len) + " bytes at offset " +
            std::to_string(off) + " in " + path + " failed: " + std::strerror(errno);
      return FKV_ERR_IO;
    }
    if (n == 0) {
      err = "short read at offset " + std::to_string(off) + " in " + path + " (past the end of the file)";
      return FKV_ERR_IO;
    }
    p += n;
    off += n;
    len -= n;
  }
  return FKV_OK;
}

}  // namespace

struct fkv_ssd_ctx {
  int num_devices = 0;
  int files_per_device = 0;
  std::vector<std::string> paths;
  std::vector<int> fd_buf, fd_direct;  // [d * F + f]; fd_direct -1 if O_DIRECT is refused
  IoPool pool;
  std::unique_ptr<IoRing> ring[2];  // [0] reads, [1] writes; null = thread pool
  std::atomic<int64_t> last_ios{0}, last_bytes{0};
};

using fkv::fail;

extern "C" {

int fkv_ssd_ctx_create(const char *const *paths, int num_devices, int files_per_device, int iouring_entries,
                       int iouring_flags, fkv_ssd_ctx **out) {
  fkv::clear_error();
  if (!out) return fail(FKV_ERR_INVALID_ARG, "null output");
  *out = nullptr;
  if (!paths || num_devices <= 0 || files_per_device <= 0)
    return fail(FKV_ERR_INVALID_ARG, "SSD context needs at least one device with at least one file");
  auto c = std::make_unique<fkv_ssd_ctx>();
  c->num_devices = num_devices;
  c->files_per_device = files_per_device;
  const int n = num_devices * files_per_device;
  for (int i = 0; i < n; ++i) {
    if (!paths[i]) return fail(FKV_ERR_INVALID_ARG, "null SSD file path");
    c->paths.emplace_back(paths[i]);
  }
  for (int i = 0; i < n; ++i) {
    const int fb = open(c->paths[i].c_str(), O_RDWR);
    if (fb < 0) {
      const std::string msg = "open " + c->paths[i] + " failed: " + std::strerror(errno);
      for (int fd : c->fd_buf) close(fd);
      for (int fd : c->fd_direct)
        if (fd >= 0) close(fd);
      return fail(FKV_ERR_IO, msg);
    }
    posix_fadvise(fb, 0, 0, POSIX_FADV_SEQUENTIAL);
    c->fd_buf.push_back(fb);
    c->fd_direct.push_back(open(c->paths[i].c_str(), O_RDWR | O_DIRECT));  // -1: filesystem refuses it
  }
  if (iouring_entries > 0) {
    for (auto &r : c->ring) {
      r.reset(new IoRing());
      if (!r->init((unsigned)iouring_entries, (unsigned)iouring_flags)) r.reset();  // thread pool instead
    }
  }
  *out = c.release();
  return FKV_OK;
}

void fkv_ssd_ctx_destroy(fkv_ssd_ctx *ctx) {
  if (!ctx) return;
  for (int fd : ctx->fd_buf) close(fd);
  for (int fd : ctx->fd_direct)
    if (fd >= 0) close(fd);
  delete ctx;
}

int fkv_transfer_kv_blocks_ssd(fkv_ssd_ctx *ctx, int start_layer, int num_layers, void *cpu_ptr,
                               int64_t cpu_pool_bytes, const int64_t *ssd_block_ids,
                               const int64_t *cpu_block_ids, int64_t num_blocks,
                               int64_t cpu_layer_stride_in_bytes, int64_t cpu_kv_stride_in_bytes,
                               int64_t ssd_layer_stride_in_bytes, int64_t ssd_kv_stride_in_bytes,
                               int64_t chunk_size_in_bytes, int64_t block_stride_in_bytes, int is_read,
                               int num_blocks_per_file, int round_robin, int num_threads_per_device,
                               int is_mla) {
  fkv::clear_error();
  (void)num_blocks_per_file;  // the reference passes it but never uses it (transfer_ssd.cpp:186-194)
  if (!ctx) return fail(FKV_ERR_INVALID_ARG, "null SSD context");
  if (num_blocks < 0 || num_layers < 0 || start_layer < 0)
    return fail(FKV_ERR_INVALID_ARG, "negative block count or layer range");
  if (num_blocks == 0 || num_layers == 0) {
    ctx->last_ios = 0;
    ctx->last_bytes = 0;
    return FKV_OK;
  }
  if (!cpu_ptr || !ssd_block_ids || !cpu_block_ids) return fail(FKV_ERR_INVALID_ARG, "null pointer argument");
  if (chunk_size_in_bytes <= 0 || block_stride_in_bytes < 0 || cpu_layer_stride_in_bytes < 0 ||
      cpu_kv_stride_in_bytes < 0 || ssd_layer_stride_in_bytes < 0 || ssd_kv_stride_in_bytes < 0)
    return fail(FKV_ERR_INVALID_ARG, "strides must be non-negative and the chunk positive");
  if (round_robin <= 0) return fail(FKV_ERR_INVALID_ARG, "round_robin must be positive");
  const int D = ctx->num_devices, F = ctx->files_per_device;
  const int KV = is_mla ? 1 : 2;
  const int threads = num_threads_per_device > 0 ? num_threads_per_device : 1;
  const int64_t last_layer = (int64_t)start_layer + num_layers - 1;

  // Per-device block lists in the caller's order, ids remapped to files.
  struct Blk {
    int file;
    int64_t fblock;
    int64_t cblock;
  };
  std::vector<std::vector<Blk>> per_dev(D);
  for (int64_t i = 0; i < num_blocks; ++i) {
    const int64_t s = ssd_block_ids[i], cb = cpu_block_ids[i];
    if (s < 0 || s > INT32_MAX || cb < 0 || cb > INT32_MAX)
      return fail(FKV_ERR_OUT_OF_RANGE, "block id " + std::to_string(s < 0 || s > INT32_MAX ? s : cb) +
                                            " outside [0, 2^31) at position " + std::to_string(i));
    const int64_t d = (s / round_robin) % D;
    const int64_t in_dev = ((s / round_robin) / D) * round_robin + s % round_robin;
    const int f = (int)(in_dev % F);
    per_dev[d].push_back({(int)d * F + f, in_dev / F, cb});
    if (cpu_pool_bytes > 0) {
      const int64_t end = cb * block_stride_in_bytes + last_layer * cpu_layer_stride_in_bytes +
                          (KV - 1) * cpu_kv_stride_in_bytes + chunk_size_in_bytes;
      if (end > cpu_pool_bytes)
        return fail(FKV_ERR_OUT_OF_RANGE, "cpu block " + std::to_string(cb) + " runs past the cpu pool");
    }
  }
  char *cpu = static_cast<char *>(cpu_ptr);
  // Chunk order that lets neighbours merge: block-major when a block's
  // chunks are contiguous, layer-major when consecutive blocks are.
  const bool block_major = !(block_stride_in_bytes == chunk_size_in_bytes);
  std::vector<std::vector<Seg>> segs(D);
  auto emit = [&](std::vector<Seg> &v, int file, int64_t off, char *p) {
    if (!v.empty()) {
      Seg &t = v.back();
      if (t.file == file && t.off + t.len == off && t.cpu + t.len == p && t.len + chunk_size_in_bytes <= kMaxSegBytes) {
        t.len += chunk_size_in_bytes;
        return;
      }
    }
    v.push_back({file, off, p, chunk_size_in_bytes});
  };
  for (int d = 0; d < D; ++d) {
    auto &v = segs[d];
    auto &bl = per_dev[d];
    if (block_major) {
      for (const Blk &b : bl)
        for (int64_t l = start_layer; l <= last_layer; ++l)
          for (int k = 0; k < KV; ++k)
            emit(v, b.file, b.fblock * block_stride_in_bytes + l * ssd_layer_stride_in_bytes + k * ssd_kv_stride_in_bytes,
                 cpu + b.cblock * block_stride_in_bytes + l * cpu_layer_stride_in_bytes + k * cpu_kv_stride_in_bytes);
    } else {
      for (int64_t l = start_layer; l <= last_layer; ++l)
        for (int k = 0; k < KV; ++k)
          for (const Blk &b : bl)
            emit(v, b.file, b.fblock * block_stride_in_bytes + l * ssd_layer_stride_in_bytes + k * ssd_kv_stride_in_bytes,
                 cpu + b.cblock * block_stride_in_bytes + l * cpu_layer_stride_in_bytes + k * cpu_kv_stride_in_bytes);
    }
  }
  // O_DIRECT reads follow the reference's rule (chunk a multiple of 4 KiB)
  // where the memory and file offsets allow it.
  const bool direct_ok = is_read && chunk_size_in_bytes % kDirectAlign == 0;
  std::vector<std::function<int(std::string &)>> jobs;
  int64_t n_ios = 0, n_bytes = 0;
  for (int d = 0; d < D; ++d) {
    auto &v = segs[d];
    if (v.empty()) continue;
    int64_t total = 0;
    for (auto &s : v) total += s.len;
    n_ios += (int64_t)v.size();
    n_bytes += total;
    const int t_use = (int)std::min<int64_t>(threads, (int64_t)v.size());
    const int64_t share = (total + t_use - 1) / t_use;
    size_t i = 0;
    for (int t = 0; t < t_use && i < v.size(); ++t) {
      const size_t first = i;
      int64_t acc = 0;
      while (i < v.size() && (acc < share || t == t_use - 1)) acc += v[i++].len;
      const Seg *sp = v.data() + first;
      const size_t cnt = i - first;
      jobs.push_back([ctx, sp, cnt, is_read, direct_ok](std::string &err) {
        for (size_t k = 0; k < cnt; ++k) {
          const Seg &s = sp[k];
          int fd = ctx->fd_buf[s.file];
          if (direct_ok && ctx->fd_direct[s.file] >= 0 && s.off % kDirectAlign == 0 &&
              reinterpret_cast<uintptr_t>(s.cpu) % kDirectAlign == 0)
            fd = ctx->fd_direct[s.file];
          if (int rc = io_all(fd, s.cpu, s.len, s.off, is_read != 0, err, ctx->paths[s.file])) return rc;
        }
        return FKV_OK;
      });
    }
  }
  std::string err;
  int rc = FKV_OK;
  if (IoRing *ring = ctx->ring[is_read ? 0 : 1].get()) {
    // Ring path: the devices' requests interleaved, so every device has
    // requests in flight.
    std::vector<Req> reqs;
    reqs.reserve((size_t)n_ios);
    for (size_t k = 0;; ++k) {
      bool any = false;
      for (int d = 0; d < D; ++d) {
        if (k >= segs[d].size()) continue;
        any = true;
        const Seg &s = segs[d][k];
        int fd = ctx->fd_buf[s.file];
        if (direct_ok && ctx->fd_direct[s.file] >= 0 && s.off % kDirectAlign == 0 &&
            reinterpret_cast<uintptr_t>(s.cpu) % kDirectAlign == 0)
          fd = ctx->fd_direct[s.file];
        reqs.push_back({fd, s.file, s.cpu, s.len, s.off});
      }
      if (!any) break;
    }
    rc = ring->run(reqs, is_read != 0, ctx->paths, err);
  } else {
    ctx->pool.ensure(D * threads);
    rc = ctx->pool.run(jobs, err);
  }
  ctx->last_ios = n_ios;
  ctx->last_bytes = n_bytes;
  if (rc != FKV_OK) return fail(rc, err);
  return FKV_OK;
}

int fkv_ssd_ctx_uses_io_uring(const fkv_ssd_ctx *ctx) {
  return ctx && ctx->ring[0] && ctx->ring[1] ? 1 : 0;
}

int fkv_ssd_last_stats(const fkv_ssd_ctx *ctx, int64_t *num_ios, int64_t *bytes) {
  if (!ctx) return fail(FKV_ERR_INVALID_ARG, "null SSD context");
  if (num_ios) *num_ios = ctx->last_ios.load();
  if (bytes) *bytes = ctx->last_bytes.load();
  return FKV_OK;
}

}  // extern "C"
