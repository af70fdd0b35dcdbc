// In-process transfer engine for one data-parallel group (one GPU, or the
// GPUs of one tensor-parallel group) — the data-plane half of FlexKV's
// TransferEngine (flexkv/transfer/transfer_engine.py:197-307) and its GPU
// workers (flexkv/transfer/worker.py:144-177, 259-342, 402-480).
//
// The reference runs a Python scheduler thread that resolves op
// dependencies on the host, pipes every op to a worker process, pins the
// block ids on every call and copies synchronously, one op at a time.
// Here one dispatcher thread owns all CUDA work of the group:
//   * a submitted graph is ordered topologically and every op is enqueued
//     at once; a dependency is a cudaStreamWaitEvent on the predecessor's
//     completion event, resolved on the GPU without a host round trip;
//   * H2D ops and D2H ops run on separate streams per GPU, so the two
//     directions share the full-duplex host link; each direction has a
//     small pool of streams (2 by default) used round robin, so the tail
//     of one small op overlaps the start of the next;
//   * the block-id tables are staged in a page-locked ring owned by the
//     engine (no per-op pinning), each slice released when its op is done;
//   * completion is detected by polling the ops' events and reported as
//     (graph_id, op_id) pairs, op_id = -1 once a whole graph is done — the
//     shape of TransferEngine.get_completed_graphs_and_ops.
// A failed op (invalid ids, CUDA error) is reported with its status; its
// completion event is still recorded so successors are not held back.
//
// SSD ops (DISK2H / H2DISK, CPUSSDDiskTransferWorker, worker.py:482-590)
// are host work: two engine I/O threads (reads, writes) run them through
// the SSD tier.  An SSD op is handed to its thread once every predecessor
// has completed; a GPU op is enqueued once each predecessor has either
// completed or been enqueued on the GPU itself (then an event wait orders
// them), so a GPU op after an SSD op waits on the host for it.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdlib>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <list>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "fkv_common.h"

namespace {

struct Op {
  int64_t graph_id = 0;
  int64_t op_id = 0;
  int type = FKV_OP_H2D;
  std::vector<int64_t> gpu_ids, cpu_ids;
  int layer_id = 0;
  int layer_gran = 0;
  std::vector<int64_t> preds;
  std::vector<cudaEvent_t> done;  // per rank
  std::vector<std::pair<size_t, size_t>> slices;  // ring slices (offset, length)
  int status = FKV_OK;
  std::string error;
  bool completed = false;
  bool host = false;        // DISK2H / H2DISK: runs on an I/O thread
  bool dispatched = false;  // enqueued (GPU) or handed to an I/O thread
  std::atomic<bool> host_done{false};
};

struct Graph {
  int64_t id = 0;
  std::vector<std::unique_ptr<Op>> ops;
  std::unordered_map<int64_t, Op *> by_id;
  int remaining = 0;
  int status = FKV_OK;
  std::string error;
};

struct Completion {
  int64_t graph_id, op_id;
  int status;
};

// Page-locked ring for id tables; slices are released in any order and
// reclaimed in allocation order.
class PinnedRing {
 public:
  int init(size_t cap) {
    cap_ = cap;
    cudaError_t e = cudaHostAlloc((void **)&buf_, cap, cudaHostAllocPortable);
    if (e != cudaSuccess) return fkv::fail_cuda(e, "cudaHostAlloc(engine ring)");
    return FKV_OK;
  }
  ~PinnedRing() {
    if (buf_) cudaFreeHost(buf_);
  }
  char *base() const { return buf_; }
  size_t capacity() const { return cap_; }
  // Reserve len bytes (16-byte granular); false when the ring is full.
  bool reserve(size_t len, size_t *off) {
    len = (len + 15) & ~size_t(15);
    if (len > cap_) return false;
    if (head_ + len > cap_) {  // skip the tail end
      if (used_ + (cap_ - head_) + len > cap_) return false;
      slices_.push_back({head_, cap_ - head_, true});
      used_ += cap_ - head_;
      head_ = 0;
    }
    if (used_ + len > cap_) return false;
    *off = head_;
    slices_.push_back({head_, len, false});
    head_ = (head_ + len) % cap_;
    used_ += len;
    return true;
  }
  void release(size_t off) {
    for (auto &s : slices_)
      if (!s.free && s.off == off) {
        s.free = true;
        break;
      }
    while (!slices_.empty() && slices_.front().free) {
      used_ -= slices_.front().len;
      slices_.pop_front();
    }
    if (slices_.empty()) head_ = 0;
  }

 private:
  struct Slice {
    size_t off, len;
    bool free;
  };
  char *buf_ = nullptr;
  size_t cap_ = 0, head_ = 0, used_ = 0;
  std::deque<Slice> slices_;
};

struct Rank {
  int device = 0;
  std::vector<cudaStream_t> h2d, d2h;  // per-direction stream pools
  size_t next_h2d = 0, next_d2h = 0;
  std::vector<void *> layer_ptrs;
  std::vector<cudaEvent_t> free_events;
};

}  // namespace

struct fkv_engine {
  fkv_engine_config cfg{};
  std::vector<Rank> ranks;
  PinnedRing ring;

  std::mutex mu;
  std::condition_variable cv_work, cv_done;
  std::deque<std::unique_ptr<Graph>> submitted;
  std::deque<Completion> completions;
  bool stop = false;
  int64_t inflight_ops = 0;
  std::thread worker;
  std::string init_error;
  int init_rc = FKV_OK;
  bool ready = false;
  bool finished = false;  // the dispatcher has returned

  // Dispatcher-thread state.
  std::unordered_map<int64_t, std::unique_ptr<Graph>> live;
  std::list<Op *> inflight;
  std::list<Op *> waiting;  // held until their predecessors allow dispatch

  // SSD I/O threads: queue 0 runs DISK2H ops, queue 1 H2DISK ops.
  std::mutex io_mu;
  std::condition_variable io_cv;
  std::deque<Op *> io_q[2];
  bool io_stop = false;
  std::thread io_th[2];
};

namespace {

int make_event(Rank &r, cudaEvent_t *out) {
  if (!r.free_events.empty()) {
    *out = r.free_events.back();
    r.free_events.pop_back();
    return FKV_OK;
  }
  FKV_CUDA(cudaEventCreateWithFlags(out, cudaEventDisableTiming));
  return FKV_OK;
}

void push_completion(fkv_engine *e, int64_t g, int64_t op, int status) {
  {
    std::lock_guard<std::mutex> lk(e->mu);
    e->completions.push_back({g, op, status});
  }
  e->cv_done.notify_all();
}

// Enqueue one op on every rank (dispatcher thread).
void dispatch(fkv_engine *e, Graph &g, Op &op, const std::unordered_map<int64_t, Op *> &by_id) {
  const fkv_engine_config &c = e->cfg;
  const int nr = (int)e->ranks.size();
  op.done.assign(nr, nullptr);
  const int L = c.num_layers;
  const int lid = op.layer_id < 0 ? 0 : op.layer_id;
  const int gran = op.layer_gran < 0 ? L - lid : op.layer_gran;
  if (op.status == FKV_OK && (lid + gran > L || gran < 0)) {
    op.status = FKV_ERR_INVALID_ARG;
    op.error = "layer range exceeds the engine's layers";
  }
  for (int r = 0; r < nr; ++r) {
    Rank &rk = e->ranks[r];
    cudaSetDevice(rk.device);
    cudaStream_t s = op.type == FKV_OP_D2H ? rk.d2h[rk.next_d2h++ % rk.d2h.size()]
                                           : rk.h2d[rk.next_h2d++ % rk.h2d.size()];
    for (int64_t p : op.preds) {
      auto it = by_id.find(p);
      if (it == by_id.end() || it->second->host) continue;  // SSD predecessors completed before dispatch
      if ((size_t)r < it->second->done.size() && it->second->done[r])
        cudaStreamWaitEvent(s, it->second->done[r], 0);
    }
    if (op.status == FKV_OK && op.type != FKV_OP_VIRTUAL && !op.gpu_ids.empty() && gran > 0) {
      fkv_transfer_desc d;
      fkv_transfer_desc_init(&d);
      d.num_blocks = (int)op.gpu_ids.size();
      d.start_layer_id = lid;
      d.num_layers = gran;
      d.is_host_to_device = op.type == FKV_OP_H2D;
      d.is_mla = c.is_mla;
      d.transfer_sms = op.type == FKV_OP_H2D ? c.transfer_sms_h2d : c.transfer_sms_d2h;
      d.use_ce_transfer = op.type == FKV_OP_H2D ? c.use_ce_h2d : c.use_ce_d2h;
      d.synchronous = 0;
      d.gpu_block_ids = op.gpu_ids.data();
      d.cpu_block_ids = op.cpu_ids.data();
      d.gpu_layer_ptrs = rk.layer_ptrs.data() + lid;
      d.cpu_ptr = c.cpu_ptr;
      d.gpu_kv_stride_in_bytes = c.gpu_kv_stride_in_bytes;
      d.gpu_block_stride_in_bytes = c.gpu_block_stride_in_bytes;
      d.cpu_kv_stride_in_bytes = c.cpu_kv_stride_in_bytes;
      d.cpu_layer_stride_in_bytes = c.cpu_layer_stride_in_bytes;
      d.cpu_block_stride_in_bytes = c.cpu_block_stride_in_bytes;
      d.cpu_startoff_inside_chunks = c.is_mla ? 0 : (int64_t)r * c.gpu_chunk_size_in_bytes;
      d.chunk_size_in_bytes = c.gpu_chunk_size_in_bytes;
      d.cpu_pool_bytes = c.cpu_pool_bytes;
      d.gpu_layer_bytes = c.gpu_layer_bytes;
      const size_t need = fkv::transfer_stage_bytes(d);
      size_t off = 0;
      // Wait for ring space: free the slices of the oldest in-flight op that
      // still holds any.  Slices are allocated in dispatch order, so that
      // op owns the ring's front slice and every pass frees space; an op
      // whose slices an earlier pass already freed (it stays in flight until
      // the poll loop retires it) is skipped.
      while (!e->ring.reserve(need, &off)) {
        Op *oldest = nullptr;
        for (Op *o : e->inflight)
          if (!o->slices.empty()) {
            oldest = o;
            break;
          }
        if (!oldest) {
          op.status = FKV_ERR_INVALID_ARG;
          op.error = "id table larger than the engine's staging ring";
          break;
        }
        for (cudaEvent_t ev : oldest->done)
          if (ev) cudaEventSynchronize(ev);
        for (auto &sl : oldest->slices) e->ring.release(sl.first);
        oldest->slices.clear();
      }
      if (op.status == FKV_OK) {
        op.slices.push_back({off, need});
        int rc = fkv::transfer_enqueue(d, s, e->ring.base() + off, need);
        if (rc != FKV_OK) {
          op.status = rc;
          op.error = std::string("rank ") + std::to_string(r) + ": " + fkv_last_error();
        }
      }
    }
    cudaEvent_t ev = nullptr;
    if (make_event(rk, &ev) == FKV_OK && cudaEventRecord(ev, s) == cudaSuccess) {
      op.done[r] = ev;
    } else {
      if (ev) rk.free_events.push_back(ev);
      op.status = FKV_ERR_CUDA;
      op.error = "could not record the op's completion event";
    }
  }
  op.dispatched = true;
  e->inflight.push_back(&op);
  (void)g;
}

// Whether op may be dispatched now (dispatcher thread).
bool ready(const Op &op, const std::unordered_map<int64_t, Op *> &by_id) {
  for (int64_t p : op.preds) {
    auto it = by_id.find(p);
    if (it == by_id.end()) continue;
    const Op *q = it->second;
    if (q->completed) continue;
    if (op.host || q->host || !q->dispatched) return false;
  }
  return true;
}

// Hand an SSD op to its I/O thread (dispatcher thread).
void dispatch_host(fkv_engine *e, Op &op) {
  op.dispatched = true;
  e->inflight.push_back(&op);
  {
    std::lock_guard<std::mutex> lk(e->io_mu);
    e->io_q[op.type == FKV_OP_DISK2H ? 0 : 1].push_back(&op);
  }
  e->io_cv.notify_all();
}

void dispatch_any(fkv_engine *e, Graph &g, Op &op) {
  if (op.host) dispatch_host(e, op);
  else dispatch(e, g, op, g.by_id);
}

// Dispatch every held op whose predecessors now allow it; the list keeps
// each graph's topological order, so chains advance in one pass.
void pump_waiting(fkv_engine *e) {
  for (auto it = e->waiting.begin(); it != e->waiting.end();) {
    Op *op = *it;
    auto git = e->live.find(op->graph_id);
    if (git != e->live.end() && ready(*op, git->second->by_id)) {
      dispatch_any(e, *git->second, *op);
      it = e->waiting.erase(it);
    } else {
      ++it;
    }
  }
}

// One SSD op through the SSD tier (I/O thread).
void run_ssd_op(fkv_engine *e, Op &op) {
  if (op.status != FKV_OK || op.gpu_ids.empty()) return;
  const fkv_engine_config &c = e->cfg;
  const int L = c.num_layers;
  const int lid = op.layer_id < 0 ? 0 : op.layer_id;
  const int gran = op.layer_gran < 0 ? L - lid : op.layer_gran;
  if (lid + gran > L || gran < 0) {
    op.status = FKV_ERR_INVALID_ARG;
    op.error = "layer range exceeds the engine's layers";
    return;
  }
  const int rc = fkv_transfer_kv_blocks_ssd(
      c.ssd_ctx, lid, gran, c.cpu_ptr, c.cpu_pool_bytes, op.gpu_ids.data(), op.cpu_ids.data(),
      (int64_t)op.gpu_ids.size(), c.cpu_layer_stride_in_bytes, c.cpu_kv_stride_in_bytes,
      c.ssd_layer_stride_in_bytes, c.ssd_kv_stride_in_bytes, c.cpu_chunk_size_in_bytes,
      c.cpu_block_stride_in_bytes, op.type == FKV_OP_DISK2H, c.ssd_num_blocks_per_file,
      c.ssd_round_robin > 0 ? c.ssd_round_robin : 1, c.ssd_threads_per_device > 0 ? c.ssd_threads_per_device : 32,
      c.is_mla);
  if (rc != FKV_OK) {
    op.status = rc;
    op.error = fkv_last_error();
  }
}

void io_main(fkv_engine *e, int q) {
  for (;;) {
    Op *op = nullptr;
    {
      std::unique_lock<std::mutex> lk(e->io_mu);
      e->io_cv.wait(lk, [&] { return e->io_stop || !e->io_q[q].empty(); });
      if (e->io_q[q].empty()) return;
      op = e->io_q[q].front();
      e->io_q[q].pop_front();
    }
    run_ssd_op(e, *op);
    op->host_done.store(true, std::memory_order_release);
    {
      std::lock_guard<std::mutex> lk(e->mu);  // pairs with the dispatcher's wait on cv_work
    }
    e->cv_work.notify_all();
  }
}

// Retire every in-flight op whose events have all fired (dispatcher thread).
bool retire(fkv_engine *e) {
  bool any = false;
  for (auto it = e->inflight.begin(); it != e->inflight.end();) {
    Op *op = *it;
    bool done = !op->host || op->host_done.load(std::memory_order_acquire);
    for (size_t r = 0; r < op->done.size() && done; ++r) {
      if (!op->done[r]) continue;
      cudaSetDevice(e->ranks[r].device);
      cudaError_t q = cudaEventQuery(op->done[r]);
      if (q == cudaErrorNotReady) {
        done = false;
      } else if (q != cudaSuccess) {
        cudaGetLastError();
        if (op->status == FKV_OK) {
          op->status = FKV_ERR_CUDA;
          op->error = cudaGetErrorString(q);
        }
      }
    }
    if (!done) {
      ++it;
      continue;
    }
    any = true;
    for (auto &sl : op->slices) e->ring.release(sl.first);
    op->slices.clear();
    op->completed = true;
    auto git = e->live.find(op->graph_id);
    push_completion(e, op->graph_id, op->op_id, op->status);
    it = e->inflight.erase(it);
    {
      std::lock_guard<std::mutex> lk(e->mu);
      --e->inflight_ops;
    }
    if (git != e->live.end()) {
      Graph &g = *git->second;
      if (op->status != FKV_OK && g.status == FKV_OK) g.status = op->status;
      if (--g.remaining == 0) {
        for (auto &o : g.ops)
          for (size_t r = 0; r < o->done.size(); ++r)
            if (o->done[r]) e->ranks[r].free_events.push_back(o->done[r]);
        push_completion(e, g.id, -1, g.status);
        e->live.erase(git);
      }
    }
  }
  return any;
}

// Order a graph's ops so every op follows its predecessors (Kahn).
bool topo_order(Graph &g, std::vector<Op *> &order, std::string &err) {
  std::unordered_map<int64_t, Op *> by_id;
  for (auto &o : g.ops) {
    if (!by_id.emplace(o->op_id, o.get()).second) {
      err = "duplicate op id " + std::to_string(o->op_id);
      return false;
    }
  }
  std::unordered_map<int64_t, int> indeg;
  std::unordered_map<int64_t, std::vector<Op *>> succ;
  for (auto &o : g.ops) {
    indeg[o->op_id] += 0;
    for (int64_t p : o->preds) {
      if (!by_id.count(p)) {
        err = "op " + std::to_string(o->op_id) + " depends on op " + std::to_string(p) +
              " outside its graph";
        return false;
      }
      indeg[o->op_id]++;
      succ[p].push_back(o.get());
    }
  }
  std::deque<Op *> q;
  for (auto &o : g.ops)
    if (indeg[o->op_id] == 0) q.push_back(o.get());
  while (!q.empty()) {
    Op *o = q.front();
    q.pop_front();
    order.push_back(o);
    for (Op *s : succ[o->op_id])
      if (--indeg[s->op_id] == 0) q.push_back(s);
  }
  if (order.size() != g.ops.size()) {
    err = "dependency cycle in graph " + std::to_string(g.id);
    return false;
  }
  return true;
}

void mark_finished(fkv_engine *e) {
  {
    std::lock_guard<std::mutex> lk(e->mu);
    e->finished = true;
  }
  e->cv_done.notify_all();
}

void engine_main(fkv_engine *e) {
  // Per-rank streams are created on this thread (it owns all CUDA work).
  int rc = FKV_OK;
  std::string msg;
  const int nstreams = e->cfg.streams_per_direction > 0 ? e->cfg.streams_per_direction : 2;
  for (auto &r : e->ranks) {
    cudaError_t ce = cudaSetDevice(r.device);
    for (int i = 0; i < nstreams && ce == cudaSuccess; ++i) {
      cudaStream_t a = nullptr, b = nullptr;
      ce = cudaStreamCreateWithFlags(&a, cudaStreamNonBlocking);
      if (ce == cudaSuccess) {
        r.h2d.push_back(a);
        ce = cudaStreamCreateWithFlags(&b, cudaStreamNonBlocking);
      }
      if (ce == cudaSuccess) r.d2h.push_back(b);
    }
    if (ce != cudaSuccess) {
      rc = FKV_ERR_CUDA;
      msg = std::string("engine stream creation: ") + cudaGetErrorString(ce);
      break;
    }
  }
  if (rc == FKV_OK) rc = e->ring.init(e->cfg.staging_bytes > 0 ? (size_t)e->cfg.staging_bytes : (32u << 20));
  if (rc != FKV_OK && msg.empty()) msg = fkv_last_error();
  {
    std::lock_guard<std::mutex> lk(e->mu);
    e->init_rc = rc;
    e->init_error = msg;
    e->ready = true;
  }
  e->cv_done.notify_all();
  if (rc != FKV_OK) {
    mark_finished(e);
    return;
  }
  // Completion-poll interval while ops are in flight: the added latency of
  // a finished op is at most this (FKV_ENGINE_POLL_US, default 10 us).
  int poll_us = 10;
  if (const char *v = std::getenv("FKV_ENGINE_POLL_US")) poll_us = std::max(1, std::atoi(v));

  for (;;) {
    std::deque<std::unique_ptr<Graph>> batch;
    {
      std::unique_lock<std::mutex> lk(e->mu);
      if (e->submitted.empty() && e->inflight.empty() && e->waiting.empty())
        e->cv_work.wait(lk, [&] { return e->stop || !e->submitted.empty(); });
      if (e->stop && e->submitted.empty() && e->inflight.empty() && e->waiting.empty()) break;
      batch.swap(e->submitted);
    }
    for (auto &gp : batch) {
      Graph &g = *gp;
      std::vector<Op *> order;
      std::string err;
      const bool ok = topo_order(g, order, err);
      g.remaining = (int)g.ops.size();
      const int64_t gid = g.id;
      if (!ok) {
        for (auto &o : g.ops) push_completion(e, gid, o->op_id, FKV_ERR_INVALID_ARG);
        push_completion(e, gid, -1, FKV_ERR_INVALID_ARG);
        std::lock_guard<std::mutex> lk(e->mu);
        e->inflight_ops -= (int64_t)g.ops.size();
        continue;
      }
      for (auto &o : g.ops) g.by_id[o->op_id] = o.get();
      e->live[gid] = std::move(gp);
      Graph &lg = *e->live[gid];
      if (lg.ops.empty()) {
        push_completion(e, gid, -1, FKV_OK);
        e->live.erase(gid);
        continue;
      }
      for (Op *o : order) {
        if (ready(*o, lg.by_id)) dispatch_any(e, lg, *o);
        else e->waiting.push_back(o);
      }
    }
    const bool progressed = retire(e);
    if (!e->waiting.empty()) pump_waiting(e);
    if (!progressed) {
      // Nothing finished: give the GPU a moment before polling again (a
      // submission or a finished SSD op wakes the loop at once).
      std::unique_lock<std::mutex> lk(e->mu);
      e->cv_work.wait_for(lk, std::chrono::microseconds(poll_us),
                          [&] { return e->stop || !e->submitted.empty(); });
    }
  }
  for (auto &r : e->ranks) {
    cudaSetDevice(r.device);
    for (cudaEvent_t ev : r.free_events) cudaEventDestroy(ev);
    for (cudaStream_t st : r.h2d) cudaStreamDestroy(st);
    for (cudaStream_t st : r.d2h) cudaStreamDestroy(st);
  }
  mark_finished(e);
}

// Stop the I/O threads (after the dispatcher drained every op).
void stop_io(fkv_engine *e) {
  {
    std::lock_guard<std::mutex> lk(e->io_mu);
    e->io_stop = true;
  }
  e->io_cv.notify_all();
  for (auto &t : e->io_th)
    if (t.joinable()) t.join();
}

}  // namespace

extern "C" {

void fkv_engine_config_init(fkv_engine_config *c) {
  std::memset(c, 0, sizeof(*c));
  c->num_ranks = 1;
  c->transfer_sms_h2d = -1;
  c->transfer_sms_d2h = -1;
}

int fkv_engine_create(const fkv_engine_config *c, fkv_engine **out) {
  fkv::clear_error();
  if (!c || !out) return fkv::fail(FKV_ERR_INVALID_ARG, "null config or output");
  *out = nullptr;
  if (c->num_ranks <= 0 || c->num_layers <= 0 || !c->gpu_layer_ptrs || !c->cpu_ptr)
    return fkv::fail(FKV_ERR_INVALID_ARG, "engine needs ranks, layers, layer pointers and a cpu pool");
  if (!c->is_mla && (int64_t)c->num_ranks * c->gpu_chunk_size_in_bytes > c->cpu_chunk_size_in_bytes &&
      c->cpu_chunk_size_in_bytes > 0)
    return fkv::fail(FKV_ERR_INVALID_ARG, "num_ranks * gpu_chunk exceeds cpu_chunk");
  int ndev = 0;
  FKV_CUDA(cudaGetDeviceCount(&ndev));
  auto e = std::make_unique<fkv_engine>();
  e->cfg = *c;
  e->ranks.resize(c->num_ranks);
  for (int r = 0; r < c->num_ranks; ++r) {
    int dev = c->device_ids ? c->device_ids[r] : r;
    if (dev < 0 || dev >= ndev)
      return fkv::fail(FKV_ERR_INVALID_ARG, "engine rank " + std::to_string(r) + " maps to missing device");
    e->ranks[r].device = dev;
    e->ranks[r].layer_ptrs.assign(c->gpu_layer_ptrs + (size_t)r * c->num_layers,
                                  c->gpu_layer_ptrs + (size_t)(r + 1) * c->num_layers);
  }
  e->cfg.gpu_layer_ptrs = nullptr;  // copied per rank
  e->cfg.device_ids = nullptr;
  fkv_engine *raw = e.get();
  if (c->ssd_ctx) {
    e->io_th[0] = std::thread(io_main, raw, 0);
    e->io_th[1] = std::thread(io_main, raw, 1);
  }
  e->worker = std::thread(engine_main, raw);
  {
    std::unique_lock<std::mutex> lk(e->mu);
    e->cv_done.wait(lk, [&] { return e->ready; });
  }
  if (e->init_rc != FKV_OK) {
    e->worker.join();
    stop_io(raw);
    return fkv::fail(e->init_rc, "engine init failed: " + e->init_error);
  }
  *out = e.release();
  return FKV_OK;
}

int fkv_engine_submit_graph(fkv_engine *e, int64_t graph_id, const fkv_engine_op *ops, int n_ops) {
  fkv::clear_error();
  if (!e) return fkv::fail(FKV_ERR_INVALID_ARG, "null engine");
  if (n_ops < 0 || (n_ops > 0 && !ops)) return fkv::fail(FKV_ERR_INVALID_ARG, "bad op array");
  auto g = std::make_unique<Graph>();
  g->id = graph_id;
  for (int i = 0; i < n_ops; ++i) {
    const fkv_engine_op &s = ops[i];
    if (s.type != FKV_OP_H2D && s.type != FKV_OP_D2H && s.type != FKV_OP_VIRTUAL && s.type != FKV_OP_DISK2H &&
        s.type != FKV_OP_H2DISK)
      return fkv::fail(FKV_ERR_INVALID_ARG, "unknown op type " + std::to_string(s.type));
    if ((s.type == FKV_OP_DISK2H || s.type == FKV_OP_H2DISK) && !e->cfg.ssd_ctx)
      return fkv::fail(FKV_ERR_INVALID_ARG, "DISK2H / H2DISK ops need an engine created with an SSD context");
    if (s.num_blocks < 0 || (s.num_blocks > 0 && (!s.gpu_block_ids || !s.cpu_block_ids)))
      return fkv::fail(FKV_ERR_INVALID_ARG, "bad block id arrays for op " + std::to_string(s.op_id));
    if (s.num_predecessors < 0 || (s.num_predecessors > 0 && !s.predecessors))
      return fkv::fail(FKV_ERR_INVALID_ARG, "bad predecessor array for op " + std::to_string(s.op_id));
    auto o = std::make_unique<Op>();
    o->graph_id = graph_id;
    o->op_id = s.op_id;
    o->type = s.type;
    o->host = s.type == FKV_OP_DISK2H || s.type == FKV_OP_H2DISK;
    if (s.type != FKV_OP_VIRTUAL && s.num_blocks > 0) {
      o->gpu_ids.assign(s.gpu_block_ids, s.gpu_block_ids + s.num_blocks);
      o->cpu_ids.assign(s.cpu_block_ids, s.cpu_block_ids + s.num_blocks);
    }
    o->layer_id = s.layer_id;
    o->layer_gran = s.layer_granularity;
    if (s.num_predecessors > 0) o->preds.assign(s.predecessors, s.predecessors + s.num_predecessors);
    g->ops.push_back(std::move(o));
  }
  {
    std::lock_guard<std::mutex> lk(e->mu);
    if (e->stop) return fkv::fail(FKV_ERR_INVALID_ARG, "engine is shutting down");
    e->inflight_ops += n_ops;
    e->submitted.push_back(std::move(g));
  }
  e->cv_work.notify_all();
  return FKV_OK;
}

int fkv_engine_poll(fkv_engine *e, int64_t *graph_ids, int64_t *op_ids, int *statuses, int max,
                    int timeout_ms, int *n_out) {
  fkv::clear_error();
  if (!e || !n_out || max < 0) return fkv::fail(FKV_ERR_INVALID_ARG, "bad poll arguments");
  *n_out = 0;
  std::unique_lock<std::mutex> lk(e->mu);
  if (e->completions.empty() && timeout_ms > 0)
    e->cv_done.wait_for(lk, std::chrono::milliseconds(timeout_ms),
                        [&] { return !e->completions.empty(); });
  int n = 0;
  while (n < max && !e->completions.empty()) {
    const Completion &c = e->completions.front();
    if (graph_ids) graph_ids[n] = c.graph_id;
    if (op_ids) op_ids[n] = c.op_id;
    if (statuses) statuses[n] = c.status;
    e->completions.pop_front();
    ++n;
  }
  *n_out = n;
  return FKV_OK;
}

int64_t fkv_engine_pending_ops(fkv_engine *e) {
  if (!e) return 0;
  std::lock_guard<std::mutex> lk(e->mu);
  return e->inflight_ops;
}

int fkv_engine_shutdown(fkv_engine *e, int timeout_ms) {
  fkv::clear_error();
  if (!e) return FKV_OK;
  {
    std::lock_guard<std::mutex> lk(e->mu);
    e->stop = true;
  }
  e->cv_work.notify_all();
  int64_t pending = 0;
  bool drained = true;
  if (timeout_ms >= 0) {
    std::unique_lock<std::mutex> lk(e->mu);
    drained = e->cv_done.wait_for(lk, std::chrono::milliseconds(timeout_ms), [&] { return e->finished; });
    pending = e->inflight_ops;
  }
  if (!drained) {
    // The dispatcher still owns e: leave it running (it exits once its ops
    // are done) and keep e allocated; the caller must not use e again.
    e->worker.detach();
    return fkv::fail(FKV_ERR_TIMEOUT, "engine did not drain its " + std::to_string(pending) +
                                          " pending ops within " + std::to_string(timeout_ms) +
                                          " ms; it was left running detached and must not be used again");
  }
  if (e->worker.joinable()) e->worker.join();
  stop_io(e);
  delete e;
  return FKV_OK;
}

void fkv_engine_destroy(fkv_engine *e) { fkv_engine_shutdown(e, -1); }

}  // extern "C"
