// Host runtime: the multi-GPU embedder and the request server (host code only; no kernels).
//
// Reference: internal/embeddings/embeddings.go — NewEmbedder builds one BertModel per device
// (:84-175); EmbedBatch splits a request across devices by token count weighted by each
// device's measured throughput (:436-553); runInferenceOnDevice cuts a device's share into
// dynamic batches (:704-731), runs them and updates the device's throughput average
// (:678-815).  The server front end caps the sequences in flight with a semaphore
// (internal/server/server.go:101).
//
// Differences, all in how the work is driven, none in what is computed:
//   - each replica has its own host thread that keeps two device batches in flight
//     (Cuda_Model_ForwardBatchAsync into pinned buffers): batch k+1 is staged and launched while
//     the device runs batch k, and batch k's vectors are collected while k+1 runs;
//   - the server's batcher joins queued requests into one batch per replica (round-robin over
//     replicas holding fewer than jobs_per_replica batches), each batch at most its replica's
//     share of the in-flight budget, so batches grow with the load;
//   - all bookkeeping is native (mutexes and condition variables), so a server feeding eight
//     replicas spends no host time per request beyond copying its ids.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../../include/fletcher_cuda.h"

// model.cu
int64_t model_hidden(CudaModelRef model);
CudaContextRef model_context(CudaModelRef model);

namespace {

int64_t now_ns() {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

using Range = std::pair<int32_t, int32_t>;

// embeddings.go:436-501: device d targets int(total * w_d / sum(w)) tokens (total / n while no
// throughput is known), at least 1; it takes at least one sequence, stops once its target is
// reached, and the last device takes the rest.  Devices past the end get nothing.
std::vector<Range> split_by_weight(const int32_t* len, int32_t n_seq, const double* w, int32_t n) {
  int64_t total = 0;
  for (int32_t i = 0; i < n_seq; i++) total += len[i];
  double tw = 0;
  for (int32_t d = 0; d < n; d++) tw += w[d];
  std::vector<Range> out;
  int32_t start = 0;
  for (int32_t d = 0; d < n; d++) {
    if (start >= n_seq) break;
    int64_t target = tw > 0 ? (int64_t)((double)total * w[d] / tw) : total / n;
    if (target == 0) target = 1;
    int32_t end = start;
    int64_t cur = 0;
    while (end < n_seq) {
      if (end == start) {
        cur += len[end++];
        continue;
      }
      if (d < n - 1 && cur >= target) break;
      cur += len[end++];
    }
    if (d == n - 1) end = n_seq;
    out.push_back({start, end});
    start = end;
  }
  return out;
}

// embeddings.go:704-731: fill a batch until max_batch sequences, or until the next sequence would
// pass max_tokens (a single longer sequence still forms its own batch).
std::vector<Range> dynamic_batches(const int32_t* len, int32_t n, int32_t max_batch, int64_t max_tokens) {
  std::vector<Range> out;
  int32_t i = 0;
  while (i < n) {
    int32_t size = 0;
    int64_t tok = 0;
    for (int32_t j = i; j < n; j++) {
      if (size >= max_batch) break;
      if (tok + len[j] > max_tokens && size > 0) break;
      tok += len[j];
      size++;
    }
    size = std::max(size, 1);
    out.push_back({i, i + size});
    i += size;
  }
  return out;
}

// One unit of work for a replica: sequences with their packed ids, the destination row of each
// sequence's vector, and a completion callback run once on the replica's thread.
struct Job {
  std::vector<int32_t> ids, lengths;
  std::vector<int64_t> cu;  // token offset of each sequence (+ the end)
  std::vector<float*> dst;  // destination row per sequence
  std::deque<Range> todo;   // device batches not yet launched
  int pending = 0;          // device batches not yet collected
  int32_t status = FLETCHER_OK;
  std::string err;
  int64_t t0 = 0;
  std::function<void(Job&)> done;

  void prepare(int32_t max_batch, int64_t max_tokens) {
    const int32_t n = (int32_t)lengths.size();
    cu.assign(n + 1, 0);
    for (int32_t i = 0; i < n; i++) cu[i + 1] = cu[i] + lengths[i];
    for (const Range& r : dynamic_batches(lengths.data(), n, max_batch, max_tokens)) todo.push_back(r);
    pending = (int)todo.size();
    t0 = now_ns();
  }
};

// The device side of one replica: two in-flight slots.  launch() stages a batch into a slot and
// starts it; collect() waits for it and exposes its [B, hidden] float32 rows.
struct Device {
  virtual ~Device() = default;
  virtual int32_t launch(int slot, const int32_t* ids, int64_t n_ids, const int32_t* lengths, int32_t B,
                         int64_t* ticket) = 0;
  virtual int32_t collect(int slot, int64_t ticket, const float** rows) = 0;
  virtual std::string error() = 0;
};

struct ModelDevice : Device {
  CudaModelRef model;
  CudaContextRef ctx;
  int64_t hidden;
  int32_t pooling;
  struct Slot {
    int32_t* ids = nullptr;
    int64_t ids_cap = 0;
    float* out = nullptr;
    int64_t out_rows = 0;
  } slots[2];
  std::string msg;

  ModelDevice(CudaModelRef m, int32_t pool) : model(m), ctx(model_context(m)), hidden(model_hidden(m)), pooling(pool) {}
  ~ModelDevice() override {
    for (Slot& s : slots) {
      if (s.ids) Cuda_HostFree(ctx, s.ids);
      if (s.out) Cuda_HostFree(ctx, s.out);
    }
  }
  int32_t launch(int k, const int32_t* ids, int64_t n_ids, const int32_t* lengths, int32_t B,
                 int64_t* ticket) override {
    Slot& s = slots[k];
    if (s.ids_cap < n_ids) {  // pinned staging grows to the largest batch seen
      if (s.ids) Cuda_HostFree(ctx, s.ids);
      s.ids_cap = std::max<int64_t>(n_ids, 1 << 14);
      s.ids = static_cast<int32_t*>(Cuda_HostAlloc(ctx, s.ids_cap * 4));
      if (!s.ids) {
        s.ids_cap = 0;
        msg = "pinned host allocation failed";
        return FLETCHER_ERR_OOM;
      }
    }
    if (s.out_rows < B) {
      if (s.out) Cuda_HostFree(ctx, s.out);
      s.out_rows = std::max<int64_t>(B, 64);
      s.out = static_cast<float*>(Cuda_HostAlloc(ctx, s.out_rows * hidden * 4));
      if (!s.out) {
        s.out_rows = 0;
        msg = "pinned host allocation failed";
        return FLETCHER_ERR_OOM;
      }
    }
    std::memcpy(s.ids, ids, n_ids * 4);
    return Cuda_Model_ForwardBatchAsync(model, s.ids, lengths, B, pooling, FLETCHER_F32, s.out, ticket);
  }
  int32_t collect(int k, int64_t ticket, const float** rows) override {
    *rows = slots[k].out;
    return Cuda_Model_Wait(model, ticket);
  }
  std::string error() override {
    if (!msg.empty()) return std::exchange(msg, std::string());
    char buf[512] = {0};
    Cuda_GetLastError(ctx, buf, sizeof(buf));
    return buf;
  }
};

// Test double: a "device" that runs one batch at a time, delay_us each, and writes
// (first id, length, replica index, 0, ...) per sequence.  A negative id fails the batch, the way
// an out-of-range id fails a model's batch.
struct FakeDevice : Device {
  int32_t index, hidden;
  int64_t delay_ns, busy_until = 0;
  struct Slot {
    std::vector<float> rows;
    int64_t ready = 0;
  } slots[2];
  std::string msg;

  FakeDevice(int32_t i, int32_t h, int64_t delay_us) : index(i), hidden(h), delay_ns(delay_us * 1000) {}
  int32_t launch(int k, const int32_t* ids, int64_t n_ids, const int32_t* lengths, int32_t B,
                 int64_t* ticket) override {
    for (int64_t t = 0; t < n_ids; t++)
      if (ids[t] < 0) {
        msg = "fake replica " + std::to_string(index) + ": negative id " + std::to_string(ids[t]);
        return FLETCHER_ERR_INVALID;
      }
    Slot& s = slots[k];
    s.rows.assign((size_t)B * hidden, 0.f);
    int64_t off = 0;
    for (int32_t i = 0; i < B; i++) {
      s.rows[(size_t)i * hidden] = (float)ids[off];
      if (hidden > 1) s.rows[(size_t)i * hidden + 1] = (float)lengths[i];
      if (hidden > 2) s.rows[(size_t)i * hidden + 2] = (float)index;
      off += lengths[i];
    }
    busy_until = std::max(busy_until, now_ns()) + delay_ns;
    s.ready = busy_until;
    *ticket = k;
    return FLETCHER_OK;
  }
  int32_t collect(int k, int64_t, const float** rows) override {
    const int64_t wait = slots[k].ready - now_ns();
    if (wait > 0) std::this_thread::sleep_for(std::chrono::nanoseconds(wait));
    *rows = slots[k].rows.data();
    return FLETCHER_OK;
  }
  std::string error() override { return std::exchange(msg, std::string()); }
};

struct Replica {
  int32_t index;
  int64_t hidden;
  std::unique_ptr<Device> dev;
  std::mutex mu;
  std::condition_variable cv;
  std::deque<Job*> queue;
  bool stop = false;
  double tput = 1.0;  // embeddings.go:197: the cold-start value, replaced by the first measurement
  bool measured = false;
  std::atomic<int64_t> jobs{0}, seqs{0};
  std::thread th;

  Replica(int32_t i, int64_t h, std::unique_ptr<Device> d) : index(i), hidden(h), dev(std::move(d)) {
    th = std::thread([this] { loop(); });
  }
  ~Replica() {
    {
      std::lock_guard<std::mutex> lk(mu);
      stop = true;
    }
    cv.notify_all();
    th.join();
  }
  void enqueue(Job* j) {
    jobs++;
    seqs += (int64_t)j->lengths.size();
    if (j->pending == 0) {  // nothing to run
      finish(*j);
      return;
    }
    {
      std::lock_guard<std::mutex> lk(mu);
      queue.push_back(j);
    }
    cv.notify_one();
  }
  double throughput() {
    std::lock_guard<std::mutex> lk(mu);
    return tput;
  }
  void set_throughput(double v) {
    std::lock_guard<std::mutex> lk(mu);
    tput = v;
    measured = true;
  }
  // embeddings.go:795-804: sequences / elapsed, first measurement replaces the default, then an
  // exponential average with alpha = 0.3.
  void finish(Job& j) {
    if (j.status == FLETCHER_OK && !j.lengths.empty()) {
      const double dt = (double)(now_ns() - j.t0) * 1e-9;
      if (dt > 0) {
        const double r = (double)j.lengths.size() / dt;
        std::lock_guard<std::mutex> lk(mu);
        tput = measured ? 0.3 * r + 0.7 * tput : r;
        measured = true;
      }
    }
    j.done(j);
  }
  void fail(Job& j, int32_t rc) {
    if (j.status == FLETCHER_OK) {
      j.status = rc;
      j.err = dev->error();
      if (j.err.empty()) j.err = "replica " + std::to_string(index) + ": error " + std::to_string(rc);
    }
  }
  void loop() {
    struct InFlight {
      int64_t ticket;
      int slot;
      Job* job;
      Range r;
      bool ok;
    };
    std::deque<Job*> todo;
    std::deque<InFlight> inflight;
    uint64_t nslot = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu);
        if (todo.empty() && inflight.empty()) cv.wait(lk, [&] { return stop || !queue.empty(); });
        while (!queue.empty()) {
          todo.push_back(queue.front());
          queue.pop_front();
        }
        if (stop && todo.empty() && inflight.empty()) return;
      }
      if (!todo.empty() && inflight.size() < 2) {
        Job* j = todo.front();
        const Range r = j->todo.front();
        j->todo.pop_front();
        if (j->todo.empty()) todo.pop_front();
        const int k = (int)(nslot++ % 2);  // FIFO collection frees the slots in this order
        InFlight f{0, k, j, r, false};
        if (j->status == FLETCHER_OK) {
          const int32_t rc = dev->launch(k, j->ids.data() + j->cu[r.first], j->cu[r.second] - j->cu[r.first],
                                         j->lengths.data() + r.first, r.second - r.first, &f.ticket);
          if (rc)
            fail(*j, rc);
          else
            f.ok = true;
        }
        inflight.push_back(f);
      } else if (!inflight.empty()) {
        const InFlight f = inflight.front();
        inflight.pop_front();
        Job& j = *f.job;
        if (f.ok) {
          const float* rows = nullptr;
          const int32_t rc = dev->collect(f.slot, f.ticket, &rows);
          if (rc) {
            fail(j, rc);
          } else if (j.status == FLETCHER_OK) {
            for (int32_t i = f.r.first; i < f.r.second; i++)
              std::memcpy(j.dst[i], rows + (size_t)(i - f.r.first) * hidden, hidden * sizeof(float));
          }
        }
        if (--j.pending == 0) finish(j);
      }
    }
  }
};

struct Embedder {
  std::vector<std::unique_ptr<Replica>> reps;
  int64_t hidden = 0;
  int32_t max_batch = 512;
  int64_t max_tokens = 65536;
  std::mutex err_mu;
  std::string last_err;

  void set_error(const std::string& e) {
    std::lock_guard<std::mutex> lk(err_mu);
    last_err = e;
  }
};

struct Req {
  int64_t arrival = 0, done = -1;
  int32_t status = FLETCHER_OK;
  int32_t nseq = 0;
  float* out = nullptr;
  std::vector<int32_t> ids, lengths;
};

struct Server {
  Embedder* emb;
  int64_t cap;
  int32_t jpr;
  int64_t share;
  std::mutex mu;
  std::condition_variable cv_disp, cv_done;
  std::deque<Req> reqs;       // ticket t is reqs[t - 1]
  std::deque<int64_t> held;   // submitted, not yet dispatched
  int64_t busy = 0;           // sequences handed to replicas and not yet returned
  std::vector<int32_t> jobs;  // batches outstanding per replica
  int32_t rr = 0;
  bool stop = false;
  FletcherServerStats st{};
  std::thread th;

  Server(Embedder* e, int64_t max_in_flight, int32_t jobs_per_replica)
      : emb(e), cap(max_in_flight), jpr(jobs_per_replica), jobs(e->reps.size(), 0) {
    // One batch takes at most its replica's share of the budget, so that every replica can hold
    // work at once under the cap.
    share = std::max<int64_t>(1, cap / ((int64_t)e->reps.size() * jpr));
    th = std::thread([this] { loop(); });
  }
  ~Server() {
    {
      std::lock_guard<std::mutex> lk(mu);
      stop = true;
    }
    cv_disp.notify_all();
    th.join();
  }

  void loop() {
    const int32_t nrep = (int32_t)jobs.size();
    std::unique_lock<std::mutex> lk(mu);
    for (;;) {
      int32_t rep = -1;
      for (int32_t k = 0; k < nrep; k++) {
        const int32_t i = (rr + k) % nrep;
        if (jobs[i] < jpr) {
          rep = i;
          break;
        }
      }
      // A batch's first request goes out within the budget, or alone when nothing runs.
      const bool go = rep >= 0 && !held.empty() &&
                      (busy + reqs[held.front() - 1].nseq <= cap || busy == 0);
      if (!go) {
        if (stop && held.empty() && busy == 0) return;
        cv_disp.wait(lk);
        continue;
      }
      std::vector<int64_t> take;
      int64_t nseq = 0;
      while (!held.empty()) {
        const int64_t n = reqs[held.front() - 1].nseq;
        if (!take.empty() && !(busy + nseq + n <= cap && nseq + n <= share)) break;
        take.push_back(held.front());
        held.pop_front();
        nseq += n;
      }
      rr = rep + 1;
      busy += nseq;
      jobs[rep]++;
      st.batches++;
      st.max_busy = std::max(st.max_busy, busy);
      if (take.size() > 1) st.max_batch_seqs = std::max(st.max_batch_seqs, nseq);
      // The requests' ids move into the job; the concatenation runs outside the lock.
      std::vector<std::vector<int32_t>> ids(take.size()), lens(take.size());
      std::vector<float*> outs(take.size());
      for (size_t i = 0; i < take.size(); i++) {
        Req& r = reqs[take[i] - 1];
        ids[i].swap(r.ids);
        lens[i].swap(r.lengths);
        outs[i] = r.out;
      }
      lk.unlock();
      Job* j = new Job;
      int64_t ntok = 0;
      for (auto& v : ids) ntok += (int64_t)v.size();
      j->ids.reserve(ntok);
      j->lengths.reserve(nseq);
      j->dst.reserve(nseq);
      for (size_t i = 0; i < take.size(); i++) {
        j->ids.insert(j->ids.end(), ids[i].begin(), ids[i].end());
        j->lengths.insert(j->lengths.end(), lens[i].begin(), lens[i].end());
        for (size_t q = 0; q < lens[i].size(); q++) j->dst.push_back(outs[i] + (int64_t)q * emb->hidden);
      }
      j->prepare(emb->max_batch, emb->max_tokens);
      j->done = [this, take = std::move(take), nseq, rep](Job& job) {
        if (job.status != FLETCHER_OK) emb->set_error(job.err);
        const int64_t t = now_ns();
        {
          std::lock_guard<std::mutex> g(mu);
          busy -= nseq;
          jobs[rep]--;
          for (int64_t tk : take) {
            Req& r = reqs[tk - 1];
            r.status = job.status;
            r.done = t;
          }
          st.completed += (int64_t)take.size();
          // Notified under the lock: once it is released the server may be destroyed.
          cv_disp.notify_all();
          cv_done.notify_all();
        }
        delete &job;
      };
      emb->reps[rep]->enqueue(j);
      lk.lock();
    }
  }
};

int32_t make_embedder(std::vector<std::unique_ptr<Device>> devs, int64_t hidden, int32_t max_batch,
                      int64_t max_tokens, CudaEmbedderRef* out) {
  auto* e = new Embedder;
  e->hidden = hidden;
  e->max_batch = max_batch > 0 ? max_batch : 512;
  e->max_tokens = max_tokens;
  for (size_t i = 0; i < devs.size(); i++)
    e->reps.emplace_back(new Replica((int32_t)i, hidden, std::move(devs[i])));
  *out = e;
  return FLETCHER_OK;
}

}  // namespace

extern "C" {

int32_t Cuda_Runtime_SplitByWeight(const int32_t* lengths, int32_t numSeqs, const double* weights, int32_t n,
                                   int32_t* ranges) {
  if (!lengths || !weights || !ranges || numSeqs < 0 || n <= 0) return -1;
  const std::vector<Range> r = split_by_weight(lengths, numSeqs, weights, n);
  for (size_t d = 0; d < r.size(); d++) {
    ranges[2 * d] = r[d].first;
    ranges[2 * d + 1] = r[d].second;
  }
  return (int32_t)r.size();
}

int32_t Cuda_Runtime_DynamicBatches(const int32_t* lengths, int32_t numSeqs, int32_t max_batch, int64_t max_tokens,
                                    int32_t* ranges, int32_t cap) {
  if (!lengths || !ranges || numSeqs < 0 || max_batch <= 0) return -1;
  const std::vector<Range> r = dynamic_batches(lengths, numSeqs, max_batch, max_tokens);
  if ((int32_t)r.size() > cap) return -1;
  for (size_t i = 0; i < r.size(); i++) {
    ranges[2 * i] = r[i].first;
    ranges[2 * i + 1] = r[i].second;
  }
  return (int32_t)r.size();
}

int32_t Cuda_Embedder_Create(const CudaModelRef* models, int32_t n, int32_t pooling, int32_t max_batch,
                             int64_t max_tokens, CudaEmbedderRef* out) {
  if (!models || n <= 0 || !out) return FLETCHER_ERR_INVALID;
  const int64_t hidden = model_hidden(models[0]);
  int64_t min_total = INT64_MAX;
  for (int32_t i = 0; i < n; i++) {
    if (!models[i] || model_hidden(models[i]) != hidden || hidden <= 0) return FLETCHER_ERR_INVALID;
    int64_t alloc = 0, total = 0;
    if (Cuda_MemGetInfo(model_context(models[i]), &alloc, &total) == FLETCHER_OK) min_total = std::min(min_total, total);
  }
  if (max_tokens <= 0) max_tokens = min_total != INT64_MAX && min_total >= (64ll << 30) ? 65536 : 16384;
  std::vector<std::unique_ptr<Device>> devs;
  for (int32_t i = 0; i < n; i++) devs.emplace_back(new ModelDevice(models[i], pooling));
  return make_embedder(std::move(devs), hidden, max_batch, max_tokens, out);
}

int32_t Cuda_Embedder_CreateFake(int32_t n, int32_t hidden, int64_t delay_us, int32_t max_batch, int64_t max_tokens,
                                 CudaEmbedderRef* out) {
  if (n <= 0 || hidden <= 0 || delay_us < 0 || !out) return FLETCHER_ERR_INVALID;
  std::vector<std::unique_ptr<Device>> devs;
  for (int32_t i = 0; i < n; i++) devs.emplace_back(new FakeDevice(i, hidden, delay_us));
  return make_embedder(std::move(devs), hidden, max_batch, max_tokens > 0 ? max_tokens : 65536, out);
}

int32_t Cuda_Embedder_Embed(CudaEmbedderRef ref, const int32_t* ids, const int32_t* lengths, int32_t numSeqs,
                            float* out) {
  auto* e = static_cast<Embedder*>(ref);
  if (!e || numSeqs < 0 || (numSeqs > 0 && (!ids || !lengths || !out))) return FLETCHER_ERR_INVALID;
  if (numSeqs == 0) return FLETCHER_OK;
  for (int32_t i = 0; i < numSeqs; i++)
    if (lengths[i] < 0) {
      e->set_error("Embed: negative length");
      return FLETCHER_ERR_INVALID;
    }
  const int32_t n = (int32_t)e->reps.size();
  std::vector<double> w(n);
  for (int32_t d = 0; d < n; d++) w[d] = e->reps[d]->throughput();
  const std::vector<Range> parts = split_by_weight(lengths, numSeqs, w.data(), n);
  std::vector<int64_t> cu(numSeqs + 1, 0);
  for (int32_t i = 0; i < numSeqs; i++) cu[i + 1] = cu[i] + lengths[i];
  struct Latch {
    std::mutex mu;
    std::condition_variable cv;
    int left;
    int32_t status = FLETCHER_OK;
    std::string err;
  };
  auto latch = std::make_shared<Latch>();
  latch->left = (int)parts.size();
  for (size_t d = 0; d < parts.size(); d++) {
    const Range r = parts[d];
    Job* j = new Job;
    j->ids.assign(ids + cu[r.first], ids + cu[r.second]);
    j->lengths.assign(lengths + r.first, lengths + r.second);
    for (int32_t i = r.first; i < r.second; i++) j->dst.push_back(out + (int64_t)i * e->hidden);
    j->prepare(e->max_batch, e->max_tokens);
    j->done = [latch](Job& job) {
      {
        std::lock_guard<std::mutex> g(latch->mu);
        if (job.status != FLETCHER_OK && latch->status == FLETCHER_OK) {
          latch->status = job.status;
          latch->err = job.err;
        }
        latch->left--;
      }
      latch->cv.notify_all();
      delete &job;
    };
    e->reps[d]->enqueue(j);
  }
  std::unique_lock<std::mutex> lk(latch->mu);
  latch->cv.wait(lk, [&] { return latch->left == 0; });
  if (latch->status != FLETCHER_OK) e->set_error(latch->err);
  return latch->status;
}

int32_t Cuda_Embedder_Throughput(CudaEmbedderRef ref, double* tput, int32_t n, int32_t set) {
  auto* e = static_cast<Embedder*>(ref);
  if (!e || !tput || n != (int32_t)e->reps.size()) return FLETCHER_ERR_INVALID;
  for (int32_t d = 0; d < n; d++) {
    if (set)
      e->reps[d]->set_throughput(tput[d]);
    else
      tput[d] = e->reps[d]->throughput();
  }
  return FLETCHER_OK;
}

int32_t Cuda_Embedder_Counts(CudaEmbedderRef ref, int64_t* jobs, int64_t* seqs, int32_t n) {
  auto* e = static_cast<Embedder*>(ref);
  if (!e || n != (int32_t)e->reps.size()) return FLETCHER_ERR_INVALID;
  for (int32_t d = 0; d < n; d++) {
    if (jobs) jobs[d] = e->reps[d]->jobs.load();
    if (seqs) seqs[d] = e->reps[d]->seqs.load();
  }
  return FLETCHER_OK;
}

int32_t Cuda_Embedder_Hidden(CudaEmbedderRef ref) {
  auto* e = static_cast<Embedder*>(ref);
  return e ? (int32_t)e->hidden : -1;
}

int32_t Cuda_Embedder_MaxBatch(CudaEmbedderRef ref, int32_t* max_batch, int64_t* max_tokens) {
  auto* e = static_cast<Embedder*>(ref);
  if (!e) return FLETCHER_ERR_INVALID;
  if (max_batch) *max_batch = e->max_batch;
  if (max_tokens) *max_tokens = e->max_tokens;
  return FLETCHER_OK;
}

int32_t Cuda_Embedder_LastError(CudaEmbedderRef ref, char* buf, int32_t len) {
  auto* e = static_cast<Embedder*>(ref);
  if (!e || !buf || len <= 0) return FLETCHER_ERR_INVALID;
  std::lock_guard<std::mutex> lk(e->err_mu);
  std::snprintf(buf, (size_t)len, "%s", e->last_err.c_str());
  return FLETCHER_OK;
}

void Cuda_Embedder_Destroy(CudaEmbedderRef ref) { delete static_cast<Embedder*>(ref); }

int32_t Cuda_Server_Create(CudaEmbedderRef ref, int32_t max_in_flight, int32_t jobs_per_replica, CudaServerRef* out) {
  auto* e = static_cast<Embedder*>(ref);
  if (!e || !out) return FLETCHER_ERR_INVALID;
  *out = new Server(e, max_in_flight > 0 ? max_in_flight : 16384, jobs_per_replica > 0 ? jobs_per_replica : 2);
  return FLETCHER_OK;
}

int64_t Cuda_Server_Clock(void) { return now_ns(); }

int32_t Cuda_Server_Submit(CudaServerRef ref, int32_t n, const int32_t* ids, const int32_t* lengths,
                           const int64_t* seq_off, const int64_t* arrival_ns, float* out, int64_t* first_ticket) {
  auto* s = static_cast<Server*>(ref);
  if (!s || n < 0 || !first_ticket || (n > 0 && (!ids || !lengths || !seq_off || !out))) return FLETCHER_ERR_INVALID;
  if (n > 0 && seq_off[0] != 0) return FLETCHER_ERR_INVALID;
  int64_t tok = 0;
  for (int32_t r = 0; r < n; r++) {
    if (seq_off[r + 1] < seq_off[r]) return FLETCHER_ERR_INVALID;
    for (int64_t i = seq_off[r]; i < seq_off[r + 1]; i++) {
      if (lengths[i] < 0) return FLETCHER_ERR_INVALID;
      tok += lengths[i];
    }
  }
  const int64_t t = now_ns();
  {
    std::lock_guard<std::mutex> lk(s->mu);
    if (s->stop) return FLETCHER_ERR_INVALID;
    *first_ticket = (int64_t)s->reqs.size() + 1;
    int64_t off = 0;
    for (int32_t r = 0; r < n; r++) {
      s->reqs.emplace_back();
      Req& q = s->reqs.back();
      q.arrival = arrival_ns ? arrival_ns[r] : t;
      q.nseq = (int32_t)(seq_off[r + 1] - seq_off[r]);
      q.out = out + seq_off[r] * s->emb->hidden;
      q.lengths.assign(lengths + seq_off[r], lengths + seq_off[r + 1]);
      int64_t nt = 0;
      for (int32_t l : q.lengths) nt += l;
      q.ids.assign(ids + off, ids + off + nt);
      off += nt;
      s->st.requests++;
      s->st.max_request_seqs = std::max<int64_t>(s->st.max_request_seqs, q.nseq);
      if (q.nseq == 0) {  // nothing to embed
        q.done = t;
        s->st.completed++;
      } else {
        s->held.push_back(*first_ticket + r);
      }
    }
  }
  (void)tok;
  s->cv_disp.notify_all();
  return FLETCHER_OK;
}

int32_t Cuda_Server_Wait(CudaServerRef ref, int64_t ticket, double timeout_s, int64_t* latency_ns) {
  auto* s = static_cast<Server*>(ref);
  if (!s) return FLETCHER_ERR_INVALID;
  std::unique_lock<std::mutex> lk(s->mu);
  if (ticket < 1 || ticket > (int64_t)s->reqs.size()) return FLETCHER_ERR_INVALID;
  auto ready = [&] { return s->reqs[ticket - 1].done >= 0; };
  if (timeout_s < 0) {
    s->cv_done.wait(lk, ready);
  } else if (!s->cv_done.wait_for(lk, std::chrono::duration<double>(timeout_s), ready)) {
    return -1;
  }
  const Req& r = s->reqs[ticket - 1];
  if (latency_ns) *latency_ns = r.done - r.arrival;
  return r.status;
}

int32_t Cuda_Server_Latencies(CudaServerRef ref, int64_t first, int64_t n, int64_t* latency_ns) {
  auto* s = static_cast<Server*>(ref);
  if (!s || !latency_ns || first < 1 || n < 0) return FLETCHER_ERR_INVALID;
  std::lock_guard<std::mutex> lk(s->mu);
  if (first + n - 1 > (int64_t)s->reqs.size()) return FLETCHER_ERR_INVALID;
  for (int64_t i = 0; i < n; i++) {
    const Req& r = s->reqs[first - 1 + i];
    latency_ns[i] = r.done < 0 ? -1 : (r.status != FLETCHER_OK ? -2 : r.done - r.arrival);
  }
  return FLETCHER_OK;
}

int32_t Cuda_Server_Drain(CudaServerRef ref) {
  auto* s = static_cast<Server*>(ref);
  if (!s) return FLETCHER_ERR_INVALID;
  std::unique_lock<std::mutex> lk(s->mu);
  s->cv_done.wait(lk, [&] { return s->st.completed == s->st.requests; });
  return FLETCHER_OK;
}

int32_t Cuda_Server_Stats(CudaServerRef ref, FletcherServerStats* st) {
  auto* s = static_cast<Server*>(ref);
  if (!s || !st) return FLETCHER_ERR_INVALID;
  std::lock_guard<std::mutex> lk(s->mu);
  *st = s->st;
  return FLETCHER_OK;
}

void Cuda_Server_Destroy(CudaServerRef ref) { delete static_cast<Server*>(ref); }

}  // extern "C"
