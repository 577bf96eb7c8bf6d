// The serving front of the library: a request queue in front of one worker thread per GPU that
// packs queued requests from many clients into varlen batches.
//
// It keeps the reference server's contract (runtime/crates/sys1rust/src/worker.rs,
// runtime/crates/sys1rust/src/http.rs:168-230) and replaces its one-request-at-a-time inference
// thread with cross-request batching over several GPUs:
//  * admission is non-blocking: a request over the concurrency cap is refused at once ("server
//    busy, try again later", HTTP 503 with Retry-After: 1 in the reference) rather than queued,
//    so what is buffered stays bounded. The permit lives from submit until the result is collected
//    or the ticket is cancelled;
//  * a request whose client went away (cancelled ticket) is dropped from the queue unrun;
//  * a failed forward fails only the requests of its batch; the worker keeps serving;
//  * with no worker running, requests fail with "inference worker is not running" (503).
// Workers take the oldest queued request and then more, in arrival order, while the batch stays
// within the token and row limits (a request longer than the token limit runs alone); an idle
// worker takes the next batch, so the load spreads over the GPUs by availability.
#pragma once
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

namespace s1c {
namespace srv {

struct Job {
  uint64_t id = 0;
  std::vector<uint32_t> ids, markers;
  uint32_t qtype = 0;
  std::vector<float> logits, pooled;
  s1c_status status = S1C_OK;
  std::string error;
  bool done = false, cancelled = false;
  double infer_ms = 0;
  int worker = -1;
};

struct Server {
  s1c_server_forward_fn fn = nullptr;
  std::vector<void*> ctx;
  int hidden = 0;
  s1c_server_opts opts{};

  std::mutex mu;
  std::condition_variable cv_work, cv_done;
  std::deque<std::shared_ptr<Job>> queue;
  std::unordered_map<uint64_t, std::shared_ptr<Job>> jobs;  // admitted, not yet collected
  uint64_t next_id = 1;
  bool stopping = false;
  std::atomic<int> alive{0};
  std::vector<std::thread> workers;
  s1c_server_stats stats{};

  void fail_queued_locked(const char* why) {
    for (auto& j : queue) {
      if (j->done) continue;
      j->status = S1C_ERR_DEAD;
      j->error = why;
      j->done = true;
    }
    queue.clear();
  }

  // Take the next batch (caller holds the lock; the queue is non-empty).
  std::vector<std::shared_ptr<Job>> take_batch_locked() {
    std::vector<std::shared_ptr<Job>> b;
    size_t tokens = 0;
    while (!queue.empty()) {
      std::shared_ptr<Job> j = queue.front();
      if (j->cancelled) {
        queue.pop_front();
        ++stats.cancelled_skipped;
        continue;
      }
      const size_t len = j->ids.size();
      if (!b.empty() && ((int64_t)(tokens + len) > opts.max_batch_tokens || (int32_t)b.size() >= opts.max_batch_rows))
        break;
      queue.pop_front();
      tokens += len;
      b.push_back(std::move(j));
    }
    return b;
  }

  // `alive` counts the workers from their creation (server_start sets it) until they exit.
  void run(int w) {
    std::vector<uint32_t> ids, mpos, qtype;
    std::vector<int32_t> cu, mcount;
    std::vector<float> logits, pooled;
    for (;;) {
      std::vector<std::shared_ptr<Job>> batch;
      {
        std::unique_lock<std::mutex> lk(mu);
        cv_work.wait(lk, [&] { return stopping || !queue.empty(); });
        if (stopping) break;
        if (opts.linger_us > 0) {
          // A short wait for more requests when the batch would be far from full.
          size_t queued = 0;
          for (auto& j : queue) queued += j->ids.size();
          if ((int64_t)queued < opts.max_batch_tokens / 2)
            cv_work.wait_for(lk, std::chrono::microseconds(opts.linger_us), [&] { return stopping; });
          if (stopping) break;
        }
        batch = take_batch_locked();
        if (batch.empty()) continue;
        ++stats.batches;
        stats.rows += batch.size();
      }
      // Pack: ids back to back, markers padded to the batch's largest marker count.
      const int n = (int)batch.size();
      int kmax = 0;
      cu.assign(1, 0);
      ids.clear();
      for (auto& j : batch) {
        ids.insert(ids.end(), j->ids.begin(), j->ids.end());
        cu.push_back((int32_t)ids.size());
        kmax = std::max(kmax, (int)j->markers.size());
      }
      mpos.assign((size_t)n * (size_t)std::max(kmax, 1), 0);
      mcount.assign(n, 0);
      qtype.assign(n, 0);
      for (int r = 0; r < n; ++r) {
        const Job& j = *batch[r];
        for (size_t k = 0; k < j.markers.size(); ++k) mpos[(size_t)r * kmax + k] = j.markers[k];
        mcount[r] = (int32_t)j.markers.size();
        qtype[r] = j.qtype;
      }
      logits.assign((size_t)n * (size_t)std::max(kmax, 1), 0.f);
      pooled.assign((size_t)n * (size_t)hidden, 0.f);
      s1c_varlen v{n, kmax, ids.data(), cu.data(), mpos.data(), mcount.data(), qtype.data()};
      const auto t0 = std::chrono::steady_clock::now();
      const char* err = nullptr;
      s1c_status st = fn(ctx[(size_t)w], &v, logits.data(), pooled.data(), &err);
      const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
      {
        std::lock_guard<std::mutex> lk(mu);
        stats.tokens += ids.size();
        if (st != S1C_OK) ++stats.failed_batches;
        for (int r = 0; r < n; ++r) {
          Job& j = *batch[r];
          j.worker = w;
          j.infer_ms = ms;
          j.status = st;
          if (st == S1C_OK) {
            j.logits.assign(logits.begin() + (size_t)r * kmax, logits.begin() + (size_t)r * kmax + j.markers.size());
            j.pooled.assign(pooled.begin() + (size_t)r * hidden, pooled.begin() + (size_t)(r + 1) * hidden);
          } else {
            j.error = err ? err : ("forward failed with status " + std::to_string(st));
          }
          j.done = true;
        }
      }
      cv_done.notify_all();
    }
    --alive;
  }
};

}  // namespace srv
}  // namespace s1c
