// Batched positional reads for the expert reader (host code only).
//
// The reference reads every merged span with one os.pread on a Python
// thread pool (streamlx/reader.py:80-100).  Here one call hands all spans of
// a read to a persistent pool of native threads that pread straight into
// the caller's (pinned) buffers; the calling thread works on its own spans
// too, so a read costs one library call instead of a Python task per span.
// Several callers (the decode thread, the prefetch thread, the sweep
// read-ahead) may read concurrently: their spans share one queue.
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <mutex>
#include <thread>
#include <vector>

#include "streamlx_cuda.h"

namespace {

struct Job {
  const int* fds;
  const int64_t* offs;
  const int64_t* sizes;
  void* const* dsts;
  std::atomic<int> remaining{0};
  std::atomic<int> err_index{-1};
  std::atomic<int> err_no{0};
  std::mutex m;
  std::condition_variable cv;
};

struct Task {
  Job* job;
  int i;
};

void run_task(const Task& t) {
  Job* j = t.job;
  const int i = t.i;
  char* dst = static_cast<char*>(j->dsts[i]);
  int64_t left = j->sizes[i], off = j->offs[i];
  while (left > 0 && j->err_index.load(std::memory_order_relaxed) < 0) {
    const ssize_t got = pread(j->fds[i], dst, (size_t)left, (off_t)off);
    if (got < 0) {
      if (errno == EINTR) continue;
      int expect = -1;
      if (j->err_index.compare_exchange_strong(expect, i)) j->err_no = errno;
      break;
    }
    if (got == 0) {  // end of file before the span ends: a short read
      int expect = -1;
      if (j->err_index.compare_exchange_strong(expect, i)) j->err_no = 0;
      break;
    }
    dst += got;
    off += got;
    left -= got;
  }
  // decrement under the job's lock: once the waiter can see zero it may
  // return and free the job, so nothing may touch it after the unlock
  std::lock_guard<std::mutex> lk(j->m);
  if (j->remaining.fetch_sub(1) == 1) j->cv.notify_all();
}

class Pool {
 public:
  void ensure_workers(int n) {
    std::lock_guard<std::mutex> lk(mu_);
    while ((int)threads_.size() < n)
      threads_.emplace_back([this] { worker(); });
  }
  void push(Job* job, int n) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      for (int i = 0; i < n; ++i) q_.push_back({job, i});
    }
    cv_.notify_all();
  }
  bool try_pop(Task* t) {
    std::lock_guard<std::mutex> lk(mu_);
    if (q_.empty()) return false;
    *t = q_.front();
    q_.pop_front();
    return true;
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& th : threads_) th.join();
  }

 private:
  void worker() {
    for (;;) {
      Task t;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [this] { return stop_ || !q_.empty(); });
        if (stop_ && q_.empty()) return;
        t = q_.front();
        q_.pop_front();
      }
      run_task(t);
    }
  }
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Task> q_;
  std::vector<std::thread> threads_;
  bool stop_ = false;
};

Pool& pool() {
  static Pool p;
  return p;
}

}  // namespace

extern "C" int slx_pread_many(const int* fds, const int64_t* offsets,
                              const int64_t* sizes, void* const* dsts, int n,
                              int threads, int* failed_index,
                              int* failed_errno) {
  if (failed_index) *failed_index = -1;
  if (failed_errno) *failed_errno = 0;
  if (n < 0 || (n > 0 && (!fds || !offsets || !sizes || !dsts)))
    return SLX_ERR_INVALID;
  if (n == 0) return SLX_OK;
  for (int i = 0; i < n; ++i)
    if (sizes[i] < 0 || offsets[i] < 0 || (sizes[i] > 0 && !dsts[i]))
      return SLX_ERR_INVALID;
  Job job;
  job.fds = fds;
  job.offs = offsets;
  job.sizes = sizes;
  job.dsts = dsts;
  job.remaining = n;
  if (threads > 1 && n > 1) {
    pool().ensure_workers(threads - 1);
    pool().push(&job, n);
    // help with whatever is queued (this job's spans or another caller's)
    Task t;
    while (job.remaining.load() > 0 && pool().try_pop(&t)) run_task(t);
    std::unique_lock<std::mutex> lk(job.m);
    job.cv.wait(lk, [&] { return job.remaining.load() == 0; });
  } else {
    for (int i = 0; i < n; ++i) run_task({&job, i});
  }
  const int bad = job.err_index.load();
  if (bad >= 0) {
    if (failed_index) *failed_index = bad;
    if (failed_errno) *failed_errno = job.err_no.load();
    return SLX_ERR_IO;
  }
  return SLX_OK;
}
