// Persistent worker pool for the host CPU kernels (no OpenMP runtime is
// required at link time).  A job is published by bumping an atomic
// generation counter; workers spin on it for a short while (a decode step
// issues its small matmuls back to back, so the next job usually arrives
// within microseconds) and only then sleep on a condition variable, and the
// caller spins on an atomic count of unfinished parts.  Dispatch therefore
// costs about a cache-line round trip instead of two futex wake-ups.
#pragma once

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace bloom {
namespace rt {

class ThreadPool {
 public:
  static ThreadPool& instance() {
    static ThreadPool pool;
    return pool;
  }
  int size() const { return static_cast<int>(workers_.size()) + 1; }
  void resize(int n);
  // Calls fn(begin, end) over [0, n) split into contiguous chunks; blocks until done.
  void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& fn);

 private:
  ThreadPool();
  ~ThreadPool();
  void stop_workers();
  void start_workers(int n);
  void worker_loop(int idx);

  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_;
  const std::function<void(int64_t, int64_t)>* job_ = nullptr;
  int64_t job_n_ = 0;
  std::atomic<int64_t> generation_{0};
  std::atomic<int> pending_{0};
  std::atomic<bool> stop_{false};
  std::atomic<int> sleepers_{0};
};

inline void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& fn) {
  ThreadPool::instance().parallel_for(n, fn);
}

}  // namespace rt
}  // namespace bloom
