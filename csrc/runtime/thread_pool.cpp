#include "thread_pool.h"

#include <chrono>
#include <cstdlib>

namespace bloom {
namespace rt {

namespace {
constexpr auto kSpin = std::chrono::microseconds(200);  // busy-wait for the next job before sleeping
inline void cpu_relax() {
#if defined(__x86_64__)
  __builtin_ia32_pause();
#endif
}
}  // namespace

ThreadPool::ThreadPool() {
  int n = static_cast<int>(std::thread::hardware_concurrency());
  if (const char* e = std::getenv("BLOOM_CPU_THREADS")) n = std::atoi(e);
  start_workers(std::max(1, n) - 1);
}

ThreadPool::~ThreadPool() { stop_workers(); }

void ThreadPool::start_workers(int n) {
  stop_ = false;
  for (int i = 0; i < n; ++i) workers_.emplace_back([this, i] { worker_loop(i); });
}

void ThreadPool::stop_workers() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  for (auto& t : workers_) t.join();
  workers_.clear();
}

void ThreadPool::resize(int n) {
  stop_workers();
  start_workers(std::max(1, n) - 1);
}

void ThreadPool::worker_loop(int idx) {
  int64_t seen = 0;
  for (;;) {
    // spin briefly, then sleep until a new generation (or stop) is published
    const auto t0 = std::chrono::steady_clock::now();
    while (generation_.load(std::memory_order_acquire) == seen && !stop_.load(std::memory_order_relaxed)) {
      if (std::chrono::steady_clock::now() - t0 > kSpin) {
        std::unique_lock<std::mutex> lk(mu_);
        ++sleepers_;
        cv_.wait(lk, [&] { return stop_.load() || generation_.load() != seen; });
        --sleepers_;
        break;
      }
      cpu_relax();
    }
    if (stop_.load()) return;
    seen = generation_.load(std::memory_order_acquire);
    const std::function<void(int64_t, int64_t)>* job = job_;
    const int64_t n = job_n_;
    const int parts = size();
    const int64_t chunk = (n + parts - 1) / parts;
    const int64_t b = std::min<int64_t>(n, (idx + 1) * chunk), e = std::min<int64_t>(n, b + chunk);
    if (b < e) (*job)(b, e);
    pending_.fetch_sub(1, std::memory_order_acq_rel);
  }
}

void ThreadPool::parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& fn) {
  if (n <= 0) return;
  if (workers_.empty() || n == 1) {
    fn(0, n);
    return;
  }
  job_ = &fn;
  job_n_ = n;
  pending_.store(static_cast<int>(workers_.size()), std::memory_order_relaxed);
  {
    std::lock_guard<std::mutex> lk(mu_);  // orders the job fields before the generation bump for sleepers
    generation_.fetch_add(1, std::memory_order_acq_rel);
  }
  if (sleepers_.load() > 0) cv_.notify_all();
  const int64_t chunk = (n + size() - 1) / size();
  fn(0, std::min<int64_t>(n, chunk));  // calling thread takes the first chunk
  while (pending_.load(std::memory_order_acquire) != 0) cpu_relax();
  job_ = nullptr;
}

}  // namespace rt
}  // namespace bloom
