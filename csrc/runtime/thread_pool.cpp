#include "thread_pool.h"

#include <cstdlib>

namespace bloom {
namespace rt {

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
    const std::function<void(int64_t, int64_t)>* job;
    int64_t n;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return stop_ || generation_ != seen; });
      if (stop_) return;
      seen = generation_;
      job = job_;
      n = job_n_;
    }
    const int parts = size();
    const int64_t chunk = (n + parts - 1) / parts;
    const int64_t b = std::min<int64_t>(n, (idx + 1) * chunk), e = std::min<int64_t>(n, b + chunk);
    if (b < e) (*job)(b, e);
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }
}

void ThreadPool::parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& fn) {
  if (n <= 0) return;
  if (workers_.empty() || n == 1) {
    fn(0, n);
    return;
  }
  {
    std::lock_guard<std::mutex> lk(mu_);
    job_ = &fn;
    job_n_ = n;
    pending_ = static_cast<int>(workers_.size());
    ++generation_;
  }
  cv_.notify_all();
  const int64_t chunk = (n + size() - 1) / size();
  fn(0, std::min<int64_t>(n, chunk));  // calling thread takes the first chunk
  std::unique_lock<std::mutex> lk(mu_);
  done_cv_.wait(lk, [&] { return pending_ == 0; });
  job_ = nullptr;
}

}  // namespace rt
}  // namespace bloom
