// Admission-side host components (C++):
//
//   RateLimiter       per-model token buckets (capacity = burst, refill at rate
//                     tokens/s; off by default).  A request of n tokens either
//                     takes them or is told how long to wait.  Defaults follow
//                     the reference (token_scheduling/rate_limiter.rs: burst
//                     32768, 200 tokens/s, per-model overrides).
//   SegmentScheduler  request classes Foreground / Realtime / Background /
//                     Maintenance served by strict priority or weighted fair
//                     queueing (weights 4/3/2/1, round-robin start), with the
//                     batch limit reduced under thermal or power pressure
//                     (reference scheduler/mod.rs:1086-1449 BloomScheduler).
//   ResourceLedger    per-device memory budgets: reservations by owner with a
//                     priority; a reservation that does not fit evicts lower
//                     priority resident owners, oldest first (reference
//                     crates/core/src/vram.rs:22-584), sized here for 180 GB
//                     of HBM per GPU.
// Time is passed in by the caller (seconds), so behaviour is deterministic
// under test.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <deque>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace bloom {
namespace rt {

class RateLimiter {
 public:
  RateLimiter(bool enabled, double burst, double rate) : enabled_(enabled), burst_(burst), rate_(rate) {
    if (burst <= 0 || rate <= 0) throw std::invalid_argument("RateLimiter: burst and rate must be positive");
  }
  void set_override(const std::string& model, double burst, double rate) { overrides_[model] = {burst, rate}; }
  // (allowed, seconds to wait before n tokens are available)
  std::pair<bool, double> try_acquire(const std::string& model, double n, double now) {
    ++requests_;
    if (!enabled_) return {true, 0.0};
    Bucket& b = bucket(model, now);
    b.tokens = std::min(b.cap, b.tokens + (now - b.last) * b.rate);
    b.last = now;
    if (b.tokens >= n) {
      b.tokens -= n;
      return {true, 0.0};
    }
    ++throttled_;
    return {false, (n - b.tokens) / b.rate};
  }
  double available(const std::string& model, double now) {
    Bucket& b = bucket(model, now);
    return std::min(b.cap, b.tokens + (now - b.last) * b.rate);
  }
  int64_t requests() const { return requests_; }
  int64_t throttled() const { return throttled_; }

 private:
  struct Bucket {
    double tokens, cap, rate, last;
  };
  Bucket& bucket(const std::string& model, double now) {
    auto it = buckets_.find(model);
    if (it != buckets_.end()) return it->second;
    double cap = burst_, rate = rate_;
    auto o = overrides_.find(model);
    if (o != overrides_.end()) {
      cap = o->second.first;
      rate = o->second.second;
    }
    return buckets_.emplace(model, Bucket{cap, cap, rate, now}).first->second;
  }
  bool enabled_;
  double burst_, rate_;
  std::map<std::string, std::pair<double, double>> overrides_;
  std::map<std::string, Bucket> buckets_;
  int64_t requests_ = 0, throttled_ = 0;
};

class SegmentScheduler {
 public:
  // classes: 0 foreground interactive, 1 realtime stream, 2 background batch, 3 maintenance
  SegmentScheduler(int base_max_batch, bool wfq) : base_(base_max_batch), wfq_(wfq) {
    if (base_max_batch < 1) throw std::invalid_argument("SegmentScheduler: batch must be >= 1");
  }
  void submit(const std::string& id, int cls) {
    if (cls < 0 || cls > 3) throw std::invalid_argument("SegmentScheduler: class 0..3");
    q_[cls].push_back(id);
  }
  // thermal: 0 nominal, 1 fair, 2 serious, 3 critical; power: 0 external, 1 battery, 2 low battery
  void set_conditions(int thermal, int power) {
    thermal_ = thermal;
    power_ = power;
  }
  int effective_max_batch() const {
    int b = base_;
    if (thermal_ == 2) b = std::max(1, b / 2);
    if (thermal_ >= 3) b = 1;
    if (power_ == 1) b = std::max(1, (b * 3) / 4);
    if (power_ >= 2) b = std::max(1, b / 2);
    return b;
  }
  std::vector<std::pair<std::string, int>> next_batch() {
    std::vector<std::pair<std::string, int>> out;
    int room = effective_max_batch();
    if (!wfq_) {
      for (int c = 0; c < 4 && room > 0; ++c)
        while (room > 0 && !q_[c].empty()) take(c, out, room);
      return out;
    }
    static const int w[4] = {4, 3, 2, 1};
    const int start = static_cast<int>(rr_++ % 4);
    for (int k = 0; k < 4 && room > 0; ++k) {  // one weighted pass from a rotating start
      const int c = (start + k) % 4;
      for (int i = 0; i < w[c] && room > 0 && !q_[c].empty(); ++i) take(c, out, room);
    }
    for (int c = 0; c < 4 && room > 0; ++c)  // leftover room: work-conserving
      while (room > 0 && !q_[c].empty()) take(c, out, room);
    return out;
  }
  std::vector<int> depths() const { return {int(q_[0].size()), int(q_[1].size()), int(q_[2].size()), int(q_[3].size())}; }

 private:
  void take(int c, std::vector<std::pair<std::string, int>>& out, int& room) {
    out.emplace_back(q_[c].front(), c);
    q_[c].pop_front();
    --room;
  }
  int base_;
  bool wfq_;
  int thermal_ = 0, power_ = 0;
  uint64_t rr_ = 0;
  std::deque<std::string> q_[4];
};

class ResourceLedger {
 public:
  void add_device(int device, int64_t capacity_bytes) { cap_[device] = capacity_bytes; }
  // Returns (ok, evicted owners).  Priority: higher value is more important.
  std::pair<bool, std::vector<std::string>> reserve(const std::string& owner, int device, int64_t bytes, int priority,
                                                    int64_t stamp) {
    auto c = cap_.find(device);
    if (c == cap_.end()) throw std::invalid_argument("ResourceLedger: unknown device");
    std::vector<std::string> evicted;
    if (bytes > c->second) return {false, evicted};
    auto used = [&] {
      int64_t u = 0;
      for (auto& r : res_)
        if (r.second.device == device) u += r.second.bytes;
      return u;
    };
    while (used() + bytes > c->second) {
      // victim: lowest priority, then oldest, among owners less important than the request
      const Res* v = nullptr;
      std::string vk;
      for (auto& r : res_) {
        if (r.second.device != device || r.second.priority >= priority) continue;
        if (v == nullptr || r.second.priority < v->priority ||
            (r.second.priority == v->priority && r.second.stamp < v->stamp)) {
          v = &r.second;
          vk = r.first;
        }
      }
      if (v == nullptr) return {false, {}};
      evicted.push_back(vk);
      res_.erase(vk);
    }
    res_[owner] = Res{device, bytes, priority, stamp};
    return {true, evicted};
  }
  bool release(const std::string& owner) { return res_.erase(owner) > 0; }
  int64_t used(int device) const {
    int64_t u = 0;
    for (auto& r : res_)
      if (r.second.device == device) u += r.second.bytes;
    return u;
  }
  int64_t free_bytes(int device) const {
    auto c = cap_.find(device);
    return c == cap_.end() ? 0 : c->second - used(device);
  }

 private:
  struct Res {
    int device;
    int64_t bytes;
    int priority;
    int64_t stamp;
  };
  std::map<int, int64_t> cap_;
  std::map<std::string, Res> res_;
};

}  // namespace rt
}  // namespace bloom

void register_admission(py::module_& m) {
  using namespace bloom::rt;
  py::class_<RateLimiter>(m, "RateLimiter")
      .def(py::init<bool, double, double>(), py::arg("enabled") = false, py::arg("burst") = 32768.0,
           py::arg("rate_per_second") = 200.0)
      .def("set_override", &RateLimiter::set_override)
      .def("try_acquire", &RateLimiter::try_acquire)
      .def("available", &RateLimiter::available)
      .def_property_readonly("requests", &RateLimiter::requests)
      .def_property_readonly("throttled", &RateLimiter::throttled);
  py::class_<SegmentScheduler>(m, "SegmentScheduler")
      .def(py::init<int, bool>(), py::arg("base_max_batch"), py::arg("weighted_fair") = true)
      .def("submit", &SegmentScheduler::submit)
      .def("set_conditions", &SegmentScheduler::set_conditions, py::arg("thermal"), py::arg("power"))
      .def("effective_max_batch", &SegmentScheduler::effective_max_batch)
      .def("next_batch", &SegmentScheduler::next_batch)
      .def("depths", &SegmentScheduler::depths);
  py::class_<ResourceLedger>(m, "ResourceLedger")
      .def(py::init<>())
      .def("add_device", &ResourceLedger::add_device)
      .def("reserve", &ResourceLedger::reserve, py::arg("owner"), py::arg("device"), py::arg("bytes"),
           py::arg("priority"), py::arg("stamp"))
      .def("release", &ResourceLedger::release)
      .def("used", &ResourceLedger::used)
      .def("free_bytes", &ResourceLedger::free_bytes);
}
