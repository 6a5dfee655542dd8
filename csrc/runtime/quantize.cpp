// Offline weight quantisers behind the bloom_quantize CLI (CPU, thread pool).
//
//   rtn_int8   per-row symmetric: scale = max|w| / 127, q = round(w / scale) + 128 (u8)
//   rtn_int4   per-group asymmetric (group g along the row): scale = (max - min) / 15,
//              zero = min, q = clamp(round((w - zero) / scale), 0, 15) (one u8 per value)
//   awq_int4   activation-aware variant without calibration data: every input
//              column gets a scale s_j = (mean |w_.j|)^0.5 normalised to geometric
//              mean 1 (large-magnitude columns, a proxy for salient activations,
//              are scaled up before rounding and keep more precision), the scaled
//              weight is quantised as rtn_int4, and the per-column scales are
//              stored so the loader divides them back out.
//
// Output tensor names follow the reference quantiser (crates/engine/src/bin/
// bloom_quantize.rs): <name>.qweight, <name>.scales, <name>.zeros, which keeps
// its output loadable by the same consumers; the arithmetic is this file's.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <algorithm>
#include <cmath>

#include "thread_pool.h"

namespace {

using bloom::rt::ThreadPool;

py::tuple rtn_int8(const torch::Tensor& w_in) {
  TORCH_CHECK(w_in.dim() == 2, "rtn_int8: 2-D weight");
  const torch::Tensor w = w_in.to(torch::kFloat).contiguous();
  const int64_t R = w.size(0), C = w.size(1);
  auto q = torch::empty({R, C}, torch::kUInt8);
  auto s = torch::empty({R, 1}, torch::kFloat);
  const float* wp = w.data_ptr<float>();
  uint8_t* qp = q.data_ptr<uint8_t>();
  float* sp = s.data_ptr<float>();
  ThreadPool::instance().parallel_for(R, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      const float* row = wp + r * C;
      float mx = 0.f;
      for (int64_t c = 0; c < C; ++c) mx = std::max(mx, std::fabs(row[c]));
      const float scale = std::max(mx / 127.f, 1e-8f);
      sp[r] = scale;
      for (int64_t c = 0; c < C; ++c) {
        const float v = std::nearbyint(row[c] / scale);
        qp[r * C + c] = static_cast<uint8_t>(std::clamp(v, -127.f, 127.f) + 128.f);
      }
    }
  });
  return py::make_tuple(q, s);
}

py::tuple rtn_int4(const torch::Tensor& w_in, int64_t group) {
  TORCH_CHECK(w_in.dim() == 2 && group > 0 && w_in.size(1) % group == 0, "rtn_int4: columns must divide by group");
  const torch::Tensor w = w_in.to(torch::kFloat).contiguous();
  const int64_t R = w.size(0), C = w.size(1), G = C / group;
  auto q = torch::empty({R, C}, torch::kUInt8);
  auto s = torch::empty({R, G}, torch::kFloat);
  auto z = torch::empty({R, G}, torch::kFloat);
  const float* wp = w.data_ptr<float>();
  uint8_t* qp = q.data_ptr<uint8_t>();
  float* sp = s.data_ptr<float>();
  float* zp = z.data_ptr<float>();
  ThreadPool::instance().parallel_for(R, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r)
      for (int64_t g = 0; g < G; ++g) {
        const float* x = wp + r * C + g * group;
        float lo = x[0], hi = x[0];
        for (int64_t j = 1; j < group; ++j) {
          lo = std::min(lo, x[j]);
          hi = std::max(hi, x[j]);
        }
        const float scale = std::max((hi - lo) / 15.f, 1e-8f);
        sp[r * G + g] = scale;
        zp[r * G + g] = lo;
        for (int64_t j = 0; j < group; ++j)
          qp[r * C + g * group + j] = static_cast<uint8_t>(std::clamp(std::nearbyint((x[j] - lo) / scale), 0.f, 15.f));
      }
  });
  return py::make_tuple(q, s, z);
}

py::tuple awq_int4(const torch::Tensor& w_in, int64_t group) {
  const torch::Tensor w = w_in.to(torch::kFloat).contiguous();
  auto col = w.abs().mean(0).clamp_min(1e-8).sqrt();            // [C]
  col = col / torch::exp(torch::log(col).mean());                 // geometric mean 1
  auto t = rtn_int4(w * col.unsqueeze(0), group);
  return py::make_tuple(t[0], t[1], t[2], col);
}

torch::Tensor dequant_int8(const torch::Tensor& q, const torch::Tensor& s) {
  return (q.to(torch::kFloat) - 128.f) * s.to(torch::kFloat);
}

torch::Tensor dequant_int4(const torch::Tensor& q, const torch::Tensor& s, const torch::Tensor& z, int64_t group,
                           const c10::optional<torch::Tensor>& col_scale) {
  const int64_t R = q.size(0), C = q.size(1);
  auto w = q.to(torch::kFloat).view({R, C / group, group}) * s.to(torch::kFloat).unsqueeze(2) +
           z.to(torch::kFloat).unsqueeze(2);
  w = w.view({R, C});
  if (col_scale.has_value() && col_scale->defined()) w = w / col_scale->to(torch::kFloat).unsqueeze(0);
  return w;
}

}  // namespace

void register_quantize(py::module_& m) {
  m.def("quantize_rtn_int8", &rtn_int8, "per-row symmetric int8 -> (q u8, scales)");
  m.def("quantize_rtn_int4", &rtn_int4, py::arg("w"), py::arg("group_size") = 128,
        "per-group asymmetric int4 -> (q u8, scales, zeros)");
  m.def("quantize_awq_int4", &awq_int4, py::arg("w"), py::arg("group_size") = 128,
        "column-scaled int4 -> (q u8, scales, zeros, column scales)");
  m.def("dequant_rtn_int8", &dequant_int8);
  m.def("dequant_int4", &dequant_int4, py::arg("q"), py::arg("scales"), py::arg("zeros"), py::arg("group_size"),
        py::arg("col_scale") = py::none());
}
