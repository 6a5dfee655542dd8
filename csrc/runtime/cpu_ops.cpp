// CPU kernels for GGUF block-quantised weights (host path for small models on
// machines without a GPU, and the oracle for the GPU dequant kernels).
//
// Block formats (GGUF / ggml, 32 elements per block):
//   Q8_0: fp16 scale d, 32 x int8 q          -> x = d * q            (34 bytes)
//   Q4_0: fp16 scale d, 16 bytes of nibbles  -> x = d * (nibble - 8) (18 bytes)
//         element j (< 16) is the low nibble of byte j, element j + 16 the high one.
//
// Q8_0 x Q8_0 dot products follow the usual scheme of quantising the
// activation row to Q8_0 on the fly and accumulating int8 products per block
// (AVX2 maddubs), matching the reference's Candle CPU quantized matmul
// (crates/engine/src/executor/candle.rs:1533-1568, candle quantized_llama).
#include <immintrin.h>
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include <cmath>
#include <cstring>

#include "thread_pool.h"

namespace py = pybind11;
using bloom::rt::parallel_for;

namespace {

inline float fp16_to_f32(uint16_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal
      exp = 127 - 15 + 1;
      while ((man & 0x400u) == 0) {
        man <<= 1;
        --exp;
      }
      man &= 0x3FFu;
      bits = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t f32_to_fp16(float f) {
  // round-to-nearest-even conversion
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  int32_t exp = static_cast<int32_t>((x >> 23) & 0xFFu) - 127 + 15;
  uint32_t man = x & 0x7FFFFFu;
  if (((x >> 23) & 0xFFu) == 0xFFu) return static_cast<uint16_t>(sign | 0x7C00u | (man ? 0x200u : 0u));
  if (exp >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
  if (exp <= 0) {
    if (exp < -10) return static_cast<uint16_t>(sign);
    man |= 0x800000u;
    const int shift = 14 - exp;
    uint32_t h = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return static_cast<uint16_t>(sign | h);
  }
  uint32_t h = (static_cast<uint32_t>(exp) << 10) | (man >> 13);
  const uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return static_cast<uint16_t>(sign | h);
}

constexpr int QK = 32;
constexpr int Q8_BYTES = 34;
constexpr int Q4_BYTES = 18;

torch::Tensor dequant_q8_0(const torch::Tensor& raw, int64_t n) {
  TORCH_CHECK(raw.scalar_type() == at::kByte && raw.is_contiguous(), "raw must be uint8");
  TORCH_CHECK(n % QK == 0 && raw.numel() >= n / QK * Q8_BYTES, "q8_0: size mismatch");
  auto out = torch::empty({n}, torch::kFloat);
  const uint8_t* p = raw.data_ptr<uint8_t>();
  float* o = out.data_ptr<float>();
  const int64_t nb = n / QK;
  parallel_for(nb, [&](int64_t b0, int64_t b1) {
  for (int64_t b = b0; b < b1; ++b) {
    const uint8_t* blk = p + b * Q8_BYTES;
    uint16_t hd;
    std::memcpy(&hd, blk, 2);
    const float d = fp16_to_f32(hd);
    const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
    for (int j = 0; j < QK; ++j) o[b * QK + j] = d * q[j];
  }
  });
  return out;
}

torch::Tensor dequant_q4_0(const torch::Tensor& raw, int64_t n) {
  TORCH_CHECK(raw.scalar_type() == at::kByte && raw.is_contiguous(), "raw must be uint8");
  TORCH_CHECK(n % QK == 0 && raw.numel() >= n / QK * Q4_BYTES, "q4_0: size mismatch");
  auto out = torch::empty({n}, torch::kFloat);
  const uint8_t* p = raw.data_ptr<uint8_t>();
  float* o = out.data_ptr<float>();
  const int64_t nb = n / QK;
  parallel_for(nb, [&](int64_t b0, int64_t b1) {
  for (int64_t b = b0; b < b1; ++b) {
    const uint8_t* blk = p + b * Q4_BYTES;
    uint16_t hd;
    std::memcpy(&hd, blk, 2);
    const float d = fp16_to_f32(hd);
    const uint8_t* q = blk + 2;
    for (int j = 0; j < 16; ++j) {
      o[b * QK + j] = d * (static_cast<int>(q[j] & 0x0F) - 8);
      o[b * QK + j + 16] = d * (static_cast<int>(q[j] >> 4) - 8);
    }
  }
  });
  return out;
}

// Quantise f32 values to Q8_0 blocks (round half away from zero, d = amax / 127).
void quantize_row_q8_0(const float* x, uint8_t* out, int64_t n) {
  for (int64_t b = 0; b < n / QK; ++b) {
    const float* xb = x + b * QK;
    float amax = 0.f;
    for (int j = 0; j < QK; ++j) amax = std::max(amax, std::fabs(xb[j]));
    const float d = amax / 127.f;
    const float id = d != 0.f ? 1.f / d : 0.f;
    uint8_t* blk = out + b * Q8_BYTES;
    const uint16_t hd = f32_to_fp16(d);
    std::memcpy(blk, &hd, 2);
    int8_t* q = reinterpret_cast<int8_t*>(blk + 2);
    for (int j = 0; j < QK; ++j) q[j] = static_cast<int8_t>(std::lround(xb[j] * id));
  }
}

torch::Tensor quantize_q8_0(const torch::Tensor& x) {
  auto xc = x.to(torch::kFloat).contiguous();
  const int64_t n = xc.numel();
  TORCH_CHECK(n % QK == 0, "quantize_q8_0: size must be a multiple of 32");
  auto out = torch::empty({n / QK * Q8_BYTES}, torch::kByte);
  const int64_t nb = n / QK;
  const float* src = xc.data_ptr<float>();
  uint8_t* dst = out.data_ptr<uint8_t>();
  parallel_for(nb, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) quantize_row_q8_0(src + b * QK, dst + b * Q8_BYTES, QK);
  });
  return out;
}

torch::Tensor quantize_q4_0(const torch::Tensor& x) {
  auto xc = x.to(torch::kFloat).contiguous();
  const int64_t n = xc.numel();
  TORCH_CHECK(n % QK == 0, "quantize_q4_0: size must be a multiple of 32");
  auto out = torch::empty({n / QK * Q4_BYTES}, torch::kByte);
  const float* src = xc.data_ptr<float>();
  uint8_t* dst = out.data_ptr<uint8_t>();
  const int64_t nb = n / QK;
  parallel_for(nb, [&](int64_t b0, int64_t b1) {
  for (int64_t b = b0; b < b1; ++b) {
    const float* xb = src + b * QK;
    // scale from the signed value of largest magnitude: x = d * (q - 8), q in [0, 15]
    float amax = 0.f, mx = 0.f;
    for (int j = 0; j < QK; ++j)
      if (std::fabs(xb[j]) > amax) {
        amax = std::fabs(xb[j]);
        mx = xb[j];
      }
    const float d = mx / -8.f;
    const float id = d != 0.f ? 1.f / d : 0.f;
    uint8_t* blk = dst + b * Q4_BYTES;
    const uint16_t hd = f32_to_fp16(d);
    std::memcpy(blk, &hd, 2);
    for (int j = 0; j < 16; ++j) {
      const int q0 = std::min(15, static_cast<int>(xb[j] * id + 8.5f));
      const int q1 = std::min(15, static_cast<int>(xb[j + 16] * id + 8.5f));
      blk[2 + j] = static_cast<uint8_t>(std::max(0, q0) | (std::max(0, q1) << 4));
    }
  }
  });
  return out;
}

// int8 dot of one Q8_0 block pair, AVX2
inline float dot_q8_block(const uint8_t* a, const uint8_t* b) {
  uint16_t ha, hb;
  std::memcpy(&ha, a, 2);
  std::memcpy(&hb, b, 2);
  const __m256i qa = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(a + 2));
  const __m256i qb = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(b + 2));
  // sign trick: |a| * sign(b, a)
  const __m256i ax = _mm256_sign_epi8(qa, qa);
  const __m256i sy = _mm256_sign_epi8(qb, qa);
  const __m256i dot16 = _mm256_maddubs_epi16(ax, sy);
  const __m256i dot32 = _mm256_madd_epi16(dot16, _mm256_set1_epi16(1));
  __m128i s = _mm_add_epi32(_mm256_castsi256_si128(dot32), _mm256_extracti128_si256(dot32, 1));
  s = _mm_hadd_epi32(s, s);
  s = _mm_hadd_epi32(s, s);
  return fp16_to_f32(ha) * fp16_to_f32(hb) * static_cast<float>(_mm_cvtsi128_si32(s));
}

// y[M, N] = x[M, K] (f32, quantised to Q8_0 per row) . W[N, K] (Q8_0 raw rows)^T
torch::Tensor q8_0_matmul(const torch::Tensor& x, const torch::Tensor& wraw, int64_t N, int64_t K) {
  TORCH_CHECK(K % QK == 0, "q8_0_matmul: K must be a multiple of 32");
  TORCH_CHECK(wraw.scalar_type() == at::kByte && wraw.is_contiguous() && wraw.numel() >= N * (K / QK) * Q8_BYTES,
              "q8_0_matmul: weight bytes");
  auto xc = x.to(torch::kFloat).contiguous().view({-1, K});
  const int64_t M = xc.size(0);
  const int64_t kb = K / QK;
  std::vector<uint8_t> xq(static_cast<size_t>(M * kb * Q8_BYTES));
  for (int64_t m = 0; m < M; ++m) quantize_row_q8_0(xc.data_ptr<float>() + m * K, xq.data() + m * kb * Q8_BYTES, K);
  auto y = torch::empty({M, N}, torch::kFloat);
  float* yp = y.data_ptr<float>();
  const uint8_t* w = wraw.data_ptr<uint8_t>();
  auto rows = [&](int64_t n0, int64_t n1) {
  for (int64_t n = n0; n < n1; ++n) {
    const uint8_t* wr = w + n * kb * Q8_BYTES;
    for (int64_t m = 0; m < M; ++m) {
      const uint8_t* xr = xq.data() + m * kb * Q8_BYTES;
      float acc = 0.f;
      for (int64_t b = 0; b < kb; ++b) acc += dot_q8_block(wr + b * Q8_BYTES, xr + b * Q8_BYTES);
      yp[m * N + n] = acc;
    }
  }
  };
  // below ~256 KB of weights one core finishes before a dispatch pays off
  if (N * K * M < (int64_t(1) << 18))
    rows(0, N);
  else
    parallel_for(N, rows);
  return y;
}

// Multimodal rotary embedding on the host (the CPU counterpart of
// csrc/kernels/mrope.cu; reference: crates/tilelang/scripts/generate_kernel.py:
// 264-338).  x [B, H, S, D] f32, cos / sin [3, B, S, D] f32; the half
// dimension is cut into sections (s0, s1, s2) taken from the temporal, height
// and width position planes; rotate-half pairs channel c with c + D/2.
torch::Tensor mrope_cpu(const torch::Tensor& x, const torch::Tensor& cos, const torch::Tensor& sin, int64_t s0,
                        int64_t s1, int64_t s2) {
  TORCH_CHECK(x.dim() == 4 && x.scalar_type() == at::kFloat, "mrope_cpu: x f32 [B, H, S, D]");
  const int64_t B = x.size(0), H = x.size(1), S = x.size(2), D = x.size(3), half = D / 2;
  TORCH_CHECK(D % 2 == 0 && s0 >= 0 && s1 >= 0 && s2 >= 0 && s0 + s1 + s2 == half, "mrope_cpu: sections");
  TORCH_CHECK(cos.scalar_type() == at::kFloat && cos.dim() == 4 && cos.size(0) == 3 && cos.size(1) == B &&
                  cos.size(2) == S && cos.size(3) == D && sin.sizes() == cos.sizes(),
              "mrope_cpu: cos / sin f32 [3, B, S, D]");
  const torch::Tensor xc = x.contiguous(), cc = cos.contiguous(), sc = sin.contiguous();
  torch::Tensor out = torch::empty_like(xc);
  const float* xp = xc.data_ptr<float>();
  const float* cp = cc.data_ptr<float>();
  const float* sp = sc.data_ptr<float>();
  float* op = out.data_ptr<float>();
  const int64_t plane = B * S * D;
  for (int64_t b = 0; b < B; ++b)
    for (int64_t h = 0; h < H; ++h)
      for (int64_t s = 0; s < S; ++s) {
        const float* xr = xp + ((b * H + h) * S + s) * D;
        float* orow = op + ((b * H + h) * S + s) * D;
        for (int64_t c = 0; c < half; ++c) {
          const int64_t comp = c < s0 ? 0 : (c < s0 + s1 ? 1 : 2);
          const int64_t cb = comp * plane + (b * S + s) * D;
          orow[c] = xr[c] * cp[cb + c] - xr[c + half] * sp[cb + c];
          orow[c + half] = xr[c + half] * cp[cb + c + half] + xr[c] * sp[cb + c + half];
        }
      }
  return out;
}

// Small host kernels kept as CPU oracles (the reference generates them as
// TileLang C++: crates/tilelang/scripts/generate_kernel.py:7-102): elementwise
// add, row-major matmul, softmax of a vector, and single-head attention with
// an online (running max / running sum) softmax.
torch::Tensor oracle_vector_add(const torch::Tensor& a, const torch::Tensor& b) {
  TORCH_CHECK(a.scalar_type() == at::kFloat && b.scalar_type() == at::kFloat && a.numel() == b.numel(),
              "vector_add: two f32 tensors of one size");
  const torch::Tensor ac = a.contiguous(), bc = b.contiguous();
  torch::Tensor c = torch::empty_like(ac);
  const float* pa = ac.data_ptr<float>();
  const float* pb = bc.data_ptr<float>();
  float* pc = c.data_ptr<float>();
  for (int64_t i = 0; i < ac.numel(); ++i) pc[i] = pa[i] + pb[i];
  return c;
}

torch::Tensor oracle_matmul(const torch::Tensor& a, const torch::Tensor& b) {
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(0) && a.scalar_type() == at::kFloat &&
                  b.scalar_type() == at::kFloat,
              "matmul: f32 [m, k] @ [k, n]");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(1);
  const torch::Tensor ac = a.contiguous(), bc = b.contiguous();
  torch::Tensor c = torch::zeros({M, N}, a.options());
  const float* pa = ac.data_ptr<float>();
  const float* pb = bc.data_ptr<float>();
  float* pc = c.data_ptr<float>();
  for (int64_t i = 0; i < M; ++i)
    for (int64_t k = 0; k < K; ++k) {
      const float x = pa[i * K + k];
      for (int64_t j = 0; j < N; ++j) pc[i * N + j] += x * pb[k * N + j];
    }
  return c;
}

torch::Tensor oracle_softmax(const torch::Tensor& x) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.numel() > 0, "softmax: non-empty f32");
  const torch::Tensor xc = x.contiguous();
  torch::Tensor y = torch::empty_like(xc);
  const float* px = xc.data_ptr<float>();
  float* py = y.data_ptr<float>();
  const int64_t n = xc.numel();
  float mx = px[0];
  for (int64_t i = 1; i < n; ++i) mx = std::max(mx, px[i]);
  double sum = 0.0;
  for (int64_t i = 0; i < n; ++i) sum += std::exp(static_cast<double>(px[i] - mx));
  for (int64_t i = 0; i < n; ++i) py[i] = static_cast<float>(std::exp(static_cast<double>(px[i] - mx)) / sum);
  return y;
}

torch::Tensor oracle_attention(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v) {
  TORCH_CHECK(q.dim() == 2 && k.sizes() == q.sizes() && v.sizes() == q.sizes() && q.scalar_type() == at::kFloat,
              "attention: f32 q, k, v [seq, head_dim]");
  const int64_t S = q.size(0), D = q.size(1);
  const torch::Tensor qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
  torch::Tensor o = torch::zeros_like(qc);
  const float* pq = qc.data_ptr<float>();
  const float* pk = kc.data_ptr<float>();
  const float* pv = vc.data_ptr<float>();
  float* po = o.data_ptr<float>();
  const float scale = 1.0f / std::sqrt(static_cast<float>(D));
  for (int64_t r = 0; r < S; ++r) {
    float m = -INFINITY, l = 0.f;
    float* orow = po + r * D;
    for (int64_t j = 0; j < S; ++j) {
      float dot = 0.f;
      for (int64_t d = 0; d < D; ++d) dot += pq[r * D + d] * pk[j * D + d];
      const float s = dot * scale;
      const float mn = std::max(m, s);
      const float alpha = std::exp(m - mn);  // rescales what was accumulated under the old max
      const float p = std::exp(s - mn);
      l = l * alpha + p;
      for (int64_t d = 0; d < D; ++d) orow[d] = orow[d] * alpha + p * pv[j * D + d];
      m = mn;
    }
    for (int64_t d = 0; d < D; ++d) orow[d] /= l;
  }
  return o;
}

}  // namespace

void register_cpu_ops(py::module_& m) {
  m.def("oracle_vector_add", &oracle_vector_add, "c = a + b (f32, host)");
  m.def("oracle_matmul", &oracle_matmul, "c = a @ b (f32 row-major, host)");
  m.def("oracle_softmax", &oracle_softmax, "softmax of a f32 vector (host)");
  m.def("oracle_attention", &oracle_attention, "single-head attention with online softmax (f32, host)");
  m.def("mrope_cpu", &mrope_cpu, "multimodal rotary embedding of x [B,H,S,D] (f32, host)");
  m.def("dequant_q8_0", &dequant_q8_0, "GGUF Q8_0 blocks -> f32");
  m.def("dequant_q4_0", &dequant_q4_0, "GGUF Q4_0 blocks -> f32");
  m.def("quantize_q8_0", &quantize_q8_0, "f32 -> GGUF Q8_0 blocks");
  m.def("quantize_q4_0", &quantize_q4_0, "f32 -> GGUF Q4_0 blocks");
  m.def("q8_0_matmul", &q8_0_matmul, "x f32 [M,K] @ Q8_0 W[N,K]^T -> f32 [M,N] (AVX2)");
  m.def("set_num_threads", [](int n) { bloom::rt::ThreadPool::instance().resize(n); });
}
