// Token sampling on the GPU.
//
// Greedy: per-row argmax (lowest index wins ties).
// Stochastic: temperature, top-k and top-p (nucleus) per row.  The kept set
// is found by a two-level histogram selection on an integer key of the
// scaled logit distance to the maximum (see sample_kernel), then one token
// is drawn from the renormalised kept distribution by inverse CDF.  Uniforms come from
// Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3",
// SC'11), keyed by the request seed and counted by the step offset, so a
// request's stream is reproducible and independent of batch position.
//
// Reference behaviour: host sampler executor/batch_executor.rs:932-1022
// (temperature, top-p, seeded PRNG) and candle LogitsProcessor
// (executor/candle.rs:2199-2203).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {
namespace {

constexpr int kThreads = 1024;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

__device__ __forceinline__ void argmax_combine(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

template <typename T>
__device__ void block_argmax(const T* row, int V, float& best_v, int& best_i) {
  __shared__ float sv[32];
  __shared__ int si[32];
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int k = threadIdx.x; k < V; k += blockDim.x) argmax_combine(v, idx, to_f(row[k]), k);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    argmax_combine(v, idx, v2, i2);
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = v;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    v = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    idx = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
      argmax_combine(v, idx, v2, i2);
    }
    if (threadIdx.x == 0) {
      sv[0] = v;
      si[0] = idx;
    }
  }
  __syncthreads();
  best_v = sv[0];
  best_i = si[0];
  __syncthreads();
}

template <typename T>
__global__ void argmax_kernel(const T* __restrict__ logits, long ld, int V, int* __restrict__ out) {
  float v;
  int i;
  block_argmax(logits + blockIdx.x * ld, V, v, i);
  if (threadIdx.x == 0) out[blockIdx.x] = i;
}

// ---- Philox4x32-10
struct U4 {
  uint32_t x, y, z, w;
};
__device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += W0;
    k1 += W1;
  }
  return c;
}
// uniform in (0, 1)
__device__ __forceinline__ float u01(uint32_t r) { return (float(r >> 8) + 0.5f) * (1.0f / 16777216.0f); }

// ---- stochastic sampling by two-level histogram selection
//
// Every logit l of a row gets an integer key = floor((mx - l) / t * 2^22 / 60)
// (0 = the maximum; logits more than 60 t below the maximum carry < e^-60 of
// the mass and get no key) and a fixed-point mass round(exp((l - mx) / t) *
// 2^32).  The kept set of top-k / top-p is a key prefix [0, key_cut]: a
// 2048-bin histogram of the key's high 11 bits (counts and masses) locates the
// bin holding the cut, a second histogram of the low 11 bits inside that bin
// locates the cut key.  The token is then drawn by inverse CDF over the
// kept keys (key order, then index order) from one Philox uniform: the same
// two histograms locate the key, an ordered pass over the row the token.
// Masses are summed as 64-bit integers, so every sum is exact and independent
// of the order of the atomic adds: a seed reproduces its tokens.  Cost: 4-6
// passes over the row and no per-token random numbers.
constexpr int kHistBins = 2048;
constexpr int kKeyBits = 22;
constexpr float kURange = 60.f;
constexpr float kKeyScale = float(1 << kKeyBits) / kURange;

struct HistSmem {
  unsigned int cnt1[kHistBins];
  unsigned long long mass1[kHistBins];
  unsigned int cnt2[kHistBins];
  unsigned long long mass2[kHistBins];
  unsigned long long wsum[32];
  unsigned int wcnt[32];
  int found;
};

__device__ __forceinline__ int key_of(float l, float mx, float inv_t) {
  const float u = (mx - l) * inv_t;
  if (!(u < kURange)) return -1;
  return min(int(u * kKeyScale), (1 << kKeyBits) - 1);
}
__device__ __forceinline__ unsigned long long mass_of(float l, float mx, float inv_t) {
  return static_cast<unsigned long long>(__expf((l - mx) * inv_t) * 4294967296.f);
}

// In-place inclusive scan of cnt[kHistBins] and mass[kHistBins] (blockDim = 1024, 2 bins per thread).
__device__ void hist_scan(unsigned int* cnt, unsigned long long* mass, HistSmem& sm) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int b0 = 2 * t;
  unsigned int c0 = cnt[b0], c1 = cnt[b0 + 1];
  unsigned long long m0 = mass[b0], m1 = mass[b0 + 1];
  unsigned int c = c0 + c1;
  unsigned long long m = m0 + m1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned int c2 = __shfl_up_sync(0xffffffffu, c, o);
    const unsigned long long m2 = __shfl_up_sync(0xffffffffu, m, o);
    if (lane >= o) {
      c += c2;
      m += m2;
    }
  }
  if (lane == 31) {
    sm.wcnt[w] = c;
    sm.wsum[w] = m;
  }
  __syncthreads();
  if (w == 0) {
    unsigned int cc = sm.wcnt[lane];
    unsigned long long mm = sm.wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned int c2 = __shfl_up_sync(0xffffffffu, cc, o);
      const unsigned long long m2 = __shfl_up_sync(0xffffffffu, mm, o);
      if (lane >= o) {
        cc += c2;
        mm += m2;
      }
    }
    sm.wcnt[lane] = cc;
    sm.wsum[lane] = mm;
  }
  __syncthreads();
  const unsigned int cbase = (w ? sm.wcnt[w - 1] : 0u) + c - (c0 + c1);
  const unsigned long long mbase = (w ? sm.wsum[w - 1] : 0ull) + m - (m0 + m1);
  cnt[b0] = cbase + c0;
  cnt[b0 + 1] = cbase + c0 + c1;
  mass[b0] = mbase + m0;
  mass[b0 + 1] = mbase + m0 + m1;
  __syncthreads();
}

// First bin whose inclusive count (by_count) or mass reaches `target` (after adding `base`).
__device__ int hist_find(const unsigned int* cnt, const unsigned long long* mass, bool by_count,
                         unsigned long long base, unsigned long long target, HistSmem& sm) {
  if (threadIdx.x == 0) sm.found = kHistBins - 1;
  __syncthreads();
  for (int b = threadIdx.x; b < kHistBins; b += blockDim.x) {
    const unsigned long long v = base + (by_count ? static_cast<unsigned long long>(cnt[b]) : mass[b]);
    const unsigned long long prev = b ? base + (by_count ? static_cast<unsigned long long>(cnt[b - 1]) : mass[b - 1])
                                      : base;
    if (v >= target && prev < target) atomicMin(&sm.found, b);
  }
  __syncthreads();
  const int r = sm.found;
  __syncthreads();
  return r;
}

// Calls f(i, logit) for every element of the row; 16-byte loads when the row
// allows them (each thread takes 8 consecutive bf16 / 4 floats per step).
template <typename T, typename F>
__device__ __forceinline__ void for_each_logit(const T* row, int V, bool vec_ok, F&& f) {
  constexpr int kVec = 16 / sizeof(T);
  int start = 0;
  if (vec_ok) {
    const int nv = V / kVec;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
      const uint4 raw = rv[v];
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int q = 0; q < kVec; ++q) f(v * kVec + q, to_f(e[q]));
    }
    start = nv * kVec;
  }
  for (int i = start + threadIdx.x; i < V; i += blockDim.x) f(i, to_f(row[i]));
}

template <typename T>
__device__ void hist_fill(const T* row, int V, bool vec_ok, float mx, float inv_t, int sel_bin, int skip,
                          unsigned int* cnt, unsigned long long* mass) {
  for (int b = threadIdx.x; b < kHistBins; b += blockDim.x) {
    cnt[b] = 0;
    mass[b] = 0;
  }
  __syncthreads();
  for_each_logit(row, V, vec_ok, [&](int i, float l) {
    const int key = key_of(l, mx, inv_t);
    if (key < 0 || i == skip) return;
    const int hi = key >> 11;
    if (sel_bin >= 0 && hi != sel_bin) return;
    const int bin = sel_bin >= 0 ? (key & (kHistBins - 1)) : hi;
    atomicAdd(&cnt[bin], 1u);
    atomicAdd(&mass[bin], mass_of(l, mx, inv_t));
  });
  __syncthreads();
}

// Block-wide exclusive scan of one 64-bit value per thread (deterministic order).
__device__ unsigned long long block_exscan_u64(unsigned long long v, HistSmem& sm, unsigned long long* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned long long x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sm.wsum[w] = x;
  __syncthreads();
  if (w == 0) {
    unsigned long long z = lane < (int)(blockDim.x >> 5) ? sm.wsum[lane] : 0ull;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, z, o);
      if (lane >= o) z += y;
    }
    sm.wsum[lane] = z;
  }
  __syncthreads();
  const unsigned long long base = (w ? sm.wsum[w - 1] : 0ull) + x - v;
  *total = sm.wsum[(blockDim.x >> 5) - 1];
  __syncthreads();
  return base;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    sample_kernel(const T* __restrict__ logits, long ld, int V, const float* __restrict__ temp,
                  const float* __restrict__ top_p, const int* __restrict__ top_k,
                  const int64_t* __restrict__ seeds, const int64_t* __restrict__ offsets,
                  const int* __restrict__ draft, int* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t hist_raw[];
  HistSmem& sm = *reinterpret_cast<HistSmem*>(hist_raw);
  const int b = blockIdx.x;
  const T* row = logits + (long)b * ld;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(row) % 16) == 0;
  float mx;
  int amax;
  block_argmax(row, V, mx, amax);
  const float t = temp[b];
  if (!(t > 0.f) || mx == -INFINITY) {
    if (threadIdx.x == 0) out[b] = amax;
    return;
  }
  const float inv_t = 1.f / t;
  const float p = top_p[b];
  const int k = top_k[b];
  const bool need_p = p > 0.f && p < 1.f;
  const bool need_k = k > 0 && k < V;
  const int d = draft ? draft[b] : -1;
  const bool has_draft = d >= 0 && d < V;
  const uint32_t k0 = static_cast<uint32_t>(seeds[b]), k1 = static_cast<uint32_t>(static_cast<uint64_t>(seeds[b]) >> 32);
  const uint64_t off = static_cast<uint64_t>(offsets[b]);

  // ---- kept set: key prefix [0, key_cut] with exact integer mass z_cut
  hist_fill(row, V, vec_ok, mx, inv_t, -1, -1, sm.cnt1, sm.mass1);
  hist_scan(sm.cnt1, sm.mass1, sm);
  int key_cut = (1 << kKeyBits) - 1;
  unsigned long long z_cut = sm.mass1[kHistBins - 1];
  int bin2 = -1;  // level-1 bin whose level-2 scan sits in cnt2 / mass2
  if (need_k && static_cast<unsigned int>(k) < sm.cnt1[kHistBins - 1]) {
    const int bk = hist_find(sm.cnt1, sm.mass1, true, 0, static_cast<unsigned long long>(k), sm);
    const unsigned int cb = bk ? sm.cnt1[bk - 1] : 0u;
    const unsigned long long mb = bk ? sm.mass1[bk - 1] : 0ull;
    hist_fill(row, V, vec_ok, mx, inv_t, bk, -1, sm.cnt2, sm.mass2);
    hist_scan(sm.cnt2, sm.mass2, sm);
    bin2 = bk;
    const int sk = hist_find(sm.cnt2, sm.mass2, true, cb, static_cast<unsigned long long>(k), sm);
    key_cut = (bk << 11) | sk;
    z_cut = mb + sm.mass2[sk];
  }
  if (need_p) {
    const unsigned long long target =
        static_cast<unsigned long long>(ceil(static_cast<double>(p) * static_cast<double>(z_cut)));
    const int bp = hist_find(sm.cnt1, sm.mass1, false, 0, target, sm);
    if (bp <= (key_cut >> 11)) {
      const unsigned long long mb = bp ? sm.mass1[bp - 1] : 0ull;
      if (bp != bin2) {
        hist_fill(row, V, vec_ok, mx, inv_t, bp, -1, sm.cnt2, sm.mass2);
        hist_scan(sm.cnt2, sm.mass2, sm);
        bin2 = bp;
      }
      const int sp = hist_find(sm.cnt2, sm.mass2, false, mb, target, sm);
      const int key_p = (bp << 11) | sp;
      if (key_p < key_cut) {
        key_cut = key_p;
        z_cut = mb + sm.mass2[sp];
      }
    }
  }

  // ---- speculative proposal: accept with probability p(d) under the kept,
  // renormalised distribution; on rejection d leaves the support, which is
  // the residual max(0, p - q) for a proposal q that is one-hot on d.
  int excluded = -1;
  int key_x = -1;
  unsigned long long m_x = 0;
  if (has_draft) {
    const float ld = to_f(row[d]);
    const int kd = key_of(ld, mx, inv_t);
    const unsigned long long md = (kd >= 0 && kd <= key_cut) ? mass_of(ld, mx, inv_t) : 0ull;
    const U4 r = philox4x32_10(U4{0xffffffffu, static_cast<uint32_t>(off), static_cast<uint32_t>(off >> 32), 0xacce97edu}, k0, k1);
    if (static_cast<double>(u01(r.x)) * static_cast<double>(z_cut) < static_cast<double>(md)) {
      if (threadIdx.x == 0) out[b] = d;
      return;
    }
    excluded = d;
    if (md > 0) {
      key_x = kd;
      m_x = md;
    }
  }
  const unsigned long long z_pick = z_cut - m_x;
  if (z_pick == 0) {  // nothing but the rejected proposal carried mass: fall back to the mode
    if (threadIdx.x == 0) out[b] = amax != excluded ? amax : (amax + 1) % V;
    return;
  }

  // ---- inverse-CDF draw over the kept keys in key order, then index order
  const U4 r = philox4x32_10(U4{0xfffffffeu, static_cast<uint32_t>(off), static_cast<uint32_t>(off >> 32), 0x5eed5eedu}, k0, k1);
  const unsigned long long u64 = (static_cast<unsigned long long>(r.x) << 32) | r.y;
  unsigned long long target = static_cast<unsigned long long>(
                                  (static_cast<unsigned __int128>(u64) * static_cast<unsigned __int128>(z_pick)) >> 64) +
                              1ull;  // uniform in [1, z_pick]
  // level 1: the bin (masses of bins >= the proposal's bin exclude it)
  if (threadIdx.x == 0) sm.found = kHistBins - 1;
  __syncthreads();
  const int cut_bin = key_cut >> 11, xb = key_x >= 0 ? (key_x >> 11) : kHistBins;
  for (int q = threadIdx.x; q <= cut_bin; q += blockDim.x) {
    const unsigned long long v = sm.mass1[q] - (q >= xb ? m_x : 0ull);
    const unsigned long long pv = q ? sm.mass1[q - 1] - (q - 1 >= xb ? m_x : 0ull) : 0ull;
    if (v >= target && pv < target) atomicMin(&sm.found, q);
  }
  __syncthreads();
  const int pb = min(sm.found, cut_bin);
  __syncthreads();
  const unsigned long long before_b = pb ? sm.mass1[pb - 1] - (pb - 1 >= xb ? m_x : 0ull) : 0ull;
  target -= before_b;
  // level 2: the sub-bin inside pb (the proposal is left out of the fill)
  hist_fill(row, V, vec_ok, mx, inv_t, pb, excluded, sm.cnt2, sm.mass2);
  hist_scan(sm.cnt2, sm.mass2, sm);
  const int sub_lim = pb == cut_bin ? (key_cut & (kHistBins - 1)) : kHistBins - 1;
  int ps = hist_find(sm.cnt2, sm.mass2, false, 0, target, sm);
  ps = min(ps, sub_lim);
  target -= ps ? sm.mass2[ps - 1] : 0ull;
  const int key_pick = (pb << 11) | ps;
  // last pass: tokens with key_pick in index order; each thread owns a contiguous chunk
  const int chunk = (V + blockDim.x - 1) / blockDim.x;
  const int i0 = threadIdx.x * chunk, i1 = min(V, i0 + chunk);
  unsigned long long mine = 0;
  for (int i = i0; i < i1; ++i) {
    const float l = to_f(row[i]);
    if (i != excluded && key_of(l, mx, inv_t) == key_pick) mine += mass_of(l, mx, inv_t);
  }
  unsigned long long tot;
  const unsigned long long pre = block_exscan_u64(mine, sm, &tot);
  if (threadIdx.x == 0) sm.found = 0x7fffffff;
  __syncthreads();
  if (pre < target && pre + mine >= target) {
    unsigned long long acc = pre;
    for (int i = i0; i < i1; ++i) {
      const float l = to_f(row[i]);
      if (i == excluded || key_of(l, mx, inv_t) != key_pick) continue;
      acc += mass_of(l, mx, inv_t);
      if (acc >= target) {
        atomicMin(&sm.found, i);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int pick = sm.found;
    if (pick == 0x7fffffff) pick = amax != excluded ? amax : (amax + 1) % V;  // rounding guard
    out[b] = pick;
  }
}

}  // namespace

// ---- constrained decoding: allowed-token masks from the host matcher
// mask [R, words] uint32, bit (t % 32) of word (t / 32) = token t allowed;
// rows[r] = the logits row of constraint r; this rank's logits hold the
// vocabulary columns [col_offset, col_offset + Vl).  Disallowed logits become
// -inf in place, so the ordinary argmax / sampler only picks allowed tokens.
namespace {
__global__ void apply_token_mask_kernel(__nv_bfloat16* __restrict__ logits, long ld, int Vl,
                                        const int* __restrict__ rows, const uint32_t* __restrict__ mask, int words,
                                        int col_offset) {
  const int r = blockIdx.y;
  __nv_bfloat16* lr = logits + (long)rows[r] * ld;
  const uint32_t* mr = mask + (long)r * words;
  const __nv_bfloat16 ninf = __ushort_as_bfloat16(0xFF80u);
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < Vl; c += gridDim.x * blockDim.x) {
    const int t = c + col_offset;
    const int w = t >> 5;
    const bool ok = w < words && ((mr[w] >> (t & 31)) & 1u);
    if (!ok) lr[c] = ninf;
  }
}
}  // namespace

void apply_token_mask(torch::Tensor& logits, const torch::Tensor& rows, const torch::Tensor& mask, int64_t col_offset) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1,
              "apply_token_mask: logits bf16 [NL, V]");
  TORCH_CHECK(rows.scalar_type() == at::kInt && rows.is_contiguous() && rows.is_cuda(), "apply_token_mask: rows int32");
  TORCH_CHECK(mask.scalar_type() == at::kInt && mask.is_contiguous() && mask.dim() == 2 && mask.is_cuda(),
              "apply_token_mask: mask int32 [R, words]");
  const int R = static_cast<int>(rows.numel());
  TORCH_CHECK(mask.size(0) >= R, "apply_token_mask: fewer mask rows than constrained rows");
  if (R == 0) return;
  const int Vl = static_cast<int>(logits.size(1));
  const at::cuda::CUDAGuard g(logits.device());
  const int bx = std::max(1, std::min(64, (Vl + 1023) / 1024));
  apply_token_mask_kernel<<<dim3(bx, R), 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0), Vl, rows.data_ptr<int>(),
      reinterpret_cast<const uint32_t*>(mask.data_ptr()), static_cast<int>(mask.size(1)), static_cast<int>(col_offset));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_rows(const torch::Tensor& logits, torch::Tensor& out) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "argmax: logits [B, V]");
  TORCH_CHECK(out.scalar_type() == at::kInt, "argmax: out int32");
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  const at::cuda::CUDAGuard g(logits.device());
  auto s = at::cuda::getCurrentCUDAStream();
  if (logits.scalar_type() == at::kFloat)
    argmax_kernel<float><<<B, kThreads, 0, s>>>(logits.data_ptr<float>(), logits.stride(0), V, out.data_ptr<int>());
  else
    argmax_kernel<__nv_bfloat16><<<B, kThreads, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), V, out.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

namespace {
void launch_sample(const torch::Tensor& logits, const torch::Tensor& temperature, const torch::Tensor& top_p,
                   const torch::Tensor& top_k, const torch::Tensor& seeds, const torch::Tensor& offsets,
                   const int* draft, torch::Tensor& out) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "sample: logits [B, V]");
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  TORCH_CHECK(temperature.scalar_type() == at::kFloat && top_p.scalar_type() == at::kFloat, "sample: f32 params");
  TORCH_CHECK(top_k.scalar_type() == at::kInt && seeds.scalar_type() == at::kLong && offsets.scalar_type() == at::kLong,
              "sample: top_k int32, seeds/offsets int64");
  TORCH_CHECK(temperature.numel() >= B && top_p.numel() >= B && top_k.numel() >= B && seeds.numel() >= B &&
                  offsets.numel() >= B && out.numel() >= B,
              "sample: per-row parameters shorter than the logits rows");
  const at::cuda::CUDAGuard g(logits.device());
  auto s = at::cuda::getCurrentCUDAStream();
  constexpr int smem = sizeof(HistSmem);
  static uint64_t configured = 0;  // per-device opt-in above 48 KB of shared memory
  const int dev = logits.get_device();
  if (!((configured >> dev) & 1u)) {
    cudaFuncSetAttribute(sample_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(sample_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured |= uint64_t(1) << dev;
  }
  if (logits.scalar_type() == at::kFloat)
    sample_kernel<float><<<B, kThreads, smem, s>>>(logits.data_ptr<float>(), logits.stride(0), V,
                                                 temperature.data_ptr<float>(), top_p.data_ptr<float>(),
                                                 top_k.data_ptr<int>(), seeds.data_ptr<int64_t>(),
                                                 offsets.data_ptr<int64_t>(), draft, out.data_ptr<int>());
  else
    sample_kernel<__nv_bfloat16><<<B, kThreads, smem, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), V, temperature.data_ptr<float>(),
        top_p.data_ptr<float>(), top_k.data_ptr<int>(), seeds.data_ptr<int64_t>(), offsets.data_ptr<int64_t>(), draft,
        out.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
}  // namespace

void sample_rows(const torch::Tensor& logits, const torch::Tensor& temperature, const torch::Tensor& top_p,
                 const torch::Tensor& top_k, const torch::Tensor& seeds, const torch::Tensor& offsets,
                 torch::Tensor& out) {
  launch_sample(logits, temperature, top_p, top_k, seeds, offsets, nullptr, out);
}

void verify_sample_rows(const torch::Tensor& logits, const torch::Tensor& temperature, const torch::Tensor& top_p,
                        const torch::Tensor& top_k, const torch::Tensor& seeds, const torch::Tensor& offsets,
                        const torch::Tensor& draft, torch::Tensor& out) {
  TORCH_CHECK(draft.scalar_type() == at::kInt && draft.numel() >= logits.size(0), "verify: draft int32 [B]");
  launch_sample(logits, temperature, top_p, top_k, seeds, offsets, draft.data_ptr<int>(), out);
}

torch::Tensor status_tensor(int64_t device) {
  static torch::Tensor per_device[64];
  TORCH_CHECK(device >= 0 && device < 64, "status: bad device");
  if (!per_device[device].defined()) {
    per_device[device] =
        torch::zeros({16}, torch::TensorOptions().dtype(torch::kInt).device(torch::kCUDA, int(device)));
  }
  return per_device[device];
}

}  // namespace bloom
