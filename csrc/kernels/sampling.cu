// Token sampling on the GPU.
//
// Greedy: per-row argmax (lowest index wins ties).
// Stochastic: temperature, top-k and top-p (nucleus) per row.  The kept set
// is found by bisection on a logit threshold (each probe is one pass of block
// reductions over the row), then one token is drawn from the renormalised
// kept distribution with the Gumbel-max trick.  Uniforms come from
// Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3",
// SC'11), keyed by the request seed and counted by (step offset, vocab index),
// so a request's stream is reproducible and independent of batch position.
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

template <typename T>
__device__ float block_sum_f(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

template <typename T>
__global__ void sample_kernel(const T* __restrict__ logits, long ld, int V, const float* __restrict__ temp,
                              const float* __restrict__ top_p, const int* __restrict__ top_k,
                              const int64_t* __restrict__ seeds, const int64_t* __restrict__ offsets,
                              const int* __restrict__ draft, int* __restrict__ out) {
  __shared__ float red[33];
  const int b = blockIdx.x;
  const T* row = logits + (long)b * ld;
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
  // Z = sum exp((l - mx)/t)
  float z = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) z += __expf((to_f(row[i]) - mx) * inv_t);
  z = block_sum_f<T>(z, red);
  // Kept set = {i : l_i >= lo}.  Top-k: largest threshold keeping >= k tokens.
  // Top-p (applied inside the top-k set): largest threshold keeping >= p of
  // that set's probability mass.  Logits below mx - 60 t carry < e^-60 of the
  // mass, so they bound the search from below.  The argmax always stays kept.
  float lo = -INFINITY;
  const bool need_p = p > 0.f && p < 1.f;
  const bool need_k = k > 0 && k < V;
  if (need_p || need_k) {
    const float floor_thr = mx - 60.f * t;
    float zk = z;
    float base = floor_thr;
    if (need_k) {
      float l0 = floor_thr, h0 = mx;
      for (int it = 0; it < 24; ++it) {
        const float mid = 0.5f * (l0 + h0);
        float cnt = 0.f;
        for (int i = threadIdx.x; i < V; i += blockDim.x) cnt += (to_f(row[i]) >= mid) ? 1.f : 0.f;
        cnt = block_sum_f<T>(cnt, red);
        if (cnt >= float(k)) l0 = mid; else h0 = mid;
      }
      base = l0;
      float m = 0.f;
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float l = to_f(row[i]);
        if (l >= base) m += __expf((l - mx) * inv_t);
      }
      zk = block_sum_f<T>(m, red);
    }
    lo = base;
    if (need_p) {
      float l0 = base, h0 = mx;
      for (int it = 0; it < 24; ++it) {
        const float mid = 0.5f * (l0 + h0);
        float mass = 0.f;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
          const float l = to_f(row[i]);
          if (l >= mid) mass += __expf((l - mx) * inv_t);
        }
        mass = block_sum_f<T>(mass, red);
        if (mass >= p * zk) l0 = mid; else h0 = mid;
      }
      lo = l0;
    }
  }
  const uint32_t k0 = static_cast<uint32_t>(seeds[b]), k1 = static_cast<uint32_t>(static_cast<uint64_t>(seeds[b]) >> 32);
  const uint64_t off = static_cast<uint64_t>(offsets[b]);
  // Speculative proposal: accept with probability p(d) of the kept,
  // renormalised distribution; on rejection d leaves the support, which is
  // the residual max(0, p - q) for a proposal q that is one-hot on d.
  int excluded = -1;
  const int d = draft ? draft[b] : -1;
  if (d >= 0 && d < V) {
    float zk = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float l = to_f(row[i]);
      if (l >= lo) zk += __expf((l - mx) * inv_t);
    }
    zk = block_sum_f<T>(zk, red);
    const float ld = to_f(row[d]);
    const float pd = (ld >= lo && zk > 0.f) ? __expf((ld - mx) * inv_t) / zk : 0.f;
    const U4 r = philox4x32_10(U4{0xffffffffu, static_cast<uint32_t>(off), static_cast<uint32_t>(off >> 32), 0xacce97edu}, k0, k1);
    if (u01(r.x) < pd) {
      if (threadIdx.x == 0) out[b] = d;
      return;
    }
    excluded = d;
  }
  // Gumbel-max over kept tokens
  float best = -INFINITY;
  int bi = amax != excluded ? amax : -1;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float l = to_f(row[i]);
    if (l < lo || i == excluded) continue;
    const U4 r = philox4x32_10(U4{static_cast<uint32_t>(i), static_cast<uint32_t>(off), static_cast<uint32_t>(off >> 32), 0x5eed5eedu}, k0, k1);
    const float gumbel = -__logf(-__logf(u01(r.x)));
    argmax_combine(best, bi, l * inv_t + gumbel, i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_combine(best, bi, v2, i2);
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    best = threadIdx.x < (blockDim.x >> 5) ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < (blockDim.x >> 5) ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      argmax_combine(best, bi, v2, i2);
    }
    if (threadIdx.x == 0) out[b] = (bi >= 0 && bi < V) ? bi : amax;
  }
}

}  // namespace

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
  if (logits.scalar_type() == at::kFloat)
    sample_kernel<float><<<B, kThreads, 0, s>>>(logits.data_ptr<float>(), logits.stride(0), V,
                                                 temperature.data_ptr<float>(), top_p.data_ptr<float>(),
                                                 top_k.data_ptr<int>(), seeds.data_ptr<int64_t>(),
                                                 offsets.data_ptr<int64_t>(), draft, out.data_ptr<int>());
  else
    sample_kernel<__nv_bfloat16><<<B, kThreads, 0, s>>>(
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
