// Encoder (BERT / MiniLM) kernels for sentence embeddings over packed
// variable-length batches (no padding tokens are computed):
//
//   bert_embed_ln      x[t] = LayerNorm(word[id] + pos[p] + type[tt])
//   varlen_attention   non-causal softmax(q k^T * scale) v per (sequence, head),
//                      head_dim <= 64, sequences up to 512 tokens; K/V of one
//                      head are staged in shared memory, one warp per query row
//   mean_pool_l2       mean over each sequence's tokens, then L2-normalise
//
// Linear layers use the tcgen05 GEMM (bias and bias+GELU epilogues).  The
// reference runs candle's padded BertModel and pools on the host
// (crates/engine/src/executor/candle.rs:177-264, server embedding.rs:505-540).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {
namespace {

__device__ __forceinline__ float block_sum_b(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[32] = t;
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

// one CTA per token; H <= 1024 (one element per thread)
__global__ void bert_embed_ln_kernel(const int* __restrict__ ids, const int* __restrict__ pos,
                                     const int* __restrict__ types, const __nv_bfloat16* __restrict__ word,
                                     const __nv_bfloat16* __restrict__ pemb, const __nv_bfloat16* __restrict__ temb,
                                     const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ b,
                                     __nv_bfloat16* __restrict__ out, int H, int V, int P, float eps) {
  __shared__ float red[33];
  const long t = blockIdx.x;
  const int i = threadIdx.x;
  int id = ids[t];
  id = id < 0 || id >= V ? 0 : id;
  int p = pos[t];
  p = p < 0 ? 0 : (p >= P ? P - 1 : p);
  const int tt = types != nullptr ? types[t] : 0;
  float v = 0.f;
  if (i < H)
    v = __bfloat162float(word[(long)id * H + i]) + __bfloat162float(pemb[(long)p * H + i]) +
        __bfloat162float(temb[(long)tt * H + i]);
  const float mean = block_sum_b(i < H ? v : 0.f, red) / H;
  const float d = i < H ? v - mean : 0.f;
  const float inv = rsqrtf(block_sum_b(d * d, red) / H + eps);
  if (i < H) out[t * H + i] = __float2bfloat16(d * inv * __bfloat162float(g[i]) + __bfloat162float(b[i]));
}

// qkv: [T, 3 * NH * D] (q | k | v); out: [T, NH * D].  grid (num_seqs, NH), block 256 threads.
template <int D>
__global__ void varlen_attention_kernel(const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ cu,
                                        __nv_bfloat16* __restrict__ out, int NH, float scale) {
  extern __shared__ float sm[];
  const int s = blockIdx.x, h = blockIdx.y;
  const int t0 = cu[s], L = cu[s + 1] - t0;
  float* Ks = sm;                 // [L][D]
  float* Vs = sm + (long)L * D;   // [L][D]
  const long ld = 3L * NH * D;
  for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
    const int j = idx / D, d = idx - j * D;
    const __nv_bfloat16* row = qkv + (long)(t0 + j) * ld;
    Ks[idx] = __bfloat162float(row[(long)NH * D + h * D + d]);
    Vs[idx] = __bfloat162float(row[2L * NH * D + h * D + d]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  constexpr int PER = (D + 31) / 32;  // dims per lane
  for (int qi = warp; qi < L; qi += nw) {
    const __nv_bfloat16* qrow = qkv + (long)(t0 + qi) * ld + h * D;
    float q[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int d = lane + 32 * k;
      q[k] = d < D ? __bfloat162float(qrow[d]) * scale : 0.f;
    }
    float m = -INFINITY, l = 0.f, o[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) o[k] = 0.f;
    for (int j = 0; j < L; ++j) {
      float sdot = 0.f;
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int d = lane + 32 * k;
        if (d < D) sdot += q[k] * Ks[j * D + d];
      }
      sdot = warp_sum(sdot);
      const float mn = fmaxf(m, sdot);
      const float corr = __expf(m - mn);
      const float p = __expf(sdot - mn);
      l = l * corr + p;
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int d = lane + 32 * k;
        o[k] = o[k] * corr + (d < D ? p * Vs[j * D + d] : 0.f);
      }
      m = mn;
    }
    __nv_bfloat16* orow = out + (long)(t0 + qi) * NH * D + h * D;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int d = lane + 32 * k;
      if (d < D) orow[d] = __float2bfloat16(o[k] / l);
    }
  }
}

// one CTA per sequence; out f32 [S, H]
__global__ void mean_pool_l2_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ cu,
                                    float* __restrict__ out, int H, int normalize) {
  __shared__ float red[33];
  const int s = blockIdx.x;
  const int t0 = cu[s], L = cu[s + 1] - t0;
  const int i = threadIdx.x;
  float acc = 0.f;
  if (i < H)
    for (int j = 0; j < L; ++j) acc += __bfloat162float(x[(long)(t0 + j) * H + i]);
  acc = L > 0 ? acc / L : 0.f;
  float nrm = 1.f;
  if (normalize) nrm = rsqrtf(fmaxf(block_sum_b(i < H ? acc * acc : 0.f, red), 1e-24f));
  if (i < H) out[(long)s * H + i] = acc * nrm;
}

}  // namespace

void bert_embed_ln(const torch::Tensor& ids, const torch::Tensor& pos, const c10::optional<torch::Tensor>& types,
                   const torch::Tensor& word, const torch::Tensor& pemb, const torch::Tensor& temb,
                   const torch::Tensor& g, const torch::Tensor& b, torch::Tensor& out, double eps) {
  const int T = ids.numel(), H = word.size(1);
  TORCH_CHECK(H <= 1024, "bert_embed_ln: hidden size <= 1024");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(ids.device());
  const int threads = ((H + 31) / 32) * 32;
  bert_embed_ln_kernel<<<T, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int>(), pos.data_ptr<int>(), types.has_value() ? types->data_ptr<int>() : nullptr,
      reinterpret_cast<const __nv_bfloat16*>(word.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(pemb.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(temb.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), H,
      word.size(0), pemb.size(0), float(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void varlen_attention(const torch::Tensor& qkv, const torch::Tensor& cu_seqlens, torch::Tensor& out, int64_t num_heads,
                      int64_t head_dim, int64_t max_len, double scale) {
  const int S = cu_seqlens.numel() - 1;
  if (S <= 0) return;
  TORCH_CHECK(head_dim == 32 || head_dim == 64, "varlen_attention: head_dim 32 or 64");
  TORCH_CHECK(max_len <= 512, "varlen_attention: sequences up to 512 tokens");
  const at::cuda::CUDAGuard guard(qkv.device());
  const size_t smem = 2 * size_t(max_len) * head_dim * sizeof(float);
  auto s = at::cuda::getCurrentCUDAStream();
  dim3 grid(S, num_heads);
  if (head_dim == 32) {
    cudaFuncSetAttribute(varlen_attention_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 512 * 32 * 4);
    varlen_attention_kernel<32><<<grid, 256, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                                                       cu_seqlens.data_ptr<int>(),
                                                       reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                       int(num_heads), float(scale));
  } else {
    cudaFuncSetAttribute(varlen_attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 512 * 64 * 4);
    varlen_attention_kernel<64><<<grid, 256, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                                                       cu_seqlens.data_ptr<int>(),
                                                       reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                       int(num_heads), float(scale));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mean_pool_l2(const torch::Tensor& x, const torch::Tensor& cu_seqlens, torch::Tensor& out, bool normalize) {
  const int S = cu_seqlens.numel() - 1, H = x.size(1);
  TORCH_CHECK(H <= 1024, "mean_pool_l2: hidden size <= 1024");
  if (S <= 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  mean_pool_l2_kernel<<<S, ((H + 31) / 32) * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), cu_seqlens.data_ptr<int>(), out.data_ptr<float>(), H,
      normalize ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
