// Multimodal rotary embedding (M-RoPE, Qwen2/3-VL) on q [B, H, S, D] and
// k [B, KVH, S, D].  The rotary half-dimension D/2 is cut into three sections
// (temporal, height, width; 24/20/20 for D = 128); channel c (and c + D/2)
// takes its cos/sin from the position component of its section:
//   cos, sin  [3, B, S, D]   (one plane per component)
//   out[c]       = x[c] * cos[comp(c)][..c]       - x[c + D/2] * sin[comp(c)][..c]
//   out[c + D/2] = x[c + D/2] * cos[comp(c)][..c + D/2] + x[c] * sin[comp(c)][..c + D/2]
// (reference: crates/tilelang/scripts/generate_kernel.py:264-338, the CPU /
// MLX mrope kernel; that kernel hard-codes D = 128 and sections 24/20/20).
// One thread per rotation pair: the partner channel is read once, both
// outputs are written.  fp32 or bf16 tensors (math in fp32).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) {
  return *p;
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ void st(T* p, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, float v) {
  *p = v;
}
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16(v);
}

template <typename T>
__global__ void mrope_kernel(const T* __restrict__ x, T* __restrict__ out, const float* __restrict__ cosv,
                             const float* __restrict__ sinv, int B, int H, int S, int D, int sec0, int sec1) {
  const int half = D / 2;
  const long pairs = (long)B * H * S * half;
  const long plane = (long)B * S * D;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < pairs; i += (long)gridDim.x * blockDim.x) {
    const int c = static_cast<int>(i % half);
    const long row = i / half;  // (b, h, s)
    const int s = static_cast<int>(row % S);
    const int b = static_cast<int>(row / ((long)S * H));
    const int comp = c < sec0 ? 0 : (c < sec0 + sec1 ? 1 : 2);
    const long base = row * D;
    const long cb = comp * plane + ((long)b * S + s) * D;
    const float x0 = ld(x + base + c), x1 = ld(x + base + c + half);
    st(out + base + c, x0 * cosv[cb + c] - x1 * sinv[cb + c]);
    st(out + base + c + half, x1 * cosv[cb + c + half] + x0 * sinv[cb + c + half]);
  }
}

void launch_one(const torch::Tensor& x, torch::Tensor& out, const torch::Tensor& cos, const torch::Tensor& sin,
                int sec0, int sec1, cudaStream_t st) {
  const int B = x.size(0), H = x.size(1), S = x.size(2), D = x.size(3);
  const long pairs = (long)B * H * S * (D / 2);
  if (pairs == 0) return;
  const int grid = static_cast<int>(std::min<long>((pairs + 255) / 256, 148L * 16));
  if (x.scalar_type() == at::kFloat)
    mrope_kernel<float><<<grid, 256, 0, st>>>(x.data_ptr<float>(), out.data_ptr<float>(), cos.data_ptr<float>(),
                                              sin.data_ptr<float>(), B, H, S, D, sec0, sec1);
  else
    mrope_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
        cos.data_ptr<float>(), sin.data_ptr<float>(), B, H, S, D, sec0, sec1);
}

}  // namespace

void mrope(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& cos, const torch::Tensor& sin,
           torch::Tensor& q_out, torch::Tensor& k_out, int64_t sec0, int64_t sec1, int64_t sec2) {
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4, "mrope: q [B, H, S, D], k [B, KVH, S, D]");
  const int B = q.size(0), S = q.size(2), D = q.size(3);
  TORCH_CHECK(k.size(0) == B && k.size(2) == S && k.size(3) == D && D % 2 == 0, "mrope: q / k shapes disagree");
  TORCH_CHECK(sec0 >= 0 && sec1 >= 0 && sec2 >= 0 && sec0 + sec1 + sec2 == D / 2,
              "mrope: the three sections must cover head_dim / 2");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && (q.scalar_type() == at::kFloat || q.scalar_type() == at::kBFloat16),
              "mrope: q and k fp32 or bf16");
  TORCH_CHECK(q_out.scalar_type() == q.scalar_type() && k_out.scalar_type() == k.scalar_type() &&
                  q_out.sizes() == q.sizes() && k_out.sizes() == k.sizes(),
              "mrope: outputs like the inputs");
  TORCH_CHECK(cos.scalar_type() == at::kFloat && sin.scalar_type() == at::kFloat && cos.dim() == 4 &&
                  cos.size(0) == 3 && cos.size(1) == B && cos.size(2) == S && cos.size(3) == D &&
                  sin.sizes() == cos.sizes(),
              "mrope: cos / sin fp32 [3, B, S, D]");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && cos.is_contiguous() && sin.is_contiguous() &&
                  q_out.is_contiguous() && k_out.is_contiguous(),
              "mrope: contiguous tensors");
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  launch_one(q, q_out, cos, sin, int(sec0), int(sec1), st);
  launch_one(k, k_out, cos, sin, int(sec0), int(sec1), st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
