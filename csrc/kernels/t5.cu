// umT5 encoder self-attention with the T5 relative position bias.
//
// scores[h, i, j] = q_i . k_j + bias[(j - i) + L - 1][h]   (no 1/sqrt(d) scale)
// keys j >= len[s] (padding) are masked; the bias table is built on the host
// per layer from the learned [32 buckets, heads] embedding with T5's
// bidirectional log buckets.  One CTA per (sequence, head, 32-query chunk):
// the head's K and V for the whole sequence sit in shared memory (rows padded
// to 66 elements so lane-per-key reads hit distinct banks), one warp per
// query row computes its scores lane-per-key, a warp softmax, and
// accumulates the output lane-per-dimension pair.  The encoder runs once per
// generation over at most 512 tokens, so this stays a CUDA-core kernel.
//
// Reference: executor/wan/t5_encoder.rs (the encoder block :295-343); the
// bias and gated-GELU FFN follow the published umT5 / T5 v1.1 definition.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops_media.h"

namespace bloom {
namespace t5 {

constexpr int kD = 64;        // head dim
constexpr int kRS = kD + 2;   // padded smem row (elements)
constexpr int kWarps = 8;
constexpr int kRowsPerCta = 32;

__global__ void __launch_bounds__(kWarps * 32) rel_attention_kernel(
    const __nv_bfloat16* __restrict__ qkv, int L, int H, const int* __restrict__ lens,
    const float* __restrict__ bias, __nv_bfloat16* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sV = sK + (long)L * kRS;
  float* sP = reinterpret_cast<float*>(sV + (long)L * kRS);  // [kWarps][L]
  float* sQ = sP + (long)kWarps * L;                           // [kWarps][64]
  const int s = blockIdx.x, h = blockIdx.y, r0 = blockIdx.z * kRowsPerCta;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = lens[s];
  const long ld = 3L * H * kD;
  const __nv_bfloat16* base = qkv + (long)s * L * ld;
  for (int idx = threadIdx.x; idx < L * (kD / 2); idx += blockDim.x) {
    const int j = idx / (kD / 2), d = (idx - j * (kD / 2)) * 2;
    const __nv_bfloat16* row = base + (long)j * ld;
    *reinterpret_cast<uint32_t*>(sK + j * kRS + d) = *reinterpret_cast<const uint32_t*>(row + (H + h) * kD + d);
    *reinterpret_cast<uint32_t*>(sV + j * kRS + d) = *reinterpret_cast<const uint32_t*>(row + (2 * H + h) * kD + d);
  }
  __syncthreads();
  float* p = sP + warp * L;
  for (int i = r0 + warp; i < min(r0 + kRowsPerCta, L); i += kWarps) {
    // q row as f32 in this warp's shared slot (broadcast reads)
    float* qs = sQ + warp * kD;
    {
      const __nv_bfloat162 qv = *reinterpret_cast<const __nv_bfloat162*>(base + (long)i * ld + h * kD + 2 * lane);
      qs[2 * lane] = __bfloat162float(qv.x);
      qs[2 * lane + 1] = __bfloat162float(qv.y);
    }
    __syncwarp();
    float mx = -INFINITY;
    for (int j = lane; j < len; j += 32) {
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < kD; d += 2) {
        const __nv_bfloat162 kk = *reinterpret_cast<const __nv_bfloat162*>(sK + j * kRS + d);
        acc += qs[d] * __bfloat162float(kk.x) + qs[d + 1] * __bfloat162float(kk.y);
      }
      const float sc = acc + bias[(long)(j - i + L - 1) * H + h];
      p[j] = sc;
      mx = fmaxf(mx, sc);
    }
    mx = warp_max(mx);
    float sum = 0.f;
    for (int j = lane; j < len; j += 32) {
      const float e = __expf(p[j] - mx);
      p[j] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    float o0 = 0.f, o1 = 0.f;
    for (int j = 0; j < len; ++j) {
      const float pj = p[j];
      const __nv_bfloat162 vv = *reinterpret_cast<const __nv_bfloat162*>(sV + j * kRS + 2 * lane);
      o0 += pj * __bfloat162float(vv.x);
      o1 += pj * __bfloat162float(vv.y);
    }
    *reinterpret_cast<uint32_t*>(out + ((long)s * L + i) * H * kD + h * kD + 2 * lane) = pack_bf16x2(o0 * inv, o1 * inv);
    __syncwarp();
  }
}

}  // namespace t5

void t5_rel_attention(const torch::Tensor& qkv, int64_t seqs, int64_t heads, const torch::Tensor& lens,
                      const torch::Tensor& bias, torch::Tensor& out) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous() && qkv.dim() == 2 &&
                  qkv.size(1) == 3 * heads * t5::kD && qkv.size(0) % seqs == 0,
              "t5_rel_attention: qkv bf16 [seqs * L, 3 * heads * 64]");
  const int L = int(qkv.size(0) / seqs);
  TORCH_CHECK(lens.scalar_type() == at::kInt && lens.numel() == seqs, "t5_rel_attention: lens int32 [seqs]");
  TORCH_CHECK(bias.scalar_type() == at::kFloat && bias.is_contiguous() && bias.numel() == (2L * L - 1) * heads,
              "t5_rel_attention: bias f32 [2L - 1, heads]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == qkv.size(0) * heads * t5::kD,
              "t5_rel_attention: out bf16 [seqs * L, heads * 64]");
  const size_t smem = (size_t)L * t5::kRS * 2 * 2 + (size_t)t5::kWarps * (L + t5::kD) * 4;
  TORCH_CHECK(smem <= 227 * 1024, "t5_rel_attention: sequence too long for shared memory");
  if (qkv.numel() == 0) return;
  const at::cuda::CUDAGuard g(qkv.device());
  C10_CUDA_CHECK(cudaFuncSetAttribute(t5::rel_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(smem)));
  dim3 grid(int(seqs), int(heads), (L + t5::kRowsPerCta - 1) / t5::kRowsPerCta);
  t5::rel_attention_kernel<<<grid, t5::kWarps * 32, smem, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), L, int(heads), lens.data_ptr<int>(),
      bias.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
