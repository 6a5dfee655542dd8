// Wan 2.1 VAE decoder (frame-wise 2-D decoder of the reference): the layout,
// normalisation and packing kernels around the tcgen05 GEMM.
//
// Reference behaviour: executor/wan/vae.rs (decoder structure :218-276,
// residual block :440-462 = GroupNorm -> SiLU -> conv3x3 -> GroupNorm ->
// SiLU -> conv3x3 + (1x1) shortcut, mid attention :124-176 over the pixels of
// each frame with one head, nearest x2 upsampling + conv3x3 :464-492,
// GroupNorm -> SiLU -> conv_out, RGB bytes :573-606).
//
// Activations are NHWC bf16 [frames, H, W, C] so a 3x3 convolution is one
// GEMM: `im2col` gathers the 9 taps of every output pixel into a row of
// [9 * C] (tap-major, channel-minor; the weights are permuted to match at
// load time), applying on the fly the pending GroupNorm (per frame and
// group statistics from `gn_stats`), the SiLU and the nearest-neighbour x2
// upsampling of the source, so none of those intermediates is ever written.
// The GEMM epilogue then adds the bias and, for the second convolution of a
// residual block, the shortcut.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops_media.h"

namespace bloom {
namespace vae {

constexpr int kThreads = 256;
constexpr int kMaxGroups = 32;

int grid_for(long n) { return int(std::min<long>((n + kThreads - 1) / kThreads, 148L * 32)); }

// Partial sums of x and x^2 per (frame, group) over a slice of the frame's
// pixels: grid (frames, slices); partial [frames][slices][G][2].  Each
// active thread keeps one 8-channel chunk for the whole slice (the thread
// count is a multiple of C / 8), so the per-channel sums are private
// registers, and the groups are then summed in a fixed order: the result
// does not depend on scheduling (no floating-point atomics).
__global__ void __launch_bounds__(kThreads) gn_partial_kernel(const __nv_bfloat16* __restrict__ x, long P, int C,
                                                               int G, int slices, float* __restrict__ partial) {
  __shared__ float red[kThreads][8][2];
  const int n = blockIdx.x, sl = blockIdx.y;
  const int cpg = C / G, c8 = C / 8;
  const int active = (kThreads / c8) * c8;  // c8 <= kThreads (C <= 2048)
  const long pix_per = (P + slices - 1) / slices;
  const long p0 = sl * pix_per, p1 = min(P, p0 + pix_per);
  const __nv_bfloat16* xf = x + (long)n * P * C;
  float s[8], q[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) s[k] = q[k] = 0.f;
  const int cc = threadIdx.x % c8;
  if (threadIdx.x < active) {
    for (long p = p0 + threadIdx.x / c8; p < p1; p += active / c8) {
      const uint4 u = *reinterpret_cast<const uint4*>(xf + p * C + cc * 8);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float v = __bfloat162float(b[k]);
        s[k] += v;
        q[k] += v * v;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    red[threadIdx.x][k][0] = threadIdx.x < active ? s[k] : 0.f;
    red[threadIdx.x][k][1] = threadIdx.x < active ? q[k] : 0.f;
  }
  __syncthreads();
  for (int g = threadIdx.x; g < G; g += kThreads) {
    float gs = 0.f, gq = 0.f;
    for (int t = 0; t < active; ++t) {
      const int c0 = (t % c8) * 8;
      if (c0 + 8 <= g * cpg || c0 >= (g + 1) * cpg) continue;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if ((c0 + k) / cpg == g) {
          gs += red[t][k][0];
          gq += red[t][k][1];
        }
    }
    partial[(((long)n * slices + sl) * G + g) * 2] = gs;
    partial[(((long)n * slices + sl) * G + g) * 2 + 1] = gq;
  }
}

// stats [frames][G][2] = (mean, rstd) from the partial sums (double precision)
__global__ void gn_finalize_kernel(const float* __restrict__ partial, int frames, int slices, int G, long count,
                                   float eps, float* __restrict__ stats) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= frames * G) return;
  const int n = i / G, g = i - n * G;
  double s = 0.0, q = 0.0;
  for (int sl = 0; sl < slices; ++sl) {
    s += partial[(((long)n * slices + sl) * G + g) * 2];
    q += partial[(((long)n * slices + sl) * G + g) * 2 + 1];
  }
  const double mean = s / count;
  const double var = fmax(q / count - mean * mean, 0.0);
  stats[i * 2] = float(mean);
  stats[i * 2 + 1] = float(1.0 / sqrt(var + eps));
}

struct NormArgs {
  const float* stats;  // [frames][G][2] or null
  const float* gamma;  // [C]
  const float* beta;   // [C]
  int G;
  int silu;
};

__device__ __forceinline__ void norm8(float (&v)[8], const NormArgs& nm, int n, int c0, int C) {
  if (nm.stats != nullptr) {
    const int cpg = C / nm.G;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = c0 + k, g = c / cpg;
      const float mean = nm.stats[(n * nm.G + g) * 2], rstd = nm.stats[(n * nm.G + g) * 2 + 1];
      v[k] = (v[k] - mean) * rstd * nm.gamma[c] + nm.beta[c];
    }
  }
  if (nm.silu) {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = v[k] / (1.f + __expf(-v[k]));
  }
}

// dst [frames * Ho * Wo, 9 * C]: row (n, y, x), column (ky * 3 + kx) * C + c =
// act(src[n, yy / up, xx / up, c]) with yy = y * stride + ky - pad_t (and
// likewise xx) in the x`up` nearest-upsampled source, zero outside it.
__global__ void __launch_bounds__(kThreads) im2col3x3_kernel(const __nv_bfloat16* __restrict__ src, int frames,
                                                              int Hs, int Ws, int C, int up, int stride, int pad_t,
                                                              int pad_l, int Ho, int Wo, const NormArgs nm,
                                                              __nv_bfloat16* __restrict__ dst) {
  const int Hu = Hs * up, Wu = Ws * up, c8 = C / 8;
  const long total = (long)frames * Ho * Wo * 9 * c8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int cc = int(i % c8);
    const long r = i / c8;
    const int tap = int(r % 9);
    const long pix = r / 9;
    const int x = int(pix % Wo), y = int((pix / Wo) % Ho), n = int(pix / ((long)Wo * Ho));
    const int yy = y * stride + tap / 3 - pad_t, xx = x * stride + tap % 3 - pad_l;
    uint4 out = make_uint4(0, 0, 0, 0);
    if (yy >= 0 && yy < Hu && xx >= 0 && xx < Wu) {
      const int sy = yy / up, sx = xx / up;
      const uint4 u = *reinterpret_cast<const uint4*>(src + (((long)n * Hs + sy) * Ws + sx) * C + cc * 8);
      if (nm.stats != nullptr || nm.silu) {
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __bfloat162float(b[k]);
        norm8(v, nm, n, cc * 8, C);
        out = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                         pack_bf16x2(v[6], v[7]));
      } else {
        out = u;
      }
    }
    *reinterpret_cast<uint4*>(dst + (pix * 9 + tap) * C + cc * 8) = out;
  }
}

// dst [frames * P, C] = act(src) (GroupNorm / SiLU applied, same layout)
__global__ void __launch_bounds__(kThreads) gn_apply_kernel(const __nv_bfloat16* __restrict__ src, int frames,
                                                             long P, int C, const NormArgs nm,
                                                             __nv_bfloat16* __restrict__ dst) {
  const int c8 = C / 8;
  const long total = (long)frames * P * c8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int cc = int(i % c8);
    const int n = int(i / c8 / P);
    const uint4 u = *reinterpret_cast<const uint4*>(src + i * 8);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __bfloat162float(b[k]);
    norm8(v, nm, n, cc * 8, C);
    *reinterpret_cast<uint4*>(dst + i * 8) =
        make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

// qkv [frames * P, 3C] -> q [frames * P, C] and one-head KV pages
// [frames * bpb][2][16][C] (frame n's pixel p in page n * bpb + p / 16)
__global__ void __launch_bounds__(kThreads) pack_attn_kernel(const __nv_bfloat16* __restrict__ qkv, int frames,
                                                              long P, int C, int bpb, __nv_bfloat16* __restrict__ q,
                                                              __nv_bfloat16* __restrict__ kv) {
  const int c8 = C / 8;
  const long total = (long)frames * P * c8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int cc = int(i % c8);
    const long row = i / c8;
    const int n = int(row / P);
    const long p = row - (long)n * P;
    const __nv_bfloat16* s = qkv + row * 3 * C + cc * 8;
    *reinterpret_cast<uint4*>(q + row * C + cc * 8) = *reinterpret_cast<const uint4*>(s);
    const long blk = (long)n * bpb + p / 16;
    const int slot = int(p % 16);
    *reinterpret_cast<uint4*>(kv + ((blk * 2 + 0) * 16 + slot) * C + cc * 8) =
        *reinterpret_cast<const uint4*>(s + C);
    *reinterpret_cast<uint4*>(kv + ((blk * 2 + 1) * 16 + slot) * C + cc * 8) =
        *reinterpret_cast<const uint4*>(s + 2 * C);
  }
}

// src [pixels, ld] bf16 (channels 0..2 = R, G, B in [-1, 1]) -> u8 [pixels, 3]
__global__ void rgb_kernel(const __nv_bfloat16* __restrict__ src, long pixels, int ld, uint8_t* __restrict__ dst) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < pixels * 3; i += (long)gridDim.x * blockDim.x) {
    const long p = i / 3;
    const int c = int(i - p * 3);
    const float v = (__bfloat162float(src[p * ld + c]) * 0.5f + 0.5f) * 255.f;
    dst[i] = uint8_t(fminf(fmaxf(v, 0.f), 255.f));
  }
}

NormArgs norm_args(const c10::optional<torch::Tensor>& stats, const c10::optional<torch::Tensor>& gamma,
                   const c10::optional<torch::Tensor>& beta, int64_t groups, bool silu, int C) {
  NormArgs nm{};
  if (stats.has_value()) {
    TORCH_CHECK(stats->scalar_type() == at::kFloat && stats->is_contiguous(), "vae: stats f32");
    TORCH_CHECK(gamma.has_value() && beta.has_value() && gamma->numel() == C && beta->numel() == C &&
                    gamma->scalar_type() == at::kFloat && beta->scalar_type() == at::kFloat,
                "vae: GroupNorm gamma / beta f32 [C]");
    TORCH_CHECK(groups > 0 && C % groups == 0, "vae: groups divide C");
    nm.stats = stats->data_ptr<float>();
    nm.gamma = gamma->data_ptr<float>();
    nm.beta = beta->data_ptr<float>();
    nm.G = int(groups);
  }
  nm.silu = silu ? 1 : 0;
  return nm;
}

}  // namespace vae

void vae_gn_stats(const torch::Tensor& x, int64_t groups, double eps, torch::Tensor& stats) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 4, "vae_gn_stats: x NHWC bf16");
  const int N = x.size(0), C = x.size(3);
  const long P = (long)x.size(1) * x.size(2);
  TORCH_CHECK(C % 8 == 0 && C <= 8 * vae::kThreads && groups > 0 && groups <= vae::kMaxGroups && C % groups == 0,
              "vae_gn_stats: C % 8 == 0, C <= 2048, groups");
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.is_contiguous() && stats.numel() == (int64_t)N * groups * 2,
              "vae_gn_stats: stats f32 [N, G, 2]");
  if (N == 0) return;
  const int slices = int(std::max<long>(1, std::min<long>(256, P * (C / 8) / (vae::kThreads * 32))));
  auto partial = torch::empty({(int64_t)N * slices * groups * 2}, x.options().dtype(at::kFloat));
  const at::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  vae::gn_partial_kernel<<<dim3(N, slices), vae::kThreads, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), P, C, int(groups), slices, partial.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  vae::gn_finalize_kernel<<<int((N * groups + 127) / 128), 128, 0, st>>>(
      partial.data_ptr<float>(), N, slices, int(groups), P * (C / groups), float(eps), stats.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void vae_im2col3x3(const torch::Tensor& src, int64_t up, const c10::optional<torch::Tensor>& stats,
                   const c10::optional<torch::Tensor>& gamma, const c10::optional<torch::Tensor>& beta,
                   int64_t groups, bool silu, torch::Tensor& dst, int64_t stride, int64_t pad_t, int64_t pad_b,
                   int64_t pad_l, int64_t pad_r) {
  TORCH_CHECK(src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.dim() == 4,
              "vae_im2col3x3: src NHWC bf16");
  const int N = src.size(0), Hs = src.size(1), Ws = src.size(2), C = src.size(3);
  TORCH_CHECK(C % 8 == 0 && (up == 1 || up == 2) && (stride == 1 || stride == 2), "vae_im2col3x3: C % 8, up, stride");
  TORCH_CHECK(pad_t >= 0 && pad_b >= 0 && pad_l >= 0 && pad_r >= 0 && pad_t <= 2 && pad_l <= 2, "vae_im2col3x3: pads");
  const int Ho = int((Hs * up + pad_t + pad_b - 3) / stride + 1), Wo = int((Ws * up + pad_l + pad_r - 3) / stride + 1);
  TORCH_CHECK(Ho > 0 && Wo > 0, "vae_im2col3x3: empty output");
  TORCH_CHECK(dst.scalar_type() == at::kBFloat16 && dst.is_contiguous() && dst.numel() == (int64_t)N * Ho * Wo * 9 * C,
              "vae_im2col3x3: dst bf16 [N * Ho * Wo, 9 * C]");
  const vae::NormArgs nm = vae::norm_args(stats, gamma, beta, groups, silu, C);
  if (stats.has_value()) TORCH_CHECK(stats->numel() == (int64_t)N * groups * 2, "vae_im2col3x3: stats [N, G, 2]");
  const long total = dst.numel() / 8;
  if (total == 0) return;
  const at::cuda::CUDAGuard g(src.device());
  vae::im2col3x3_kernel<<<vae::grid_for(total), vae::kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), N, Hs, Ws, C, int(up), int(stride), int(pad_t),
      int(pad_l), Ho, Wo, nm, reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void vae_gn_apply(const torch::Tensor& src, const torch::Tensor& stats, const torch::Tensor& gamma,
                  const torch::Tensor& beta, int64_t groups, bool silu, torch::Tensor& dst) {
  TORCH_CHECK(src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.dim() == 4,
              "vae_gn_apply: src NHWC bf16");
  const int N = src.size(0), C = src.size(3);
  const long P = (long)src.size(1) * src.size(2);
  TORCH_CHECK(dst.scalar_type() == at::kBFloat16 && dst.is_contiguous() && dst.numel() == src.numel(),
              "vae_gn_apply: dst like src");
  TORCH_CHECK(C % 8 == 0 && stats.numel() == (int64_t)N * groups * 2, "vae_gn_apply: C % 8, stats [N, G, 2]");
  const vae::NormArgs nm = vae::norm_args(stats, gamma, beta, groups, silu, C);
  const long total = src.numel() / 8;
  if (total == 0) return;
  const at::cuda::CUDAGuard g(src.device());
  vae::gn_apply_kernel<<<vae::grid_for(total), vae::kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), N, P, C, nm,
      reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void vae_pack_attn(const torch::Tensor& qkv, int64_t frames, int64_t channels, torch::Tensor& q, torch::Tensor& kv) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous() && qkv.dim() == 2 &&
                  qkv.size(1) == 3 * channels && qkv.size(0) % frames == 0,
              "vae_pack_attn: qkv bf16 [frames * P, 3C]");
  const long P = qkv.size(0) / frames;
  const int C = int(channels);
  const int bpb = int((P + 15) / 16);
  TORCH_CHECK(C % 8 == 0, "vae_pack_attn: C % 8 == 0");
  TORCH_CHECK(q.is_contiguous() && q.numel() == qkv.size(0) * C, "vae_pack_attn: q [frames * P, C]");
  TORCH_CHECK(kv.is_contiguous() && kv.numel() >= frames * bpb * 2 * 16 * C, "vae_pack_attn: kv pages");
  const long total = qkv.size(0) * (C / 8);
  if (total == 0) return;
  const at::cuda::CUDAGuard g(qkv.device());
  vae::pack_attn_kernel<<<vae::grid_for(total), vae::kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), int(frames), P, C, bpb,
      reinterpret_cast<__nv_bfloat16*>(q.data_ptr()), reinterpret_cast<__nv_bfloat16*>(kv.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void vae_rgb(const torch::Tensor& src, torch::Tensor& dst) {
  TORCH_CHECK(src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.stride(1) == 1 && src.size(1) >= 3,
              "vae_rgb: src bf16 [pixels, >= 3]");
  TORCH_CHECK(dst.scalar_type() == at::kByte && dst.is_contiguous() && dst.numel() == src.size(0) * 3,
              "vae_rgb: dst u8 [pixels, 3]");
  const long pixels = src.size(0);
  if (pixels == 0) return;
  const at::cuda::CUDAGuard g(src.device());
  vae::rgb_kernel<<<vae::grid_for(pixels * 3), vae::kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), pixels, int(src.stride(0)), dst.data_ptr<uint8_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
