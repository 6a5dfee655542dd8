// Dequantisers for the non-GGUF weight formats and the 8-bit KV-cache rows.
//
//   int4_flat_dequant   AWQ / GPTQ int4 in the flat layout the reference's
//                       CPU fallback and Metal shader use
//                       (executor/metal_quant.rs:256-383): element id is
//                       nibble id % 8 of qweight[id / 8]; its group g is
//                       id / 128 (AWQ) or g_idx[id] (GPTQ); the zero point is
//                       nibble g % 8 of qzeros[g / 8];
//                       w = (q - z) * scales[g].  Out-of-range words, scales
//                       or group indices give 0, out-of-range zeros give z = 0,
//                       as in the reference.
//   gptq_dequant        GPTQ checkpoints as stored by HF / AutoGPTQ:
//                       qweight int32 [K/8, N] (8 K-rows per word),
//                       qzeros int32 [G, N/8], scales [G, N], g_idx [K];
//                       zero points are stored minus one (v1 format):
//                       W[n, k] = (q - (z + 1)) * s.  Output W [N, K] bf16,
//                       the nn.Linear layout the tcgen05 GEMM consumes.
//   awq_dequant         AWQ "GEMM" checkpoints: qweight int32 [K, N/8] with
//                       the nibble order 0,2,4,6,1,3,5,7 inside a word,
//                       qzeros int32 [K/group, N/8] (same order),
//                       scales [K/group, N]; W[n, k] = (q - z) * s.
//   bnb4_dequant        bitsandbytes 4-bit codes: two codes per byte, high
//                       nibble first (core/quantization.rs:474-560), value =
//                       codebook[code] * scale[block]; the scale has one entry
//                       per `block` output elements (one entry = per-tensor).
//   kv_row_quant/deq    8-bit KV rows.  int8: symmetric per row
//                       (core/quantization.rs:396-470): scale = max|x| / 127
//                       (1 for an all-zero row), q = clamp(round(x / scale),
//                       -128, 127), x' = q * scale.  fp8: e4m3 with
//                       scale = max|x| / 448 (1 for an all-zero row).
//
// All kernels are memory-bound elementwise passes with grid-stride loops.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include <algorithm>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {
namespace {

__device__ __forceinline__ uint32_t nib(uint32_t w, int i) { return (w >> (4 * i)) & 0xFu; }

template <typename T>
__device__ __forceinline__ T to_out(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float v) {
  return __float2bfloat16(v);
}
template <>
__device__ __forceinline__ __half to_out<__half>(float v) {
  return __float2half(v);
}
template <>
__device__ __forceinline__ float to_out<float>(float v) {
  return v;
}

template <typename T>
__global__ void int4_flat_dequant_kernel(const uint32_t* __restrict__ qw, long nqw, const float* __restrict__ sc,
                                         long nsc, const uint32_t* __restrict__ qz, long nqz,
                                         const int32_t* __restrict__ gidx, long ngidx, long n, T* __restrict__ out) {
  for (long id = blockIdx.x * (long)blockDim.x + threadIdx.x; id < n; id += (long)gridDim.x * blockDim.x) {
    float v = 0.f;
    const long wi = id >> 3;
    if (wi < nqw) {
      const uint32_t q = nib(qw[wi], static_cast<int>(id & 7));
      long g;
      bool ok = true;
      if (gidx != nullptr) {
        ok = id < ngidx;
        g = ok ? static_cast<long>(static_cast<uint32_t>(gidx[id])) : 0;
      } else {
        g = id >> 7;
      }
      if (ok && g < nsc) {
        const long zi = g >> 3;
        const uint32_t z = zi < nqz ? nib(qz[zi], static_cast<int>(g & 7)) : 0u;
        v = (static_cast<float>(q) - static_cast<float>(z)) * sc[g];
      }
    }
    out[id] = to_out<T>(v);
  }
}

// One thread per (n, 8 consecutive k): reads one qweight word, writes 16 bytes.
__global__ void gptq_dequant_kernel(const int32_t* __restrict__ qw, const int32_t* __restrict__ qz,
                                    const __half* __restrict__ sc, const int32_t* __restrict__ gidx, int K, int N,
                                    __nv_bfloat16* __restrict__ out) {
  const long total = (long)(K / 8) * N;
  for (long t = blockIdx.x * (long)blockDim.x + threadIdx.x; t < total; t += (long)gridDim.x * blockDim.x) {
    const int n = static_cast<int>(t % N);
    const int kw = static_cast<int>(t / N);
    const uint32_t w = static_cast<uint32_t>(qw[(long)kw * N + n]);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = kw * 8 + i;
      const int g = gidx[k];
      const uint32_t z = nib(static_cast<uint32_t>(qz[(long)g * (N / 8) + n / 8]), n & 7) + 1u;
      v[i] = (static_cast<float>(nib(w, i)) - static_cast<float>(z)) * __half2float(sc[(long)g * N + n]);
    }
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(out + (long)n * K + kw * 8) = o;
  }
}

// AWQ packs 8 output columns per word in the order 0,2,4,6,1,3,5,7: column j
// of a group of 8 sits in nibble kAwqNibble[j].
__constant__ int kAwqNibble[8] = {0, 4, 1, 5, 2, 6, 3, 7};

// One thread per (k, 8 consecutive n): reads one qweight word and one zero word.
__global__ void awq_dequant_kernel(const int32_t* __restrict__ qw, const int32_t* __restrict__ qz,
                                   const __half* __restrict__ sc, int K, int N, int group,
                                   __nv_bfloat16* __restrict__ out) {
  const long total = (long)K * (N / 8);
  for (long t = blockIdx.x * (long)blockDim.x + threadIdx.x; t < total; t += (long)gridDim.x * blockDim.x) {
    const int nw = static_cast<int>(t % (N / 8));
    const int k = static_cast<int>(t / (N / 8));
    const int g = k / group;
    const uint32_t w = static_cast<uint32_t>(qw[(long)k * (N / 8) + nw]);
    const uint32_t z = static_cast<uint32_t>(qz[(long)g * (N / 8) + nw]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = nw * 8 + j;
      const int s = kAwqNibble[j];
      const float v =
          (static_cast<float>(nib(w, s)) - static_cast<float>(nib(z, s))) * __half2float(sc[(long)g * N + n]);
      out[(long)n * K + k] = __float2bfloat16(v);
    }
  }
}

// bitsandbytes 4-bit code books: NF4 (the normal-float quantiles of the QLoRA
// data type, as bitsandbytes publishes them) and FP4 (bitsandbytes' code order).
__constant__ float kNf4[16] = {-1.0f,
                               -0.6961928009986877f,
                               -0.5250730514526367f,
                               -0.39491748809814453f,
                               -0.28444138169288635f,
                               -0.18477343022823334f,
                               -0.09105003625154495f,
                               0.0f,
                               0.07958029955625534f,
                               0.16093020141124725f,
                               0.24611230194568634f,
                               0.33791524171829224f,
                               0.44070982933044434f,
                               0.5626170039176941f,
                               0.7229568362236023f,
                               1.0f};
__constant__ float kFp4[16] = {0.0f,  0.0625f,  8.0f,  12.0f,  4.0f,  6.0f,  2.0f,  3.0f,
                               -0.0f, -0.0625f, -8.0f, -12.0f, -4.0f, -6.0f, -2.0f, -3.0f};

template <bool NF4>
__global__ void bnb4_dequant_kernel(const uint8_t* __restrict__ packed, long nbytes, const float* __restrict__ scale,
                                    long block, __nv_bfloat16* __restrict__ out) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nbytes; i += (long)gridDim.x * blockDim.x) {
    const uint32_t b = packed[i];
    const long e0 = 2 * i;
    const float s0 = scale[e0 / block], s1 = scale[(e0 + 1) / block];
    const float c0 = NF4 ? kNf4[b >> 4] : kFp4[b >> 4];
    const float c1 = NF4 ? kNf4[b & 15u] : kFp4[b & 15u];
    *reinterpret_cast<uint32_t*>(out + e0) = pack_bf16x2(c0 * s0, c1 * s1);
  }
}

// Row quantisers: one warp per row.
template <bool FP8>
__global__ void kv_row_quant_kernel(const __nv_bfloat16* __restrict__ x, long rows, int cols, uint8_t* __restrict__ q,
                                    float* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const long warps = (long)gridDim.x * (blockDim.x / 32);
  for (long r = blockIdx.x * (long)(blockDim.x / 32) + (threadIdx.x >> 5); r < rows; r += warps) {
    const __nv_bfloat16* xr = x + r * cols;
    float mx = 0.f;
    for (int c = lane; c < cols; c += 32) mx = fmaxf(mx, fabsf(__bfloat162float(xr[c])));
    mx = warp_max(mx);
    const float scale = mx > 0.f ? mx / (FP8 ? 448.f : 127.f) : 1.f;
    const float inv = 1.f / scale;
    if (lane == 0) scales[r] = scale;
    uint8_t* qr = q + r * cols;
    for (int c = lane; c < cols; c += 32) {
      const float v = __bfloat162float(xr[c]) * inv;
      if constexpr (FP8) {
        const __nv_fp8_e4m3 f(v);
        qr[c] = *reinterpret_cast<const uint8_t*>(&f);
      } else {
        const float rq = fminf(fmaxf(roundf(v), -128.f), 127.f);
        qr[c] = static_cast<uint8_t>(static_cast<int8_t>(rq));
      }
    }
  }
}

template <bool FP8>
__global__ void kv_row_dequant_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scales, long rows,
                                      int cols, __nv_bfloat16* __restrict__ out) {
  const long n = rows * cols;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float s = scales[i / cols];
    float v;
    if constexpr (FP8) {
      __nv_fp8_e4m3 f;
      *reinterpret_cast<uint8_t*>(&f) = q[i];
      v = static_cast<float>(f);
    } else {
      v = static_cast<float>(static_cast<int8_t>(q[i]));
    }
    out[i] = __float2bfloat16(v * s);
  }
}

int grid_for(long n, int threads) {
  const long b = (n + threads - 1) / threads;
  return static_cast<int>(std::max<long>(1, std::min<long>(b, 148L * 16)));
}

}  // namespace

void int4_flat_dequant(const torch::Tensor& qweight, const torch::Tensor& scales, const torch::Tensor& qzeros,
                       const c10::optional<torch::Tensor>& g_idx, torch::Tensor& out) {
  TORCH_CHECK(qweight.is_cuda() && scales.is_cuda() && qzeros.is_cuda() && out.is_cuda(),
              "int4 dequant: CUDA tensors");
  TORCH_CHECK(qweight.scalar_type() == at::kInt && qzeros.scalar_type() == at::kInt, "int4 dequant: int32 words");
  TORCH_CHECK(scales.scalar_type() == at::kFloat, "int4 dequant: fp32 scales");
  TORCH_CHECK(qweight.is_contiguous() && scales.is_contiguous() && qzeros.is_contiguous() && out.is_contiguous(),
              "int4 dequant: contiguous tensors");
  const long n = out.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int32_t* gi = nullptr;
  long ng = 0;
  if (g_idx.has_value() && g_idx->defined()) {
    TORCH_CHECK(g_idx->scalar_type() == at::kInt && g_idx->is_contiguous(), "int4 dequant: g_idx int32");
    gi = g_idx->data_ptr<int32_t>();
    ng = g_idx->numel();
  }
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(qweight.data_ptr<int32_t>());
  const uint32_t* qz = reinterpret_cast<const uint32_t*>(qzeros.data_ptr<int32_t>());
  const int g = grid_for(n, 256);
  switch (out.scalar_type()) {
    case at::kBFloat16:
      int4_flat_dequant_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(
          qw, qweight.numel(), scales.data_ptr<float>(), scales.numel(), qz, qzeros.numel(), gi, ng, n,
          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
      break;
    case at::kHalf:
      int4_flat_dequant_kernel<__half><<<g, 256, 0, st>>>(qw, qweight.numel(), scales.data_ptr<float>(),
                                                          scales.numel(), qz, qzeros.numel(), gi, ng, n,
                                                          reinterpret_cast<__half*>(out.data_ptr()));
      break;
    case at::kFloat:
      int4_flat_dequant_kernel<float><<<g, 256, 0, st>>>(qw, qweight.numel(), scales.data_ptr<float>(),
                                                         scales.numel(), qz, qzeros.numel(), gi, ng, n,
                                                         out.data_ptr<float>());
      break;
    default:
      TORCH_CHECK(false, "int4 dequant: out must be bf16, fp16 or fp32");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gptq_dequant(const torch::Tensor& qweight, const torch::Tensor& qzeros, const torch::Tensor& scales,
                  const torch::Tensor& g_idx, torch::Tensor& out) {
  TORCH_CHECK(qweight.scalar_type() == at::kInt && qzeros.scalar_type() == at::kInt, "gptq: int32 words");
  TORCH_CHECK(scales.scalar_type() == at::kHalf && g_idx.scalar_type() == at::kInt, "gptq: fp16 scales, int32 g_idx");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2, "gptq: out bf16 [N, K]");
  const int N = out.size(0), K = out.size(1);
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "gptq: K and N must be multiples of 8");
  TORCH_CHECK(qweight.size(0) == K / 8 && qweight.size(1) == N, "gptq: qweight [K/8, N]");
  TORCH_CHECK(qzeros.size(1) == N / 8 && scales.size(1) == N && qzeros.size(0) == scales.size(0),
              "gptq: qzeros [G, N/8], scales [G, N]");
  TORCH_CHECK(g_idx.numel() == K, "gptq: g_idx [K]");
  TORCH_CHECK(qweight.is_contiguous() && qzeros.is_contiguous() && scales.is_contiguous() && g_idx.is_contiguous() &&
                  out.is_contiguous(),
              "gptq: contiguous tensors");
  if (out.numel() == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  gptq_dequant_kernel<<<grid_for((long)(K / 8) * N, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      qweight.data_ptr<int32_t>(), qzeros.data_ptr<int32_t>(), reinterpret_cast<const __half*>(scales.data_ptr()),
      g_idx.data_ptr<int32_t>(), K, N, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void awq_dequant(const torch::Tensor& qweight, const torch::Tensor& qzeros, const torch::Tensor& scales,
                 int64_t group, torch::Tensor& out) {
  TORCH_CHECK(qweight.scalar_type() == at::kInt && qzeros.scalar_type() == at::kInt, "awq: int32 words");
  TORCH_CHECK(scales.scalar_type() == at::kHalf, "awq: fp16 scales");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2, "awq: out bf16 [N, K]");
  const int N = out.size(0), K = out.size(1);
  TORCH_CHECK(N % 8 == 0 && group > 0 && K % group == 0, "awq: N multiple of 8, K multiple of the group");
  TORCH_CHECK(qweight.size(0) == K && qweight.size(1) == N / 8, "awq: qweight [K, N/8]");
  TORCH_CHECK(qzeros.size(0) == K / group && qzeros.size(1) == N / 8, "awq: qzeros [K/group, N/8]");
  TORCH_CHECK(scales.size(0) == K / group && scales.size(1) == N, "awq: scales [K/group, N]");
  TORCH_CHECK(qweight.is_contiguous() && qzeros.is_contiguous() && scales.is_contiguous() && out.is_contiguous(),
              "awq: contiguous tensors");
  if (out.numel() == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  awq_dequant_kernel<<<grid_for((long)K * (N / 8), 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      qweight.data_ptr<int32_t>(), qzeros.data_ptr<int32_t>(), reinterpret_cast<const __half*>(scales.data_ptr()), K,
      N, int(group), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void bnb4_dequant(const torch::Tensor& packed, const torch::Tensor& scale, int64_t block, bool nf4,
                  torch::Tensor& out) {
  TORCH_CHECK(packed.scalar_type() == at::kByte && packed.is_contiguous(), "bnb4: packed uint8");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.is_contiguous(), "bnb4: fp32 scale");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == 2 * packed.numel(),
              "bnb4: out bf16 with two elements per byte");
  TORCH_CHECK(block > 0 && scale.numel() * block >= out.numel(), "bnb4: one scale per block of outputs");
  if (packed.numel() == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int g = grid_for(packed.numel(), 256);
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (nf4)
    bnb4_dequant_kernel<true><<<g, 256, 0, st>>>(packed.data_ptr<uint8_t>(), packed.numel(), scale.data_ptr<float>(),
                                                 block, o);
  else
    bnb4_dequant_kernel<false><<<g, 256, 0, st>>>(packed.data_ptr<uint8_t>(), packed.numel(),
                                                  scale.data_ptr<float>(), block, o);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_row_quant(const torch::Tensor& x, torch::Tensor& q, torch::Tensor& scales, bool fp8) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(), "kv quant: x bf16 [rows, cols]");
  TORCH_CHECK(q.scalar_type() == at::kByte && q.sizes() == x.sizes() && q.is_contiguous(), "kv quant: q uint8");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.numel() == x.size(0), "kv quant: fp32 scale per row");
  if (x.numel() == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const long rows = x.size(0);
  const int grid = static_cast<int>(std::min<long>((rows + 7) / 8, 148L * 16));
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  if (fp8)
    kv_row_quant_kernel<true><<<grid, 256, 0, st>>>(xp, rows, x.size(1), q.data_ptr<uint8_t>(),
                                                    scales.data_ptr<float>());
  else
    kv_row_quant_kernel<false><<<grid, 256, 0, st>>>(xp, rows, x.size(1), q.data_ptr<uint8_t>(),
                                                     scales.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_row_dequant(const torch::Tensor& q, const torch::Tensor& scales, torch::Tensor& out, bool fp8) {
  TORCH_CHECK(q.scalar_type() == at::kByte && q.dim() == 2 && q.is_contiguous(), "kv dequant: q uint8 [rows, cols]");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.numel() == q.size(0), "kv dequant: fp32 scale per row");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.sizes() == q.sizes() && out.is_contiguous(),
              "kv dequant: out bf16");
  if (q.numel() == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int g = grid_for(q.numel(), 256);
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (fp8)
    kv_row_dequant_kernel<true><<<g, 256, 0, st>>>(q.data_ptr<uint8_t>(), scales.data_ptr<float>(), q.size(0),
                                                   q.size(1), o);
  else
    kv_row_dequant_kernel<false><<<g, 256, 0, st>>>(q.data_ptr<uint8_t>(), scales.data_ptr<float>(), q.size(0),
                                                    q.size(1), o);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
