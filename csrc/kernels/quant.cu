// GGUF block-quantised weights on the GPU: Q8_0 and Q4_0 (32-element blocks,
// one fp16 scale each), kept quantised in HBM.
//
// Device layout (repacked from the GGUF blocks at load, bit-exact): the
// scales of a row form an fp16 plane [N, K/32]; the quants an aligned plane
// -- Q8_0: int8 [N, K] (value = q * d); Q4_0: uint8 [N, K/2] where byte j of a
// block holds element j in its low nibble and element j + 16 in its high
// nibble (value = (nibble - 8) * d), exactly the GGUF block order.  Splitting
// the 34 / 18-byte blocks into planes makes every load 16-byte aligned.
//
//   qgemv      decode (M <= 8 tokens): y = x W^T straight from the quantised
//              rows -- each warp owns two weight rows (for SwiGLU the gate row
//              and its up row), its lanes stride over the 32-element blocks,
//              dequantise in registers and accumulate fp32 for every token;
//              weights are read from HBM exactly once per call.
//   qdequant   prefill: rows -> bf16 scratch that the tcgen05 GEMM consumes.
//
// Reference behaviour: candle quantized qmatmul (executor/candle.rs:1533-1568)
// and the CPU Q8_0 / Q4_0 dequantisers (GGML block formats).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp16.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {
namespace {

constexpr int kWarps = 8;

template <int KIND>
__device__ __forceinline__ void load_block(const uint8_t* qs, long row, int nbk, int blk, float (&w)[32]) {
  if constexpr (KIND == 0) {  // Q8_0: 32 int8
    const int4* p = reinterpret_cast<const int4*>(qs + (row * nbk + blk) * 32);
    const int4 a = p[0], b = p[1];
    const int8_t* ea = reinterpret_cast<const int8_t*>(&a);
    const int8_t* eb = reinterpret_cast<const int8_t*>(&b);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      w[j] = float(ea[j]);
      w[16 + j] = float(eb[j]);
    }
  } else {  // Q4_0: 16 bytes, low nibbles = elements 0..15, high = 16..31
    const int4 a = *reinterpret_cast<const int4*>(qs + (row * nbk + blk) * 16);
    const uint8_t* e = reinterpret_cast<const uint8_t*>(&a);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      w[j] = float(int(e[j] & 0x0F) - 8);
      w[16 + j] = float(int(e[j] >> 4) - 8);
    }
  }
}

// EPI: 0 bf16 out, 2 SwiGLU (row pair = gate, up), 4 residual add
template <int KIND, int EPI, int MT>
__global__ void __launch_bounds__(kWarps * 32)
    qgemv_kernel(const __nv_bfloat16* __restrict__ x, int M, int K, const uint8_t* __restrict__ qs,
                 const __half* __restrict__ sc, int N, __nv_bfloat16* __restrict__ out, long ldo,
                 const __nv_bfloat16* __restrict__ resid, long ldr) {
  const int warp = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int nbk = K / 32;
  // two weight rows per warp
  long r0, r1;
  int f0, f1;  // output columns
  if constexpr (EPI == 2) {
    const int f = warp;  // output feature
    if (f >= N / 2) return;
    const int g = f / 16, j = f % 16;
    r0 = long(g) * 32 + j;       // gate row
    r1 = r0 + 16;                // up row
    f0 = f1 = f;
  } else {
    r0 = long(warp) * 2;
    if (r0 >= N) return;
    r1 = r0 + 1 < N ? r0 + 1 : r0;
    f0 = int(r0);
    f1 = int(r0 + 1);
  }
  float acc0[MT], acc1[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc0[m] = acc1[m] = 0.f;
  for (int blk = lane; blk < nbk; blk += 32) {
    float w0[32], w1[32];
    load_block<KIND>(qs, r0, nbk, blk, w0);
    load_block<KIND>(qs, r1, nbk, blk, w1);
    const float d0 = __half2float(sc[r0 * nbk + blk]);
    const float d1 = __half2float(sc[r1 * nbk + blk]);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m >= M) break;
      const int4* xp = reinterpret_cast<const int4*>(x + long(m) * K + blk * 32);
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int4 raw = xp[v];
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float xv = __bfloat162float(e[q]);
          s0 = fmaf(w0[v * 8 + q], xv, s0);
          s1 = fmaf(w1[v * 8 + q], xv, s1);
        }
      }
      acc0[m] = fmaf(s0, d0, acc0[m]);
      acc1[m] = fmaf(s1, d1, acc1[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    acc0[m] = warp_sum(acc0[m]);
    acc1[m] = warp_sum(acc1[m]);
  }
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m >= M) break;
      if constexpr (EPI == 2) {
        out[long(m) * ldo + f0] = __float2bfloat16(silu(acc0[m]) * acc1[m]);
      } else {
        float a = acc0[m], b = acc1[m];
        if constexpr (EPI == 4) {
          a += __bfloat162float(resid[long(m) * ldr + f0]);
          if (f1 < N) b += __bfloat162float(resid[long(m) * ldr + f1]);
        }
        out[long(m) * ldo + f0] = __float2bfloat16(a);
        if (f1 < N) out[long(m) * ldo + f1] = __float2bfloat16(b);
      }
    }
  }
}

template <int KIND>
__global__ void qdequant_kernel(const uint8_t* __restrict__ qs, const __half* __restrict__ sc, long nblocks,
                                __nv_bfloat16* __restrict__ out) {
  const long b = blockIdx.x * long(blockDim.x) + threadIdx.x;
  if (b >= nblocks) return;
  float w[32];
  if constexpr (KIND == 0) {
    const int4* p = reinterpret_cast<const int4*>(qs + b * 32);
    const int4 a = p[0], c = p[1];
    const int8_t* ea = reinterpret_cast<const int8_t*>(&a);
    const int8_t* ec = reinterpret_cast<const int8_t*>(&c);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      w[j] = float(ea[j]);
      w[16 + j] = float(ec[j]);
    }
  } else {
    const int4 a = *reinterpret_cast<const int4*>(qs + b * 16);
    const uint8_t* e = reinterpret_cast<const uint8_t*>(&a);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      w[j] = float(int(e[j] & 0x0F) - 8);
      w[16 + j] = float(int(e[j] >> 4) - 8);
    }
  }
  const float d = __half2float(sc[b]);
  int4 o[4];
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(o);
#pragma unroll
  for (int j = 0; j < 32; ++j) ob[j] = __float2bfloat16(w[j] * d);
  int4* dst = reinterpret_cast<int4*>(out + b * 32);
#pragma unroll
  for (int v = 0; v < 4; ++v) dst[v] = o[v];
}

template <int KIND, int EPI>
void launch_qgemv(int MT, dim3 grid, cudaStream_t s, const __nv_bfloat16* x, int M, int K, const uint8_t* qs,
                  const __half* sc, int N, __nv_bfloat16* out, long ldo, const __nv_bfloat16* resid, long ldr) {
  switch (MT) {
    case 1: qgemv_kernel<KIND, EPI, 1><<<grid, kWarps * 32, 0, s>>>(x, M, K, qs, sc, N, out, ldo, resid, ldr); break;
    case 2: qgemv_kernel<KIND, EPI, 2><<<grid, kWarps * 32, 0, s>>>(x, M, K, qs, sc, N, out, ldo, resid, ldr); break;
    case 4: qgemv_kernel<KIND, EPI, 4><<<grid, kWarps * 32, 0, s>>>(x, M, K, qs, sc, N, out, ldo, resid, ldr); break;
    default: qgemv_kernel<KIND, EPI, 8><<<grid, kWarps * 32, 0, s>>>(x, M, K, qs, sc, N, out, ldo, resid, ldr); break;
  }
}

}  // namespace

void qgemv(const torch::Tensor& x, const torch::Tensor& qs, const torch::Tensor& scales, int64_t kind,
           torch::Tensor& out, int64_t epi, const c10::optional<torch::Tensor>& resid) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "qgemv: x bf16 contiguous");
  TORCH_CHECK(scales.scalar_type() == at::kHalf && scales.is_contiguous() && qs.is_contiguous(), "qgemv: layout");
  const int M = x.size(0), K = x.size(1), N = scales.size(0);
  TORCH_CHECK(M >= 1 && M <= 8, "qgemv: 1..8 tokens (larger batches dequantise into the tcgen05 GEMM)");
  TORCH_CHECK(K % 32 == 0 && scales.size(1) == K / 32, "qgemv: K must be whole 32-element blocks");
  TORCH_CHECK(kind == 0 ? qs.numel() == (int64_t)N * K : qs.numel() == (int64_t)N * K / 2, "qgemv: quant plane size");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(-1) == 1, "qgemv: out bf16");
  const __nv_bfloat16* rp = nullptr;
  long ldr = 0;
  if (epi == kEpiResidual) {
    TORCH_CHECK(resid.has_value() && resid->scalar_type() == at::kBFloat16, "qgemv: residual epilogue needs resid");
    rp = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
    ldr = resid->stride(0);
  } else {
    TORCH_CHECK(epi == kEpiBF16 || epi == kEpiSwiGLU, "qgemv: bf16, SwiGLU or residual epilogue");
  }
  if (epi == kEpiSwiGLU) TORCH_CHECK(N % 32 == 0 && out.size(-1) == N / 2, "qgemv swiglu: out [M, N/2]");
  const at::cuda::CUDAGuard g(x.device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const int warps = epi == kEpiSwiGLU ? N / 2 : (N + 1) / 2;
  const dim3 grid((warps + kWarps - 1) / kWarps);
  const int MT = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* qp = reinterpret_cast<const uint8_t*>(qs.data_ptr());
  auto* sp = reinterpret_cast<const __half*>(scales.data_ptr());
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const long ldo = out.stride(0);
  if (kind == 0) {
    if (epi == kEpiSwiGLU) launch_qgemv<0, 2>(MT, grid, s, xp, M, K, qp, sp, N, op, ldo, rp, ldr);
    else if (epi == kEpiResidual) launch_qgemv<0, 4>(MT, grid, s, xp, M, K, qp, sp, N, op, ldo, rp, ldr);
    else launch_qgemv<0, 0>(MT, grid, s, xp, M, K, qp, sp, N, op, ldo, rp, ldr);
  } else {
    TORCH_CHECK(kind == 1, "qgemv: kind 0 (Q8_0) or 1 (Q4_0)");
    if (epi == kEpiSwiGLU) launch_qgemv<1, 2>(MT, grid, s, xp, M, K, qp, sp, N, op, ldo, rp, ldr);
    else if (epi == kEpiResidual) launch_qgemv<1, 4>(MT, grid, s, xp, M, K, qp, sp, N, op, ldo, rp, ldr);
    else launch_qgemv<1, 0>(MT, grid, s, xp, M, K, qp, sp, N, op, ldo, rp, ldr);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qdequant(const torch::Tensor& qs, const torch::Tensor& scales, int64_t kind, torch::Tensor& out) {
  TORCH_CHECK(scales.scalar_type() == at::kHalf && scales.is_contiguous() && qs.is_contiguous(), "qdequant: layout");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous(), "qdequant: out bf16 contiguous");
  const long nblocks = scales.numel();
  TORCH_CHECK(out.numel() == nblocks * 32, "qdequant: out must hold N*K elements");
  if (nblocks == 0) return;
  const at::cuda::CUDAGuard g(qs.device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const int threads = 256;
  const long blocks = (nblocks + threads - 1) / threads;
  auto* qp = reinterpret_cast<const uint8_t*>(qs.data_ptr());
  auto* sp = reinterpret_cast<const __half*>(scales.data_ptr());
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (kind == 0)
    qdequant_kernel<0><<<blocks, threads, 0, s>>>(qp, sp, nblocks, op);
  else
    qdequant_kernel<1><<<blocks, threads, 0, s>>>(qp, sp, nblocks, op);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
