// Encoder (BERT / MiniLM) kernels for sentence embeddings over packed
// variable-length batches (no padding tokens are computed):
//
//   bert_embed_ln      x[t] = LayerNorm(word[id] + pos[p] + type[tt])
//   varlen_attention   non-causal softmax(q k^T * scale) v per (sequence, head),
//                      head_dim 32 / 64, sequences up to 512 tokens: tensor-core
//                      (mma.sync) FlashAttention-2 tiles over the head's K / V
//                      staged in shared memory; a scalar one-warp-per-query
//                      kernel remains for unaligned inputs (BLOOM_BERT_ATTN_TC=0)
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

// Kernels below are instantiated for bf16 (the tensor-core path) and fp32
// (the full-precision path: fp32 weights and activations end to end).
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

// one CTA per token; H <= 1024 (one element per thread)
template <typename T>
__global__ void bert_embed_ln_kernel(const int* __restrict__ ids, const int* __restrict__ pos,
                                     const int* __restrict__ types, const T* __restrict__ word,
                                     const T* __restrict__ pemb, const T* __restrict__ temb,
                                     const T* __restrict__ g, const T* __restrict__ b,
                                     T* __restrict__ out, int H, int V, int P, float eps) {
  __shared__ float red[33];
  const long t = blockIdx.x;
  const int i = threadIdx.x;
  int id = ids[t];
  id = id < 0 || id >= V ? 0 : id;
  int p = pos[t];
  p = p < 0 ? 0 : (p >= P ? P - 1 : p);
  const int tt = types != nullptr ? types[t] : 0;
  float v = 0.f;
  if (i < H) v = to_f(word[(long)id * H + i]) + to_f(pemb[(long)p * H + i]) + to_f(temb[(long)tt * H + i]);
  const float mean = block_sum_b(i < H ? v : 0.f, red) / H;
  const float d = i < H ? v - mean : 0.f;
  const float inv = rsqrtf(block_sum_b(d * d, red) / H + eps);
  if (i < H) out[t * H + i] = from_f<T>(d * inv * to_f(g[i]) + to_f(b[i]));
}

// fp32 path: out = LayerNorm(delta + resid) per row; one CTA per row, H <= 1024
__global__ void ln_residual_f32_kernel(const float* __restrict__ delta, const float* __restrict__ resid,
                                       const float* __restrict__ g, const float* __restrict__ b,
                                       float* __restrict__ out, int H, float eps) {
  __shared__ float red[33];
  const long t = blockIdx.x;
  const int i = threadIdx.x;
  const float v = i < H ? delta[t * H + i] + resid[t * H + i] : 0.f;
  const float mean = block_sum_b(v, red) / H;
  const float d = i < H ? v - mean : 0.f;
  const float inv = rsqrtf(block_sum_b(d * d, red) / H + eps);
  if (i < H) out[t * H + i] = d * inv * g[i] + b[i];
}

// fp32 path: exact (erf) GELU in place
__global__ void gelu_f32_kernel(float* __restrict__ x, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = x[i];
    x[i] = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
  }
}

// qkv: [T, 3 * NH * D] (q | k | v); out: [T, NH * D].  grid (num_seqs, NH), block 256 threads.
template <int D, typename T>
__global__ void varlen_attention_kernel(const T* __restrict__ qkv, const int* __restrict__ cu,
                                        T* __restrict__ out, int NH, float scale) {
  extern __shared__ float sm[];
  const int s = blockIdx.x, h = blockIdx.y;
  const int t0 = cu[s], L = cu[s + 1] - t0;
  float* Ks = sm;                 // [L][D]
  float* Vs = sm + (long)L * D;   // [L][D]
  const long ld = 3L * NH * D;
  for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
    const int j = idx / D, d = idx - j * D;
    const T* row = qkv + (long)(t0 + j) * ld;
    Ks[idx] = to_f(row[(long)NH * D + h * D + d]);
    Vs[idx] = to_f(row[2L * NH * D + h * D + d]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  constexpr int PER = (D + 31) / 32;  // dims per lane
  for (int qi = warp; qi < L; qi += nw) {
    const T* qrow = qkv + (long)(t0 + qi) * ld + h * D;
    float q[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int d = lane + 32 * k;
      q[k] = d < D ? to_f(qrow[d]) * scale : 0.f;
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
    T* orow = out + (long)(t0 + qi) * NH * D + h * D;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int d = lane + 32 * k;
      if (d < D) orow[d] = from_f<T>(o[k] / l);
    }
  }
}

// Tensor-core variant (mma.sync m16n8k16, bf16 in, f32 accumulate) for
// head_dim 32 / 64: grid (num_seqs, NH, query tiles of 64 rows), 4 warps of
// 16 query rows.  The head's K and V rows (zero-padded to a multiple of 16
// keys) are staged in shared memory as bf16; each warp runs FlashAttention-2
// style over 16-key tiles: S = Q K^T into registers, online softmax in the
// base-2 domain, P re-packed from the S accumulators straight into the A
// operand of P V.  Keys past the sequence end are masked to -inf.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_raw(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  __nv_bfloat162 v;
  v.x = lo;
  v.y = hi;
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int D>
__global__ void __launch_bounds__(128) varlen_attention_tc_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                                  const int* __restrict__ cu,
                                                                  __nv_bfloat16* __restrict__ out, int NH,
                                                                  float scale_log2) {
  constexpr int KC = D / 16;  // k-chunks of Q K^T
  constexpr int NB = D / 8;   // n-blocks of the output
  extern __shared__ __align__(16) uint8_t smraw[];
  const int s = blockIdx.x, h = blockIdx.y;
  const int t0 = cu[s], L = cu[s + 1] - t0;
  const int q0 = blockIdx.z * 64;
  if (q0 >= L) return;
  const int Lp = (L + 15) & ~15;
  // rows padded by 8 elements (16 bytes): the 8 key rows one MMA fragment
  // load touches then fall into distinct shared-memory banks
  constexpr int RS = D + 8;
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(smraw);  // [Lp][RS]
  __nv_bfloat16* Vs = Ks + (long)Lp * RS;                       // [Lp][RS]
  const long ld = 3L * NH * D;
  constexpr int VEC = D / 8;  // 16-byte vectors per row
  for (int idx = threadIdx.x; idx < Lp * VEC; idx += blockDim.x) {
    const int j = idx / VEC, c = idx - j * VEC;
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (j < L) {
      const __nv_bfloat16* row = qkv + (long)(t0 + j) * ld;
      kv = *reinterpret_cast<const uint4*>(row + (long)NH * D + h * D + c * 8);
      vv = *reinterpret_cast<const uint4*>(row + 2L * NH * D + h * D + c * 8);
    }
    *reinterpret_cast<uint4*>(Ks + (long)j * RS + c * 8) = kv;
    *reinterpret_cast<uint4*>(Vs + (long)j * RS + c * 8) = vv;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;  // this thread's two query rows
  if (q0 + warp * 16 >= L) return;
  // Q fragments (A operand, row-major 16 x 16 per k-chunk)
  uint32_t qf[KC][4];
  const __nv_bfloat16* qb = qkv + (long)t0 * ld + h * D;
  const __nv_bfloat16 zero = __float2bfloat16(0.f);
#pragma unroll
  for (int kc = 0; kc < KC; ++kc) {
    const int c0 = kc * 16 + t4 * 2;
    const __nv_bfloat16* p0 = qb + (long)r0 * ld;
    const __nv_bfloat16* p1 = qb + (long)r1 * ld;
    const bool v0 = r0 < L, v1 = r1 < L;
    qf[kc][0] = v0 ? *reinterpret_cast<const uint32_t*>(p0 + c0) : pack_raw(zero, zero);
    qf[kc][1] = v1 ? *reinterpret_cast<const uint32_t*>(p1 + c0) : pack_raw(zero, zero);
    qf[kc][2] = v0 ? *reinterpret_cast<const uint32_t*>(p0 + c0 + 8) : pack_raw(zero, zero);
    qf[kc][3] = v1 ? *reinterpret_cast<const uint32_t*>(p1 + c0 + 8) : pack_raw(zero, zero);
  }
  float o[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  for (int kt = 0; kt < Lp; kt += 16) {
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      const __nv_bfloat16* krow = Ks + (long)(kt + nt * 8 + g) * RS;  // key n = g of this n-block
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + kc * 16 + t4 * 2);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + kc * 16 + t4 * 2 + 8);
        mma16816(sc[nt], qf[kc], b0, b1);
      }
    }
    // scale, mask, online softmax (rows r0: elements 0,1; r1: elements 2,3)
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kt + nt * 8 + t4 * 2 + (e & 1);
        sc[nt][e] = key < L ? sc[nt][e] * scale_log2 : -INFINITY;
        if (e < 2) mx0 = fmaxf(mx0, sc[nt][e]);
        else mx1 = fmaxf(mx1, sc[nt][e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = exp2f(m0 - mx0), c1 = exp2f(m1 - mx1);  // m = -inf at the start: exp2(-inf) = 0
    m0 = mx0;
    m1 = mx1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(sc[nt][e] - (e < 2 ? mx0 : mx1));
        sc[nt][e] = p;
        if (e < 2) ps0 += p;
        else ps1 += p;
      }
    l0 = l0 * c0 + ps0;  // per-thread partial row sums; combined over the quad at the end
    l1 = l1 * c1 + ps1;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      o[nb][0] *= c0;
      o[nb][1] *= c0;
      o[nb][2] *= c1;
      o[nb][3] *= c1;
    }
    // P (16 q x 16 keys) as the A operand of P V
    uint32_t pa[4];
    pa[0] = pack_bf16(sc[0][0], sc[0][1]);
    pa[1] = pack_bf16(sc[0][2], sc[0][3]);
    pa[2] = pack_bf16(sc[1][0], sc[1][1]);
    pa[3] = pack_bf16(sc[1][2], sc[1][3]);
    const __nv_bfloat16* v0r = Vs + (long)(kt + t4 * 2) * RS;  // keys t4*2, t4*2+1 (and +8, +9)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int d = nb * 8 + g;
      const uint32_t b0 = pack_raw(v0r[d], v0r[RS + d]);
      const uint32_t b1 = pack_raw(v0r[8 * RS + d], v0r[9 * RS + d]);
      mma16816(o[nb], pa, b0, b1);
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.f / l0, i1 = 1.f / l1;
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    const int d = nb * 8 + t4 * 2;
    if (r0 < L)
      *reinterpret_cast<uint32_t*>(out + (long)(t0 + r0) * NH * D + h * D + d) = pack_bf16(o[nb][0] * i0, o[nb][1] * i0);
    if (r1 < L)
      *reinterpret_cast<uint32_t*>(out + (long)(t0 + r1) * NH * D + h * D + d) = pack_bf16(o[nb][2] * i1, o[nb][3] * i1);
  }
}

// one CTA per sequence; out f32 [S, H]
template <typename T>
__global__ void mean_pool_l2_kernel(const T* __restrict__ x, const int* __restrict__ cu,
                                    float* __restrict__ out, int H, int normalize) {
  __shared__ float red[33];
  const int s = blockIdx.x;
  const int t0 = cu[s], L = cu[s + 1] - t0;
  const int i = threadIdx.x;
  float acc = 0.f;
  if (i < H)
    for (int j = 0; j < L; ++j) acc += to_f(x[(long)(t0 + j) * H + i]);
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
  TORCH_CHECK(out.scalar_type() == word.scalar_type(), "bert_embed_ln: out and tables share a dtype");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(ids.device());
  const int threads = ((H + 31) / 32) * 32;
  auto st = at::cuda::getCurrentCUDAStream();
  const int* tp = types.has_value() ? types->data_ptr<int>() : nullptr;
  if (word.scalar_type() == at::kFloat) {
    bert_embed_ln_kernel<float><<<T, threads, 0, st>>>(
        ids.data_ptr<int>(), pos.data_ptr<int>(), tp, word.data_ptr<float>(), pemb.data_ptr<float>(),
        temb.data_ptr<float>(), g.data_ptr<float>(), b.data_ptr<float>(), out.data_ptr<float>(), H, word.size(0),
        pemb.size(0), float(eps));
  } else {
    TORCH_CHECK(word.scalar_type() == at::kBFloat16, "bert_embed_ln: bf16 or fp32 tables");
    bert_embed_ln_kernel<__nv_bfloat16><<<T, threads, 0, st>>>(
        ids.data_ptr<int>(), pos.data_ptr<int>(), tp, reinterpret_cast<const __nv_bfloat16*>(word.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(pemb.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(temb.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), H, word.size(0), pemb.size(0), float(eps));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ln_residual_f32(const torch::Tensor& delta, const torch::Tensor& resid, const torch::Tensor& g,
                     const torch::Tensor& b, torch::Tensor& out, double eps) {
  TORCH_CHECK(delta.scalar_type() == at::kFloat && resid.scalar_type() == at::kFloat && delta.is_contiguous() &&
                  resid.is_contiguous() && out.is_contiguous(), "ln_residual_f32: contiguous fp32 [T, H]");
  const int T = delta.size(0), H = delta.size(1);
  TORCH_CHECK(H <= 1024, "ln_residual_f32: hidden size <= 1024");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(delta.device());
  ln_residual_f32_kernel<<<T, ((H + 31) / 32) * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      delta.data_ptr<float>(), resid.data_ptr<float>(), g.data_ptr<float>(), b.data_ptr<float>(),
      out.data_ptr<float>(), H, float(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gelu_f32_(torch::Tensor& x) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous(), "gelu_f32_: contiguous fp32");
  const long n = x.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  const int blocks = static_cast<int>(std::min<long>((n + 255) / 256, 148L * 16));
  gelu_f32_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void varlen_attention(const torch::Tensor& qkv, const torch::Tensor& cu_seqlens, torch::Tensor& out, int64_t num_heads,
                      int64_t head_dim, int64_t max_len, double scale) {
  const int S = cu_seqlens.numel() - 1;
  if (S <= 0) return;
  TORCH_CHECK(head_dim == 32 || head_dim == 64, "varlen_attention: head_dim 32 or 64");
  TORCH_CHECK(max_len <= 512, "varlen_attention: sequences up to 512 tokens");
  const at::cuda::CUDAGuard guard(qkv.device());
  auto s = at::cuda::getCurrentCUDAStream();
  static const bool tc = [] {
    const char* e = std::getenv("BLOOM_BERT_ATTN_TC");
    return e == nullptr || std::atoi(e) != 0;
  }();
  const bool aligned = reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0 && qkv.is_contiguous() &&
                       out.is_contiguous() && reinterpret_cast<uintptr_t>(out.data_ptr()) % 4 == 0;
  if (tc && aligned && qkv.scalar_type() == at::kBFloat16) {
    const int Lp = int((max_len + 15) / 16 * 16);
    const size_t smem_tc = 2 * size_t(Lp) * (head_dim + 8) * sizeof(__nv_bfloat16);
    dim3 g3(S, num_heads, int((max_len + 63) / 64));
    if (head_dim == 32) {
      cudaFuncSetAttribute(varlen_attention_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 512 * 40 * 2);
      varlen_attention_tc_kernel<32><<<g3, 128, smem_tc, s>>>(
          reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), cu_seqlens.data_ptr<int>(),
          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(num_heads), float(scale * 1.4426950408889634));
    } else {
      cudaFuncSetAttribute(varlen_attention_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 512 * 72 * 2);
      varlen_attention_tc_kernel<64><<<g3, 128, smem_tc, s>>>(
          reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), cu_seqlens.data_ptr<int>(),
          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(num_heads), float(scale * 1.4426950408889634));
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const size_t smem = 2 * size_t(max_len) * head_dim * sizeof(float);
  dim3 grid(S, num_heads);
  if (qkv.scalar_type() == at::kFloat) {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "varlen_attention: fp32 qkv needs an fp32 output");
    if (head_dim == 32) {
      cudaFuncSetAttribute(varlen_attention_kernel<32, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           2 * 512 * 32 * 4);
      varlen_attention_kernel<32, float><<<grid, 256, smem, s>>>(qkv.data_ptr<float>(), cu_seqlens.data_ptr<int>(),
                                                                 out.data_ptr<float>(), int(num_heads), float(scale));
    } else {
      cudaFuncSetAttribute(varlen_attention_kernel<64, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           2 * 512 * 64 * 4);
      varlen_attention_kernel<64, float><<<grid, 256, smem, s>>>(qkv.data_ptr<float>(), cu_seqlens.data_ptr<int>(),
                                                                 out.data_ptr<float>(), int(num_heads), float(scale));
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  if (head_dim == 32) {
    cudaFuncSetAttribute(varlen_attention_kernel<32, __nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         2 * 512 * 32 * 4);
    varlen_attention_kernel<32, __nv_bfloat16><<<grid, 256, smem, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), cu_seqlens.data_ptr<int>(),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(num_heads), float(scale));
  } else {
    cudaFuncSetAttribute(varlen_attention_kernel<64, __nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         2 * 512 * 64 * 4);
    varlen_attention_kernel<64, __nv_bfloat16><<<grid, 256, smem, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), cu_seqlens.data_ptr<int>(),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(num_heads), float(scale));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mean_pool_l2(const torch::Tensor& x, const torch::Tensor& cu_seqlens, torch::Tensor& out, bool normalize) {
  const int S = cu_seqlens.numel() - 1, H = x.size(1);
  TORCH_CHECK(H <= 1024, "mean_pool_l2: hidden size <= 1024");
  if (S <= 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kFloat)
    mean_pool_l2_kernel<float><<<S, ((H + 31) / 32) * 32, 0, st>>>(x.data_ptr<float>(), cu_seqlens.data_ptr<int>(),
                                                                  out.data_ptr<float>(), H, normalize ? 1 : 0);
  else
    mean_pool_l2_kernel<__nv_bfloat16><<<S, ((H + 31) / 32) * 32, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), cu_seqlens.data_ptr<int>(), out.data_ptr<float>(), H,
        normalize ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
