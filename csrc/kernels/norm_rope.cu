// Memory-bound per-token kernels: RMSNorm (with fused residual add and fused
// split-K reduction), LayerNorm (BERT), embedding gather, and RoPE fused with
// the paged KV-cache write.
//
// Reference behaviour: RMSNorm qwen_streaming.rs:300-324, rotary
// qwen_streaming.rs:74-116,387 (HF rotate_half convention), KV append
// qwen_streaming.rs:394-409 / paged write scheduler/paged_cache.rs:208-308
// (host f32 blocks there; HBM-resident bf16 pages here).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {

namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
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

// x: [M, H] bf16 (row stride ldx), out [M, H] (row stride ldo)
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long ldx, const __nv_bfloat16* __restrict__ w,
                               __nv_bfloat16* __restrict__ out, long ldo, int H, float eps) {
  extern __shared__ float buf[];  // H floats
  __shared__ float red[33];
  const long row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = __bfloat162float(xr[i]);
    buf[i] = v;
    ss += v * v;
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[row * ldo + i] = __float2bfloat16(buf[i] * inv * __bfloat162float(w[i]));
}

// residual[M,H] += delta (bf16 [M,H] or f32 partials [S,M,H]); out = rmsnorm(residual) * w
template <bool kF32Partials>
__global__ void add_rmsnorm_kernel(const void* __restrict__ delta, int S, long ldd, __nv_bfloat16* __restrict__ resid,
                                   long ldr, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                   long ldo, int M, int H, float eps) {
  extern __shared__ float buf[];
  __shared__ float red[33];
  const long row = blockIdx.x;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float d;
    if constexpr (kF32Partials) {
      const float* dp = reinterpret_cast<const float*>(delta);
      d = 0.f;
      for (int s = 0; s < S; ++s) d += dp[((long)s * M + row) * H + i];
    } else {
      d = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(delta)[row * ldd + i]);
    }
    // the residual stream is stored in bf16 (as the checkpoint's dtype)
    const __nv_bfloat16 nb = __float2bfloat16(__bfloat162float(resid[row * ldr + i]) + d);
    resid[row * ldr + i] = nb;
    const float v = __bfloat162float(nb);
    buf[i] = v;
    ss += v * v;
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[row * ldo + i] = __float2bfloat16(buf[i] * inv * __bfloat162float(w[i]));
}

// Vectorised variants: one 16-byte vector (8 x bf16) per thread, the row held
// in registers (H <= 8192, H % 8 == 0, 16-byte aligned rows).
__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 t = __bfloat1622float2(h[k]);
    f[2 * k] = t.x;
    f[2 * k + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
  return u;
}

template <int kMode>  // 0: plain rmsnorm(x); 1: residual += bf16 delta; 2: residual += sum of f32 partials
__global__ void rmsnorm_vec_kernel(const void* __restrict__ delta, int S, long ldd, __nv_bfloat16* __restrict__ resid,
                                   long ldr, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                   long ldo, int M, int H, float eps) {
  __shared__ float red[33];
  const long row = blockIdx.x;
  const int i = threadIdx.x * 8;
  const bool active = i < H;
  float v[8];
  float ss = 0.f;
  if (active) {
    uint4 r = *reinterpret_cast<const uint4*>(resid + row * ldr + i);
    bf16x8_to_f32(r, v);
    if constexpr (kMode == 1) {
      float d[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(delta) + row * ldd + i), d);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] += d[k];
    } else if constexpr (kMode == 2) {
      const float* dp = reinterpret_cast<const float*>(delta);
      for (int sidx = 0; sidx < S; ++sidx) {
        const float4 a = *reinterpret_cast<const float4*>(dp + ((long)sidx * M + row) * H + i);
        const float4 b = *reinterpret_cast<const float4*>(dp + ((long)sidx * M + row) * H + i + 4);
        v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
        v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
      }
    }
    if constexpr (kMode != 0) {
      // the residual stream is stored in bf16 (the checkpoint dtype); normalise the rounded value
      const uint4 nb = f32_to_bf16x8(v);
      *reinterpret_cast<uint4*>(resid + row * ldr + i) = nb;
      bf16x8_to_f32(nb, v);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += v[k] * v[k];
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / H + eps);
  if (active) {
    float wf[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(w + i), wf);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = v[k] * inv * wf[k];
    *reinterpret_cast<uint4*>(out + row * ldo + i) = f32_to_bf16x8(v);
  }
}

bool vec_ok(int H, const void* p, long ld) {
  return (H % 8 == 0) && H <= 8192 && (reinterpret_cast<uintptr_t>(p) % 16 == 0) && (ld % 8 == 0);
}
int vec_threads(int H) { return ((H / 8 + 31) / 32) * 32; }

// LayerNorm with optional residual input (x + resid), affine.
__global__ void layernorm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r,
                                 const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ b,
                                 __nv_bfloat16* __restrict__ out, int H, float eps) {
  extern __shared__ float buf[];
  __shared__ float red[33];
  const long row = blockIdx.x;
  float s = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = __bfloat162float(x[row * H + i]);
    if (r != nullptr) v += __bfloat162float(r[row * H + i]);
    buf[i] = v;
    s += v;
  }
  const float mean = block_sum(s, red) / H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float d = buf[i] - mean;
    ss += d * d;
  }
  const float inv = rsqrtf(block_sum(ss, red) / H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[row * H + i] =
        __float2bfloat16((buf[i] - mean) * inv * __bfloat162float(w[i]) + __bfloat162float(b[i]));
}

__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table, long V,
                                 int H, __nv_bfloat16* __restrict__ out, int* status) {
  const long t = blockIdx.x;
  const long id = ids[t];
  const bool ok = id >= 0 && id < V;  // always bounded: an unknown id embeds as zeros
  if (threadIdx.x == 0) kcheck(ok, status);
  // 16-byte vectors when H is a multiple of 8
  if ((H & 7) == 0) {
    const uint4* src = reinterpret_cast<const uint4*>(table + (ok ? id : 0) * H);
    uint4* dst = reinterpret_cast<uint4*>(out + t * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = ok ? src[i] : make_uint4(0, 0, 0, 0);
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x)
      out[t * H + i] = ok ? table[id * H + i] : __float2bfloat16(0.f);
  }
}

// One warp per head.  Lane l owns dims {l, l+32, l+64, l+96} of a 128-dim
// head, so the rotate_half pairs (d, d+64) stay inside the lane.
// qkv row layout: [q heads | k heads | v heads] x 128.
// cos_sin: [max_pos, 128] f32 = [cos(0..63) | sin(0..63)].
// kv cache: [L, NB, 2, KVH, 16, 128].
// Q8: the cache is int8 with a per-(token, head) fp32 scale (symmetric,
// absmax / 127).  Per layer and block: K pages [KVH][16 tokens][D], V pages
// [KVH][D][16 tokens] (dim-major, so a V page is read as the k = token operand
// of P V without a transpose), then the scales [2][KVH][16] fp32.
// `layer_stride` is then in bytes and `block_bytes` the block's byte size.
template <int D, bool Q8 = false>
__global__ void rope_kv_write_kernel(const __nv_bfloat16* __restrict__ qkv, long ldq, const int64_t* __restrict__ pos,
                                     const int* __restrict__ slots, const float* __restrict__ cos_sin,
                                     __nv_bfloat16* __restrict__ q_out, void* __restrict__ cache_v,
                                     long layer_stride, int nq, int nkv, const __nv_bfloat16* __restrict__ qn,
                                     const __nv_bfloat16* __restrict__ kn, float eps, long max_pos,
                                     long cache_slots, int* status, long block_bytes = 0) {
  __nv_bfloat16* cache = reinterpret_cast<__nv_bfloat16*>(cache_v);
  constexpr int NV = D / 32;  // values per lane: dims lane + 32 i
  const long t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  long p = pos[t];
  p = p < 0 ? 0 : (p >= max_pos ? max_pos - 1 : p);  // the table bounds every read
  int slot = slots != nullptr ? slots[t] : -1;
  if (slot >= 0 && !kcheck(slot < cache_slots, status)) slot = -1;
  const float* cs = cos_sin + p * D;  // [cos(D/2) | sin(D/2)]
  const __nv_bfloat16* row = qkv + t * ldq;
  for (int h = warp; h < nq + 2 * nkv; h += nwarps) {
    const __nv_bfloat16* src = row + (long)h * D;
    float v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = __bfloat162float(src[lane + 32 * i]);
    const bool is_q = h < nq;
    const bool is_k = !is_q && h < nq + nkv;
    if (is_q || is_k) {
      const __nv_bfloat16* nw = is_q ? qn : kn;
      if (nw != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) ss += v[i] * v[i];
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss / D + eps);
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = v[i] * inv * __bfloat162float(nw[lane + 32 * i]);
      }
      // rotate-half pairs (d, d + D/2)
#pragma unroll
      for (int i = 0; i < NV / 2; ++i) {
        const int d = lane + 32 * i;
        const float c = cs[d], s = cs[D / 2 + d];
        const float x1 = v[i], x2 = v[i + NV / 2];
        v[i] = x1 * c - x2 * s;
        v[i + NV / 2] = x2 * c + x1 * s;
      }
    }
    if (is_q) {
      __nv_bfloat16* dst = q_out + (t * nq + h) * D;
#pragma unroll
      for (int i = 0; i < NV; ++i) dst[lane + 32 * i] = __float2bfloat16(v[i]);
    } else if (slot >= 0) {
      const int kvsel = is_k ? 0 : 1;
      const int kh = is_k ? h - nq : h - nq - nkv;
      const long blk = slot >> 4, off = slot & 15;
      if constexpr (Q8) {
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const float inv = am > 0.f ? 127.f / am : 0.f;
        uint8_t* bp = reinterpret_cast<uint8_t*>(cache_v) + layer_stride + blk * block_bytes;
        int8_t* page = reinterpret_cast<int8_t*>(bp) + (long)((kvsel * nkv + kh) * 16) * D;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int q = max(-127, min(127, __float2int_rn(v[i] * inv)));
          const int d = lane + 32 * i;
          // K rows in natural order (operands of int8 Q K^T MMAs); V rows (one
          // per dimension, 16 tokens) in fp16 fragment order (q8_perm16)
          if (is_k) page[off * D + d] = static_cast<int8_t>(q);
          else page[d * 16 + q8_perm16(static_cast<int>(off))] = static_cast<int8_t>(q);
        }
        if (lane == 0)
          reinterpret_cast<float*>(bp + 2L * nkv * 16 * D)[(kvsel * nkv + kh) * 16 + off] = am / 127.f;
      } else {
        __nv_bfloat16* dst = cache + layer_stride + (((blk * 2 + kvsel) * nkv + kh) * 16 + off) * D;
#pragma unroll
        for (int i = 0; i < NV; ++i) dst[lane + 32 * i] = __float2bfloat16(v[i]);
      }
    }
  }
}

}  // namespace

void rmsnorm(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& out, double eps) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "rmsnorm: x bf16 [M,H]");
  const int M = x.size(0), H = x.size(1);
  if (M == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  if (vec_ok(H, x.data_ptr(), x.stride(0)) && vec_ok(H, out.data_ptr(), out.stride(0))) {
    // plain rmsnorm: read x through the "residual" slot, no write-back
    rmsnorm_vec_kernel<0><<<M, vec_threads(H), 0, at::cuda::getCurrentCUDAStream()>>>(
        nullptr, 0, 0, reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
        out.stride(0), M, H, float(eps));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  rmsnorm_kernel<<<M, kNormThreads, H * sizeof(float), at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      out.stride(0), H, float(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void add_rmsnorm(const torch::Tensor& delta, torch::Tensor& residual, const torch::Tensor& w, torch::Tensor& out,
                 double eps) {
  TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && residual.dim() == 2, "add_rmsnorm: residual bf16 [M,H]");
  const int M = residual.size(0), H = residual.size(1);
  if (M == 0) return;
  const at::cuda::CUDAGuard g(residual.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const size_t sm = H * sizeof(float);
  const bool vec = vec_ok(H, residual.data_ptr(), residual.stride(0)) && vec_ok(H, out.data_ptr(), out.stride(0)) &&
                   vec_ok(H, delta.data_ptr(), delta.dim() == 2 ? delta.stride(0) : H);
  if (vec) {
    if (delta.scalar_type() == at::kFloat) {
      TORCH_CHECK(delta.is_contiguous() && delta.numel() % ((int64_t)M * H) == 0, "add_rmsnorm: f32 partials [S,M,H]");
      rmsnorm_vec_kernel<2><<<M, vec_threads(H), 0, stream>>>(
          delta.data_ptr(), int(delta.numel() / ((int64_t)M * H)), H,
          reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()), residual.stride(0),
          reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
          out.stride(0), M, H, float(eps));
    } else {
      TORCH_CHECK(delta.scalar_type() == at::kBFloat16 && delta.stride(1) == 1, "add_rmsnorm: delta bf16 [M,H]");
      rmsnorm_vec_kernel<1><<<M, vec_threads(H), 0, stream>>>(
          delta.data_ptr(), 1, delta.stride(0), reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()),
          residual.stride(0), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), M, H, float(eps));
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  if (delta.scalar_type() == at::kFloat) {
    TORCH_CHECK(delta.is_contiguous() && delta.numel() % ((int64_t)M * H) == 0, "add_rmsnorm: f32 partials [S,M,H]");
    const int S = delta.numel() / ((int64_t)M * H);
    add_rmsnorm_kernel<true><<<M, kNormThreads, sm, stream>>>(
        delta.data_ptr(), S, H, reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()), residual.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
        out.stride(0), M, H, float(eps));
  } else {
    TORCH_CHECK(delta.scalar_type() == at::kBFloat16 && delta.stride(1) == 1, "add_rmsnorm: delta bf16 [M,H]");
    add_rmsnorm_kernel<false><<<M, kNormThreads, sm, stream>>>(
        delta.data_ptr(), 1, delta.stride(0), reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()),
        residual.stride(0), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), M, H, float(eps));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void layernorm(const torch::Tensor& x, const c10::optional<torch::Tensor>& resid, const torch::Tensor& w,
               const torch::Tensor& b, torch::Tensor& out, double eps) {
  TORCH_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16, "layernorm: x contiguous bf16");
  const int H = x.size(-1);
  const int M = x.numel() / H;
  if (M == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  const __nv_bfloat16* r = nullptr;
  if (resid.has_value() && resid->defined()) {
    TORCH_CHECK(resid->is_contiguous() && resid->numel() == x.numel(), "layernorm: resid shape");
    r = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
  }
  layernorm_kernel<<<M, kNormThreads, H * sizeof(float), at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), r, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), H,
      float(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embedding(const torch::Tensor& ids, const torch::Tensor& table, torch::Tensor& out) {
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "embedding: ids int32");
  TORCH_CHECK(table.scalar_type() == at::kBFloat16 && table.is_contiguous(), "embedding: table bf16");
  const int T = ids.numel();
  if (T == 0) return;
  const at::cuda::CUDAGuard g(ids.device());
  embedding_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()), table.size(0), table.size(1),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), check_word(ids.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_kv_write(const torch::Tensor& qkv, const torch::Tensor& positions, const torch::Tensor& slot_mapping,
                   const torch::Tensor& cos_sin, torch::Tensor& q_out, torch::Tensor& kv_cache, int64_t layer,
                   int64_t num_q_heads, int64_t num_kv_heads, const c10::optional<torch::Tensor>& q_norm,
                   const c10::optional<torch::Tensor>& k_norm, double eps) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1, "rope: qkv bf16 [T, *]");
  const int hd = int(kv_cache.size(5));
  TORCH_CHECK(hd == 128 || hd == 64, "rope: head_dim must be 128 or 64");
  TORCH_CHECK(qkv.size(1) >= (num_q_heads + 2 * num_kv_heads) * hd, "rope: qkv narrower than the heads");
  TORCH_CHECK(positions.scalar_type() == at::kLong, "rope: positions int64");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kInt, "rope: slot_mapping int32");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == hd, "rope: cos_sin f32 [P, head_dim]");
  TORCH_CHECK(kv_cache.dim() == 6 && kv_cache.size(3) == num_kv_heads, "rope: kv_cache [L,NB,2,KVH,16,head_dim]");
  const int T = qkv.size(0);
  if (T == 0) return;
  const at::cuda::CUDAGuard g(qkv.device());
  const long layer_stride = layer * kv_cache.stride(0);
  const __nv_bfloat16* qn = (q_norm.has_value() && q_norm->defined())
                                ? reinterpret_cast<const __nv_bfloat16*>(q_norm->data_ptr())
                                : nullptr;
  const __nv_bfloat16* kn = (k_norm.has_value() && k_norm->defined())
                                ? reinterpret_cast<const __nv_bfloat16*>(k_norm->data_ptr())
                                : nullptr;
  auto kern = hd == 128 ? rope_kv_write_kernel<128, false> : rope_kv_write_kernel<64, false>;
  kern<<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), positions.data_ptr<int64_t>(),
      slot_mapping.data_ptr<int>(), cos_sin.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(kv_cache.data_ptr()), layer_stride, int(num_q_heads), int(num_kv_heads), qn,
      kn, float(eps), cos_sin.size(0), kv_cache.size(1) * 16, check_word(qkv.device().index()), 0L);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_kv_write_q8(const torch::Tensor& qkv, const torch::Tensor& positions, const torch::Tensor& slot_mapping,
                      const torch::Tensor& cos_sin, torch::Tensor& q_out, torch::Tensor& kv_cache, int64_t layer,
                      int64_t num_q_heads, int64_t num_kv_heads, const c10::optional<torch::Tensor>& q_norm,
                      const c10::optional<torch::Tensor>& k_norm, double eps) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1, "rope_q8: qkv bf16 [T, *]");
  constexpr int hd = 128;
  TORCH_CHECK(kv_cache.scalar_type() == at::kByte && kv_cache.dim() == 3 && kv_cache.is_contiguous(),
              "rope_q8: int8 kv cache [L, NB, block_bytes] uint8");
  const long bb = kv_cache.size(2);
  TORCH_CHECK(bb == 2L * num_kv_heads * 16 * (hd + 4), "rope_q8: block bytes do not match 2 x KVH x 16 x (128 + 4)");
  TORCH_CHECK(qkv.size(1) >= (num_q_heads + 2 * num_kv_heads) * hd, "rope_q8: qkv narrower than the heads");
  TORCH_CHECK(positions.scalar_type() == at::kLong && slot_mapping.scalar_type() == at::kInt, "rope_q8: index dtypes");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == hd, "rope_q8: cos_sin f32 [P, 128]");
  const int T = qkv.size(0);
  if (T == 0) return;
  const at::cuda::CUDAGuard g(qkv.device());
  const __nv_bfloat16* qn = (q_norm.has_value() && q_norm->defined())
                                ? reinterpret_cast<const __nv_bfloat16*>(q_norm->data_ptr())
                                : nullptr;
  const __nv_bfloat16* kn = (k_norm.has_value() && k_norm->defined())
                                ? reinterpret_cast<const __nv_bfloat16*>(k_norm->data_ptr())
                                : nullptr;
  rope_kv_write_kernel<hd, true><<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), positions.data_ptr<int64_t>(),
      slot_mapping.data_ptr<int>(), cos_sin.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
      kv_cache.data_ptr(), layer * kv_cache.stride(0), int(num_q_heads), int(num_kv_heads), qn, kn, float(eps),
      cos_sin.size(0), kv_cache.size(1) * 16, check_word(qkv.device().index()), bb);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
