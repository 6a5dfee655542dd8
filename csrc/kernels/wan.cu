// Wan 2.1 text-to-video DiT: the element-wise and layout kernels around the
// tcgen05 GEMMs and the paged tensor-core attention.
//
// Reference behaviour: executor/wan/dit.rs (WanAttentionBlock::forward
// :727-773 with the six AdaLN modulation rows, Head::forward :804-818,
// rope_apply :201-313 with the head dim split into temporal / height / width
// pairs, WanRMSNorm over the full model dim :334-346, WanLayerNorm :383-400,
// patch embedding :866-869 and unpatchify :1000-1037), and
// executor/wan/scheduler.rs (flow-matching Euler step :76-93).
//
// The residual stream stays in fp32 [T, D] (T = batch x tokens); every
// GEMM input is produced in bf16 by the kernel that finishes the previous
// step, so each block is: residual_norm -> qkv GEMM -> qkv_norm_rope (q and
// paged K / V) -> attention -> o GEMM -> residual_norm (gate, norm3) ->
// q GEMM -> q norm -> cross attention over the cached text K / V -> o GEMM
// -> residual_norm (modulated norm2) -> FFN GEMMs (GELU epilogue) ->
// residual_norm (gate, next block's modulated norm1).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops_media.h"

namespace bloom {
namespace wan {

constexpr int kThreads = 256;
constexpr int kMaxChunks = 4;  // 8-element chunks per thread: D <= 8192

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) s += red[w];
  return s;
}

struct ResArgs {
  float* x;                    // [T, D] f32 residual (in / out)
  const __nv_bfloat16* delta;  // [T, D] or null
  const float* gmod;           // gate = gmod[gi * D + d] + ge[b * gbs + gi * gis + d]
  const float* ge;
  int gi;
  long gbs, gis;
  int mode;  // 0: y = x; 1: y = LN(x) * w + b; 2: y = LN(x) * (1 + scale) + shift
  const float* lw;
  const float* lb;
  const float* nmod;  // shift / scale rows: nmod[i * D + d] + ne[b * ebs + i * eis + d]
  const float* ne;
  int ish, isc;
  long ebs, eis;
  int D, S;
  float eps;
  __nv_bfloat16* y;
};

__global__ void __launch_bounds__(kThreads) residual_norm_kernel(const ResArgs a) {
  __shared__ float red[kThreads / 32];
  const long row = blockIdx.x;
  const int b = int(row / a.S);
  const int nch = a.D / 8;
  float v[kMaxChunks][8];
  float s1 = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = threadIdx.x + kThreads * i;
#pragma unroll
    for (int k = 0; k < 8; ++k) v[i][k] = 0.f;
    if (c >= nch) continue;
    float* xp = a.x + row * a.D + c * 8;
    const float4 x0 = *reinterpret_cast<const float4*>(xp);
    const float4 x1 = *reinterpret_cast<const float4*>(xp + 4);
    v[i][0] = x0.x, v[i][1] = x0.y, v[i][2] = x0.z, v[i][3] = x0.w;
    v[i][4] = x1.x, v[i][5] = x1.y, v[i][6] = x1.z, v[i][7] = x1.w;
    if (a.delta != nullptr) {
      const uint4 u = *reinterpret_cast<const uint4*>(a.delta + row * a.D + c * 8);
      const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float g = 1.f;
        if (a.gi >= 0) {
          const int d = c * 8 + k;
          g = a.gmod[a.gi * a.D + d] + a.ge[b * a.gbs + a.gi * a.gis + d];
        }
        v[i][k] += __bfloat162float(db[k]) * g;
      }
      *reinterpret_cast<float4*>(xp) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
      *reinterpret_cast<float4*>(xp + 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) s1 += v[i][k];
  }
  float mean = 0.f, inv = 1.f;
  if (a.mode != 0) {
    mean = block_sum(s1, red) / a.D;
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = threadIdx.x + kThreads * i;
      if (c >= nch) continue;
#pragma unroll
      for (int k = 0; k < 8; ++k) s2 += (v[i][k] - mean) * (v[i][k] - mean);
    }
    inv = rsqrtf(block_sum(s2, red) / a.D + a.eps);
  }
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = threadIdx.x + kThreads * i;
    if (c >= nch) continue;
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int d = c * 8 + k;
      float t = v[i][k];
      if (a.mode == 1) {
        t = (t - mean) * inv * (a.lw ? a.lw[d] : 1.f) + (a.lb ? a.lb[d] : 0.f);
      } else if (a.mode == 2) {
        const float sc = a.nmod[a.isc * a.D + d] + a.ne[b * a.ebs + a.isc * a.eis + d];
        const float sh = a.nmod[a.ish * a.D + d] + a.ne[b * a.ebs + a.ish * a.eis + d];
        t = (t - mean) * inv * (1.f + sc) + sh;
      }
      o[k] = t;
    }
    *reinterpret_cast<uint4*>(a.y + row * a.D + c * 8) = make_uint4(
        pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
  }
}

// The same step with one warp per row (8 rows per 256-thread CTA): warp
// shuffles instead of block barriers, and no idle threads for D = 1536 /
// 3072 (the CTA-per-row kernel leaves 64 of 256 threads idle at D = 1536).
// CPL = 8-element chunks per lane (D <= 256 * CPL).
template <int CPL>
__global__ void __launch_bounds__(kThreads) residual_norm_warp_kernel(const ResArgs a, long T) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * (kThreads / 32) + warp;
  if (row >= T) return;
  const int b = int(row / a.S);
  const int nch = a.D / 8;
  float v[CPL][8];
  float s1 = 0.f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
#pragma unroll
    for (int k = 0; k < 8; ++k) v[i][k] = 0.f;
    if (c >= nch) continue;
    float* xp = a.x + row * a.D + c * 8;
    const float4 x0 = *reinterpret_cast<const float4*>(xp);
    const float4 x1 = *reinterpret_cast<const float4*>(xp + 4);
    v[i][0] = x0.x, v[i][1] = x0.y, v[i][2] = x0.z, v[i][3] = x0.w;
    v[i][4] = x1.x, v[i][5] = x1.y, v[i][6] = x1.z, v[i][7] = x1.w;
    if (a.delta != nullptr) {
      const uint4 u = *reinterpret_cast<const uint4*>(a.delta + row * a.D + c * 8);
      const __nv_bfloat16* db = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float g = 1.f;
        if (a.gi >= 0) {
          const int d = c * 8 + k;
          g = a.gmod[a.gi * a.D + d] + a.ge[b * a.gbs + a.gi * a.gis + d];
        }
        v[i][k] += __bfloat162float(db[k]) * g;
      }
      *reinterpret_cast<float4*>(xp) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
      *reinterpret_cast<float4*>(xp + 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) s1 += v[i][k];
  }
  float mean = 0.f, inv = 1.f;
  if (a.mode != 0) {
    mean = warp_sum(s1) / a.D;
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      if (lane + 32 * i >= nch) continue;
#pragma unroll
      for (int k = 0; k < 8; ++k) s2 += (v[i][k] - mean) * (v[i][k] - mean);
    }
    inv = rsqrtf(warp_sum(s2) / a.D + a.eps);
  }
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = lane + 32 * i;
    if (c >= nch) continue;
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int d = c * 8 + k;
      float t = v[i][k];
      if (a.mode == 1) {
        t = (t - mean) * inv * (a.lw ? a.lw[d] : 1.f) + (a.lb ? a.lb[d] : 0.f);
      } else if (a.mode == 2) {
        const float sc = a.nmod[a.isc * a.D + d] + a.ne[b * a.ebs + a.isc * a.eis + d];
        const float sh = a.nmod[a.ish * a.D + d] + a.ne[b * a.ebs + a.ish * a.eis + d];
        t = (t - mean) * inv * (1.f + sc) + sh;
      }
      o[k] = t;
    }
    *reinterpret_cast<uint4*>(a.y + row * a.D + c * 8) = make_uint4(
        pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
  }
}

struct QkvArgs {
  const __nv_bfloat16* src;
  long ld;
  int q_col, k_col, v_col;  // column of the q / k / v part (-1: absent)
  int nh, hd, D;
  const float* qw;
  const float* kw;
  float eps;
  int head_norm;       // 1: RMSNorm over each head (weights [hd]); 0: over the whole model dim (weights [D])
  const float2* rope;  // [positions][hd / 2] (cos, sin) of each pair's own axis frequency, or null
  int rope_rows;       // positions in the table (larger positions are clamped)
  int pt, ph;          // pairs [0, pt) rotate with the frame index, [pt, pt + ph) the row, the rest the column
  int gf, gh, gw;      // token grid (positions from the token index) when pos3 is null
  const int* pos3;     // [S_out][3] (frame, row, column) of each output token, or null
  int S;               // src rows per sample
  int S_out, off;      // output tokens per sample; these rows land at [off, off + S)
  __nv_bfloat16* q_out;  // [B * S_out, nh, hd]
  __nv_bfloat16* kv;     // pages [NB][2][nh][16][hd]
  int bpb;               // pages per sample
};

// One CTA per src row: RMSNorm of q and k (over the model dim or per head),
// RoPE on (even, odd) pairs, q -> q_out, k / v -> pages.  Sums are formed
// in a fixed order (no atomics), so results do not depend on scheduling.
__global__ void __launch_bounds__(kThreads) qkv_norm_rope_kernel(const QkvArgs a) {
  __shared__ float red[kThreads / 32];
  extern __shared__ float sq[];  // head_norm: [D / 2] pair squares, then [nh] head sums
  const long row = blockIdx.x;
  const int b = int(row / a.S), n = int(row - (long)b * a.S);
  const int no = a.off + n;
  const long orow = (long)b * a.S_out + no;
  int pf, ph_, pw;
  if (a.pos3 != nullptr) {
    pf = a.pos3[no * 3];
    ph_ = a.pos3[no * 3 + 1];
    pw = a.pos3[no * 3 + 2];
  } else {
    const int hw = a.gh * a.gw;
    pf = n / hw;
    ph_ = (n / a.gw) % a.gh;
    pw = n % a.gw;
  }
  const int half = a.hd / 2;
  const int np = a.D / 2;
  const __nv_bfloat16* s = a.src + row * a.ld;
  const int blk = b * a.bpb + no / 16, slot = no % 16;

  auto rot = [&](int P, float& x0, float& x1) {
    if (a.rope == nullptr) return;
    const int p = P % half;
    const int pos = min(max(p < a.pt ? pf : (p < a.pt + a.ph ? ph_ : pw), 0), a.rope_rows - 1);
    const float2 cs = a.rope[(long)pos * half + p];
    const float r0 = x0 * cs.x - x1 * cs.y;
    const float r1 = x0 * cs.y + x1 * cs.x;
    x0 = r0;
    x1 = r1;
  };
  float* hsum = sq + np;
  for (int part = 0; part < 2; ++part) {  // 0: q, 1: k
    const int col = part == 0 ? a.q_col : a.k_col;
    if (col < 0) continue;
    const float* w = part == 0 ? a.qw : a.kw;
    float inv_all = 1.f;
    if (w != nullptr && !a.head_norm) {
      float ss = 0.f;
      for (int P = threadIdx.x; P < np; P += kThreads) {
        const __nv_bfloat162 t = *reinterpret_cast<const __nv_bfloat162*>(s + col + 2 * P);
        const float x0 = __bfloat162float(t.x), x1 = __bfloat162float(t.y);
        ss += x0 * x0 + x1 * x1;
      }
      inv_all = rsqrtf(block_sum(ss, red) / a.D + a.eps);
    } else if (w != nullptr) {
      __syncthreads();  // sq / hsum reuse across parts
      for (int P = threadIdx.x; P < np; P += kThreads) {
        const __nv_bfloat162 t = *reinterpret_cast<const __nv_bfloat162*>(s + col + 2 * P);
        const float x0 = __bfloat162float(t.x), x1 = __bfloat162float(t.y);
        sq[P] = x0 * x0 + x1 * x1;
      }
      __syncthreads();
      for (int h = threadIdx.x; h < a.nh; h += kThreads) {
        float acc = 0.f;
        for (int i = 0; i < half; ++i) acc += sq[h * half + i];
        hsum[h] = rsqrtf(acc / a.hd + a.eps);
      }
      __syncthreads();
    }
    for (int P = threadIdx.x; P < np; P += kThreads) {
      const __nv_bfloat162 t = *reinterpret_cast<const __nv_bfloat162*>(s + col + 2 * P);
      const int h = (2 * P) / a.hd, d = 2 * P - h * a.hd;
      float x0 = __bfloat162float(t.x), x1 = __bfloat162float(t.y);
      if (w != nullptr) {
        const float inv = a.head_norm ? hsum[h] : inv_all;
        const int wi = a.head_norm ? d : 2 * P;
        x0 *= inv * w[wi];
        x1 *= inv * w[wi + 1];
      }
      rot(P, x0, x1);
      __nv_bfloat16* dst = part == 0 ? a.q_out + (orow * a.nh + h) * a.hd + d
                                     : a.kv + (((long)blk * 2 + 0) * a.nh + h) * 16 * a.hd + slot * a.hd + d;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(x0, x1);
    }
  }
  if (a.v_col >= 0) {
    for (int P = threadIdx.x; P < np; P += kThreads) {
      const int h = (2 * P) / a.hd, d = 2 * P - h * a.hd;
      *reinterpret_cast<uint32_t*>(a.kv + (((long)blk * 2 + 1) * a.nh + h) * 16 * a.hd + slot * a.hd + d) =
          *reinterpret_cast<const uint32_t*>(s + a.v_col + 2 * P);
    }
  }
}

// Full-model-dim norms (head_norm == 0) with one warp per src row: the
// squares are summed with shuffles, the pairs re-read from L1 for the write.
__global__ void __launch_bounds__(kThreads) qkv_norm_rope_warp_kernel(const QkvArgs a, long T) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * (kThreads / 32) + warp;
  if (row >= T) return;
  const int b = int(row / a.S), n = int(row - (long)b * a.S);
  const int no = a.off + n;
  const long orow = (long)b * a.S_out + no;
  int pf, ph_, pw;
  if (a.pos3 != nullptr) {
    pf = a.pos3[no * 3];
    ph_ = a.pos3[no * 3 + 1];
    pw = a.pos3[no * 3 + 2];
  } else {
    const int hw = a.gh * a.gw;
    pf = n / hw;
    ph_ = (n / a.gw) % a.gh;
    pw = n % a.gw;
  }
  const int half = a.hd / 2, np = a.D / 2;
  const __nv_bfloat16* s = a.src + row * a.ld;
  const int blk = b * a.bpb + no / 16, slot = no % 16;
  for (int part = 0; part < 2; ++part) {
    const int col = part == 0 ? a.q_col : a.k_col;
    if (col < 0) continue;
    const float* w = part == 0 ? a.qw : a.kw;
    float inv = 1.f;
    if (w != nullptr) {
      float ss = 0.f;
      for (int P = lane; P < np; P += 32) {
        const __nv_bfloat162 t = *reinterpret_cast<const __nv_bfloat162*>(s + col + 2 * P);
        const float x0 = __bfloat162float(t.x), x1 = __bfloat162float(t.y);
        ss += x0 * x0 + x1 * x1;
      }
      inv = rsqrtf(warp_sum(ss) / a.D + a.eps);
    }
    for (int P = lane; P < np; P += 32) {
      const __nv_bfloat162 t = *reinterpret_cast<const __nv_bfloat162*>(s + col + 2 * P);
      float x0 = __bfloat162float(t.x) * inv, x1 = __bfloat162float(t.y) * inv;
      if (w != nullptr) {
        x0 *= w[2 * P];
        x1 *= w[2 * P + 1];
      }
      if (a.rope != nullptr) {
        const int p = P % half;
        const int pos = min(max(p < a.pt ? pf : (p < a.pt + a.ph ? ph_ : pw), 0), a.rope_rows - 1);
        const float2 cs = a.rope[(long)pos * half + p];
        const float r0 = x0 * cs.x - x1 * cs.y, r1 = x0 * cs.y + x1 * cs.x;
        x0 = r0;
        x1 = r1;
      }
      const int h = (2 * P) / a.hd, d = 2 * P - h * a.hd;
      __nv_bfloat16* dst = part == 0 ? a.q_out + (orow * a.nh + h) * a.hd + d
                                     : a.kv + (((long)blk * 2 + 0) * a.nh + h) * 16 * a.hd + slot * a.hd + d;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(x0, x1);
    }
  }
  if (a.v_col >= 0) {
    for (int P = lane; P < np; P += 32) {
      const int h = (2 * P) / a.hd, d = 2 * P - h * a.hd;
      *reinterpret_cast<uint32_t*>(a.kv + (((long)blk * 2 + 1) * a.nh + h) * 16 * a.hd + slot * a.hd + d) =
          *reinterpret_cast<const uint32_t*>(s + a.v_col + 2 * P);
    }
  }
}

// latent f32 [B, C, F, H, W] -> tokens bf16 [B * F * (H/2) * (W/2), C * 4],
// column c * 4 + i * 2 + j = latent[b, c, f, 2h + i, 2w + j] (the 1x2x2 patch
// conv's weight layout [dim, C, 1, 2, 2] flattened)
__global__ void patchify_kernel(const float* __restrict__ lat, __nv_bfloat16* __restrict__ tok, int B, int C, int F,
                                int H, int W) {
  const int H2 = H / 2, W2 = W / 2;
  const long total = (long)B * F * H2 * W2 * C * 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int col = int(i % (C * 4));
    const long t = i / (C * 4);
    const int w2 = int(t % W2), h2 = int((t / W2) % H2), f = int((t / ((long)W2 * H2)) % F);
    const int b = int(t / ((long)W2 * H2 * F));
    const int c = col / 4, pi = (col / 2) % 2, pj = col % 2;
    tok[i] = __float2bfloat16(lat[((((long)b * C + c) * F + f) * H + 2 * h2 + pi) * W + 2 * w2 + pj]);
  }
}

// head output bf16 [preds * S, C * 4] (token-major, column c * 4 + i * 2 + j)
// -> velocity v (preds == 2: v = u + g (c - u), rows [0, S) conditional,
// [S, 2S) unconditional); latent f32 [C, F, H, W] += dt * v.
__global__ void unpatchify_step_kernel(const __nv_bfloat16* __restrict__ ho, int preds, float g, float dt,
                                       float* __restrict__ lat, int C, int F, int H, int W) {
  const int H2 = H / 2, W2 = W / 2;
  const long S = (long)F * H2 * W2;
  const long total = (long)C * F * H * W;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int x = int(i % W), y = int((i / W) % H), f = int((i / ((long)W * H)) % F), c = int(i / ((long)W * H * F));
    const long t = ((long)f * H2 + y / 2) * W2 + x / 2;
    const int col = c * 4 + (y % 2) * 2 + (x % 2);
    float v = __bfloat162float(ho[t * C * 4 + col]);
    if (preds == 2) {
      const float u = __bfloat162float(ho[(S + t) * C * 4 + col]);
      v = u + g * (v - u);
    }
    lat[i] += dt * v;
  }
}

__global__ void silu_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = __bfloat162float(x[i]);
    y[i] = __float2bfloat16(v / (1.f + __expf(-v)));
  }
}

int grid_for(long n) { return int(std::min<long>((n + 255) / 256, 148L * 16)); }

}  // namespace wan

static const float* fptr(const c10::optional<torch::Tensor>& t, const char* what) {
  if (!t.has_value()) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous(), what, ": f32 contiguous");
  return t->data_ptr<float>();
}

void wan_residual_norm(torch::Tensor& x, const c10::optional<torch::Tensor>& delta,
                       const c10::optional<torch::Tensor>& gate_mod, const c10::optional<torch::Tensor>& gate_e,
                       int64_t gate_idx, int64_t gate_batch_stride, int64_t gate_idx_stride, int64_t mode, const c10::optional<torch::Tensor>& ln_w,
                       const c10::optional<torch::Tensor>& ln_b, const c10::optional<torch::Tensor>& mod,
                       const c10::optional<torch::Tensor>& e, int64_t shift_idx, int64_t scale_idx,
                       int64_t e_batch_stride, int64_t e_idx_stride, int64_t rows_per_batch, double eps,
                       torch::Tensor& y) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && x.dim() == 2, "wan_residual_norm: x f32 [T, D]");
  const int T = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0 && D <= 8 * wan::kThreads * wan::kMaxChunks, "wan_residual_norm: D % 8 == 0, <= 8192");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.sizes() == x.sizes(), "wan_residual_norm: y");
  if (delta.has_value())
    TORCH_CHECK(delta->scalar_type() == at::kBFloat16 && delta->is_contiguous() && delta->sizes() == x.sizes(),
                "wan_residual_norm: delta bf16 like x");
  TORCH_CHECK(mode >= 0 && mode <= 2, "wan_residual_norm: mode 0 / 1 / 2");
  TORCH_CHECK(gate_idx < 0 || (gate_mod.has_value() && gate_e.has_value()), "wan_residual_norm: gate sources");
  TORCH_CHECK(mode != 2 || (mod.has_value() && e.has_value()), "wan_residual_norm: modulation sources");
  TORCH_CHECK(rows_per_batch > 0, "wan_residual_norm: rows per batch");
  if (T == 0) return;
  wan::ResArgs a{};
  a.x = x.data_ptr<float>();
  a.delta = delta.has_value() ? reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr()) : nullptr;
  a.gmod = fptr(gate_mod, "gate modulation");
  a.ge = fptr(gate_e, "gate e");
  a.gi = int(gate_idx);
  a.gbs = gate_batch_stride;
  a.gis = gate_idx_stride;
  a.mode = int(mode);
  a.lw = fptr(ln_w, "ln weight");
  a.lb = fptr(ln_b, "ln bias");
  a.nmod = fptr(mod, "modulation");
  a.ne = fptr(e, "e");
  a.ish = int(shift_idx);
  a.isc = int(scale_idx);
  a.ebs = e_batch_stride;
  a.eis = e_idx_stride;
  a.D = D;
  a.S = int(rows_per_batch);
  a.eps = float(eps);
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  const at::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int nch = D / 8;
  const int blocks = (T + wan::kThreads / 32 - 1) / (wan::kThreads / 32);
  // warp per row pays off with many rows of moderate width (Wan: 15,600 x 1,536: 85.0 vs 86.6 ms per
  // DiT step); few wide rows (LongCat: 1,536 x 3,072) keep a CTA per row (3.36 vs 3.68 ms per pass)
  if (T >= 4096 && nch <= 64)
    wan::residual_norm_warp_kernel<2><<<blocks, wan::kThreads, 0, st>>>(a, T);
  else if (T >= 4096 && nch <= 192)
    wan::residual_norm_warp_kernel<6><<<blocks, wan::kThreads, 0, st>>>(a, T);
  else
    wan::residual_norm_kernel<<<T, wan::kThreads, 0, st>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void wan_qkv_norm_rope(const torch::Tensor& src, int64_t q_col, int64_t k_col, int64_t v_col, int64_t heads,
                       int64_t head_dim, const c10::optional<torch::Tensor>& q_w,
                       const c10::optional<torch::Tensor>& k_w, double eps,
                       const c10::optional<torch::Tensor>& rope_tab, int64_t rope_pt, int64_t rope_ph,
                       int64_t grid_f, int64_t grid_h, int64_t grid_w, int64_t rows_per_batch,
                       const c10::optional<torch::Tensor>& q_out, const c10::optional<torch::Tensor>& kv,
                       int64_t blocks_per_batch, bool head_norm, const c10::optional<torch::Tensor>& pos3,
                       int64_t out_rows_per_batch, int64_t out_offset) {
  TORCH_CHECK(src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.stride(1) == 1 && src.stride(0) % 2 == 0,
              "wan_qkv_norm_rope: src bf16 [T, cols]");
  const int T = src.size(0);
  const int D = int(heads * head_dim);
  TORCH_CHECK(head_dim % 2 == 0 && D % 2 == 0, "wan_qkv_norm_rope: even head dim");
  const int64_t S_out = out_rows_per_batch > 0 ? out_rows_per_batch : rows_per_batch;
  TORCH_CHECK(out_offset >= 0 && out_offset + rows_per_batch <= S_out, "wan_qkv_norm_rope: output placement");
  TORCH_CHECK(rows_per_batch > 0 && T % rows_per_batch == 0, "wan_qkv_norm_rope: rows per batch");
  const int64_t B = T / rows_per_batch;
  for (int64_t c : {q_col, k_col, v_col})
    TORCH_CHECK(c < 0 || (c % 2 == 0 && c + D <= src.size(1)), "wan_qkv_norm_rope: column range");
  TORCH_CHECK(q_col < 0 || (q_out.has_value() && q_out->is_contiguous() && q_out->numel() >= B * S_out * D),
              "wan_qkv_norm_rope: q_out [B * S_out, heads, head_dim]");
  TORCH_CHECK((k_col < 0 && v_col < 0) || (kv.has_value() && kv->is_contiguous()), "wan_qkv_norm_rope: kv pages");
  if (kv.has_value()) {
    const int64_t nblk = (B - 1) * blocks_per_batch + (S_out + 15) / 16;
    TORCH_CHECK(kv->numel() >= nblk * 2 * D * 16, "wan_qkv_norm_rope: kv pages too small");
  }
  if (head_norm) {
    if (q_w.has_value()) TORCH_CHECK(q_w->numel() == head_dim, "wan_qkv_norm_rope: per-head q weights [head_dim]");
    if (k_w.has_value()) TORCH_CHECK(k_w->numel() == head_dim, "wan_qkv_norm_rope: per-head k weights [head_dim]");
  } else {
    if (q_w.has_value()) TORCH_CHECK(q_w->numel() == D, "wan_qkv_norm_rope: q weights [D]");
    if (k_w.has_value()) TORCH_CHECK(k_w->numel() == D, "wan_qkv_norm_rope: k weights [D]");
  }
  if (pos3.has_value()) {
    TORCH_CHECK(pos3->scalar_type() == at::kInt && pos3->is_contiguous() && pos3->numel() == S_out * 3,
                "wan_qkv_norm_rope: pos3 int32 [S_out, 3]");
  } else {
    TORCH_CHECK(grid_f * grid_h * grid_w == rows_per_batch, "wan_qkv_norm_rope: grid");
  }
  const int64_t maxpos = pos3.has_value() ? 1 : std::max({grid_f, grid_h, grid_w});
  if (rope_tab.has_value())
    TORCH_CHECK(rope_tab->scalar_type() == at::kFloat && rope_tab->is_contiguous() &&
                    rope_tab->numel() >= maxpos * head_dim && rope_tab->numel() % head_dim == 0,
                "wan_qkv_norm_rope: rope table [positions, head_dim / 2, 2] f32");
  if (T == 0) return;
  wan::QkvArgs a{};
  a.src = reinterpret_cast<const __nv_bfloat16*>(src.data_ptr());
  a.ld = src.stride(0);
  a.q_col = int(q_col);
  a.k_col = int(k_col);
  a.v_col = int(v_col);
  a.nh = int(heads);
  a.hd = int(head_dim);
  a.D = D;
  a.qw = fptr(q_w, "q norm");
  a.kw = fptr(k_w, "k norm");
  a.eps = float(eps);
  a.head_norm = head_norm ? 1 : 0;
  a.rope = rope_tab.has_value() ? reinterpret_cast<const float2*>(rope_tab->data_ptr<float>()) : nullptr;
  a.rope_rows = rope_tab.has_value() ? int(rope_tab->numel() / head_dim) : 0;
  a.pt = int(rope_pt);
  a.ph = int(rope_ph);
  a.gf = int(grid_f);
  a.gh = int(grid_h);
  a.gw = int(grid_w);
  a.pos3 = pos3.has_value() ? pos3->data_ptr<int>() : nullptr;
  a.S = int(rows_per_batch);
  a.S_out = int(S_out);
  a.off = int(out_offset);
  a.q_out = q_out.has_value() ? reinterpret_cast<__nv_bfloat16*>(q_out->data_ptr()) : nullptr;
  a.kv = kv.has_value() ? reinterpret_cast<__nv_bfloat16*>(kv->data_ptr()) : nullptr;
  a.bpb = int(blocks_per_batch);
  const size_t smem = head_norm ? (size_t(D / 2) + size_t(heads)) * sizeof(float) : 0;
  TORCH_CHECK(smem <= 48 * 1024, "wan_qkv_norm_rope: model dim too large for per-head norms");
  const at::cuda::CUDAGuard g(src.device());
  if (head_norm) {
    wan::qkv_norm_rope_kernel<<<T, wan::kThreads, smem, at::cuda::getCurrentCUDAStream()>>>(a);
  } else {
    const int blocks = (T + wan::kThreads / 32 - 1) / (wan::kThreads / 32);
    wan::qkv_norm_rope_warp_kernel<<<blocks, wan::kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a, T);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void wan_patchify(const torch::Tensor& latent, torch::Tensor& tokens) {
  TORCH_CHECK(latent.scalar_type() == at::kFloat && latent.is_contiguous() && latent.dim() == 5,
              "wan_patchify: latent f32 [B, C, F, H, W]");
  const int B = latent.size(0), C = latent.size(1), F = latent.size(2), H = latent.size(3), W = latent.size(4);
  TORCH_CHECK(H % 2 == 0 && W % 2 == 0, "wan_patchify: even H, W");
  TORCH_CHECK(tokens.scalar_type() == at::kBFloat16 && tokens.is_contiguous() &&
                  tokens.numel() == (int64_t)B * F * (H / 2) * (W / 2) * C * 4,
              "wan_patchify: tokens bf16 [B*F*H/2*W/2, C*4]");
  const long n = tokens.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard g(latent.device());
  wan::patchify_kernel<<<wan::grid_for(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      latent.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(tokens.data_ptr()), B, C, F, H, W);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void wan_unpatchify_step(const torch::Tensor& head_out, int64_t preds, double guidance, double dt,
                         torch::Tensor& latent) {
  TORCH_CHECK(latent.scalar_type() == at::kFloat && latent.is_contiguous() && latent.dim() == 4,
              "wan_unpatchify_step: latent f32 [C, F, H, W]");
  const int C = latent.size(0), F = latent.size(1), H = latent.size(2), W = latent.size(3);
  TORCH_CHECK(preds == 1 || preds == 2, "wan_unpatchify_step: 1 or 2 predictions");
  TORCH_CHECK(head_out.scalar_type() == at::kBFloat16 && head_out.is_contiguous() &&
                  head_out.numel() == preds * (int64_t)F * (H / 2) * (W / 2) * C * 4,
              "wan_unpatchify_step: head output bf16 [preds * tokens, C * 4]");
  const long n = latent.numel();
  const at::cuda::CUDAGuard g(latent.device());
  wan::unpatchify_step_kernel<<<wan::grid_for(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(head_out.data_ptr()), int(preds), float(guidance), float(dt),
      latent.data_ptr<float>(), C, F, H, W);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void silu_bf16(const torch::Tensor& x, torch::Tensor& out) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 && x.is_contiguous() &&
                  out.is_contiguous() && x.numel() == out.numel(),
              "silu_bf16: contiguous bf16 tensors of one size");
  const long n = x.numel();
  if (n == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  wan::silu_kernel<<<wan::grid_for(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
