// Mixture-of-experts routing, dispatch and combine for top-k softmax routers
// (Qwen3-MoE: 128 experts, top-8, normalised top-k probabilities).
//
//   moe_route    per token: softmax over the router logits, top-k, optional
//                renormalisation; tokens routed to this rank's experts
//                [e0, e0 + E_local) take a slot in their expert (atomic count)
//   moe_plan     one CTA: exclusive scan of the expert counts into row
//                offsets, then the tile lists of the two grouped GEMMs
//                (gate_up with SwiGLU, down) -- built on the device, so the
//                whole layer needs no host round trip and can be graph-captured
//   moe_gather   copies each routed token row into its expert's segment of
//                the sorted activation matrix
//   moe_combine  out[t] = sum over the token's local experts of
//                weight * expert output (fp32 accumulation)
//
// Expert parallelism: every rank routes all tokens identically, computes only
// its local experts, and the per-rank partial outputs are summed by the fused
// reduce-scatter/all-gather kernel (csrc/kernels/comm.cu), which also adds
// the residual and applies the next RMSNorm.  With activations already
// replicated by attention's tensor-parallel all-gather, that moves
// 2 (t-1)/t * H * 2 bytes per token instead of the k * H * 2 bytes a token
// all-to-all would send.  The reference has no MoE model or router at all.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {
namespace {

constexpr int kMaxTopK = 16;

// Router softmax + top-k of one token by one warp, in registers: each lane
// holds experts lane, lane + 32, ... (E <= 32 * NV); k rounds of a warp-wide
// arg-max (lowest index wins ties), the owner lane marks its winner in a bit
// mask.  Lane k returns the k-th choice and its (optionally renormalised)
// probability.
template <int NV>
__device__ __forceinline__ void route_token_warp(const float* __restrict__ row, int E, int K, int norm, int lane,
                                                 int& my_id, float& my_p) {
  float v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int e = lane + 32 * i;
    const float x = e < E ? row[e] : -INFINITY;
    v[i] = x == x ? x : -INFINITY;  // a NaN logit ranks last
  }
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < NV; ++i) mx = fmaxf(mx, v[i]);
  mx = warp_max(mx);
  float z = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) z += (lane + 32 * i < E) ? __expf(v[i] - mx) : 0.f;
  z = warp_sum(z);
  uint32_t taken = 0u;
  float psum = 0.f;
  my_id = 0;
  my_p = 0.f;
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((taken >> i) & 1u) && (v[i] > best || (v[i] == best && e < bi))) {
        best = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (b2 > best || (b2 == best && i2 < bi)) {
        best = b2;
        bi = i2;
      }
    }
    if (bi < E && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    const float p = __expf(best - mx) / z;
    psum += p;
    if (lane == k) {
      my_id = bi;
      my_p = p;
    }
  }
  if (norm) my_p /= psum;
}

// one warp per token
__global__ void moe_route_kernel(const float* __restrict__ logits, int T, int E, int K, int norm, int e0, int El,
                                 int* __restrict__ topk_ids, float* __restrict__ topk_w, int* __restrict__ slot,
                                 int* __restrict__ counts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  int id;
  float p;
  route_token_warp<8>(logits + (long)warp * E, E, K, norm, lane, id, p);
  if (lane < K) {
    topk_ids[(long)warp * K + lane] = id;
    topk_w[(long)warp * K + lane] = p;
    int s = -1;
    if (id >= e0 && id < e0 + El) s = atomicAdd(counts + (id - e0), 1);
    slot[(long)warp * K + lane] = s;
  }
}

// single CTA of 1024 threads
__global__ void moe_plan_kernel(int* __restrict__ counts, int El, int* __restrict__ offsets, int bn, int ft_gu,
                                int ft_d, int4* __restrict__ tiles_gu, int* __restrict__ n_gu, int4* __restrict__ tiles_d,
                                int* __restrict__ n_d, int max_tiles) {
  __shared__ int off_s[1025];
  __shared__ int cnt_gu, cnt_d;
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < El; ++e) {
      off_s[e] = acc;
      acc += counts[e];
    }
    off_s[El] = acc;
    cnt_gu = 0;
    cnt_d = 0;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= El; e += blockDim.x) offsets[e] = off_s[e];
  __syncthreads();
  for (int e = threadIdx.x; e < El; e += blockDim.x) {
    const int c = off_s[e + 1] - off_s[e];
    const int ntt = (c + bn - 1) / bn;
    for (int tt = 0; tt < ntt; ++tt) {
      const int r0 = off_s[e] + tt * bn;
      const int r1 = off_s[e + 1];
      for (int f = 0; f < ft_gu; ++f) {
        const int i = atomicAdd(&cnt_gu, 1);
        if (i < max_tiles) tiles_gu[i] = make_int4(e, f, r0, r1);
      }
      for (int f = 0; f < ft_d; ++f) {
        const int i = atomicAdd(&cnt_d, 1);
        if (i < max_tiles) tiles_d[i] = make_int4(e, f, r0, r1);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *n_gu = min(cnt_gu, max_tiles);
    *n_d = min(cnt_d, max_tiles);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < El; e += blockDim.x) counts[e] = 0;  // ready for the next layer
}

// one CTA per token; H/8 threads (16-byte vectors)
__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int H, int K, int e0, int El,
                                  const int* __restrict__ topk_ids, const int* __restrict__ slot,
                                  const int* __restrict__ offsets, int* __restrict__ pos,
                                  __nv_bfloat16* __restrict__ xs, long xs_rows, int* status) {
  const int t = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(x + (long)t * H);
  for (int j = 0; j < K; ++j) {
    const int s = slot[(long)t * K + j];
    if (s < 0) {
      if (threadIdx.x == 0) pos[(long)t * K + j] = -1;
      continue;
    }
    const int e = topk_ids[(long)t * K + j] - e0;
    if (!kcheck(e >= 0 && e < El, status)) {
      if (threadIdx.x == 0) pos[(long)t * K + j] = -1;
      continue;
    }
    const int r = offsets[e] + s;
    if (!kcheck(r >= 0 && r < xs_rows, status)) {
      if (threadIdx.x == 0) pos[(long)t * K + j] = -1;
      continue;
    }
    if (threadIdx.x == 0) pos[(long)t * K + j] = r;
    uint4* dst = reinterpret_cast<uint4*>(xs + (long)r * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
  }
}

// out[t] = sum_j w[t, j] * ys[pos[t, j]].  With push pointers the row goes
// straight to its owner rank's slot [rank][t % rows] over NVLink (16-byte
// stores, then a system-scope fence), like the row-parallel GEMM's push
// epilogue, so the collective that follows reduces local memory only.
struct CombinePush {
  unsigned long long p[8];
  int world, rank, rows;
};

__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ ys, int H, int K, const int* __restrict__ pos,
                                   const float* __restrict__ topk_w, __nv_bfloat16* __restrict__ out, long ys_rows,
                                   int* status, const CombinePush push) {
  const int t = blockIdx.x;
  __nv_bfloat16* dst = out + (long)t * H;
  if (push.world > 0) {
    const int owner = t / push.rows, lr = t - owner * push.rows;
    dst = reinterpret_cast<__nv_bfloat16*>(push.p[owner]) + ((long)push.rank * push.rows + lr) * H;
  }
  if ((H & 7) == 0) {
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < K; ++j) {
        const int r = pos[(long)t * K + j];
        if (r < 0 || !kcheck(r < ys_rows, status)) continue;
        const float w = topk_w[(long)t * K + j];
        const uint4 u = *reinterpret_cast<const uint4*>(ys + (long)r * H + c * 8);
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(h2[k]);
          acc[2 * k] += w * f.x;
          acc[2 * k + 1] += w * f.y;
        }
      }
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
      *reinterpret_cast<uint4*>(dst + c * 8) = o;
    }
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      float acc = 0.f;
      for (int j = 0; j < K; ++j) {
        const int r = pos[(long)t * K + j];
        if (r >= 0 && kcheck(r < ys_rows, status)) acc += topk_w[(long)t * K + j] * __bfloat162float(ys[(long)r * H + i]);
      }
      dst[i] = __float2bfloat16(acc);
    }
  }
  if (push.world > 0) __threadfence_system();  // pushed rows performed before the collective's ready signal
}

}  // namespace

void moe_route(const torch::Tensor& logits, int64_t top_k, bool norm, int64_t e0, int64_t e_local,
               torch::Tensor& topk_ids, torch::Tensor& topk_w, torch::Tensor& slot, torch::Tensor& counts) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous(), "moe_route: f32 logits");
  TORCH_CHECK(top_k >= 1 && top_k <= kMaxTopK, "moe_route: top_k in [1, 16]");
  TORCH_CHECK(logits.size(1) <= 256 && logits.size(1) >= top_k, "moe_route: top_k <= experts <= 256");
  const int T = logits.size(0), E = logits.size(1);
  if (T == 0) return;
  const at::cuda::CUDAGuard g(logits.device());
  const int threads = 256;
  const int blocks = (T * 32 + threads - 1) / threads;
  moe_route_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), T, E, int(top_k), norm ? 1 : 0, int(e0), int(e_local), topk_ids.data_ptr<int>(),
      topk_w.data_ptr<float>(), slot.data_ptr<int>(), counts.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_plan(torch::Tensor& counts, torch::Tensor& offsets, int64_t bn, int64_t ft_gu, int64_t ft_d,
              torch::Tensor& tiles_gu, torch::Tensor& n_gu, torch::Tensor& tiles_d, torch::Tensor& n_d) {
  const int El = counts.numel();
  TORCH_CHECK(El <= 1024, "moe_plan: at most 1024 local experts");
  TORCH_CHECK(tiles_gu.size(0) == tiles_d.size(0) && tiles_gu.size(1) == 4, "moe_plan: tiles [n, 4] int32");
  const at::cuda::CUDAGuard g(counts.device());
  moe_plan_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      counts.data_ptr<int>(), El, offsets.data_ptr<int>(), int(bn), int(ft_gu), int(ft_d),
      reinterpret_cast<int4*>(tiles_gu.data_ptr<int>()), n_gu.data_ptr<int>(),
      reinterpret_cast<int4*>(tiles_d.data_ptr<int>()), n_d.data_ptr<int>(), int(tiles_gu.size(0)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_gather(const torch::Tensor& x, int64_t e0, int64_t e_local, const torch::Tensor& topk_ids,
                const torch::Tensor& slot, const torch::Tensor& offsets, torch::Tensor& pos, torch::Tensor& xs) {
  const int T = x.size(0), H = x.size(1), K = topk_ids.size(1);
  TORCH_CHECK(H % 8 == 0 && x.is_contiguous(), "moe_gather: contiguous x, H % 8 == 0");
  if (T == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  moe_gather_kernel<<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), H, K, int(e0), int(e_local), topk_ids.data_ptr<int>(),
      slot.data_ptr<int>(), offsets.data_ptr<int>(), pos.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(xs.data_ptr()),
      long(xs.numel() / H), check_word(x.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_combine(const torch::Tensor& ys, const torch::Tensor& pos, const torch::Tensor& topk_w, torch::Tensor& out,
                 const std::vector<int64_t>& push_ptrs, int64_t push_rank, int64_t push_rows) {
  const int T = out.size(0), H = out.size(1), K = pos.size(1);
  if (T == 0) return;
  const at::cuda::CUDAGuard g(out.device());
  CombinePush push{};
  if (!push_ptrs.empty()) {
    TORCH_CHECK(push_ptrs.size() <= 8 && push_rank >= 0 && push_rank < (int64_t)push_ptrs.size(),
                "moe_combine push: up to 8 ranks");
    TORCH_CHECK(push_rows > 0 && push_rows * (int64_t)push_ptrs.size() >= T, "moe_combine push: rows cover T");
    TORCH_CHECK(H % 8 == 0, "moe_combine push: H must be a multiple of 8");
    for (size_t r = 0; r < push_ptrs.size(); ++r) {
      TORCH_CHECK(push_ptrs[r] % 16 == 0, "moe_combine push: peer buffers must be 16-byte aligned");
      push.p[r] = static_cast<unsigned long long>(push_ptrs[r]);
    }
    push.world = static_cast<int>(push_ptrs.size());
    push.rank = static_cast<int>(push_rank);
    push.rows = static_cast<int>(push_rows);
  }
  moe_combine_kernel<<<T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(ys.data_ptr()), H, K, pos.data_ptr<int>(), topk_w.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), long(ys.numel() / H), check_word(out.device().index()), push);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
