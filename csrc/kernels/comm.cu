// Tensor-parallel collectives fused with their compute, over NVLink / NVSwitch
// peer memory (one process per GPU; buffers mapped on every rank).
//
//   tp_allreduce_rmsnorm: the row-parallel GEMM (o_proj / down_proj) leaves its
//   partial sums in a peer-mapped buffer; this kernel
//     A. tells every peer "my partial is complete" and waits (bounded) for theirs,
//     B. for the token rows this rank owns, sums the partials of all ranks with
//        16-byte P2P loads, adds the residual, applies RMSNorm,
//     C. writes the normalised rows into every rank's input buffer with 16-byte
//        P2P stores (the all-gather), then the last CTA waits (bounded) until
//        every peer finished writing into this rank's buffer.
//   That is reduce-scatter + residual + RMSNorm + all-gather in one launch, and
//   every byte crosses NVLink once per direction: 2 (t-1)/t * T * H * 2 bytes.
//
//   tp_allgather_rows: all-gather of row slices (used for logits / hidden states).
//
// Synchronisation: per-rank flag words in the peer-mapped buffer carry a
// monotonically increasing epoch kept in device memory (advanced by the last
// CTA of every launch), so the same launch works inside CUDA graphs.  Every
// wait is bounded by %globaltimer; a wait that gives up sets
// kStatusCommTimeout in the caller's status word and the kernel returns, so a
// dead peer can never hang this GPU.
//
// Replaces the reference's no-op CollectiveOps / TensorCollectiveOps
// (crates/engine/src/core/parallelism.rs:105-178).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {
namespace comm {

constexpr int kMaxRanks = 8;

struct Peers {
  uint64_t p[kMaxRanks];
};

// Flag block layout (uint32 words) at the start of every rank's flag region:
//   [0, 8)    ready[src]   written by peer src: its partial for epoch e is complete
//   [8, 16)   done[src]    written by peer src: its all-gather stores into this rank are complete
//   [16]      epoch        local: number of completed fused collectives
//   [17]      cta counter  local: CTAs of the current launch that finished
constexpr int kReady = 0, kDone = 8, kEpoch = 16, kCtaCount = 17;
constexpr int kFlagWords = 32;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until flags[base + r] >= target for every rank r.
__device__ bool wait_flags(const uint32_t* flags, int base, int world, uint32_t target, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < world; ++r) {
    while (ld_acquire_sys(flags + base + r) < target) {
      if (globaltimer_ns() - t0 > timeout_ns) return false;
    }
  }
  return true;
}

struct ARArgs {
  Peers partial;  // bf16 [T, H] partial sums, one buffer per rank
  Peers xout;     // bf16 [T, H] normalised output, one buffer per rank (all-gathered)
  Peers flags;    // uint32 flag blocks, one per rank
  __nv_bfloat16* resid;  // local residual [T, H] (rows this rank owns are the valid ones)
  const __nv_bfloat16* w;
  int rank, world, T, H, rows_per_rank;
  float eps;
  uint64_t timeout_ns;
  int* status;
  // 1: the row-parallel GEMM already pushed every rank's partial rows of this
  // rank's slice into the local buffer as [world][rows_per_rank][H] slots
  // (reduce-scatter fused into the GEMM epilogue); phase B then reads local
  // memory only.  0: partials are [T, H] in each rank's own buffer (pulled).
  int pushed;
};

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

// grid: a fixed number of CTAs striding over the owned rows; block: H/8 threads
// (one 16-byte vector each; up to 1024 threads at H = 8192, so the kernel is
// held to the 64 registers a 1024-thread block can have)
__global__ void __launch_bounds__(1024) tp_allreduce_rmsnorm_kernel(const ARArgs a) {
  __shared__ float red[33];
  __shared__ int ok_s, last_s;
  __shared__ uint32_t epoch_s;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(a.flags.p[a.rank]);
  if (threadIdx.x == 0) {
    epoch_s = my_flags[kEpoch];
    ok_s = 1;
  }
  __syncthreads();
  const uint32_t target = epoch_s + 1;
  // A. every CTA announces readiness (idempotent) so no CTA depends on another being scheduled
  if (threadIdx.x < a.world)
    st_release_sys(reinterpret_cast<uint32_t*>(a.flags.p[threadIdx.x]) + kReady + a.rank, target);
  if (threadIdx.x == 0) {
    if (!wait_flags(my_flags, kReady, a.world, target, a.timeout_ns)) {
      ok_s = 0;
      atomicOr(a.status, kStatusCommTimeout);
    }
  }
  __syncthreads();
  const int i = threadIdx.x * 8;
  const bool active = i < a.H;
  float wf[8];
  if (active) bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.w + i), wf);
  for (int lr = blockIdx.x; ok_s && lr < a.rows_per_rank; lr += gridDim.x) {
    const int row = a.rank * a.rows_per_rank + lr;
    if (row >= a.T) break;
    // B. reduce this rank's rows over all ranks' partials, residual add, RMSNorm
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (active) {
      uint4 parts[kMaxRanks];
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < a.world)
          parts[r] = a.pushed ? *reinterpret_cast<const uint4*>(
                                    reinterpret_cast<const __nv_bfloat16*>(a.partial.p[a.rank]) +
                                    ((long)r * a.rows_per_rank + lr) * a.H + i)
                              : *reinterpret_cast<const uint4*>(
                                    reinterpret_cast<const __nv_bfloat16*>(a.partial.p[r]) + (long)row * a.H + i);
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < a.world) {
          float f[8];
          bf16x8_to_f32(parts[r], f);
#pragma unroll
          for (int k = 0; k < 8; ++k) v[k] += f[k];
        }
      float rs[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.resid + (long)row * a.H + i), rs);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] += rs[k];
      const uint4 nb = f32_to_bf16x8(v);
      *reinterpret_cast<uint4*>(a.resid + (long)row * a.H + i) = nb;
      bf16x8_to_f32(nb, v);
    }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += v[k] * v[k];
    const float inv = rsqrtf(block_sum(ss, red) / a.H + a.eps);
    if (active) {
      float o8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) o8[k] = v[k] * inv * wf[k];
      const uint4 o = f32_to_bf16x8(o8);
      // C. all-gather: the normalised row goes to every rank's input buffer
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < a.world)
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.xout.p[r]) + (long)row * a.H + i) = o;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(reinterpret_cast<int*>(my_flags + kCtaCount), 1);
    last_s = (prev == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (last_s && threadIdx.x == 0) {
    my_flags[kCtaCount] = 0;
    __threadfence_system();
    for (int r = 0; r < a.world; ++r)
      st_release_sys(reinterpret_cast<uint32_t*>(a.flags.p[r]) + kDone + a.rank, target);
    if (!wait_flags(my_flags, kDone, a.world, target, a.timeout_ns)) atomicOr(a.status, kStatusCommTimeout);
    my_flags[kEpoch] = target;  // stream order makes the next launch see it
    __threadfence();
  }
}

// All-gather of row slices: rank r owns rows [r*rows_per_rank, ...) of src (local,
// [T, C] bf16) and writes them into every rank's dst buffer (peer mapped).
struct AGArgs {
  Peers dst;
  Peers flags;
  const uint4* src;  // local rows, 16-byte vectors
  int rank, world, T, C16, rows_per_rank;  // C16 = row bytes / 16
  uint64_t timeout_ns;
  int* status;
};

__global__ void tp_allgather_rows_kernel(const AGArgs a) {
  __shared__ int last_s;
  __shared__ uint32_t epoch_s;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(a.flags.p[a.rank]);
  if (threadIdx.x == 0) epoch_s = my_flags[kEpoch];
  __syncthreads();
  const uint32_t target = epoch_s + 1;
  const int r0 = a.rank * a.rows_per_rank;
  const int r1 = min(a.T, r0 + a.rows_per_rank);
  const long n = (long)(r1 > r0 ? r1 - r0 : 0) * a.C16;
  for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < n; idx += (long)gridDim.x * blockDim.x) {
    const long off = (long)r0 * a.C16 + idx;
    const uint4 v = a.src[off];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < a.world) reinterpret_cast<uint4*>(a.dst.p[r])[off] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(reinterpret_cast<int*>(my_flags + kCtaCount), 1);
    last_s = (prev == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (last_s && threadIdx.x == 0) {
    my_flags[kCtaCount] = 0;
    __threadfence_system();
    for (int r = 0; r < a.world; ++r)
      st_release_sys(reinterpret_cast<uint32_t*>(a.flags.p[r]) + kDone + a.rank, target);
    if (!wait_flags(my_flags, kDone, a.world, target, a.timeout_ns)) atomicOr(a.status, kStatusCommTimeout);
    my_flags[kEpoch] = target;
    __threadfence();
  }
}

// Stand-alone bounded barrier (used by tests of the timeout path and at start-up).
__global__ void tp_barrier_kernel(Peers flags, int rank, int world, uint64_t timeout_ns, int* status) {
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(flags.p[rank]);
  const uint32_t target = my_flags[kEpoch] + 1;
  __threadfence_system();
  for (int r = 0; r < world; ++r) st_release_sys(reinterpret_cast<uint32_t*>(flags.p[r]) + kDone + rank, target);
  if (!wait_flags(my_flags, kDone, world, target, timeout_ns)) atomicOr(status, kStatusCommTimeout);
  my_flags[kEpoch] = target;
}

Peers to_peers(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() >= 1 && v.size() <= kMaxRanks, "1..8 ranks supported");
  Peers p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = static_cast<uint64_t>(v[i]);
  return p;
}

}  // namespace comm

int64_t tp_flag_words() { return comm::kFlagWords; }

void tp_allreduce_rmsnorm(const std::vector<int64_t>& partial_ptrs, const std::vector<int64_t>& x_ptrs,
                          const std::vector<int64_t>& flag_ptrs, int64_t rank, torch::Tensor& residual,
                          const torch::Tensor& w, double eps, int64_t T, double timeout_s,
                          const torch::Tensor& status, bool pushed) {
  const int world = static_cast<int>(partial_ptrs.size());
  TORCH_CHECK(x_ptrs.size() == partial_ptrs.size() && flag_ptrs.size() == partial_ptrs.size(), "rank count mismatch");
  TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && residual.is_contiguous(), "residual bf16 contiguous");
  const int H = residual.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8192, "H must be a multiple of 8 and <= 8192");
  if (T <= 0) return;
  const at::cuda::CUDAGuard g(residual.device());
  comm::ARArgs a;
  a.partial = comm::to_peers(partial_ptrs);
  a.xout = comm::to_peers(x_ptrs);
  a.flags = comm::to_peers(flag_ptrs);
  a.resid = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  a.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  a.rank = int(rank);
  a.world = world;
  a.T = int(T);
  a.H = H;
  a.rows_per_rank = int((T + world - 1) / world);
  a.eps = float(eps);
  a.timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  a.status = status.data_ptr<int>();
  a.pushed = pushed ? 1 : 0;
  const int threads = ((H / 8 + 31) / 32) * 32;
  // a fixed, fully resident grid striding over the owned rows keeps the number
  // of flag waits and remote ready-signals independent of the batch size
  const int blocks = std::max(1, std::min(a.rows_per_rank, 2 * 148));
  comm::tp_allreduce_rmsnorm_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_allgather_rows(const torch::Tensor& src, const std::vector<int64_t>& dst_ptrs,
                       const std::vector<int64_t>& flag_ptrs, int64_t rank, int64_t T, double timeout_s,
                       const torch::Tensor& status) {
  const int world = static_cast<int>(dst_ptrs.size());
  TORCH_CHECK(src.is_contiguous() && (src.size(-1) * src.element_size()) % 16 == 0, "rows must be 16-byte multiples");
  if (T <= 0) return;
  const at::cuda::CUDAGuard g(src.device());
  comm::AGArgs a;
  a.dst = comm::to_peers(dst_ptrs);
  a.flags = comm::to_peers(flag_ptrs);
  a.src = reinterpret_cast<const uint4*>(src.data_ptr());
  a.rank = int(rank);
  a.world = world;
  a.T = int(T);
  a.C16 = int(src.size(-1) * src.element_size() / 16);
  a.rows_per_rank = int((T + world - 1) / world);
  a.timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  a.status = status.data_ptr<int>();
  const long n = (long)a.rows_per_rank * a.C16;
  const int blocks = int(std::min<long>(148, std::max<long>(1, (n + 255) / 256)));
  comm::tp_allgather_rows_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_barrier(const std::vector<int64_t>& flag_ptrs, int64_t rank, double timeout_s, const torch::Tensor& status) {
  const at::cuda::CUDAGuard g(status.device());
  comm::tp_barrier_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(
      comm::to_peers(flag_ptrs), int(rank), int(flag_ptrs.size()), static_cast<uint64_t>(timeout_s * 1e9),
      status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
