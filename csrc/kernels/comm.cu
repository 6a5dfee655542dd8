// Tensor-parallel collectives fused with their compute, over NVLink / NVSwitch
// peer memory (one process per GPU; buffers mapped on every rank).
//
//   tp_allreduce_rmsnorm: the row-parallel GEMM (o_proj / down_proj) leaves its
//   partial sums in a peer-mapped buffer; this kernel
//     A. tells every peer "my partial is complete" and waits (bounded) for theirs,
//     B. for the token rows this rank owns, sums the partials of all ranks with
//        16-byte P2P loads, adds the residual, applies RMSNorm,
//     C. writes the normalised rows into every rank's input buffer with 16-byte
//        P2P stores (the all-gather), then every block waits (bounded) until
//        the same block of every peer finished writing into this rank's buffer.
//   Each block synchronises only with the same block index on the peers (its
//   own ready / done / epoch words), so a launch has no CTA counter and no
//   serial last-CTA hand-off, and the kernel is launched with programmatic
//   stream serialisation so its start overlaps the producing GEMM's tail.
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
// Poisoning: a timed-out wait also sets the local poison word.  From then on
// every collective launch on this rank does nothing but set
// kStatusCommPoisoned, and the epoch no longer advances, so a late peer can
// never pair its epoch with a stale one here and read overwritten partials:
// it times out on this rank's missing "done" flag and poisons itself too.
// The host reads the status word after each step, fails the step's requests
// and stops using the communicator (falls back to NCCL or rebuilds it).
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
//   [18]      poison       local: nonzero once a wait of this rank timed out
//   [19]      done count   written by every peer block of a deferred all-gather (red.add)
//   [20]      done expect  local: done count the next reader of the rows waits for
constexpr int kReady = 0, kDone = 8, kEpoch = 16, kCtaCount = 17, kPoison = kFlagPoison;
static_assert(kFlagDoneCount == 19 && kFlagDoneExpect == 20, "flag block layout");
// Per-block flags of tp_allreduce_rmsnorm (block b of a launch pairs only with
// block b of every peer, so no CTA counter and no last-CTA hand-off):
//   [kBlkReady + src * kMaxArBlocks + b]  written by peer src's block b: its partials are complete
//   [kBlkDone  + src * kMaxArBlocks + b]  written by peer src's block b: its all-gather stores here are complete
//   [kBlkEpoch + b]                       local: completed launches that had a block b
constexpr int kMaxArBlocks = 2 * 148;
constexpr int kBlkReady = 32, kBlkDone = kBlkReady + kMaxRanks * kMaxArBlocks,
              kBlkEpoch = kBlkDone + kMaxRanks * kMaxArBlocks;
constexpr int kFlagWords = ((kBlkEpoch + kMaxArBlocks + 63) / 64) * 64;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool poisoned(const uint32_t* my_flags) {
  return *reinterpret_cast<const volatile uint32_t*>(my_flags + kPoison) != 0u;
}
__device__ __forceinline__ void poison(uint32_t* my_flags, int* status) {
  *reinterpret_cast<volatile uint32_t*>(my_flags + kPoison) = 1u;
  __threadfence();
  atomicOr(status, kStatusCommTimeout);
}

// Launch-end bookkeeping shared by the collectives: the last CTA to finish
// signals "done" to every peer, waits (bounded) for theirs and advances the
// epoch -- unless the communicator is poisoned, in which case it only resets
// the CTA counter.
__device__ void finish_collective(uint32_t* my_flags, const uint64_t (&peer_flags)[8], int rank, int world,
                                  uint32_t target, uint64_t timeout_ns, int* status, int* last_s);

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

// Bounded wait until *flag >= target.
__device__ bool wait_flag(const uint32_t* flag, uint32_t target, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(flag) < target) {
    if (globaltimer_ns() - t0 > timeout_ns) return false;
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
  // optional phase timeline of block 0 (tp_ar_set_trace): 4 %globaltimer
  // stamps per launch -- entry, ready wait passed, rows written, done wait
  // passed -- at [(epoch % trace_cap) * 4]
  unsigned long long* trace;
  int trace_cap;
  // 1: do not wait for the peers' rows here; every block adds 1 to every
  // rank's done count after its stores, and the next kernel that reads the
  // rows (a GEMM given wait_flags) waits for the count instead
  int defer_done;
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
  __shared__ int ok_s, fail_s;
  __shared__ uint32_t target_s;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(a.flags.p[a.rank]);
  const int blk = blockIdx.x;
  // Launched with programmatic stream serialisation: nothing before this wait
  // may read what an earlier kernel writes (the previous collective may still
  // be finishing when the producing GEMM lets this launch start), so the
  // poison word, this block's epoch, the partials and the residual are all
  // read after it.
  griddep_wait();
  griddep_launch_dependents();  // the next GEMM may stage its weights meanwhile
  if (threadIdx.x == 0) {
    ok_s = poisoned(my_flags) ? 0 : 1;
    fail_s = 0;
    if (!ok_s) atomicOr(a.status, kStatusCommPoisoned);
    target_s = my_flags[kBlkEpoch + blk] + 1;
  }
  __syncthreads();
  if (!ok_s) return;  // poisoned communicator: touch nothing
  const uint32_t target = target_s;
  const bool tr = a.trace != nullptr && blk == 0 && threadIdx.x == 0;
  unsigned long long* trs = tr ? a.trace + (target % a.trace_cap) * 4 : nullptr;
  if (tr) trs[0] = globaltimer_ns();
  // A. this block tells block `blk` of every rank that this rank's partials are
  // complete (the producing GEMM finished before this launch), and thread r
  // waits for rank r's signal: one flag pair per (block, rank), no CTA counter
  if (threadIdx.x < a.world) {
    const int r = threadIdx.x;
    st_release_sys(reinterpret_cast<uint32_t*>(a.flags.p[r]) + kBlkReady + a.rank * kMaxArBlocks + blk, target);
    if (!wait_flag(my_flags + kBlkReady + r * kMaxArBlocks + blk, target, a.timeout_ns)) fail_s = 1;
  }
  __syncthreads();
  if (fail_s) {
    if (threadIdx.x == 0) poison(my_flags, a.status);
    return;
  }
  if (tr) trs[1] = globaltimer_ns();
  const int i = threadIdx.x * 8;
  const bool active = i < a.H;
  float wf[8];
  if (active) bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.w + i), wf);
  for (int lr = blk; lr < a.rows_per_rank; lr += gridDim.x) {
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
  // D. the block's stores (all threads, ordered before the release by the
  // barrier; release is cumulative) are announced to block `blk` of every
  // rank, and thread r waits until rank r's block `blk` finished writing here.
  // Every rank launches the same grid, so when all blocks pass, every row of
  // this rank's input buffer has arrived.
  __syncthreads();
  if (tr) trs[2] = globaltimer_ns();
  if (a.defer_done) {
    if (threadIdx.x < a.world) {
      uint32_t* cnt = reinterpret_cast<uint32_t*>(a.flags.p[threadIdx.x]) + kFlagDoneCount;
      asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(cnt) : "memory");
    }
    if (threadIdx.x == 0) {
      if (blk == 0) my_flags[kFlagDoneExpect] += gridDim.x * a.world;  // read after this launch completes
      my_flags[kBlkEpoch + blk] = target;
      if (tr) trs[3] = globaltimer_ns();
    }
    return;
  }
  if (threadIdx.x < a.world) {
    const int r = threadIdx.x;
    st_release_sys(reinterpret_cast<uint32_t*>(a.flags.p[r]) + kBlkDone + a.rank * kMaxArBlocks + blk, target);
    if (!wait_flag(my_flags + kBlkDone + r * kMaxArBlocks + blk, target, a.timeout_ns)) fail_s = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (fail_s) poison(my_flags, a.status);
    else my_flags[kBlkEpoch + blk] = target;  // stream order makes the next launch see it
    if (tr) trs[3] = globaltimer_ns();
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
  __shared__ int last_s, ok_s;
  __shared__ uint32_t epoch_s;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(a.flags.p[a.rank]);
  if (threadIdx.x == 0) {
    epoch_s = my_flags[kEpoch];
    ok_s = poisoned(my_flags) ? 0 : 1;
    if (!ok_s) atomicOr(a.status, kStatusCommPoisoned);
  }
  __syncthreads();
  if (!ok_s) return;
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
  if (threadIdx.x == 0) finish_collective(my_flags, a.flags.p, a.rank, a.world, target, a.timeout_ns, a.status, &last_s);
}

// Stand-alone bounded barrier (used by tests of the timeout path and at start-up).
__global__ void tp_barrier_kernel(Peers flags, int rank, int world, uint64_t timeout_ns, int* status) {
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(flags.p[rank]);
  if (poisoned(my_flags)) {
    atomicOr(status, kStatusCommPoisoned);
    return;
  }
  const uint32_t target = my_flags[kEpoch] + 1;
  __threadfence_system();
  for (int r = 0; r < world; ++r) st_release_sys(reinterpret_cast<uint32_t*>(flags.p[r]) + kDone + rank, target);
  if (!wait_flags(my_flags, kDone, world, target, timeout_ns)) {
    poison(my_flags, status);
    return;
  }
  my_flags[kEpoch] = target;
}

__device__ void finish_collective(uint32_t* my_flags, const uint64_t (&peer_flags)[8], int rank, int world,
                                  uint32_t target, uint64_t timeout_ns, int* status, int* last_s) {
  const int prev = atomicAdd(reinterpret_cast<int*>(my_flags + kCtaCount), 1);
  *last_s = (prev == (int)gridDim.x - 1);
  if (!*last_s) return;
  my_flags[kCtaCount] = 0;
  if (poisoned(my_flags)) return;  // a CTA of this launch timed out: no done signal, no epoch advance
  __threadfence_system();
  for (int r = 0; r < world; ++r) st_release_sys(reinterpret_cast<uint32_t*>(peer_flags[r]) + kDone + rank, target);
  if (!wait_flags(my_flags, kDone, world, target, timeout_ns)) {
    poison(my_flags, status);
    return;
  }
  my_flags[kEpoch] = target;  // stream order makes the next launch see it
  __threadfence();
}

// ---------------------------------------------------------------- last-layer logits
// Status agreement: every rank's status word travels with its logits share, and
// each rank writes the OR of all ranks' words next to the sampled tokens, so all
// ranks see the same error bits after a step and fail the same requests.

__device__ __forceinline__ void argmax_pair(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

struct ArgmaxGatherArgs {
  Peers slots;  // per rank: uint2 [world][max_rows + 1]; entry [r][row] = (value bits, global index) from rank r,
                // entry [r][max_rows] = rank r's status word
  Peers flags;
  const __nv_bfloat16* logits;  // local vocabulary shard [NL, ld]
  long ld;
  int Vl, vocab_offset;
  int rank, world, NL, max_rows;
  int* out;  // int32 [NL + 1]: greedy tokens, then the OR of every rank's status word
  int* status;
  uint64_t timeout_ns;
};

// One CTA per logits row: argmax over the local shard, the (value, index) pair
// stored into every rank's slot array with 8-byte P2P stores; the last CTA to
// finish exchanges "done" flags (bounded) and reduces the world pairs of every
// row (largest value, lowest global index on ties: the single-GPU argmax rule).
__global__ void __launch_bounds__(1024) tp_argmax_gather_kernel(const ArgmaxGatherArgs a) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ int ok_s, last_s;
  __shared__ uint32_t epoch_s;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(a.flags.p[a.rank]);
  if (threadIdx.x == 0) {
    epoch_s = my_flags[kEpoch];
    ok_s = poisoned(my_flags) ? 0 : 1;
    if (!ok_s) {
      atomicOr(a.status, kStatusCommPoisoned);
      if (blockIdx.x == 0) a.out[a.NL] = atomicOr(a.status, 0);
    }
  }
  __syncthreads();
  if (!ok_s) return;
  const uint32_t target = epoch_s + 1;
  const int row = blockIdx.x;
  const __nv_bfloat16* lr = a.logits + (long)row * a.ld;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int k = threadIdx.x; k < a.Vl; k += blockDim.x) argmax_pair(v, idx, __bfloat162float(lr[k]), k);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) argmax_pair(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = v;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    v = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    idx = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      argmax_pair(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
    // lanes 0..world-1 each store the pair into one rank's slots
    if (threadIdx.x < a.world) {
      const uint2 pr = make_uint2(__float_as_uint(v), static_cast<uint32_t>(idx + a.vocab_offset));
      reinterpret_cast<uint2*>(a.slots.p[threadIdx.x])[(long)a.rank * (a.max_rows + 1) + row] = pr;
      if (row == 0)
        reinterpret_cast<uint2*>(a.slots.p[threadIdx.x])[(long)a.rank * (a.max_rows + 1) + a.max_rows] =
            make_uint2(static_cast<uint32_t>(atomicOr(a.status, 0)), 0u);
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(reinterpret_cast<int*>(my_flags + kCtaCount), 1);
    last_s = (prev == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (!last_s) return;
  if (threadIdx.x == 0) {
    my_flags[kCtaCount] = 0;
    ok_s = 0;
    if (!poisoned(my_flags)) {
      __threadfence_system();
      for (int r = 0; r < a.world; ++r)
        st_release_sys(reinterpret_cast<uint32_t*>(a.flags.p[r]) + kDone + a.rank, target);
      if (wait_flags(my_flags, kDone, a.world, target, a.timeout_ns)) {
        ok_s = 1;
        my_flags[kEpoch] = target;
      } else {
        poison(my_flags, a.status);
      }
    }
  }
  __syncthreads();
  const uint2* mine = reinterpret_cast<const uint2*>(a.slots.p[a.rank]);
  if (!ok_s) {
    if (threadIdx.x == 0) a.out[a.NL] = atomicOr(a.status, 0);
    return;
  }
  for (int r = threadIdx.x; r < a.NL; r += blockDim.x) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int q = 0; q < a.world; ++q) {
      const volatile uint32_t* pr = reinterpret_cast<const volatile uint32_t*>(mine + (long)q * (a.max_rows + 1) + r);
      argmax_pair(bv, bi, __uint_as_float(pr[0]), static_cast<int>(pr[1]));
    }
    a.out[r] = bi;
  }
  if (threadIdx.x == 0) {
    int st = 0;
    for (int q = 0; q < a.world; ++q)
      st |= static_cast<int>(*reinterpret_cast<const volatile uint32_t*>(mine + (long)q * (a.max_rows + 1) + a.max_rows));
    a.out[a.NL] = st | atomicOr(a.status, 0);
  }
}

struct GatherColsArgs {
  Peers dst;       // per rank: bf16 [max_rows, V] full-vocabulary logits
  Peers stat;      // per rank: int32 [world] status words
  Peers flags;
  const uint4* src;  // local shard rows, 16-byte vectors
  long src_ld16;     // source row stride in 16-byte vectors
  int cols16;        // shard width in 16-byte vectors (Vl * 2 / 16)
  long dst_ld16;     // destination row stride in 16-byte vectors (V * 2 / 16)
  int rank, world, NL;
  int* out_status;  // local int32: OR of every rank's status word
  int* status;
  uint64_t timeout_ns;
};

// Vocabulary-parallel logits -> full rows on every rank: each rank stores its
// [NL, Vl] shard at columns [rank * Vl, (rank + 1) * Vl) of every rank's
// buffer with 16-byte P2P stores; the stochastic sampler then runs locally on
// identical rows with identical Philox streams, so the ranks agree.
__global__ void __launch_bounds__(256) tp_gather_cols_kernel(const GatherColsArgs a) {
  __shared__ int ok_s, last_s;
  __shared__ uint32_t epoch_s;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(a.flags.p[a.rank]);
  if (threadIdx.x == 0) {
    epoch_s = my_flags[kEpoch];
    ok_s = poisoned(my_flags) ? 0 : 1;
    if (!ok_s) {
      atomicOr(a.status, kStatusCommPoisoned);
      if (blockIdx.x == 0) *a.out_status = atomicOr(a.status, 0);
    }
  }
  __syncthreads();
  if (!ok_s) return;
  const uint32_t target = epoch_s + 1;
  const long n = (long)a.NL * a.cols16;
  for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
    const long r = e / a.cols16, c = e - r * a.cols16;
    const uint4 v = a.src[r * a.src_ld16 + c];
    const long off = r * a.dst_ld16 + (long)a.rank * a.cols16 + c;
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q)
      if (q < a.world) reinterpret_cast<uint4*>(a.dst.p[q])[off] = v;
  }
  if (blockIdx.x == 0 && threadIdx.x < a.world)
    reinterpret_cast<int*>(a.stat.p[threadIdx.x])[a.rank] = atomicOr(a.status, 0);
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) finish_collective(my_flags, a.flags.p, a.rank, a.world, target, a.timeout_ns, a.status, &last_s);
  __syncthreads();
  if (last_s && threadIdx.x == 0) {
    int st = atomicOr(a.status, 0);
    if (!poisoned(my_flags))
      for (int q = 0; q < a.world; ++q) st |= reinterpret_cast<const volatile int*>(a.stat.p[a.rank])[q];
    *a.out_status = st;
  }
}

Peers to_peers(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() >= 1 && v.size() <= kMaxRanks, "1..8 ranks supported");
  Peers p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = static_cast<uint64_t>(v[i]);
  return p;
}

}  // namespace comm

int64_t tp_flag_words() { return comm::kFlagWords; }

static unsigned long long* g_ar_trace = nullptr;
static int g_ar_trace_cap = 0;
void tp_ar_set_trace(const c10::optional<torch::Tensor>& buf) {
  if (buf.has_value() && buf->defined()) {
    TORCH_CHECK(buf->scalar_type() == at::kLong && buf->is_cuda() && buf->numel() >= 4, "trace: int64 [n * 4] CUDA");
    g_ar_trace = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
    g_ar_trace_cap = static_cast<int>(buf->numel() / 4);
  } else {
    g_ar_trace = nullptr;
    g_ar_trace_cap = 0;
  }
}

void tp_allreduce_rmsnorm(const std::vector<int64_t>& partial_ptrs, const std::vector<int64_t>& x_ptrs,
                          const std::vector<int64_t>& flag_ptrs, int64_t rank, torch::Tensor& residual,
                          const torch::Tensor& w, double eps, int64_t T, double timeout_s,
                          const torch::Tensor& status, bool pushed, bool defer_done) {
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
  a.defer_done = defer_done ? 1 : 0;
  a.trace = g_ar_trace;
  a.trace_cap = g_ar_trace_cap;
  const int threads = ((H / 8 + 31) / 32) * 32;
  // a fixed, fully resident grid striding over the owned rows keeps the number
  // of flag waits and remote ready-signals independent of the batch size
  const int blocks = std::max(1, std::min(a.rows_per_rank, comm::kMaxArBlocks));
  static const int env_pdl = [] {
    const char* e = std::getenv("BLOOM_PDL");
    return e ? std::atoi(e) : 1;
  }();
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cfg.attrs = attr;
  cfg.numAttrs = env_pdl ? 1 : 0;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, comm::tp_allreduce_rmsnorm_kernel, a));
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

void tp_argmax_gather(const torch::Tensor& logits, int64_t vocab_offset, const std::vector<int64_t>& slot_ptrs,
                      int64_t max_rows, const std::vector<int64_t>& flag_ptrs, int64_t rank, torch::Tensor& out,
                      double timeout_s, const torch::Tensor& status) {
  const int world = static_cast<int>(slot_ptrs.size());
  TORCH_CHECK(flag_ptrs.size() == slot_ptrs.size(), "rank count mismatch");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1, "logits bf16 [NL, V]");
  TORCH_CHECK(out.scalar_type() == at::kInt && out.numel() >= logits.size(0) + 1, "out int32 [NL + 1]");
  const int NL = static_cast<int>(logits.size(0));
  TORCH_CHECK(NL <= max_rows, "more logits rows than the slot array holds");
  if (NL <= 0) return;
  const at::cuda::CUDAGuard g(logits.device());
  comm::ArgmaxGatherArgs a;
  a.slots = comm::to_peers(slot_ptrs);
  a.flags = comm::to_peers(flag_ptrs);
  a.logits = reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr());
  a.ld = logits.stride(0);
  a.Vl = static_cast<int>(logits.size(1));
  a.vocab_offset = static_cast<int>(vocab_offset);
  a.rank = int(rank);
  a.world = world;
  a.NL = NL;
  a.max_rows = static_cast<int>(max_rows);
  a.out = out.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  comm::tp_argmax_gather_kernel<<<NL, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_gather_cols(const torch::Tensor& logits, const std::vector<int64_t>& dst_ptrs, int64_t dst_cols,
                    const std::vector<int64_t>& stat_ptrs, const std::vector<int64_t>& flag_ptrs, int64_t rank,
                    torch::Tensor& out_status, double timeout_s, const torch::Tensor& status) {
  const int world = static_cast<int>(dst_ptrs.size());
  TORCH_CHECK(flag_ptrs.size() == dst_ptrs.size() && stat_ptrs.size() == dst_ptrs.size(), "rank count mismatch");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1, "logits bf16 [NL, V]");
  TORCH_CHECK((logits.size(1) * 2) % 16 == 0 && (logits.stride(0) * 2) % 16 == 0 && (dst_cols * 2) % 16 == 0,
              "rows must be 16-byte multiples");
  TORCH_CHECK(logits.size(1) * world == dst_cols, "shard width x ranks must equal the full row");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0, "logits must be 16-byte aligned");
  const int NL = static_cast<int>(logits.size(0));
  if (NL <= 0) return;
  const at::cuda::CUDAGuard g(logits.device());
  comm::GatherColsArgs a;
  a.dst = comm::to_peers(dst_ptrs);
  a.stat = comm::to_peers(stat_ptrs);
  a.flags = comm::to_peers(flag_ptrs);
  a.src = reinterpret_cast<const uint4*>(logits.data_ptr());
  a.src_ld16 = logits.stride(0) * 2 / 16;
  a.cols16 = static_cast<int>(logits.size(1) * 2 / 16);
  a.dst_ld16 = dst_cols * 2 / 16;
  a.rank = int(rank);
  a.world = world;
  a.NL = NL;
  a.out_status = out_status.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  const long n = (long)NL * a.cols16;
  const int blocks = int(std::min<long>(2 * 148, std::max<long>(1, (n + 255) / 256)));
  comm::tp_gather_cols_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
