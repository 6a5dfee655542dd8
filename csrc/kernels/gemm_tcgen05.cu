// Dense bf16 GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   y[M, N] = x[M, K] @ w[N, K]^T        (nn.Linear layout, both K-major)
//
// The UMMA "A" operand is the weight tile (128 output features = UMMA M) and
// the "B" operand is the token tile (BN tokens = UMMA N, 16..256).  Putting the
// features on the 128-lane M side keeps tiny decode batches (M = 1..256
// tokens) on the tensor cores with no padding of the token dimension beyond a
// multiple of 16, and the same kernel covers large prefill batches with
// 128 x 256 tiles.  The accumulator lives in TMEM (lane = feature, column =
// token) and is double-buffered so the epilogue of tile i overlaps the MMAs of
// tile i+1.
//
// Warp roles (192 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + UMMA issuer (one elected lane)
//   warps 2..5  epilogue: tcgen05.ld of their TMEM lane quarter, fused
//               epilogue (bias / SwiGLU / residual / fp32 split-K partials)
//
// Replaces the reference's library GEMMs behind candle Linear layers
// (crates/engine/src/executor/qwen_streaming.rs:216-298, candle-transformers
// llama/qwen2/qwen3), which never had an sm_100 code path.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "bloom/common.cuh"
#include "bloom/ops.h"
#include "bloom/tma_host.h"

namespace bloom {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;

struct Args {
  int M, N, K;
  int num_feat_tiles, num_tok_tiles, splits, kb_per_split, num_kb;
  void* out;
  long ldo;
  const __nv_bfloat16* resid;
  long ldr;
  const __nv_bfloat16* bias;
  int* status;
  float* fix_ws;     // split-K fixup: [tiles, splits, BN, 128] fp32 partial accumulators
  int* fix_count;    // split-K fixup: (arrived, written) counters per output tile (self-resetting)
  int fixup;         // 1: splits > 1 with the last-arriving CTA reducing and running the epilogue
  // grouped mode (MoE experts): a device-built tile list replaces the regular
  // tile grid.  tiles[i] = (group, feat_tile, first token row, token row limit),
  // the A operand of group g starts at row g * rows_per_group.
  const int4* tiles;
  const int* num_tiles_dev;
  int rows_per_group;
  // L2 policy of the weight (A) tiles: 0 evict-first (each weight tile is
  // read by one token tile: decode), 1 normal (several token tiles re-read it
  // while it is hot: prefill), 2 evict-last.
  int wpol;
  int tok_group;  // token tiles per raster group (see decode_tile)
  // optional timeline (%globaltimer ns) of each CTA's first work item:
  // [entry, setup done, first stage landed, last MMA issued, accumulator seen
  // by the epilogue, epilogue done (cluster split-K: slice parked), cluster
  // reduction done, 0] x gridDim.x
  unsigned long long* trace;
  int vec;     // output / residual rows allow 16-byte vector access
  int csplit;  // > 1: cluster split-K, one tile per cluster of csplit CTAs (one K-slice each)
  int pdl;     // launched with programmatic stream serialization (weights prefetched before the wait)
  // Tensor-parallel reduce-scatter push (bf16 epilogue only): token row t is
  // owned by rank t / push_rows; its partial sum goes straight to that rank's
  // buffer over NVLink, into slot [push_rank][t % push_rows] of its
  // [world][push_rows][ldo] layout, while the rest of the GEMM runs.
  unsigned long long push[8];
  int push_world, push_rank, push_rows;
  int gelu_tanh;  // kEpiGelu: 1 = tanh approximation, 0 = erf; kEpiSwiGLU: 1 = GeGLU gate
  // Activations written by a deferred tensor-parallel all-gather: before the
  // first activation tile, the producer waits (bounded) until every peer's
  // rows arrived (wait_deferred_rows on this rank's flag block); nullptr = none
  uint32_t* wait_flags;
  uint64_t wait_timeout_ns;
};

// Row `tok` of the bf16 output: local, or the owner's slot for this rank (push).
__device__ __forceinline__ __nv_bfloat16* out_row_bf16(const Args& a, int tok) {
  if (a.push_world > 0) {
    const int owner = tok / a.push_rows;
    const int lr = tok - owner * a.push_rows;
    return reinterpret_cast<__nv_bfloat16*>(a.push[owner]) + ((long)a.push_rank * a.push_rows + lr) * a.ldo;
  }
  return reinterpret_cast<__nv_bfloat16*>(a.out) + (long)tok * a.ldo;
}

__device__ __forceinline__ void trace_mark(const Args& a, int slot) {
  if (a.trace != nullptr) a.trace[blockIdx.x * 8 + slot] = globaltimer_ns();
}

struct Tile {
  int ft, tt, sp, tok0, tok_end, arow;
};

template <int BN>
struct Cfg {
  static constexpr int kStages = BN >= 256 ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

// Tile order: splits fastest, then token tiles, then feature tiles, with the
// token tiles taken in groups of tok_group: all feature tiles of one group of
// token tiles run before the next group starts, so the activations of the
// group stay L2-resident while the weights stream past (a wave of the
// persistent grid touches tok_group token tiles and ~grid/tok_group weight tiles).
__device__ __forceinline__ void decode_tile(const Args& a, int t, int& feat_tile, int& tok_tile, int& split) {
  split = t % a.splits;
  const int rest = t / a.splits;
  const int per_group = a.tok_group * a.num_feat_tiles;
  const int g = rest / per_group;
  const int in = rest - g * per_group;
  const int gsize = min(a.tok_group, a.num_tok_tiles - g * a.tok_group);
  feat_tile = in / gsize;
  tok_tile = g * a.tok_group + (in - feat_tile * gsize);
}

template <int BN>
__device__ __forceinline__ Tile get_tile(const Args& a, int t) {
  Tile r;
  if (a.tiles != nullptr) {
    const int4 d = a.tiles[t];
    r.ft = d.y;
    r.tt = 0;
    r.sp = 0;
    r.tok0 = d.z;
    r.tok_end = d.w;
    r.arow = d.x * a.rows_per_group + d.y * BM;
  } else {
    decode_tile(a, t, r.ft, r.tt, r.sp);
    r.tok0 = r.tt * BN;
    r.tok_end = a.M;
    r.arow = r.ft * BM;
  }
  return r;
}

// Per-warp transpose scratch of the epilogue: 16 tokens x 32 features fp32,
// rows padded to 36 floats (conflict-free row writes and float4 column reads).
constexpr int kScrStride = 36;
constexpr int kScrFloats = 16 * kScrStride;

__device__ __forceinline__ void store8_bf16(__nv_bfloat16* dst, const float (&x)[8], int n, bool vec) {
  if (vec && n >= 8) {
    uint4 w;
    w.x = pack_bf16x2(x[0], x[1]);
    w.y = pack_bf16x2(x[2], x[3]);
    w.z = pack_bf16x2(x[4], x[5]);
    w.w = pack_bf16x2(x[6], x[7]);
    *reinterpret_cast<uint4*>(dst) = w;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k < n) dst[k] = __float2bfloat16(x[k]);
  }
}
__device__ __forceinline__ void store8_f32(float* dst, const float (&x)[8], int n, bool vec) {
  if (vec && n >= 8) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(x[4], x[5], x[6], x[7]);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k < n) dst[k] = x[k];
  }
}

// Runs the fused epilogue of columns [cbeg, cend) of one output tile.
// `load(c, v)` supplies the fp32 accumulator of columns [c, c+16) for this
// thread's row (feature): straight from TMEM, or summed over split-K partials.
// The accumulator holds one feature per lane and one token per column, the
// output is token-major, so each 32-feature x 16-token block is transposed
// through the warp's scratch and written as 16-byte vectors (8 features of one
// token per lane) instead of 2-byte scalars.
template <int BN, int EPI, typename Loader>
__device__ __forceinline__ void epilogue_tile(const Args& a, const Tile& tl, int q, int lane, float* scr, int cbeg,
                                              int cend, Loader&& load) {
  const int tok0 = tl.tok0;
  const int tok_end = tl.tok_end;
  if constexpr (EPI == kEpiSwiGLU) {
    // Weight rows are interleaved per 32-row group: 16 gate rows then the 16
    // matching up rows, so gate and up of one feature sit in lanes l and l+16.
    const int nout = a.N / 2;
    const int r = lane >> 1, fo = (lane & 1) * 8;
    const int f = tl.ft * (BM / 2) + q * 16 + fo;
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
    for (int c = cbeg; c < cend; c += 16) {
      if (tok0 + c >= tok_end) break;
      float v[16];
      load(c, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float up = __shfl_down_sync(0xffffffffu, v[j], 16);
        // lanes >= 16 write unused columns; gelu_tanh: the GeGLU gate (kEpiGeGLU)
        const float gate = a.gelu_tanh
                               ? 0.5f * v[j] * (1.f + tanhf(0.7978845608028654f * (v[j] + 0.044715f * v[j] * v[j] * v[j])))
                               : silu(v[j]);
        scr[j * kScrStride + lane] = gate * up;
      }
      __syncwarp();
      const int tok = tok0 + c + r;
      if (tok < tok_end && f < nout) {
        float x[8];
        *reinterpret_cast<float4*>(x) = *reinterpret_cast<const float4*>(scr + r * kScrStride + fo);
        *reinterpret_cast<float4*>(x + 4) = *reinterpret_cast<const float4*>(scr + r * kScrStride + fo + 4);
        store8_bf16(out + (long)tok * a.ldo + f, x, nout - f, a.vec);
      }
      __syncwarp();
    }
  } else {
    const int fo = (lane & 3) * 8;
    const int f = tl.ft * BM + q * 32 + fo;
    const int nf = a.N - f;  // features of this lane's group of 8 inside the matrix
    float bias[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) bias[k] = 0.f;
    if constexpr (EPI == kEpiBF16 || EPI == kEpiF32 || EPI == kEpiGelu || EPI == kEpiResidual) {
      if (a.bias != nullptr) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k < nf) bias[k] = __bfloat162float(a.bias[f + k]);
      }
    }
    for (int c = cbeg; c < cend; c += 16) {
      if (tok0 + c >= tok_end) break;
      float v[16];
      load(c, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) scr[j * kScrStride + lane] = v[j];
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int r = (lane >> 2) + 8 * i;
        const int tok = tok0 + c + r;
        if (tok >= tok_end || nf <= 0) continue;
        float x[8];
        *reinterpret_cast<float4*>(x) = *reinterpret_cast<const float4*>(scr + r * kScrStride + fo);
        *reinterpret_cast<float4*>(x + 4) = *reinterpret_cast<const float4*>(scr + r * kScrStride + fo + 4);
        if constexpr (EPI == kEpiBF16) {
#pragma unroll
          for (int k = 0; k < 8; ++k) x[k] += bias[k];
          store8_bf16(out_row_bf16(a, tok) + f, x, nf, a.vec);
        } else if constexpr (EPI == kEpiF32) {
#pragma unroll
          for (int k = 0; k < 8; ++k) x[k] += bias[k];
          store8_f32(reinterpret_cast<float*>(a.out) + (long)tok * a.ldo + f, x, nf, a.vec);
        } else if constexpr (EPI == kEpiPartialF32) {
          store8_f32(reinterpret_cast<float*>(a.out) + ((long)tl.sp * a.M + tok) * a.N + f, x, nf, a.vec);
        } else if constexpr (EPI == kEpiResidual) {
#pragma unroll
          for (int k = 0; k < 8; ++k) x[k] += bias[k];
          const __nv_bfloat16* rp = a.resid + (long)tok * a.ldr + f;
          if (a.vec && nf >= 8) {
            const uint4 rv = *reinterpret_cast<const uint4*>(rp);
            const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] += __bfloat162float(rb[k]);
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k)
              if (k < nf) x[k] += __bfloat162float(rp[k]);
          }
          store8_bf16(reinterpret_cast<__nv_bfloat16*>(a.out) + (long)tok * a.ldo + f, x, nf, a.vec);
        } else if constexpr (EPI == kEpiGelu) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float y = x[k] + bias[k];
            // 0.7978845608 = sqrt(2 / pi), the tanh form's scale (Hendrycks & Gimpel, 2016)
            x[k] = a.gelu_tanh ? 0.5f * y * (1.f + tanhf(0.7978845608028654f * (y + 0.044715f * y * y * y)))
                               : 0.5f * y * (1.f + erff(y * 0.7071067811865476f));
          }
          store8_bf16(reinterpret_cast<__nv_bfloat16*>(a.out) + (long)tok * a.ldo + f, x, nf, a.vec);
        }
      }
      __syncwarp();
    }
  }
}

// Named barrier of the four epilogue warps (threads 64..191).
__device__ __forceinline__ void epi_barrier() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Same barrier, returning whether any epilogue thread passed `pred` = true, so
// the four warps always leave the tile loop together (no warp can be left
// waiting at a later named barrier after another one gave up).
__device__ __forceinline__ bool epi_barrier_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, 1, 128, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred))
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Asynchronous 16-byte store into a cluster peer's shared memory that counts
// its bytes on the peer's mbarrier (complete_tx).
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, float x, float y, float z, float w,
                                            uint32_t cluster_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   cluster_addr),
               "f"(x), "f"(y), "f"(z), "f"(w), "r"(cluster_bar)
               : "memory");
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Args a) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::kStages * C::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + C::kStages * C::kBBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kStages;
  uint64_t* tfull = bars + 2 * C::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* recv = drain + 1;  // cluster split-K: the peers' partial slices have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ __align__(16) float epi_scr[4 * kScrFloats];
  bool csplit_armed = false;  // epilogue thread passed the first cluster barrier

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    trace_mark(a, 0);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    mbar_init(drain, 1);
    mbar_init(recv, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) trace_mark(a, 1);

  const int total = a.tiles != nullptr ? *a.num_tiles_dev : a.num_feat_tiles * a.num_tok_tiles * a.splits;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = a.wpol == 0 ? l2_policy_evict_first()
                                         : (a.wpol == 2 ? l2_policy_evict_last() : l2_policy_evict_normal());
      const uint64_t pol_x = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_par = 0;
      bool ok = true;
      // Under programmatic dependent launch the weight tiles of the first
      // k-blocks are requested before waiting for the previous kernel (they
      // do not depend on it); the activation tiles follow after the wait.
      int pre = 0;
      if (a.pdl) {
        if (static_cast<int>(blockIdx.x) < total) {
          const Tile tl = get_tile<BN>(a, blockIdx.x);
          const int kb0 = tl.sp * a.kb_per_split;
          pre = min(C::kStages, min(kb0 + a.kb_per_split, a.num_kb) - kb0);
          for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], C::kStageBytes);
            tma_load_2d_hint(sA + i * C::kABytes, &tmA, &full[i], (kb0 + i) * BK, tl.arow, pol_w);
          }
        }
        griddep_wait();
      }
      wait_deferred_rows(a.wait_flags, a.wait_timeout_ns, a.status);
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const Tile tl = get_tile<BN>(a, t);
        const int kb0 = tl.sp * a.kb_per_split;
        const int kb1 = min(kb0 + a.kb_per_split, a.num_kb);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!(t == static_cast<int>(blockIdx.x) && kb - kb0 < pre)) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, a.status, kStatusGemmTimeout)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
            tma_load_2d_hint(sA + stage * C::kABytes, &tmA, &full[stage], kb * BK, tl.arow, pol_w);
          }
          tma_load_2d_hint(sB + stage * C::kBBytes, &tmB, &full[stage], kb * BK, tl.tok0, pol_x);
          issued_mask |= 1u << stage;
          issued_par = phase ? (issued_par | (1u << stage)) : (issued_par & ~(1u << stage));
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < C::kStages; ++s)
          if ((issued_mask >> s) & 1u) mbar_drain(&full[s], (issued_par >> s) & 1u);
      }
      griddep_launch_dependents();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued_any = false;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const Tile tl = get_tile<BN>(a, t);
        const int kb0 = tl.sp * a.kb_per_split;
        const int kb1 = min(kb0 + a.kb_per_split, a.num_kb);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, a.status, kStatusGemmTimeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, a.status, kStatusGemmTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!issued_any) trace_mark(a, 2);
          const uint64_t adesc = umma_desc_sw128(smem_u32(sA + stage * C::kABytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + stage * C::kBBytes));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 bf16 = 32 bytes along K inside the 128-byte swizzle atom
            umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          if (t == blockIdx.x && kb == kb1 - 1) trace_mark(a, 3);
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok && issued_any) {
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  } else {
    const int q = warp & 3;  // a warp may only touch TMEM lanes [32*(warp%4), +32)
    const int row = q * 32 + lane;
    float* scr = epi_scr + q * kScrFloats;
    __shared__ int fix_last;
    int acc = 0;
    uint32_t acc_phase = 0;
    if (a.pdl) griddep_wait();  // outputs, residuals and fixup state belong to the stream order
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const Tile tl = get_tile<BN>(a, t);
      const int ft = tl.ft, tt = tl.tt, sp = tl.sp;
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, a.status, kStatusGemmTimeout);
      if (epi_barrier_or(!ok)) break;
      tc_fence_after();
      const bool first_item = t == blockIdx.x;
      if (first_item && threadIdx.x == 64) trace_mark(a, 4);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      auto from_tmem = [&](int c, float (&v)[16]) {
        tmem_ld_32x32b_x16(taddr + c, v);
        tmem_wait_ld();
      };
      if (a.csplit > 1) {
        // cluster split-K.  CTA r of the cluster owns token columns
        // [r * per, (r + 1) * per) of the tile.  Every CTA writes the other
        // owners' columns of its K-slice accumulator to an L2-resident
        // workspace (fp32 as [column / 4][row] float4, so each warp store
        // covers 512 contiguous bytes), the cluster barrier
        // publishes them, and each owner fetches its S-1 incoming slices with
        // one bulk copy into its (idle) ring memory, adds them to its own
        // columns straight from TMEM and runs the epilogue.  The reduction
        // runs in all S CTAs at once; the cluster guarantees they are resident.
        const int S = a.csplit;
        const int rank = static_cast<int>(cluster_ctarank());
        const int per = ((BN / 16 + S - 1) / S) * 16;
        const int cb = min(BN, rank * per), ce = min(BN, (rank + 1) * per);
        const long slab = (long)BM * per;  // floats of one (owner, source) slice
        float* wtile = a.fix_ws + ((long)tl.ft * a.num_tok_tiles + tl.tt) * S * (S - 1) * slab;
        for (int i2 = 1; i2 < S; ++i2) {
          const int d = rank + i2 < S ? rank + i2 : rank + i2 - S;  // stagger the destinations
          const int cbd = min(BN, d * per), ced = min(BN, (d + 1) * per);
          const int slot = rank < d ? rank : rank - 1;
          float4* dst = reinterpret_cast<float4*>(wtile + (d * (S - 1) + slot) * slab) + row;
          for (int c = cbd; c < ced; c += 16) {
            if (tl.tok0 + c >= tl.tok_end) break;
            float v[16];
            from_tmem(c, v);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              __stcg(dst + (((c - cbd) >> 2) + k) * BM,
                     make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
          }
        }
        const uint32_t bytes = static_cast<uint32_t>((S - 1) * slab * 4);
        if (threadIdx.x == 64) mbar_arrive_expect_tx(recv, bytes);
        __threadfence();
        if (threadIdx.x == 64) trace_mark(a, 5);
        cluster_sync_all();  // the peers' slices of this CTA's columns are in L2
        csplit_armed = true;
        if (threadIdx.x == 64) trace_mark(a, 7);
        if (threadIdx.x == 64) {
          asm volatile("fence.proxy.async.global;" ::: "memory");  // generic writes -> bulk-copy reads
          bulk_load(smem, wtile + (long)rank * (S - 1) * slab, bytes, recv);
        }
        const bool got = mbar_wait(recv, 0, abort_flag, a.status, kStatusGemmTimeout);
        if (!epi_barrier_or(!got)) {
          const float4* mine = reinterpret_cast<const float4*>(smem) + row;
          auto summed = [&](int c, float (&v)[16]) {
            from_tmem(c, v);
            for (int sl = 0; sl < S - 1; ++sl) {
              const float4* p = mine + sl * (slab / 4) + ((c - cb) >> 2) * BM;
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float4 x = p[k * BM];
                v[4 * k] += x.x;
                v[4 * k + 1] += x.y;
                v[4 * k + 2] += x.z;
                v[4 * k + 3] += x.w;
              }
            }
          };
          epilogue_tile<BN, EPI>(a, tl, q, lane, scr, cb, ce, summed);
          if (threadIdx.x == 64) trace_mark(a, 6);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      } else if (!a.fixup) {
        epilogue_tile<BN, EPI>(a, tl, q, lane, scr, 0, BN, from_tmem);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      } else {
        // split-K fixup.  Splits arrive in completion order; the last one to
        // arrive keeps its accumulator in TMEM and waits (bounded) only for the
        // splits that already arrived and are writing their fp32 partials to
        // the L2-resident workspace, so no CTA ever waits on one that may not
        // be running.  It then sums the partials and runs the fused epilogue.
        const long tile_id = (long)ft * a.num_tok_tiles + tt;
        int* arrive = a.fix_count + 2 * tile_id;
        int* written = arrive + 1;
        if (threadIdx.x == 64) fix_last = atomicAdd(arrive, 1);
        epi_barrier();
        const int slot = fix_last;  // arrival index (read before anyone rewrites fix_last)
        const bool last = (slot == a.splits - 1);
        // partial layout per (tile, slot): [BN/4][128 rows] float4, coalesced across a warp
        float4* ws4 = reinterpret_cast<float4*>(a.fix_ws) + (tile_id * a.splits) * (BN / 4) * BM;
        const int tok0 = tt * BN;
        bool timed_out = false;
        if (!last) {
          float4* mine = ws4 + (long)slot * (BN / 4) * BM + row;
          for (int c = 0; c < BN; c += 16) {
            if (tok0 + c >= a.M) break;
            float v[16];
            from_tmem(c, v);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              __stcg(mine + (long)((c >> 2) + j) * BM, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
          __threadfence();
          epi_barrier();
          if (threadIdx.x == 64) atomicAdd(written, 1);
        } else {
          if (threadIdx.x == 64) {
            const uint64_t t0 = globaltimer_ns();
            while (true) {
              int w;
              asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(w) : "l"(written) : "memory");
              if (w >= a.splits - 1) break;
              if (globaltimer_ns() - t0 > kLocalWaitTimeoutNs) {
                atomicOr(a.status, kStatusGemmTimeout);
                timed_out = true;
                break;
              }
            }
          }
          timed_out = epi_barrier_or(timed_out);
          __threadfence();
          if (!timed_out) {
            const float4* parts = ws4 + row;
            auto summed = [&](int c, float (&v)[16]) {
              float4 acc4[4] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f),
                                make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
              for (int s2 = 0; s2 < a.splits - 1; ++s2) {
                const float4* p = parts + ((long)s2 * (BN / 4) + (c >> 2)) * BM;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float4 q4 = __ldcg(p + (long)j * BM);
                  acc4[j].x += q4.x;
                  acc4[j].y += q4.y;
                  acc4[j].z += q4.z;
                  acc4[j].w += q4.w;
                }
              }
              from_tmem(c, v);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                v[4 * j] += acc4[j].x;
                v[4 * j + 1] += acc4[j].y;
                v[4 * j + 2] += acc4[j].z;
                v[4 * j + 3] += acc4[j].w;
              }
            };
            epilogue_tile<BN, EPI>(a, tl, q, lane, scr, 0, BN, summed);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
          epi_barrier();
          if (threadIdx.x == 64) {  // leave the counters at zero for the next launch
            *arrive = 0;
            *written = 0;
          }
        }
        epi_barrier();  // fix_last is rewritten by the next tile
        if (timed_out) break;
      }
      if (first_item && a.csplit <= 1) {
        epi_barrier();
        if (threadIdx.x == 64) trace_mark(a, 5);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  // every thread of the cluster takes part in the split-K cluster barrier
  // (epilogue warps that reached their tile took it above)
  if (a.csplit > 1 && !csplit_armed) cluster_sync_all();
  // pushed rows are performed at system scope before the kernel completes
  if (a.push_world > 0 && warp >= 2) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------- 2-CTA (cta_group::2) variant
// A CTA pair (cluster of 2) computes a 256-row x BN-token tile: each CTA
// stages its 128 weight rows and BN/2 of the tokens, the leader (rank 0)
// issues tcgen05.mma.cta_group::2 with M = 256, the tensor cores of both SMs
// read both halves, and each CTA's TMEM receives its 128 rows x BN columns.
// Per FLOP each SM fills 2/3 of the shared memory of the one-CTA 128 x 256
// tile.  Every TMA load is a plain (non-multicast) load into the issuing
// CTA's own shared memory that signals the leader's full barrier; the
// leader's MMA completion is committed separately to each CTA's barrier.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* tm, uint32_t leader_bar, int x, int y,
                                                 uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(leader_bar), "r"(x), "r"(y), "l"(hint)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on a barrier (own or the peer's, shared::cluster address) when the
// leader's prior tcgen05 operations complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

template <int BN>
struct Cfg2 {
  static constexpr int kABytes = BM * BK * 2;         // this CTA's 128 weight rows
  static constexpr int kBBytes = (BN / 2) * BK * 2;   // this CTA's half of the tokens
  static constexpr int kStageBytes = kABytes + kBBytes;
  // deep rings for small (decode) token tiles: more k-blocks in flight per SM
  static constexpr int kStages = (200 * 1024) / kStageBytes > 12 ? 12 : (200 * 1024) / kStageBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Args a) {
  using C = Cfg2<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::kStages * C::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + C::kStages * C::kBBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kStages;
  uint64_t* tfull = bars + 2 * C::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ __align__(16) float epi_scr[4 * kScrFloats];

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t peer = rank ^ 1u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);  // the four epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nft2 = (a.N + 2 * BM - 1) / (2 * BM);
  const int total = nft2 * a.num_tok_tiles;
  // pair tile t -> (256-row feature tile, token tile), token tiles in raster groups
  auto tile_of = [&](int t, int& ft2, int& tt) {
    const int per_group = a.tok_group * nft2;
    const int g = t / per_group;
    const int in = t - g * per_group;
    const int gsize = min(a.tok_group, a.num_tok_tiles - g * a.tok_group);
    ft2 = in / gsize;
    tt = g * a.tok_group + (in - ft2 * gsize);
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = a.wpol == 0 ? l2_policy_evict_first()
                                         : (a.wpol == 2 ? l2_policy_evict_last() : l2_policy_evict_normal());
      const uint64_t pol_x = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_par = 0;
      bool ok = true;
      wait_deferred_rows(a.wait_flags, a.wait_timeout_ns, a.status);
      for (int t = pair; t < total && ok; t += npairs) {
        int ft2, tt;
        tile_of(t, ft2, tt);
        const int arow = ft2 * 2 * BM + static_cast<int>(rank) * BM;
        const int brow = tt * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < a.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, a.status, kStatusGemmTimeout)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::kStageBytes);
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);  // the leader's full barrier
          tma_load_2d_pair(sA + stage * C::kABytes, &tmA, fb, kb * BK, arow, pol_w);
          tma_load_2d_pair(sB + stage * C::kBBytes, &tmB, fb, kb * BK, brow, pol_x);
          issued_mask |= 1u << stage;
          issued_par = phase ? (issued_par | (1u << stage)) : (issued_par & ~(1u << stage));
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        for (int s = 0; s < C::kStages; ++s)
          if ((issued_mask >> s) & 1u) mbar_drain(&full[s], (issued_par >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = umma_idesc_bf16(2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued_any = false;
      for (int t = pair; t < total && ok; t += npairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, a.status, kStatusGemmTimeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < a.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, a.status, kStatusGemmTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sA + stage * C::kABytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + stage * C::kBBytes));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          issued_any = true;
          const uint32_t eb = smem_u32(&empty[stage]);
          umma_commit_pair(eb);
          umma_commit_pair(mapa_shared(eb, peer));
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t tb = smem_u32(&tfull[acc]);
        umma_commit_pair(tb);
        umma_commit_pair(mapa_shared(tb, peer));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok && issued_any) {
        umma_commit_pair(smem_u32(drain));
        mbar_drain(drain, 0);
      }
    }
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t leader_tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t leader_tempty1 = mapa_shared(smem_u32(&tempty[1]), 0);
    for (int t = pair; t < total; t += npairs) {
      int ft2, tt;
      tile_of(t, ft2, tt);
      Tile tl;
      tl.ft = ft2 * 2 + static_cast<int>(rank);
      tl.tt = tt;
      tl.sp = 0;
      tl.tok0 = tt * BN;
      tl.tok_end = a.M;
      tl.arow = tl.ft * BM;
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, a.status, kStatusGemmTimeout);
      if (epi_barrier_or(!ok)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      auto from_tmem = [&](int c, float (&v)[16]) {
        tmem_ld_32x32b_x16(taddr + c, v);
        tmem_wait_ld();
      };
      epilogue_tile<BN, EPI>(a, tl, q, lane, epi_scr + q * kScrFloats, 0, BN, from_tmem);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  if (a.push_world > 0 && warp >= 2) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no remote arrival or MMA into this CTA is outstanding past this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

template <int BN, int EPI>
int launch_pair(const CUtensorMap& tmA, const CUtensorMap& tmB, const Args& a, int tiles, cudaStream_t stream) {
  auto kern = gemm_pair_kernel<BN, EPI>;
  static uint64_t configured = 0;
  static int max_clusters[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = Cfg2<BN>::kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!((configured >> dev) & 1u)) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg2<BN>::kSmem);
    cfg.gridDim = dim3(2 * 74, 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = 0;
    max_clusters[dev] = n;
    configured |= uint64_t(1) << dev;
  }
  const int clusters = std::min(max_clusters[dev], tiles);
  if (clusters <= 0) return 0;  // cluster launch unavailable: the caller uses the one-CTA kernel
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, a) == cudaSuccess ? 1 : 0;
}

template <int BN, int EPI>
void launch(const CUtensorMap& tmA, const CUtensorMap& tmB, const Args& a, int grid, cudaStream_t stream) {
  auto kern = gemm_tn_kernel<BN, EPI>;
  static uint64_t configured = 0;  // one bit per device, per template instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((configured >> dev) & 1u)) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::kSmem);
    configured |= uint64_t(1) << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (a.pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (a.csplit > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = a.csplit;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = Cfg<BN>::kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = n;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tmA, tmB, a));
}

// Clusters of `cs` one-CTA GEMM blocks that can be resident at once (0 if a
// cluster launch is unavailable); cached per device, token tile and size.
template <int BN>
int max_active_clusters(int cs) {
  static int cache[64][9];
  static bool init[64][9];
  int dev = 0;
  cudaGetDevice(&dev);
  if (cs < 1 || cs > 8 || dev >= 64) return 0;
  if (!init[dev][cs]) {
    auto kern = gemm_tn_kernel<BN, kEpiBF16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::kSmem);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(cs * 16, 1, 1);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = Cfg<BN>::kSmem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 0) {
      cudaGetLastError();
      n = 0;
    }
    cache[dev][cs] = n;
    init[dev][cs] = true;
  }
  return cache[dev][cs];
}

// Shared-memory ring bytes of the one-CTA kernel (the cluster split-K receive area).
int ring_bytes_bn(int bn) {
  switch (bn) {
    case 16: return Cfg<16>::kStages * Cfg<16>::kStageBytes;
    case 32: return Cfg<32>::kStages * Cfg<32>::kStageBytes;
    case 64: return Cfg<64>::kStages * Cfg<64>::kStageBytes;
    case 128: return Cfg<128>::kStages * Cfg<128>::kStageBytes;
    default: return Cfg<256>::kStages * Cfg<256>::kStageBytes;
  }
}

int max_active_clusters_bn(int bn, int cs) {
  switch (bn) {
    case 16: return max_active_clusters<16>(cs);
    case 32: return max_active_clusters<32>(cs);
    case 64: return max_active_clusters<64>(cs);
    case 128: return max_active_clusters<128>(cs);
    default: return max_active_clusters<256>(cs);
  }
}

template <int EPI>
void dispatch_bn(int bn, const CUtensorMap& tmA, const CUtensorMap& tmB, const Args& a, int grid, cudaStream_t s) {
  switch (bn) {
    case 16: launch<16, EPI>(tmA, tmB, a, grid, s); break;
    case 32: launch<32, EPI>(tmA, tmB, a, grid, s); break;
    case 64: launch<64, EPI>(tmA, tmB, a, grid, s); break;
    case 128: launch<128, EPI>(tmA, tmB, a, grid, s); break;
    default: launch<256, EPI>(tmA, tmB, a, grid, s); break;
  }
}

}  // namespace gemm

// Timeline buffer for the next plain (non-pair) GEMM launches; see Args::trace.
static unsigned long long* g_gemm_trace = nullptr;

void gemm_set_trace(const c10::optional<torch::Tensor>& buf) {
  if (buf.has_value() && buf->defined()) {
    TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong && buf->numel() >= 8 * 1024,
                "gemm trace: int64 CUDA tensor of >= 8192 elements");
    g_gemm_trace = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
  } else {
    g_gemm_trace = nullptr;
  }
}

int gemm_max_active_clusters(int64_t bn, int64_t cluster_size) {
  return gemm::max_active_clusters_bn(int(bn), int(cluster_size));
}

int gemm_pick_bn(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

int gemm_tiles(int M, int N, int epi) {
  const int bn = gemm_pick_bn(M);
  const int ntok = (M + bn - 1) / bn;
  const int nrows = N;  // SwiGLU: N counts interleaved gate+up rows
  (void)epi;
  return ntok * ((nrows + gemm::BM - 1) / gemm::BM);
}

int64_t gemm_fixup_ws_floats(int64_t M, int64_t N, int64_t splits, int64_t bn_override) {
  const int bn = bn_override > 0 ? int(bn_override) : gemm_pick_bn(int(M));
  const int64_t tiles = ((M + bn - 1) / bn) * ((N + gemm::BM - 1) / gemm::BM);
  // last-arriver fixup: one partial tile per split; cluster split-K: S-1
  // column slices per owner
  const int64_t per = ((bn / 16 + splits - 1) / splits) * 16;
  return std::max(tiles * splits * bn * gemm::BM, tiles * splits * (splits - 1) * gemm::BM * per);
}

int gemm_default_splits(int M, int N, int K, int device) {
  const int tiles = gemm_tiles(M, N, kEpiPartialF32);
  const int num_kb = (K + gemm::BK - 1) / gemm::BK;
  const int sms = num_sms(device);
  if (tiles >= sms) return 1;
  int splits = sms / tiles;  // whole waves only
  splits = std::min(splits, std::max(1, num_kb / 8));
  return std::max(1, std::min(splits, 16));
}

void gemm_out(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& out, int64_t epi,
              const c10::optional<torch::Tensor>& resid, const c10::optional<torch::Tensor>& bias, int64_t splits,
              const torch::Tensor& status, const c10::optional<torch::Tensor>& fix_ws,
              const c10::optional<torch::Tensor>& fix_count, int64_t bn_override,
              const std::vector<int64_t>& push_ptrs, int64_t push_rank, int64_t push_rows, int64_t wait_flags,
              double wait_timeout_s) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && out.is_cuda(), "gemm: tensors must be on CUDA");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm: x and w must be bf16");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2, "gemm: x [M,K], w [N,K]");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "gemm: inner dim must be contiguous");
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "gemm: K mismatch");
  TORCH_CHECK(K % 8 == 0, "gemm: K must be a multiple of 8");
  if (M == 0) return;
  const bool gelu_tanh = epi == kEpiGeluTanh || epi == kEpiGeGLU;
  if (epi == kEpiGeluTanh) epi = kEpiGelu;
  if (epi == kEpiGeGLU) epi = kEpiSwiGLU;
  const at::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  int bn = gemm_pick_bn(M);
  if (bn_override > 0) {
    TORCH_CHECK(bn_override == 16 || bn_override == 32 || bn_override == 64 || bn_override == 128 ||
                    bn_override == 256,
                "gemm: token tile must be 16, 32, 64, 128 or 256");
    bn = int(bn_override);
  }
  gemm::Args a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.gelu_tanh = gelu_tanh ? 1 : 0;
  a.num_kb = (K + gemm::BK - 1) / gemm::BK;
  a.num_feat_tiles = (N + gemm::BM - 1) / gemm::BM;
  a.num_tok_tiles = (M + bn - 1) / bn;
  a.splits = 1;
  a.kb_per_split = a.num_kb;
  a.out = out.data_ptr();
  a.ldo = out.dim() >= 2 ? out.stride(out.dim() - 2) : N;
  a.resid = nullptr;
  a.ldr = 0;
  a.bias = nullptr;
  a.status = status.data_ptr<int>();
  a.fix_ws = nullptr;
  a.fix_count = nullptr;
  a.fixup = 0;
  a.tiles = nullptr;
  a.num_tiles_dev = nullptr;
  a.rows_per_group = 0;
  a.wpol = a.num_tok_tiles > 1 ? 1 : 0;
  a.trace = g_gemm_trace;
  a.csplit = 1;
  a.push_world = 0;
  a.push_rank = 0;
  a.push_rows = 0;
  a.wait_flags = reinterpret_cast<uint32_t*>(static_cast<uintptr_t>(wait_flags));
  a.wait_timeout_ns = static_cast<uint64_t>(wait_timeout_s * 1e9);
  for (int r = 0; r < 8; ++r) a.push[r] = 0;
  if (!push_ptrs.empty()) {
    TORCH_CHECK(epi == kEpiBF16 && !bias.has_value(), "gemm push: plain bf16 epilogue only");
    TORCH_CHECK(push_ptrs.size() <= 8 && push_rank >= 0 && push_rank < (int64_t)push_ptrs.size(),
                "gemm push: up to 8 ranks");
    TORCH_CHECK(push_rows > 0 && push_rows * (int64_t)push_ptrs.size() >= M, "gemm push: rows per rank cover M");
    TORCH_CHECK(out.dim() == 2 && out.size(1) == N && out.stride(1) == 1 && out.stride(0) == N,
                "gemm push: out [M, N] contiguous rows (the peers' slot pitch)");
    for (size_t r = 0; r < push_ptrs.size(); ++r) {
      TORCH_CHECK(push_ptrs[r] % 16 == 0, "gemm push: peer buffers must be 16-byte aligned");
      a.push[r] = static_cast<unsigned long long>(push_ptrs[r]);
    }
    a.push_world = static_cast<int>(push_ptrs.size());
    a.push_rank = static_cast<int>(push_rank);
    a.push_rows = static_cast<int>(push_rows);
  }
  {
    static const int env_pdl = [] {
      const char* e = std::getenv("BLOOM_PDL");
      return e ? std::atoi(e) : 1;
    }();
    a.pdl = env_pdl;
  }
  {
    // 16-byte vector stores need aligned rows: 8 bf16 / 4 fp32 elements
    const int esz = out.element_size();
    a.vec = (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0) && ((a.ldo * esz) % 16 == 0) &&
            (epi == kEpiPartialF32 ? (N * 4) % 16 == 0 : true);
    if (epi == kEpiResidual && resid.has_value())
      a.vec = a.vec && reinterpret_cast<uintptr_t>(resid->data_ptr()) % 16 == 0 && (resid->stride(0) * 2) % 16 == 0;
  }
  // 8 token tiles per raster group: measured on M=8192 prefill GEMMs (N 4096-28672,
  // K 4096-14336) as 10-15 % faster than one group, with 2.3x fewer DRAM reads
  a.tok_group = std::min(a.num_tok_tiles, 8);
  {
    static const int env_group = [] {
      const char* e = std::getenv("BLOOM_GEMM_TOK_GROUP");
      return e ? std::atoi(e) : 0;
    }();
    if (env_group > 0) a.tok_group = std::min(env_group, a.num_tok_tiles);
  }
  {
    static const int env_wpol = [] {
      const char* e = std::getenv("BLOOM_GEMM_WPOL");
      return e ? std::atoi(e) : -1;
    }();
    if (env_wpol >= 0 && env_wpol <= 2) a.wpol = env_wpol;
  }

  switch (epi) {
    case kEpiBF16:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(-1) == N, "gemm: out must be bf16 [M,N]");
      break;
    case kEpiF32:
      TORCH_CHECK(out.scalar_type() == at::kFloat && out.size(-1) == N, "gemm: out must be f32 [M,N]");
      break;
    case kEpiSwiGLU:
      TORCH_CHECK(N % 32 == 0, "gemm swiglu: interleaved N must be a multiple of 32");
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(-1) == N / 2, "gemm swiglu: out [M, N/2] bf16");
      break;
    case kEpiPartialF32: {
      TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous(), "gemm partial: out must be contiguous f32");
      int s = splits > 0 ? int(splits) : 1;
      s = std::min(s, a.num_kb);
      a.kb_per_split = (a.num_kb + s - 1) / s;
      a.splits = (a.num_kb + a.kb_per_split - 1) / a.kb_per_split;
      TORCH_CHECK(out.numel() >= (int64_t)a.splits * M * N, "gemm partial: workspace too small");
      TORCH_CHECK(a.splits == s, "gemm partial: split count ", s, " not realisable for K=", K);
      break;
    }
    case kEpiGelu:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(-1) == N, "gemm gelu: out must be bf16 [M,N]");
      break;
    case kEpiResidual:
      TORCH_CHECK(resid.has_value(), "gemm residual epilogue needs resid");
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(-1) == N, "gemm: out must be bf16 [M,N]");
      a.resid = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
      a.ldr = resid->stride(0);
      break;
    default:
      TORCH_CHECK(false, "gemm: unknown epilogue ", epi);
  }
  static const int env_csplit = [] {
    const char* e = std::getenv("BLOOM_GEMM_CSPLIT");
    return e ? std::atoi(e) : 1;
  }();
  if (epi != kEpiPartialF32 && splits > 1) {
    // split-K: the K-slices of one tile run as one thread-block cluster and
    // reduce through distributed shared memory (up to 8 slices), otherwise
    // with an in-kernel fixup (the last arriving split reduces + runs the epilogue)
    int s = std::min<int>(int(splits), a.num_kb);
    a.kb_per_split = (a.num_kb + s - 1) / s;
    a.splits = (a.num_kb + a.kb_per_split - 1) / a.kb_per_split;
    // clusters only when every tile's cluster is resident at once (a second
    // wave of clusters would double the kernel time)
    const int per = ((bn / 16 + a.splits - 1) / a.splits) * 16;
    const int64_t recv_bytes = (int64_t)(a.splits - 1) * gemm::BM * per * 4;
    const int64_t tiles = (int64_t)a.num_feat_tiles * a.num_tok_tiles;
    if (a.splits > 1 && a.splits <= 8 && env_csplit && recv_bytes <= gemm::ring_bytes_bn(bn) &&
        tiles <= gemm::max_active_clusters_bn(bn, a.splits) && fix_ws.has_value() &&
        fix_ws->scalar_type() == at::kFloat &&
        fix_ws->numel() >= tiles * a.splits * (a.splits - 1) * gemm::BM * per) {
      a.csplit = a.splits;
      a.fix_ws = fix_ws->data_ptr<float>();
    } else if (a.splits > 1) {
      TORCH_CHECK(fix_ws.has_value() && fix_count.has_value(), "gemm split-K fixup needs a workspace");
      const int64_t tiles = (int64_t)a.num_feat_tiles * a.num_tok_tiles;
      TORCH_CHECK(fix_ws->scalar_type() == at::kFloat &&
                      fix_ws->numel() >= tiles * a.splits * bn * gemm::BM,
                  "gemm fixup workspace too small: need ", tiles * a.splits * bn * gemm::BM, " floats");
      TORCH_CHECK(fix_count->scalar_type() == at::kInt && fix_count->numel() >= 2 * tiles,
                  "gemm fixup counters too small");
      a.fix_ws = fix_ws->data_ptr<float>();
      a.fix_count = fix_count->data_ptr<int>();
      a.fixup = 1;
    }
  }
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N, "gemm: bias must be bf16 [N]");
    a.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }

  const CUtensorMap tmA = make_tmap_bf16_2d(w.data_ptr(), K, N, w.stride(0) * 2, gemm::BK, gemm::BM);
  // 2-CTA tiles (256 weight rows per CTA pair) for large, unsplit GEMMs
  {
    static const int env_pair = [] {
      const char* e = std::getenv("BLOOM_GEMM_PAIR");
      return e ? std::atoi(e) : 1;
    }();
    const int pair_tiles = ((N + 2 * gemm::BM - 1) / (2 * gemm::BM)) * a.num_tok_tiles;
    if (env_pair && a.splits == 1 && epi != kEpiPartialF32 && bn >= 32 && pair_tiles >= 74) {
      const CUtensorMap tmB2 = make_tmap_bf16_2d(x.data_ptr(), K, M, x.stride(0) * 2, gemm::BK, bn / 2);
      int done = 0;
      if (bn == 256) {
        switch (epi) {
          case kEpiBF16: done = gemm::launch_pair<256, kEpiBF16>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiF32: done = gemm::launch_pair<256, kEpiF32>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiSwiGLU: done = gemm::launch_pair<256, kEpiSwiGLU>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiResidual: done = gemm::launch_pair<256, kEpiResidual>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiGelu: done = gemm::launch_pair<256, kEpiGelu>(tmA, tmB2, a, pair_tiles, stream); break;
        }
      } else if (bn == 128) {
        switch (epi) {
          case kEpiBF16: done = gemm::launch_pair<128, kEpiBF16>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiF32: done = gemm::launch_pair<128, kEpiF32>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiSwiGLU: done = gemm::launch_pair<128, kEpiSwiGLU>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiResidual: done = gemm::launch_pair<128, kEpiResidual>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiGelu: done = gemm::launch_pair<128, kEpiGelu>(tmA, tmB2, a, pair_tiles, stream); break;
        }
      } else if (bn == 64) {  // decode-sized batches: more CTA pairs instead of split-K
        switch (epi) {
          case kEpiBF16: done = gemm::launch_pair<64, kEpiBF16>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiSwiGLU: done = gemm::launch_pair<64, kEpiSwiGLU>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiResidual: done = gemm::launch_pair<64, kEpiResidual>(tmA, tmB2, a, pair_tiles, stream); break;
          default: break;
        }
      } else {
        switch (epi) {
          case kEpiBF16: done = gemm::launch_pair<32, kEpiBF16>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiSwiGLU: done = gemm::launch_pair<32, kEpiSwiGLU>(tmA, tmB2, a, pair_tiles, stream); break;
          case kEpiResidual: done = gemm::launch_pair<32, kEpiResidual>(tmA, tmB2, a, pair_tiles, stream); break;
          default: break;
        }
      }
      if (done) {
        C10_CUDA_KERNEL_LAUNCH_CHECK();
        return;
      }
    }
  }
  const CUtensorMap tmB = make_tmap_bf16_2d(x.data_ptr(), K, M, x.stride(0) * 2, gemm::BK, bn);
  const int total = a.num_feat_tiles * a.num_tok_tiles * a.splits;
  // cluster split-K runs one tile per cluster (grid = all tiles); otherwise persistent
  const int grid = a.csplit > 1 ? total : std::min(total, num_sms(x.get_device()));
  switch (epi) {
    case kEpiBF16: gemm::dispatch_bn<kEpiBF16>(bn, tmA, tmB, a, grid, stream); break;
    case kEpiF32: gemm::dispatch_bn<kEpiF32>(bn, tmA, tmB, a, grid, stream); break;
    case kEpiSwiGLU: gemm::dispatch_bn<kEpiSwiGLU>(bn, tmA, tmB, a, grid, stream); break;
    case kEpiPartialF32: gemm::dispatch_bn<kEpiPartialF32>(bn, tmA, tmB, a, grid, stream); break;
    case kEpiResidual: gemm::dispatch_bn<kEpiResidual>(bn, tmA, tmB, a, grid, stream); break;
    case kEpiGelu: gemm::dispatch_bn<kEpiGelu>(bn, tmA, tmB, a, grid, stream); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom

namespace bloom {

// Grouped GEMM for MoE experts: out[r] = x[r] @ w[g]^T for the rows r of every
// tile in the device-built list (g = tile.x); w is [G * rows_per_group, K].
void gemm_grouped_out(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& out, int64_t epi,
                      const torch::Tensor& tiles, const torch::Tensor& num_tiles, int64_t rows_per_group, int64_t bn,
                      const torch::Tensor& status) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "grouped gemm: bf16");
  TORCH_CHECK(epi == kEpiBF16 || epi == kEpiSwiGLU, "grouped gemm: bf16 or SwiGLU epilogue");
  TORCH_CHECK(tiles.scalar_type() == at::kInt && tiles.dim() == 2 && tiles.size(1) == 4, "tiles int32 [n, 4]");
  TORCH_CHECK(bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 256, "grouped gemm: bad token tile");
  const int M = x.size(0), K = x.size(1);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  gemm::Args a{};
  a.M = M;
  a.N = int(rows_per_group);
  a.K = K;
  a.num_kb = (K + gemm::BK - 1) / gemm::BK;
  a.kb_per_split = a.num_kb;
  a.splits = 1;
  a.num_feat_tiles = 1;
  a.num_tok_tiles = 1;
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.status = status.data_ptr<int>();
  a.tiles = reinterpret_cast<const int4*>(tiles.data_ptr<int>());
  a.num_tiles_dev = num_tiles.data_ptr<int>();
  a.rows_per_group = int(rows_per_group);
  a.wpol = 0;
  a.tok_group = 1;
  a.trace = nullptr;
  a.csplit = 1;
  a.pdl = 0;  // the tile list is written by the previous kernel
  a.vec = reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0 && (out.stride(0) * 2) % 16 == 0;
  const CUtensorMap tmA = make_tmap_bf16_2d(w.data_ptr(), K, w.size(0), w.stride(0) * 2, gemm::BK, gemm::BM);
  const CUtensorMap tmB = make_tmap_bf16_2d(x.data_ptr(), K, M, x.stride(0) * 2, gemm::BK, int(bn));
  const int grid = num_sms(x.get_device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (epi == kEpiSwiGLU)
    gemm::dispatch_bn<kEpiSwiGLU>(int(bn), tmA, tmB, a, grid, stream);
  else
    gemm::dispatch_bn<kEpiBF16>(int(bn), tmA, tmB, a, grid, stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
