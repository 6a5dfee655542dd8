// Paged attention over the HBM-resident KV cache.
//
// Cache layout (one tensor per model): [L, NB, 2, KVH, 16, 128] bf16, i.e. a
// 16-token page of one KV head is a contiguous 4 KiB block.  Pages are moved
// with 2D TMA tiles (box 64 dims x 16 tokens, 128-byte swizzle) so the
// ldmatrix reads that feed the tensor cores are bank-conflict free.
//
// head_dim 128 or 64 (template parameter D).
//
// Decode / speculative verify (q_len 1..8): one CTA per (sequence, KV head,
// split); the q heads of a GQA group and the q positions of the request are
// packed into the 16-row M dimension of m16n8k16 MMAs, so every KV page is
// read from HBM exactly once per step.  Each warp streams its own pages
// through a private TMA ring; warps and splits are merged flash-decoding style.
// This op is HBM-bound (arithmetic intensity ~4 FLOP/B at GQA 4), so its
// roofline is the page bytes at HBM bandwidth, not tensor throughput.
//
// Prefill (chunked, with cached prefix pages): FlashAttention-2 style, 64 query
// rows per CTA, 64-token KV tiles (4 pages) double buffered through TMA.
//
// Reference behaviour: scheduler/paged_cache.rs:565-748 (host f32 SDPA with
// repeat_kv), qwen_streaming.rs:413-424 (naive SDPA), causal + GQA semantics.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"
#include "bloom/tma_host.h"

#include <mutex>

namespace bloom {
namespace attn {

constexpr int D = 128;
constexpr int PAGE = 16;
constexpr float kNegBig = -1e30f;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
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
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Byte address of element (tok, d) (d multiple of 8) inside a page tile that
// TMA wrote as two 2 KiB boxes (dims 0-63, 64-127) with the 128-byte swizzle.
__device__ __forceinline__ uint32_t page_addr(uint32_t base, int tok, int d) {
  return base + ((d >> 6) << 11) + (tok << 7) + (((((d & 63) >> 3) ^ (tok & 7))) << 4);
}

struct DecodeArgs {
  const __nv_bfloat16* q;  // [B*ql, nq, 128]
  __nv_bfloat16* out;      // [B*ql, nq, 128]
  const int* block_table;
  int bt_stride;
  const int* seq_lens;  // kv length per sequence, including the ql new tokens
  float* part;          // [B, nkv * hc, splits, 32, 130] (o[128], m, l)
  int nq, nkv, ql, splits;
  int hc;               // CTAs per KV head, each taking G / hc of its q heads (G * ql > 32)
  float scale_log2;
  int* status;
  int num_blocks;       // pages in the cache (index checks only)
  // int8 cache (decode_q8_kernel): this layer's [NB][block bytes] region and
  // the block size in bytes (K pages, dim-major V pages, then fp32 scales)
  const uint8_t* q8_base;
  long q8_block_bytes;
};

// Row r of the packed M dimension -> (q position qi, head-in-group hh).
template <int D, int MT, int NWARPS, int NST>
__global__ void __launch_bounds__(NWARPS * 32)
    decode_kernel(const __grid_constant__ CUtensorMap tmKV, const DecodeArgs a) {
  constexpr int kStageBytes = 2 * PAGE * D * 2;  // K + V page = 8 KiB
  const int b = blockIdx.x, vkh = blockIdx.y, split = blockIdx.z;
  const int kh = vkh / a.hc;  // KV head whose pages this CTA streams
  const int warp = warp_id(), lane = lane_id();
  const int g = lane >> 2, t4 = lane & 3;
  const int G = a.nq / (a.nkv * a.hc);  // q heads handled by this CTA: vkh * G ...
  const int R = a.ql * G;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wsm = smem + warp * NST * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NWARPS * NST * kStageBytes) + warp * NST;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;

  const int kv_len = a.seq_lens[b];
  const int n_pages = (kv_len + PAGE - 1) / PAGE;
  const int pps = (n_pages + a.splits - 1) / a.splits;
  const int p0 = split * pps;
  const int p1 = min(p0 + pps, n_pages);
  const int first = p0 + warp;
  const int my_n = (p1 > first) ? (p1 - first + NWARPS - 1) / NWARPS : 0;
  const int* bt = a.block_table + (long)b * a.bt_stride;

  if (lane == 0) {
    for (int s = 0; s < NST; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int i) {
    const int s = i % NST;
    const int page = first + i * NWARPS;
    int blk = bt[page];
    if (!kcheck(blk >= 0 && blk < a.num_blocks, a.status)) blk = 0;
    const int rowK = ((blk * 2 + 0) * a.nkv + kh) * PAGE;
    const int rowV = ((blk * 2 + 1) * a.nkv + kh) * PAGE;
    uint8_t* st = wsm + s * kStageBytes;
    constexpr int kPageB = PAGE * D * 2;  // one page of one KV head: 2 KiB boxes of 64 dims
    mbar_arrive_expect_tx(&bars[s], kStageBytes);
    tma_load_2d(st, &tmKV, &bars[s], 0, rowK);
    if constexpr (D == 128) tma_load_2d(st + 2048, &tmKV, &bars[s], 64, rowK);
    tma_load_2d(st + kPageB, &tmKV, &bars[s], 0, rowV);
    if constexpr (D == 128) tma_load_2d(st + kPageB + 2048, &tmKV, &bars[s], 64, rowV);
  };
  if (lane == 0) {
    for (int i = 0; i < NST && i < my_n; ++i) issue(i);
  }

  // Q fragments (A operand), rows beyond R are zero.
  uint32_t qf[MT][D / 16][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + g + 8 * hr;
      const __nv_bfloat16* qrow = nullptr;
      if (r < R) {
        const int qi = r / G, hh = r - qi * G;
        qrow = a.q + ((long)(b * a.ql + qi) * a.nq + vkh * G + hh) * D;
      }
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int d = ks * 16 + 2 * t4;
        qf[mt][ks][hr] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d) : 0u;
        qf[mt][ks][hr + 2] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d + 8) : 0u;
      }
    }
  }

  float m_run[MT][2], l_run[MT][2];
  float o[MT][D / 8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    m_run[mt][0] = m_run[mt][1] = kNegBig;
    l_run[mt][0] = l_run[mt][1] = 0.f;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[mt][n][0] = o[mt][n][1] = o[mt][n][2] = o[mt][n][3] = 0.f;
  }
  // causal limit per packed row: kv index must be <= kv_len - ql + qi
  int limit[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + g + 8 * hr;
      limit[mt][hr] = (r < R) ? kv_len - a.ql + r / G : -1;
    }

  int i = 0;
  for (; i < my_n; ++i) {
    const int s = i % NST;
    if (!mbar_wait(&bars[s], (i / NST) & 1, &abort_flag, a.status, kStatusAttnTimeout)) break;
    const uint32_t sK = smem_u32(wsm + s * kStageBytes);
    const uint32_t sV = sK + PAGE * D * 2;
    const int tok_base = (first + i * NWARPS) * PAGE;

    float sc[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[mt][nt][0] = sc[mt][nt][1] = sc[mt][nt][2] = sc[mt][nt][3] = 0.f;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(page_addr(sK, 8 * nt + (lane & 7), 32 * j + 8 * (lane >> 3)), b0, b1, b2, b3);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma_bf16_16816(sc[mt][nt], qf[mt][2 * j], b0, b1);
          mma_bf16_16816(sc[mt][nt], qf[mt][2 * j + 1], b2, b3);
        }
      }
    }

    uint32_t pa[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float x[4];
        float mx = kNegBig;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int idx = tok_base + 8 * nt + 2 * t4 + e;
            float v = sc[mt][nt][2 * hr + e] * a.scale_log2;
            if (idx > limit[mt][hr]) v = -INFINITY;
            x[nt * 2 + e] = v;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[mt][hr], mx);
        const float alpha = exp2f(m_run[mt][hr] - m_new);
        m_run[mt][hr] = m_new;
        float ps = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          x[k] = exp2f(x[k] - m_new);
          ps += x[k];
        }
        l_run[mt][hr] = l_run[mt][hr] * alpha + ps;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[mt][n][2 * hr] *= alpha;
          o[mt][n][2 * hr + 1] *= alpha;
        }
        // A fragment of P: [row g | row g+8] x [tokens 0-7 | 8-15]
        pa[mt][hr] = pack_bf16(x[0], x[1]);      // tokens 2t4, 2t4+1 (n-tile 0)
        pa[mt][hr + 2] = pack_bf16(x[2], x[3]);  // tokens 8+2t4.. (n-tile 1)
      }
    }

#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(page_addr(sV, (lane & 7) + 8 * ((lane >> 3) & 1), 16 * j + 8 * (lane >> 4)), b0, b1, b2, b3);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma_bf16_16816(o[mt][2 * j], pa[mt], b0, b1);
        mma_bf16_16816(o[mt][2 * j + 1], pa[mt], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0 && i + NST < my_n) {
      fence_proxy_async();
      issue(i + NST);
    }
  }
  if (i < my_n) {  // aborted: drain the loads this warp still has in flight
    if (lane == 0)
      for (int k = i; k < my_n && k < i + NST; ++k) mbar_drain(&bars[k % NST], (k / NST) & 1);
  }

  // finish row sums across the quad
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float l = l_run[mt][hr];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      l_run[mt][hr] = l;
    }

  __syncthreads();
  // cross-warp merge through shared memory: per warp [MT*16 rows][128 o + m + l]
  constexpr int RS = D + 2;
  float* cm = reinterpret_cast<float*>(smem);
  float* wbuf = cm + warp * (MT * 16 * RS);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + g + 8 * hr;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        wbuf[r * RS + 8 * n + 2 * t4] = o[mt][n][2 * hr];
        wbuf[r * RS + 8 * n + 2 * t4 + 1] = o[mt][n][2 * hr + 1];
      }
      if (t4 == 0) {
        wbuf[r * RS + D] = m_run[mt][hr];
        wbuf[r * RS + D + 1] = l_run[mt][hr];
      }
    }
  __syncthreads();
  const int rows = min(R, MT * 16);
  for (int idx = threadIdx.x; idx < rows * D; idx += NWARPS * 32) {
    const int r = idx / D, d = idx - r * D;
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) M = fmaxf(M, cm[w * MT * 16 * RS + r * RS + D]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) {
      const float* wb = cm + w * MT * 16 * RS + r * RS;
      const float sc = exp2f(wb[D] - M);
      L += wb[D + 1] * sc;
      O += wb[d] * sc;
    }
    if (a.splits == 1) {
      const int qi = r / G, hh = r - qi * G;
      a.out[((long)(b * a.ql + qi) * a.nq + vkh * G + hh) * D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
    } else {
      float* pr = a.part + ((((long)b * a.nkv * a.hc + vkh) * a.splits + split) * 32 + r) * RS;
      pr[d] = O;
      if (d == 0) {
        pr[D] = M;
        pr[D + 1] = L;
      }
    }
  }
}

template <int D>
__global__ void decode_combine_kernel(const float* __restrict__ part, __nv_bfloat16* __restrict__ out, int nq,
                                      int nkv, int ql, int splits) {
  constexpr int RS = D + 2;
  const int b = blockIdx.x, kh = blockIdx.y;
  const int G = nq / nkv, R = ql * G;
  const float* base = part + (((long)b * nkv + kh) * splits) * 32 * RS;
  for (int idx = threadIdx.x; idx < R * D; idx += blockDim.x) {
    const int r = idx / D, d = idx - r * D;
    float M = kNegBig;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, base[((long)s * 32 + r) * RS + D]);
    float L = 0.f, O = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float* pr = base + ((long)s * 32 + r) * RS;
      const float sc = exp2f(pr[D] - M);
      L += pr[D + 1] * sc;
      O += pr[d] * sc;
    }
    const int qi = r / G, hh = r - qi * G;
    out[((long)(b * ql + qi) * nq + kh * G + hh) * D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
  }
}

// ---------------------------------------------------------------- prefill
struct PrefillArgs {
  const __nv_bfloat16* q;  // [T, nq, 128]
  __nv_bfloat16* out;      // [T, nq, 128]
  const int* block_table;
  int bt_stride;
  const int* ctx_lens;     // total kv length per sequence after this chunk
  const int* cu_q;         // [S+1] query token offsets
  const int* tile_seq;     // per work tile: sequence index
  const int* tile_start;   // per work tile: first query row (local to the sequence)
  int nq, nkv;
  float scale_log2;
  int causal;
  int* status;
  int num_blocks;          // pages in the cache (index checks only)
};

constexpr int kPfWarps = 4;
constexpr int kPfRows = 16 * kPfWarps;  // 64 query rows per CTA
constexpr int kPfKv = 64;               // kv tokens per tile (4 pages)
template <int D>
constexpr int pf_stage_bytes() { return 2 * kPfKv * D * 2; }  // K + V tile: 32 KiB at D = 128
constexpr int kPfStages = 2;

template <int D>
__global__ void __launch_bounds__(kPfWarps * 32)
    prefill_kernel(const __grid_constant__ CUtensorMap tmKV, const PrefillArgs a) {
  const int tile = blockIdx.x, h = blockIdx.y;
  const int warp = warp_id(), lane = lane_id();
  const int g = lane >> 2, t4 = lane & 3;
  const int G = a.nq / a.nkv;
  const int kh = h / G;
  const int s_idx = a.tile_seq[tile];
  const int row0 = a.tile_start[tile] + kPfRows * blockIdx.z;  // 128-row tiles run as two 64-row halves
  const int q_begin = a.cu_q[s_idx];
  const int q_len = a.cu_q[s_idx + 1] - q_begin;
  const int ctx = a.ctx_lens[s_idx];
  const int* bt = a.block_table + (long)s_idx * a.bt_stride;
  const int n_pages = (ctx + PAGE - 1) / PAGE;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kPfStageBytes = pf_stage_bytes<D>();
  constexpr int kHalf = kPfKv * D * 2;   // K (or V) part of a stage
  constexpr int kPageB = PAGE * D * 2;   // one page of one KV head
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPfStages * kPfStageBytes);
  __shared__ int abort_flag;

  // kv range this tile needs
  const int last_row = min(row0 + kPfRows, q_len) - 1;
  const int kv_end = a.causal ? min(ctx, ctx - q_len + last_row + 1) : ctx;
  const int n_kt = (kv_end + kPfKv - 1) / kPfKv;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kPfStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int kt) {
    const int s = kt % kPfStages;
    uint8_t* st = smem + s * kPfStageBytes;
    mbar_arrive_expect_tx(&bars[s], kPfStageBytes);
#pragma unroll
    for (int pg = 0; pg < 4; ++pg) {
      const int page = kt * 4 + pg;
      int blk = bt[page < n_pages ? page : 0];
      if (!kcheck(blk >= 0 && blk < a.num_blocks, a.status)) blk = 0;
      const int rowK = ((blk * 2 + 0) * a.nkv + kh) * PAGE;
      const int rowV = ((blk * 2 + 1) * a.nkv + kh) * PAGE;
      tma_load_2d(st + pg * kPageB, &tmKV, &bars[s], 0, rowK);
      if constexpr (D == 128) tma_load_2d(st + pg * kPageB + 2048, &tmKV, &bars[s], 64, rowK);
      tma_load_2d(st + kHalf + pg * kPageB, &tmKV, &bars[s], 0, rowV);
      if constexpr (D == 128) tma_load_2d(st + kHalf + pg * kPageB + 2048, &tmKV, &bars[s], 64, rowV);
    }
  };
  if (threadIdx.x == 0)
    for (int kt = 0; kt < kPfStages && kt < n_kt; ++kt) issue(kt);

  // Q fragments for rows row0 + 16*warp + {g, g+8}
  uint32_t qf[D / 16][4];
  int qpos[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int lr = row0 + 16 * warp + g + 8 * hr;
    const bool valid = lr < q_len;
    qpos[hr] = valid ? (a.causal ? ctx - q_len + lr : ctx - 1) : -1;
    const __nv_bfloat16* qrow = valid ? a.q + ((long)(q_begin + lr) * a.nq + h) * D : nullptr;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int d = ks * 16 + 2 * t4;
      qf[ks][hr] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d) : 0u;
      qf[ks][hr + 2] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + d + 8) : 0u;
    }
  }

  float m_run[2] = {kNegBig, kNegBig}, l_run[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  int kt = 0;
  bool ok = true;
  for (; kt < n_kt; ++kt) {
    const int s = kt % kPfStages;
    if (!mbar_wait(&bars[s], (kt / kPfStages) & 1, &abort_flag, a.status, kStatusAttnTimeout)) {
      ok = false;
    }
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    const uint32_t sK = smem_u32(smem + s * kPfStageBytes);
    const uint32_t sV = sK + kHalf;
    const int kv0 = kt * kPfKv;
    // skip whole tiles above the diagonal for this warp
    const bool warp_active = (qpos[0] >= kv0) || (qpos[1] >= kv0);
    if (__any_sync(0xffffffffu, warp_active)) {
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int tok = 8 * nt + (lane & 7);
        const uint32_t pbase = sK + (tok >> 4) * kPageB;
#pragma unroll
        for (int j = 0; j < D / 32; ++j) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(page_addr(pbase, tok & 15, 32 * j + 8 * (lane >> 3)), b0, b1, b2, b3);
          mma_bf16_16816(sc[nt], qf[2 * j], b0, b1);
          mma_bf16_16816(sc[nt], qf[2 * j + 1], b2, b3);
        }
      }
      uint32_t pa[4][4];
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float mx = kNegBig;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int idx = kv0 + 8 * nt + 2 * t4 + e;
            float v = sc[nt][2 * hr + e] * a.scale_log2;
            if (idx > qpos[hr] || idx >= ctx) v = -INFINITY;
            sc[nt][2 * hr + e] = v;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[hr], mx);
        const float alpha = exp2f(m_run[hr] - m_new);
        m_run[hr] = m_new;
        float ps = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float p = exp2f(sc[nt][2 * hr + e] - m_new);
            sc[nt][2 * hr + e] = p;
            ps += p;
          }
        l_run[hr] = l_run[hr] * alpha + ps;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[n][2 * hr] *= alpha;
          o[n][2 * hr + 1] *= alpha;
        }
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        pa[kk][0] = pack_bf16(sc[2 * kk][0], sc[2 * kk][1]);
        pa[kk][1] = pack_bf16(sc[2 * kk][2], sc[2 * kk][3]);
        pa[kk][2] = pack_bf16(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
        pa[kk][3] = pack_bf16(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t pbase = sV + kk * kPageB;
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(page_addr(pbase, (lane & 7) + 8 * ((lane >> 3) & 1), 16 * j + 8 * (lane >> 4)), b0, b1, b2, b3);
          mma_bf16_16816(o[2 * j], pa[kk], b0, b1);
          mma_bf16_16816(o[2 * j + 1], pa[kk], b2, b3);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && kt + kPfStages < n_kt) {
      fence_proxy_async();
      issue(kt + kPfStages);
    }
  }
  if (!ok && threadIdx.x == 0) {
    for (int k = kt; k < n_kt && k < kt + kPfStages; ++k) mbar_drain(&bars[k % kPfStages], (k / kPfStages) & 1);
  }

#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = l_run[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int lr = row0 + 16 * warp + g + 8 * hr;
    if (lr < q_len && ok) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = a.out + ((long)(q_begin + lr) * a.nq + h) * D;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        *reinterpret_cast<uint32_t*>(orow + 8 * n + 2 * t4) = pack_bf16(o[n][2 * hr] * inv, o[n][2 * hr + 1] * inv);
      }
    }
  }
}

// ---------------------------------------------------------------- int8 KV decode
// Same work split, ring and merge as decode_kernel (head_dim 128), over an
// int8 cache with one fp32 scale per (token, head).  Per page a warp's TMA
// ring brings the K page [16 tokens][128] (128-byte swizzle), the V page
// [128 dims][16 tokens] (dim-major) and the 2 x 16 scales (bulk copies):
// 4.1 KB instead of 8 KB.  Q K^T runs as int8 MMAs (m16n8k32, s32
// accumulators): q is quantised per row once per CTA, K bytes are the B
// operand as stored, and S = q scale x K scale x the integer dot product.
// V pages are stored in fp16 fragment order (q8_perm16), so each thread gets
// the four bytes of a B fragment with one 32-bit shared load and turns them
// into fp16 with a byte permute and a subtraction; P V runs in fp16 with P
// carrying the V scales (times 2^8, divided out with the row sum).  The
// running max is rescaled lazily (only when it grows by more than 2^4).
// Four int8 values (bytes of w) -> two f16x2 registers {b0, b1} and {b2, b3},
// exactly: x + 128 is placed in the low mantissa byte of the fp16 1024.0
// (0x64xx = 1024 + (x + 128)), then 1152.0 is subtracted.
__device__ __forceinline__ void i8x4_f16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  lo = __byte_perm(u, 0x64646464u, 0x4140);
  hi = __byte_perm(u, 0x64646464u, 0x4342);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  __half2 l = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
  __half2 h = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
  lo = *reinterpret_cast<uint32_t*>(&l);
  hi = *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t b) {
  const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b));
  return pack_f16(f.x, f.y);
}

template <int MT, int NWARPS, int NST>
__global__ void __launch_bounds__(NWARPS * 32)
    decode_q8_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     const DecodeArgs a) {
  constexpr int D = 128;
  constexpr int kPageB = PAGE * D;      // one int8 page of one KV head: 2 KB
  constexpr int kStageBytes = 2 * kPageB;
  constexpr int kRing = NWARPS * NST * kStageBytes;
  constexpr int kScl = NWARPS * NST * 128;  // 16 K + 16 V scales per stage
  constexpr int kMerge = NWARPS * MT * 16 * (D + 2) * 4;
  constexpr int kBarOff = (kRing + kScl > kMerge ? kRing + kScl : kMerge);
  const int b = blockIdx.x, vkh = blockIdx.y, split = blockIdx.z;
  const int kh = vkh / a.hc;
  const int warp = warp_id(), lane = lane_id();
  const int g = lane >> 2, t4 = lane & 3;
  const int G = a.nq / (a.nkv * a.hc);
  const int R = a.ql * G;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wsm = smem + warp * NST * kStageBytes;
  float* wscl = reinterpret_cast<float*>(smem + kRing) + warp * NST * 32;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff) + warp * NST;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;

  const int kv_len = a.seq_lens[b];
  const int n_pages = (kv_len + PAGE - 1) / PAGE;
  const int pps = (n_pages + a.splits - 1) / a.splits;
  const int p0 = split * pps;
  const int p1 = min(p0 + pps, n_pages);
  const int first = p0 + warp;
  const int my_n = (p1 > first) ? (p1 - first + NWARPS - 1) / NWARPS : 0;
  const int* bt = a.block_table + (long)b * a.bt_stride;
  const long rpbK = a.q8_block_bytes / D;   // K-map rows (128 B) per block
  const long rpbV = a.q8_block_bytes / 16;  // V-map rows (16 B) per block

  if (lane == 0) {
    for (int s = 0; s < NST; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int i) {
    const int s = i % NST;
    const int page = first + i * NWARPS;
    int blk = bt[page];
    if (!kcheck(blk >= 0 && blk < a.num_blocks, a.status)) blk = 0;
    uint8_t* st = wsm + s * kStageBytes;
    mbar_arrive_expect_tx(&bars[s], kStageBytes + 128);
    tma_load_2d(st, &tmK, &bars[s], 0, static_cast<int>(blk * rpbK + kh * PAGE));
    tma_load_2d(st + kPageB, &tmV, &bars[s], 0, static_cast<int>(blk * rpbV + (long)(a.nkv + kh) * D));
    const uint8_t* sc = a.q8_base + (long)blk * a.q8_block_bytes + 2L * a.nkv * PAGE * D;
    bulk_load(wscl + s * 32, sc + kh * PAGE * 4, 64, &bars[s]);
    bulk_load(wscl + s * 32 + 16, sc + (a.nkv + kh) * PAGE * 4, 64, &bars[s]);
  };
  if (lane == 0) {
    for (int i = 0; i < NST && i < my_n; ++i) issue(i);
  }

  // q rows quantised to int8 per row (absmax / 127) for the int8 Q K^T MMAs:
  // A fragment of m16n8k32, chunk kc of 32 dims: rows g / g+8, bytes 4t4..4t4+3
  // and 16+4t4..16+4t4+3 of the chunk
  uint32_t qf[MT][D / 32][4];
  float qscale[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + g + 8 * hr;
      const __nv_bfloat16* qrow = nullptr;
      if (r < R) {
        const int qi = r / G, hh = r - qi * G;
        qrow = a.q + ((long)(b * a.ql + qi) * a.nq + vkh * G + hh) * D;
      }
      float qv[D / 32][8];
      float am = 0.f;
#pragma unroll
      for (int kc = 0; kc < D / 32; ++kc)
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int d = kc * 32 + h2 * 16 + 4 * t4;
          uint2 u = qrow ? *reinterpret_cast<const uint2*>(qrow + d) : make_uint2(0u, 0u);
          const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
          const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
          qv[kc][4 * h2 + 0] = f0.x;
          qv[kc][4 * h2 + 1] = f0.y;
          qv[kc][4 * h2 + 2] = f1.x;
          qv[kc][4 * h2 + 3] = f1.y;
#pragma unroll
          for (int e = 0; e < 4; ++e) am = fmaxf(am, fabsf(qv[kc][4 * h2 + e]));
        }
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      const float inv = am > 0.f ? 127.f / am : 0.f;
      qscale[mt][hr] = am / 127.f;
#pragma unroll
      for (int kc = 0; kc < D / 32; ++kc)
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint32_t w = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int qi8 = max(-127, min(127, __float2int_rn(qv[kc][4 * h2 + e] * inv)));
            w |= (static_cast<uint32_t>(qi8) & 0xffu) << (8 * e);
          }
          qf[mt][kc][hr + 2 * h2] = w;  // a0 / a1: bytes 4t4.. of rows g / g+8; a2 / a3: bytes 16+4t4..
        }
    }
  }

  float m_run[MT][2], l_run[MT][2];
  float o[MT][D / 8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    m_run[mt][0] = m_run[mt][1] = kNegBig;
    l_run[mt][0] = l_run[mt][1] = 0.f;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[mt][n][0] = o[mt][n][1] = o[mt][n][2] = o[mt][n][3] = 0.f;
  }
  int limit[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + g + 8 * hr;
      limit[mt][hr] = (r < R) ? kv_len - a.ql + r / G : -1;
    }

  int i = 0;
  for (; i < my_n; ++i) {
    const int s = i % NST;
    if (!mbar_wait(&bars[s], (i / NST) & 1, &abort_flag, a.status, kStatusAttnTimeout)) break;
    const uint8_t* kp = wsm + s * kStageBytes;
    const uint8_t* vp = kp + kPageB;
    const float* ksc = wscl + s * 32;
    const float* vsc = ksc + 16;
    const int tok_base = (first + i * NWARPS) * PAGE;
    float skc[2][2], svc[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        skc[nt][e] = ksc[8 * nt + 2 * t4 + e];
        svc[nt][e] = vsc[8 * nt + 2 * t4 + e] * 256.f;
      }

    int sci[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sci[mt][nt][0] = sci[mt][nt][1] = sci[mt][nt][2] = sci[mt][nt][3] = 0;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int tok = 8 * nt + g;
      const uint8_t* row = kp + tok * D;
#pragma unroll
      for (int kc = 0; kc < D / 32; ++kc) {
        // 128-byte swizzle: 16-byte chunks 2kc and 2kc+1 of row tok, bytes 4t4..4t4+3 of each
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(row + (((2 * kc) ^ (tok & 7)) << 4) + 4 * t4);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(row + (((2 * kc + 1) ^ (tok & 7)) << 4) + 4 * t4);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) mma_s8_16832(sci[mt][nt], qf[mt][kc], b0, b1);
      }
    }
    float sc[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[mt][nt][e] = static_cast<float>(sci[mt][nt][e]) * qscale[mt][e >> 1];

    uint32_t pa[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float x[4];
        float mx = kNegBig;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int idx = tok_base + 8 * nt + 2 * t4 + e;
            float v = sc[mt][nt][2 * hr + e] * skc[nt][e] * a.scale_log2;
            if (idx > limit[mt][hr]) v = -INFINITY;
            x[nt * 2 + e] = v;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        // lazy rescaling: the running max only moves (and O, l are rescaled)
        // when a score exceeds it by more than 2^4; p <= 16 otherwise
        if (mx > m_run[mt][hr] + 4.f) {
          const float alpha = exp2f(m_run[mt][hr] - mx);
          m_run[mt][hr] = mx;
          l_run[mt][hr] *= alpha;
#pragma unroll
          for (int n = 0; n < D / 8; ++n) {
            o[mt][n][2 * hr] *= alpha;
            o[mt][n][2 * hr + 1] *= alpha;
          }
        }
        const float m_use = m_run[mt][hr];
        float ps = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          x[k] = exp2f(x[k] - m_use);
          ps += x[k];
        }
        l_run[mt][hr] += ps;
        // P carries the V scales times 2^8 (undone with 1 / l at the end):
        // p * scale * 256 stays a normal fp16 number for V absmax from ~1e-2
        // up to ~2000 (p <= 16)
        pa[mt][hr] = pack_f16(x[0] * svc[0][0], x[1] * svc[0][1]);
        pa[mt][hr + 2] = pack_f16(x[2] * svc[1][0], x[3] * svc[1][1]);
      }
    }

#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      // dim nb*8+g: its 16 tokens in fragment order, this thread's four at 4t4
      const uint32_t w = *reinterpret_cast<const uint32_t*>(vp + (nb * 8 + g) * PAGE + 4 * t4);
      uint32_t b0, b1;
      i8x4_f16x2(w, b0, b1);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) mma_f16_16816(o[mt][nb], pa[mt], b0, b1);
    }
    __syncwarp();
    if (lane == 0 && i + NST < my_n) {
      fence_proxy_async();
      issue(i + NST);
    }
  }
  if (i < my_n) {
    if (lane == 0)
      for (int k = i; k < my_n && k < i + NST; ++k) mbar_drain(&bars[k % NST], (k / NST) & 1);
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float l = l_run[mt][hr];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      l_run[mt][hr] = l;
    }
  __syncthreads();
  constexpr int RS = D + 2;
  float* cm = reinterpret_cast<float*>(smem);
  float* wbuf = cm + warp * (MT * 16 * RS);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + g + 8 * hr;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        wbuf[r * RS + 8 * n + 2 * t4] = o[mt][n][2 * hr];
        wbuf[r * RS + 8 * n + 2 * t4 + 1] = o[mt][n][2 * hr + 1];
      }
      if (t4 == 0) {
        wbuf[r * RS + D] = m_run[mt][hr];
        wbuf[r * RS + D + 1] = l_run[mt][hr] * 256.f;  // O holds sum p * (v scale * 2^8) * x
      }
    }
  __syncthreads();
  const int rows = min(R, MT * 16);
  for (int idx = threadIdx.x; idx < rows * D; idx += NWARPS * 32) {
    const int r = idx / D, d = idx - r * D;
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) M = fmaxf(M, cm[w * MT * 16 * RS + r * RS + D]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) {
      const float* wb = cm + w * MT * 16 * RS + r * RS;
      const float scl = exp2f(wb[D] - M);
      L += wb[D + 1] * scl;
      O += wb[d] * scl;
    }
    if (a.splits == 1) {
      const int qi = r / G, hh = r - qi * G;
      a.out[((long)(b * a.ql + qi) * a.nq + vkh * G + hh) * D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
    } else {
      float* pr = a.part + ((((long)b * a.nkv * a.hc + vkh) * a.splits + split) * 32 + r) * RS;
      pr[d] = O;
      if (d == 0) {
        pr[D] = M;
        pr[D + 1] = L;
      }
    }
  }
}

template <int MT, int NWARPS, int NST>
void launch_decode_q8(const CUtensorMap& tmK, const CUtensorMap& tmV, const DecodeArgs& a, int B, cudaStream_t stream) {
  constexpr int D = 128;
  constexpr int kRing = NWARPS * NST * 2 * PAGE * D;
  constexpr int kScl = NWARPS * NST * 128;
  constexpr int kMerge = NWARPS * MT * 16 * (D + 2) * 4;
  constexpr int kBarOff = (kRing + kScl > kMerge ? kRing + kScl : kMerge);
  constexpr int smem = kBarOff + NWARPS * NST * 8 + 1024;
  auto kern = decode_q8_kernel<MT, NWARPS, NST>;
  static uint64_t configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((configured >> dev) & 1u)) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured |= uint64_t(1) << dev;
  }
  dim3 grid(B, a.nkv * a.hc, a.splits);
  kern<<<grid, NWARPS * 32, smem, stream>>>(tmK, tmV, a);
}

// Prefill over an int8 cache: the pages a step's prefill sequences read are
// dequantised into a bf16 scratch cache laid out [S x W pages][2][KVH][16][128]
// (sequence s, page p -> scratch block s * W + p), and the prefill kernels run
// on it with the block table {s * W + p}.  grid (W, S), 256 threads.
__global__ void kv_dequant_pages_q8_kernel(const uint8_t* __restrict__ layer_base, long block_bytes, int nkv,
                                           const int* __restrict__ bt, int bt_stride, const int* __restrict__ ctx,
                                           int W, __nv_bfloat16* __restrict__ scratch, int num_blocks,
                                           int* status) {
  constexpr int D = 128;
  const int p = blockIdx.x, s = blockIdx.y;
  if (p * PAGE >= ctx[s]) return;
  int blk = bt[(long)s * bt_stride + p];
  if (!kcheck(blk >= 0 && blk < num_blocks, status)) blk = 0;
  const uint8_t* bp = layer_base + (long)blk * block_bytes;
  const float* scl = reinterpret_cast<const float*>(bp + 2L * nkv * PAGE * D);
  __nv_bfloat16* dst = scratch + ((long)s * W + p) * 2 * nkv * PAGE * D;
  const int n = 2 * nkv * PAGE * D;
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    // e = ((kv * nkv + kh) * 16 + tok) * D + d in the bf16 page layout
    const int d = e % D, tok = (e / D) % PAGE, kvh = e / (D * PAGE);
    const int kv = kvh / nkv;
    const int8_t* page = reinterpret_cast<const int8_t*>(bp) + (long)kvh * PAGE * D;
    const int8_t q = kv == 0 ? page[tok * D + d] : page[d * PAGE + q8_perm16(tok)];
    dst[e] = __float2bfloat16(static_cast<float>(q) * scl[kvh * PAGE + tok]);
  }
}

CUtensorMap kv_tmap(const torch::Tensor& kv_cache, int64_t layer) {
  TORCH_CHECK(kv_cache.dim() == 6 && kv_cache.size(2) == 2 && kv_cache.size(4) == PAGE &&
                  (kv_cache.size(5) == 128 || kv_cache.size(5) == 64),
              "kv_cache must be [L, NB, 2, KVH, 16, 128 or 64]");
  TORCH_CHECK(kv_cache.is_contiguous() && kv_cache.scalar_type() == at::kBFloat16, "kv_cache contiguous bf16");
  const uint64_t rows = (uint64_t)kv_cache.size(1) * 2 * kv_cache.size(3) * PAGE;
  TORCH_CHECK(rows < (1ull << 31), "kv_cache too many rows per layer for int32 TMA coordinates");
  const auto* base = reinterpret_cast<const __nv_bfloat16*>(kv_cache.data_ptr()) + layer * kv_cache.stride(0);
  const int hd = int(kv_cache.size(5));
  return make_tmap_bf16_2d(base, hd, rows, hd * 2, 64, PAGE);
}

template <int D, int MT, int NWARPS, int NST>
void launch_decode(const CUtensorMap& tm, const DecodeArgs& a, int B, cudaStream_t stream) {
  constexpr int kStage = 2 * PAGE * D * 2;
  constexpr int ring = NWARPS * NST * kStage > NWARPS * MT * 16 * (D + 2) * 4 ? NWARPS * NST * kStage
                                                                              : NWARPS * MT * 16 * (D + 2) * 4;
  static_assert(ring == NWARPS * NST * kStage, "the cross-warp merge buffer must fit in the stage ring");
  constexpr int smem = ring + NWARPS * NST * 8 + 1024;
  auto kern = decode_kernel<D, MT, NWARPS, NST>;
  static uint64_t configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((configured >> dev) & 1u)) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured |= uint64_t(1) << dev;
  }
  dim3 grid(B, a.nkv * a.hc, a.splits);
  kern<<<grid, NWARPS * 32, smem, stream>>>(tm, a);
}

}  // namespace attn

int64_t decode_head_chunks(int64_t num_q_heads, int64_t num_kv_heads, int64_t q_len) {
  if (num_kv_heads <= 0 || q_len < 1 || num_q_heads % num_kv_heads) return 0;
  const int64_t G = num_q_heads / num_kv_heads;
  for (int64_t hc = 1; hc <= G; ++hc)
    if (G % hc == 0 && (G / hc) * q_len <= 32) return hc;
  return 0;
}

int64_t decode_attention_splits(int64_t batch, int64_t num_kv_heads, int64_t max_pages, int64_t device) {
  const int64_t ctas = batch * num_kv_heads;
  const int64_t target = 2 * num_sms(int(device));
  if (ctas <= 0 || ctas >= target) return 1;
  int64_t s = (target + ctas - 1) / ctas;
  // at least 4 pages per warp-quad per split on long contexts
  const int64_t max_s = std::max<int64_t>(1, max_pages / 8);
  return std::max<int64_t>(1, std::min<int64_t>(s, std::min<int64_t>(max_s, 64)));
}

void paged_decode_attention(const torch::Tensor& q, const torch::Tensor& kv_cache, int64_t layer,
                            const torch::Tensor& block_table, const torch::Tensor& seq_lens, torch::Tensor& out,
                            int64_t q_len, int64_t splits, torch::Tensor& workspace, double scale,
                            const torch::Tensor& status) {
  const int hd = int(q.size(-1));
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && (hd == 128 || hd == 64),
              "decode: q [T, nq, 128 or 64] bf16");
  TORCH_CHECK(kv_cache.size(5) == hd, "decode: q and kv_cache head_dim differ");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.stride(1) == 1, "decode: block_table int32");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt, "decode: seq_lens int32");
  const int B = seq_lens.size(0);
  if (B == 0) return;
  const int nq = q.size(-2);
  const int nkv = kv_cache.size(3);
  TORCH_CHECK(nq % nkv == 0, "decode: nq must be a multiple of nkv");
  const int G = nq / nkv;
  const int hc = int(decode_head_chunks(nq, nkv, q_len));
  TORCH_CHECK(hc > 0, "decode: no split of the ", G, " q heads per kv head fits 32 rows at q_len ", q_len);
  TORCH_CHECK(q.numel() / (nq * hd) == B * q_len, "decode: q rows must equal batch * q_len");
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();

  attn::DecodeArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = block_table.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.nq = nq;
  a.nkv = nkv;
  a.ql = int(q_len);
  a.hc = hc;
  a.splits = std::max<int>(1, int(splits));
  a.scale_log2 = float(scale * 1.4426950408889634);
  a.status = status.data_ptr<int>();
  a.num_blocks = int(kv_cache.size(1));
  a.part = nullptr;
  if (a.splits > 1) {
    TORCH_CHECK(workspace.scalar_type() == at::kFloat &&
                    workspace.numel() >= (int64_t)B * nkv * hc * a.splits * 32 * (hd + 2),
                "decode: workspace too small");
    a.part = workspace.data_ptr<float>();
  }
  const CUtensorMap tm = attn::kv_tmap(kv_cache, layer);
  const bool mt1 = (G / hc) * q_len <= 16;
  if (hd == 128) {
    if (mt1) attn::launch_decode<128, 1, 4, 3>(tm, a, B, stream);
    else attn::launch_decode<128, 2, 4, 3>(tm, a, B, stream);
  } else {
    if (mt1) attn::launch_decode<64, 1, 4, 3>(tm, a, B, stream);
    else attn::launch_decode<64, 2, 4, 3>(tm, a, B, stream);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (a.splits > 1) {
    // each (kv head, head chunk) pair acts as its own "kv head" of G / hc q heads
    if (hd == 128)
      attn::decode_combine_kernel<128><<<dim3(B, nkv * hc), 256, 0, stream>>>(a.part, a.out, nq, nkv * hc, a.ql,
                                                                             a.splits);
    else
      attn::decode_combine_kernel<64><<<dim3(B, nkv * hc), 256, 0, stream>>>(a.part, a.out, nq, nkv * hc, a.ql,
                                                                            a.splits);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

void paged_decode_attention_q8(const torch::Tensor& q, const torch::Tensor& kv_cache, int64_t layer,
                               int64_t num_kv_heads, const torch::Tensor& block_table, const torch::Tensor& seq_lens,
                               torch::Tensor& out, int64_t q_len, int64_t splits, torch::Tensor& workspace,
                               double scale, const torch::Tensor& status) {
  constexpr int hd = 128;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.size(-1) == hd, "decode_q8: q [T, nq, 128] bf16");
  TORCH_CHECK(kv_cache.scalar_type() == at::kByte && kv_cache.dim() == 3 && kv_cache.is_contiguous(),
              "decode_q8: int8 kv cache [L, NB, block_bytes] uint8");
  const int nkv = int(num_kv_heads);
  const long bb = kv_cache.size(2);
  TORCH_CHECK(bb == 2L * nkv * 16 * (hd + 4), "decode_q8: block bytes do not match 2 x KVH x 16 x (128 + 4)");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.stride(1) == 1, "decode_q8: block_table int32");
  const int B = seq_lens.size(0);
  if (B == 0) return;
  const int nq = q.size(-2);
  TORCH_CHECK(nq % nkv == 0, "decode_q8: nq must be a multiple of nkv");
  const int hc = int(decode_head_chunks(nq, nkv, q_len));
  TORCH_CHECK(hc > 0, "decode_q8: no split of the q heads per kv head fits 32 rows at q_len ", q_len);
  TORCH_CHECK(q.numel() / (nq * hd) == B * q_len, "decode_q8: q rows must equal batch * q_len");
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const uint8_t* base = kv_cache.data_ptr<uint8_t>() + layer * kv_cache.stride(0);
  const uint64_t total = static_cast<uint64_t>(kv_cache.size(1)) * bb;
  TORCH_CHECK(total / 16 < (1ull << 31), "decode_q8: cache layer too large for int32 TMA coordinates");
  const CUtensorMap tmK = make_tmap_2d(base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, hd, total / hd, hd, hd, attn::PAGE,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tmV = make_tmap_2d(base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 16, total / 16, 16, 16, hd,
                                       CU_TENSOR_MAP_SWIZZLE_NONE);
  attn::DecodeArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = block_table.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.nq = nq;
  a.nkv = nkv;
  a.ql = int(q_len);
  a.hc = hc;
  a.splits = std::max<int>(1, int(splits));
  a.scale_log2 = float(scale * 1.4426950408889634);
  a.status = status.data_ptr<int>();
  a.num_blocks = int(kv_cache.size(1));
  a.q8_base = base;
  a.q8_block_bytes = bb;
  a.part = nullptr;
  if (a.splits > 1) {
    TORCH_CHECK(workspace.scalar_type() == at::kFloat &&
                    workspace.numel() >= (int64_t)B * nkv * hc * a.splits * 32 * (hd + 2),
                "decode_q8: workspace too small");
    a.part = workspace.data_ptr<float>();
  }
  const bool mt1 = (nq / nkv / hc) * q_len <= 16;
  if (mt1) attn::launch_decode_q8<1, 4, 3>(tmK, tmV, a, B, stream);
  else attn::launch_decode_q8<2, 4, 3>(tmK, tmV, a, B, stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (a.splits > 1) {
    attn::decode_combine_kernel<128><<<dim3(B, nkv * hc), 256, 0, stream>>>(a.part, a.out, nq, nkv * hc, a.ql,
                                                                           a.splits);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

void kv_dequant_pages_q8(const torch::Tensor& kv_cache, int64_t layer, int64_t num_kv_heads,
                         const torch::Tensor& block_table, const torch::Tensor& ctx_lens, int64_t W,
                         torch::Tensor& scratch, const torch::Tensor& status) {
  TORCH_CHECK(kv_cache.scalar_type() == at::kByte && kv_cache.dim() == 3 && kv_cache.is_contiguous(),
              "kv_dequant_q8: int8 kv cache [L, NB, block_bytes] uint8");
  const int S = ctx_lens.size(0);
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.stride(1) == 1 && block_table.size(1) <= W,
              "kv_dequant_q8: block table int32 [S, <= W]");
  TORCH_CHECK(scratch.scalar_type() == at::kBFloat16 && scratch.is_contiguous() &&
                  scratch.numel() >= (int64_t)S * W * 2 * num_kv_heads * 16 * 128,
              "kv_dequant_q8: scratch bf16 [S * W, 2, KVH, 16, 128]");
  if (S == 0) return;
  const at::cuda::CUDAGuard guard(kv_cache.device());
  attn::kv_dequant_pages_q8_kernel<<<dim3(int(block_table.size(1)), S), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      kv_cache.data_ptr<uint8_t>() + layer * kv_cache.stride(0), kv_cache.size(2), int(num_kv_heads),
      block_table.data_ptr<int>(), int(block_table.stride(0)), ctx_lens.data_ptr<int>(), int(W),
      reinterpret_cast<__nv_bfloat16*>(scratch.data_ptr()), int(kv_cache.size(1)), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void paged_prefill_attention(const torch::Tensor& q, const torch::Tensor& kv_cache, int64_t layer,
                             const torch::Tensor& block_table, const torch::Tensor& ctx_lens,
                             const torch::Tensor& cu_seqlens_q, const torch::Tensor& tile_seq,
                             const torch::Tensor& tile_start, torch::Tensor& out, double scale, bool causal,
                             const torch::Tensor& status) {
  const int hd = int(q.size(-1));
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && (hd == 128 || hd == 64),
              "prefill: q [T, nq, 128 or 64] bf16");
  TORCH_CHECK(kv_cache.size(5) == hd, "prefill: q and kv_cache head_dim differ");
  const int n_tiles = tile_seq.size(0);
  if (n_tiles == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  attn::PrefillArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = block_table.stride(0);
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.cu_q = cu_seqlens_q.data_ptr<int>();
  a.tile_seq = tile_seq.data_ptr<int>();
  a.tile_start = tile_start.data_ptr<int>();
  a.nq = q.size(-2);
  a.nkv = kv_cache.size(3);
  a.scale_log2 = float(scale * 1.4426950408889634);
  a.causal = causal ? 1 : 0;
  a.status = status.data_ptr<int>();
  a.num_blocks = int(kv_cache.size(1));
  const CUtensorMap tm = attn::kv_tmap(kv_cache, layer);
  constexpr int smem128 = attn::kPfStages * attn::pf_stage_bytes<128>() + 64 + 1024;
  constexpr int smem64 = attn::kPfStages * attn::pf_stage_bytes<64>() + 64 + 1024;
  static uint64_t configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((configured >> dev) & 1u)) {
    cudaFuncSetAttribute(attn::prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem128);
    cudaFuncSetAttribute(attn::prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem64);
    configured |= uint64_t(1) << dev;
  }
  if (hd == 128)
    attn::prefill_kernel<128><<<dim3(n_tiles, a.nq, 2), attn::kPfWarps * 32, smem128, stream>>>(tm, a);
  else
    attn::prefill_kernel<64><<<dim3(n_tiles, a.nq, 2), attn::kPfWarps * 32, smem64, stream>>>(tm, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom

// ============================================================================
// Allocation-free entry point: bloom_paged_decode_attention_noalloc
//
// This entry point has no counterpart in the reference; it is an addition of
// this library.
//
// Who needs it: some callers cannot allocate GPU memory at the moment they
// want to run attention.  Examples are a host application that hands this
// library a fixed memory budget and forbids cudaMalloc after start-up, code
// that runs on a stream whose memory pool belongs to another framework, and
// plain C programs that load this library without PyTorch (so there is no
// caching allocator to borrow scratch from).  The regular entry point takes
// its split-K scratch from the caller as a torch tensor; this one takes it
// from a fixed array compiled into the library instead, and it never calls
// cudaMalloc, cudaFree or any allocating routine.
//
// What it computes: exactly what paged_decode_attention computes (the same
// kernels), for q [batch * q_len, num_q_heads, 128] bf16 against one layer of
// the paged cache [num_blocks, 2, num_kv_heads, 16, 128] bf16, writing
// out [batch * q_len, num_q_heads, 128] bf16.  The caller owns q, out, the
// cache, the block table and the sequence lengths.
//
// Limits and rules:
//  * Scratch is kNoAllocScratchFloats fp32 values (8 MiB) per GPU, held by
//    every GPU that loads the library until the process exits.  A call needs
//    batch * num_kv_heads * splits * 32 * 130 floats when splits > 1; larger
//    requests are rejected with BLOOM_NOALLOC_TOO_LARGE and nothing runs.
//  * All calls on a device share that one array, and it keeps whatever the
//    last call left in it.  Two calls whose kernels overlap on the GPU (two
//    streams, no ordering between them) race on the scratch and give wrong
//    results; order them on one stream or with events.  Nothing in the
//    scratch has to start at zero: every partial is written before it is read.
//  * The first call on a device does the set-up for that device: it looks up
//    the device address of the array with cudaGetSymbolAddress (host code
//    must never pass the array's name itself to a kernel: on the host that
//    name is only a stand-in) and clears the status word.  Make that first
//    call on each device before any stream capture begins.
//  * Waits inside the kernel are bounded; a wait that gives up sets a bit in
//    a status word that bloom_noalloc_status() reads and clears.
// ============================================================================
namespace bloom {
namespace noalloc {

constexpr long long kNoAllocScratchFloats = 1ll << 21;  // 8 MiB
static __device__ __align__(256) float g_scratch[kNoAllocScratchFloats];
static __device__ __align__(256) int g_status[16];

struct DeviceState {
  float* scratch = nullptr;
  int* status = nullptr;
  bool ready = false;
};
static DeviceState g_dev[64];
static std::mutex g_mu;

// Once per device, with that device current: resolve the arrays' device addresses.
static int setup_device(int dev) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_dev[dev].ready) return 0;
  void* scratch = nullptr;
  void* status = nullptr;
  if (cudaGetSymbolAddress(&scratch, g_scratch) != cudaSuccess) return -3;
  if (cudaGetSymbolAddress(&status, g_status) != cudaSuccess) return -3;
  if (cudaMemset(status, 0, sizeof(int) * 16) != cudaSuccess) return -3;
  g_dev[dev].scratch = static_cast<float*>(scratch);
  g_dev[dev].status = static_cast<int*>(status);
  g_dev[dev].ready = true;
  return 0;
}

}  // namespace noalloc
}  // namespace bloom

// Return codes and declarations: csrc/include/bloom/noalloc.h
#include "bloom/noalloc.h"

extern "C" __attribute__((visibility("default"))) int bloom_paged_decode_attention_noalloc(
    const void* q, void* out, const void* kv_layer, long long num_blocks, int num_q_heads, int num_kv_heads,
    const int* block_table, int block_table_stride, const int* seq_lens, int batch, int q_len, int splits,
    float scale, void* stream) {
  using namespace bloom;
  if (q == nullptr || out == nullptr || kv_layer == nullptr || block_table == nullptr || seq_lens == nullptr)
    return BLOOM_NOALLOC_BAD_ARGUMENT;
  if (batch <= 0 || num_blocks <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || q_len < 1 ||
      num_q_heads % num_kv_heads != 0 || block_table_stride <= 0)
    return BLOOM_NOALLOC_BAD_ARGUMENT;
  if ((num_q_heads / num_kv_heads) * q_len > 32) return BLOOM_NOALLOC_BAD_ARGUMENT;
  if (batch > 65535 || num_kv_heads > 65535) return BLOOM_NOALLOC_BAD_ARGUMENT;
  if (splits < 1) splits = 1;
  if (splits > 65535) return BLOOM_NOALLOC_BAD_ARGUMENT;
  if (splits > 1 && (long long)batch * num_kv_heads * splits * 32 * (attn::D + 2) > noalloc::kNoAllocScratchFloats)
    return BLOOM_NOALLOC_TOO_LARGE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BLOOM_NOALLOC_CUDA_ERROR;
  if (noalloc::setup_device(dev) != 0) return BLOOM_NOALLOC_CUDA_ERROR;

  const unsigned long long rows = (unsigned long long)num_blocks * 2 * num_kv_heads * attn::PAGE;
  if (rows >= (1ull << 31)) return BLOOM_NOALLOC_BAD_ARGUMENT;
  CUtensorMap tm;
  try {
    tm = make_tmap_bf16_2d(kv_layer, attn::D, rows, attn::D * 2, 64, attn::PAGE);
  } catch (...) {
    return BLOOM_NOALLOC_TENSOR_MAP_ERROR;
  }
  attn::DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.block_table = block_table;
  a.bt_stride = block_table_stride;
  a.seq_lens = seq_lens;
  a.nq = num_q_heads;
  a.nkv = num_kv_heads;
  a.ql = q_len;
  a.hc = 1;
  a.splits = splits;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.status = noalloc::g_dev[dev].status;
  a.part = splits > 1 ? noalloc::g_dev[dev].scratch : nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((num_q_heads / num_kv_heads) * q_len <= 16)
    attn::launch_decode<attn::D, 1, 4, 3>(tm, a, batch, s);
  else
    attn::launch_decode<attn::D, 2, 4, 3>(tm, a, batch, s);
  if (cudaGetLastError() != cudaSuccess) return BLOOM_NOALLOC_LAUNCH_ERROR;
  if (splits > 1) {
    attn::decode_combine_kernel<attn::D><<<dim3(batch, num_kv_heads), 256, 0, s>>>(a.part, a.out, num_q_heads, num_kv_heads,
                                                                          q_len, splits);
    if (cudaGetLastError() != cudaSuccess) return BLOOM_NOALLOC_LAUNCH_ERROR;
  }
  return BLOOM_NOALLOC_OK;
}

// Reads and clears the allocation-free entry point's status word on the
// current device (bit 2: an attention wait gave up).  Synchronous: it first
// waits for all work on the device (cudaDeviceSynchronize), so a call queued
// on any stream -- a non-blocking stream or a per-thread default stream
// included -- has finished and set its bits before the word is read.  Do not
// call it while a stream of this device is being captured.
extern "C" __attribute__((visibility("default"))) int bloom_noalloc_status(int* bits) {
  using namespace bloom;
  int dev = 0;
  if (bits == nullptr || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BLOOM_NOALLOC_BAD_ARGUMENT;
  if (noalloc::setup_device(dev) != 0) return BLOOM_NOALLOC_CUDA_ERROR;
  if (cudaDeviceSynchronize() != cudaSuccess) return BLOOM_NOALLOC_CUDA_ERROR;
  if (cudaMemcpy(bits, noalloc::g_dev[dev].status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return BLOOM_NOALLOC_CUDA_ERROR;
  if (cudaMemset(noalloc::g_dev[dev].status, 0, sizeof(int)) != cudaSuccess) return BLOOM_NOALLOC_CUDA_ERROR;
  return BLOOM_NOALLOC_OK;
}
