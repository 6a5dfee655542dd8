// Gemma4 text decoder kernels: wide attention heads (head_dim 256 on sliding
// layers, 512 on global layers), sliding-window masks, attention and final
// logit soft-capping, q/k/v RMSNorm with partial RoPE, and the "sandwich"
// residual norms of the Gemma block.
//
// Reference behaviour: executor/gemma4.rs (Config :175-336, RotaryEmbedding
// :405-465, Attention::forward :668-761 incl. soft-capping :731-735,
// DecoderLayer::forward :892-910, Model::forward :1040-1063, masks
// :913-949).  The reference runs these as candle tensor ops over a growing or
// rotating per-sequence KV cache; here the KV cache is paged in HBM and each
// step is a handful of fused kernels.
//
// KV cache: one bf16 tensor [L, NB, E] whose layer slice holds, per 16-token
// block, K pages [KVH][16][D] then V pages [KVH][16][D] (E is the largest
// layer's 2 * KVH * 16 * D; sliding and global layers use different KVH / D).
//
// wide_attention_kernel<D>: one CTA = 64 query rows x 128 output dims of one
// KV head.  Decode packs (q position, GQA head) pairs into the rows (every
// KV tile is read once per KV head); prefill takes 64 query tokens of one q
// head (the scheduler's 128-row prefill tiles as two halves).  K tiles of 32
// keys x D dims and the matching 32 x 128 V slice are double buffered in
// shared memory with cp.async; S = Q K^T and O += P V run on m16n8k16 bf16
// MMAs with fp32 accumulation and an online (flash) softmax.  head_dim / 128
// CTAs share one query tile, each producing one 128-dim slice of the output
// (S is recomputed per slice: 1.5x / 2.5x the minimum MMA work at D = 256 /
// 512, in exchange for 64 accumulator registers per thread at any D).  Decode
// splits the key range over up to 16 CTAs and merges (o, m, l) partials.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"

namespace bloom {
namespace gemma {

constexpr int PAGE = 16;
constexpr int kRows = 64;   // query rows per CTA (4 warps x 16)
constexpr int kKeys = 32;   // keys per KV tile (two pages)
constexpr int kDC = 128;    // output dims per CTA
constexpr int kThreads = 128;
constexpr int kMaxSplits = 16;
constexpr float kNegBig = -1e30f;
constexpr float kLog2e = 1.4426950408889634f;

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
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

struct WideArgs {
  const __nv_bfloat16* q;    // [rows, nq, D]
  __nv_bfloat16* out;        // [rows, nq, D]
  const __nv_bfloat16* kv;   // this layer's [NB, E] slice
  long block_stride;         // E: elements per block in one layer
  int nq, nkv, num_blocks;
  const int* block_table;
  int bt_stride;
  // decode: sequence b has ql query rows (b * ql ...) and kv length seq_lens[b]
  const int* seq_lens;
  int ql;
  // prefill: the scheduler's 128-row tiles over variable-length sequences
  const int* cu_q;
  const int* ctx_lens;
  const int* tile_seq;
  const int* tile_start;
  int prefill;
  int causal;       // 0: every row sees keys [0, kv_len) (window ignored)
  int window;       // > 0: key j is visible to the query at position p iff p - window < j <= p
  float scale;      // score scale before soft-capping
  float softcap;    // > 0: s = softcap * tanh(s / softcap)
  int splits;       // decode: key-range splits (partials in part)
  float* part;      // [gridDim.x * gridDim.y * splits * 64 * (128 + 2)]
  int* status;
};

template <int D, int ROWS, int STAGES>
struct Smem {
  static constexpr int kQS = D + 8;    // padded row stride (elements): ldmatrix rows hit distinct banks
  static constexpr int kVS = kDC + 8;
  static constexpr int kQBytes = ROWS * kQS * 2;
  static constexpr int kKBytes = kKeys * kQS * 2;
  static constexpr int kVBytes = kKeys * kVS * 2;
  static constexpr int kStage = kKBytes + kVBytes;
  static constexpr int kTotal = kQBytes + STAGES * kStage;
};

// ROWS query rows per CTA (64 = 4 computing warps; 16 = decode rows of one
// KV head, one computing warp while all four load), STAGES-deep cp.async
// ring of K / V tiles (one barrier per tile: a stage is refilled right after
// the barrier that follows its last use).
template <int D, int ROWS, int STAGES>
__global__ void __launch_bounds__(kThreads) wide_attention_kernel(const WideArgs a) {
  using S = Smem<D, ROWS, STAGES>;
  constexpr int kRows = ROWS;
  constexpr int NDC = D / kDC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int G = a.nq / a.nkv;

  // ---- which rows, which KV head, which output slice
  int kh, dc, split = 0, nrows, kv_len;
  int seq;
  long qrow0 = 0;   // prefill: first q token row
  int pos0 = 0;     // prefill: position of row 0
  int rbase = 0;    // decode: packed-row offset of this CTA
  int qb = 0;       // decode: sequence's first q row (b * ql)
  int h_pf = 0;     // prefill: the q head
  if (a.prefill) {
    const int tile = blockIdx.x;
    h_pf = blockIdx.y / NDC;
    dc = blockIdx.y - h_pf * NDC;
    kh = h_pf / G;
    seq = a.tile_seq[tile];
    const int lr0 = a.tile_start[tile] + kRows * blockIdx.z;
    const int q_begin = a.cu_q[seq];
    const int q_len = a.cu_q[seq + 1] - q_begin;
    kv_len = a.ctx_lens[seq];
    nrows = min(kRows, q_len - lr0);
    qrow0 = q_begin + lr0;
    pos0 = kv_len - q_len + lr0;
  } else {
    seq = blockIdx.x;
    const int R = a.ql * G;
    const int nrt = (R + kRows - 1) / kRows;
    const int per_kh = nrt * NDC;
    kh = blockIdx.y / per_kh;
    const int rem = blockIdx.y - kh * per_kh;
    const int rt = rem / NDC;
    dc = rem - rt * NDC;
    split = blockIdx.z;
    rbase = rt * kRows;
    nrows = min(kRows, R - rbase);
    kv_len = a.seq_lens[seq];
    qb = seq * a.ql;
  }
  // position and q row of packed row r
  auto row_pos = [&](int r) -> int {
    if (a.prefill) return pos0 + r;
    return kv_len - a.ql + (rbase + r) / G;
  };
  auto row_q = [&](int r) -> long {
    if (a.prefill) return (qrow0 + r) * a.nq + h_pf;
    const int rr = rbase + r, qi = rr / G, hh = rr - qi * G;
    return (long)(qb + qi) * a.nq + kh * G + hh;
  };

  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t sQa = smem_u32(smem);
  const uint32_t sStage = sQa + S::kQBytes;

  // key range of the tile's rows (rows are in increasing position order)
  const int p_first = nrows > 0 ? row_pos(0) : 0;
  const int p_last = nrows > 0 ? row_pos(nrows - 1) : -1;
  const int lo = (a.causal && a.window > 0) ? max(0, p_first - a.window + 1) : 0;
  const int hi = a.causal ? min(p_last + 1, kv_len) : (nrows > 0 ? kv_len : 0);
  const int kt0 = lo / kKeys;
  const int kt_all = hi > lo ? (hi + kKeys - 1) / kKeys - kt0 : 0;
  const int per_split = (kt_all + a.splits - 1) / a.splits;
  const int ka = kt0 + split * per_split;
  const int kb = min(kt0 + kt_all, ka + per_split);
  const int n_kt = max(0, kb - ka);
  const int n_pages = (kv_len + PAGE - 1) / PAGE;
  const int* bt = a.block_table + (long)seq * a.bt_stride;

  // ---- Q tile -> shared (rows past nrows are zero)
  for (int c = threadIdx.x; c < kRows * (D / 8); c += kThreads) {
    const int r = c / (D / 8), d8 = c - r * (D / 8);
    const uint32_t dst = sQa + (r * S::kQS + d8 * 8) * 2;
    if (r < nrows) {
      cp_async16(dst, a.q + row_q(r) * D + d8 * 8);
    } else {
      *reinterpret_cast<uint4*>(smem + (r * S::kQS + d8 * 8) * 2) = make_uint4(0, 0, 0, 0);
    }
  }
  auto load_tile = [&](int kt, int stage) {
    const uint32_t sK = sStage + stage * S::kStage;
    const uint32_t sV = sK + S::kKBytes;
    uint8_t* gK = smem + S::kQBytes + stage * S::kStage;
    uint8_t* gV = gK + S::kKBytes;
#pragma unroll
    for (int pg = 0; pg < 2; ++pg) {
      const int page = kt * 2 + pg;
      const bool live = page < n_pages;
      int blk = 0;
      if (live) {
        blk = bt[page];
        if (!kcheck(blk >= 0 && blk < a.num_blocks, a.status)) blk = 0;
      }
      const __nv_bfloat16* kp = a.kv + (long)blk * a.block_stride + (long)kh * PAGE * D;
      const __nv_bfloat16* vp = a.kv + (long)blk * a.block_stride + (long)(a.nkv + kh) * PAGE * D + dc * kDC;
      for (int c = threadIdx.x; c < PAGE * (D / 8); c += kThreads) {
        const int t = c / (D / 8), d8 = c - t * (D / 8);
        const int row = pg * PAGE + t;
        if (live)
          cp_async16(sK + (row * S::kQS + d8 * 8) * 2, kp + (long)t * D + d8 * 8);
        else
          *reinterpret_cast<uint4*>(gK + (row * S::kQS + d8 * 8) * 2) = make_uint4(0, 0, 0, 0);
      }
      for (int c = threadIdx.x; c < PAGE * (kDC / 8); c += kThreads) {
        const int t = c / (kDC / 8), d8 = c - t * (kDC / 8);
        const int row = pg * PAGE + t;
        if (live)
          cp_async16(sV + (row * S::kVS + d8 * 8) * 2, vp + (long)t * D + d8 * 8);
        else
          *reinterpret_cast<uint4*>(gV + (row * S::kVS + d8 * 8) * 2) = make_uint4(0, 0, 0, 0);
      }
    }
  };
#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) {
    if (st < n_kt) load_tile(ka + st, st);
    cp_async_commit();  // the Q tile rides in the first group
  }

  // per-thread rows g and g + 8 of this warp's 16
  int pos[2];
  bool rvalid[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = warp * 16 + g + 8 * hr;
    rvalid[hr] = r < nrows;
    pos[hr] = rvalid[hr] ? row_pos(r) : -1;
  }
  float m_run[2] = {kNegBig, kNegBig}, l_run[2] = {0.f, 0.f};
  float o[kDC / 8][4];
#pragma unroll
  for (int n = 0; n < kDC / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const float sl2 = a.scale * kLog2e;
  const bool warp_live = warp * 16 < nrows;

  for (int i = 0; i < n_kt; ++i) {
    const int stage = i % STAGES;
    cp_async_wait<STAGES - 2>();  // tile i (and Q) landed
    __syncthreads();              // ... for every thread; stage (i - 1) % STAGES is free again
    if (i + STAGES - 1 < n_kt) load_tile(ka + i + STAGES - 1, (i + STAGES - 1) % STAGES);
    cp_async_commit();
    if (warp_live) {
      const uint32_t sK = sStage + stage * S::kStage;
      const uint32_t sV = sK + S::kKBytes;
      const int k0 = (ka + i) * kKeys;
      float sc[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll 2
      for (int ks = 0; ks < D / 32; ++ks) {
        uint32_t a0[4], a1[4];
        const uint32_t qa = sQa + ((warp * 16 + (lane & 15)) * S::kQS + 32 * ks + 8 * (lane >> 4)) * 2;
        ldsm_x4(qa, a0[0], a0[1], a0[2], a0[3]);
        ldsm_x4(qa + 32, a1[0], a1[1], a1[2], a1[3]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(sK + ((8 * nt + (lane & 7)) * S::kQS + 32 * ks + 8 * (lane >> 3)) * 2, b0, b1, b2, b3);
          mma16816(sc[nt], a0, b0, b1);
          mma16816(sc[nt], a1, b2, b3);
        }
      }
      uint32_t pa[2][4];
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float x[4][2];
        float mx = kNegBig;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = k0 + 8 * nt + 2 * t4 + e;
            float v = sc[nt][2 * hr + e];
            if (a.softcap > 0.f) {
              v = a.softcap * tanhf(v * a.scale / a.softcap) * kLog2e;
            } else {
              v *= sl2;
            }
            const bool vis = a.causal ? (j <= pos[hr] && (a.window <= 0 || j > pos[hr] - a.window))
                                      : (rvalid[hr] && j < kv_len);
            v = vis ? v : -INFINITY;
            x[nt][e] = v;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[hr], mx);
        const float alpha = exp2f(m_run[hr] - m_new);
        m_run[hr] = m_new;
        float ps = 0.f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            x[nt][e] = exp2f(x[nt][e] - m_new);
            ps += x[nt][e];
          }
        l_run[hr] = l_run[hr] * alpha + ps;
#pragma unroll
        for (int n = 0; n < kDC / 8; ++n) {
          o[n][2 * hr] *= alpha;
          o[n][2 * hr + 1] *= alpha;
        }
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          pa[kk][hr] = pack2(x[2 * kk][0], x[2 * kk][1]);
          pa[kk][hr + 2] = pack2(x[2 * kk + 1][0], x[2 * kk + 1][1]);
        }
      }
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
#pragma unroll
        for (int j = 0; j < kDC / 16; ++j) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sV + ((16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1)) * S::kVS + 16 * j + 8 * (lane >> 4)) * 2,
                    b0, b1, b2, b3);
          mma16816(o[2 * j], pa[kk], b0, b1);
          mma16816(o[2 * j + 1], pa[kk], b2, b3);
        }
    }
  }
  cp_async_wait<0>();

#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = l_run[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l_run[hr] = l;
  }
  constexpr int RS = kDC + 2;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    if (!rvalid[hr]) continue;
    const int r = warp * 16 + g + 8 * hr;
    if (a.splits == 1) {
      const float inv = l_run[hr] > 0.f ? 1.f / l_run[hr] : 0.f;
      __nv_bfloat16* orow = a.out + row_q(r) * D + dc * kDC;
#pragma unroll
      for (int n = 0; n < kDC / 8; ++n)
        *reinterpret_cast<uint32_t*>(orow + 8 * n + 2 * t4) = pack2(o[n][2 * hr] * inv, o[n][2 * hr + 1] * inv);
    } else {
      float* pr = a.part + ((((long)blockIdx.x * gridDim.y + blockIdx.y) * a.splits + split) * kRows + r) * RS;
#pragma unroll
      for (int n = 0; n < kDC / 8; ++n) {
        pr[8 * n + 2 * t4] = o[n][2 * hr];
        pr[8 * n + 2 * t4 + 1] = o[n][2 * hr + 1];
      }
      if (t4 == 0) {
        pr[kDC] = m_run[hr];
        pr[kDC + 1] = l_run[hr];
      }
    }
  }
}

// Merge the decode key-range splits: one CTA per (sequence, row tile / slice).
template <int D, int ROWS>
__global__ void wide_combine_kernel(const WideArgs a) {
  constexpr int kRows = ROWS;
  constexpr int NDC = D / kDC;
  constexpr int RS = kDC + 2;
  const int G = a.nq / a.nkv;
  const int R = a.ql * G;
  const int nrt = (R + kRows - 1) / kRows;
  const int per_kh = nrt * NDC;
  const int kh = blockIdx.y / per_kh;
  const int rem = blockIdx.y - kh * per_kh;
  const int rt = rem / NDC, dc = rem - rt * NDC;
  const int nrows = min(kRows, R - rt * kRows);
  const float* base = a.part + ((long)blockIdx.x * gridDim.y + blockIdx.y) * a.splits * kRows * RS;
  for (int idx = threadIdx.x; idx < nrows * kDC; idx += blockDim.x) {
    const int r = idx / kDC, d = idx - r * kDC;
    float M = kNegBig;
    for (int s = 0; s < a.splits; ++s) M = fmaxf(M, base[((long)s * kRows + r) * RS + kDC]);
    float L = 0.f, O = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float* pr = base + ((long)s * kRows + r) * RS;
      const float w = exp2f(pr[kDC] - M);
      L += pr[kDC + 1] * w;
      O += pr[d] * w;
    }
    const int rr = rt * kRows + r, qi = rr / G, hh = rr - qi * G;
    a.out[((long)(blockIdx.x * a.ql + qi) * a.nq + kh * G + hh) * D + dc * kDC + d] =
        __float2bfloat16(L > 0.f ? O / L : 0.f);
  }
}

// ---------------------------------------------------------------- q/k/v write
// One warp per (token, head): heads [0, nq) are q heads, [nq, nq + nkv) KV
// heads.  q -> rmsnorm * q_w -> RoPE on the first `rot` dims -> q_out.
// k -> rmsnorm * k_w -> RoPE -> K page; v (or the raw k row when the layer
// has no v projection) -> rmsnorm without scale -> V page.  RoPE pairs
// (i, i + rot/2) for i < rot/2 (the rotate-half convention) with the angles
// of cs [max_pos, 2, rot/2] (cos then sin).
template <int D>
__global__ void __launch_bounds__(256) qkv_write_kernel(
    const __nv_bfloat16* __restrict__ qkv, long ld, int T, int nq, int nkv, int rot, const int64_t* __restrict__ pos,
    const int* __restrict__ slots, const float* __restrict__ cs, int max_pos, const __nv_bfloat16* __restrict__ qw,
    const __nv_bfloat16* __restrict__ kw, float eps, int k_eq_v, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ kv, long block_stride, int num_blocks, int* status) {
  constexpr int PER = D / 32;  // elements per lane: 8 or 16 (chunks of 8 at lane * 8 + 256 * c)
  __shared__ float rowbuf[8][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long item = (long)blockIdx.x * 8 + warp;
  const int nh = nq + nkv;
  if (item >= (long)T * nh) return;
  const int t = int(item / nh), h = int(item - (long)t * nh);
  const bool is_q = h < nq;
  const int kh = h - nq;
  const __nv_bfloat16* src = qkv + (long)t * ld + (long)h * D;  // q head h, or k head kh (at column (nq + kh) * D)
  float* rb = rowbuf[warp];
  int p = int(pos[t]);
  if (!kcheck(p >= 0 && p < max_pos, status)) p = 0;
  const float* cosp = cs + (long)p * rot;
  const float* sinp = cosp + rot / 2;
  const int half = rot / 2;

  auto load = [&](const __nv_bfloat16* s, float (&v)[PER]) {
#pragma unroll
    for (int c = 0; c < PER / 8; ++c) {
      const uint4 u = *reinterpret_cast<const uint4*>(s + lane * 8 + 256 * c);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[c * 8 + k] = __bfloat162float(b[k]);
    }
  };
  auto rms_inv = [&](const float (&v)[PER]) {
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) ss += v[k] * v[k];
    ss = warp_sum(ss);
    return rsqrtf(ss / D + eps);
  };
  // normalise (optionally scaled), stage in shared memory, rotate, pack
  auto norm_rope = [&](float (&v)[PER], const __nv_bfloat16* w, bool rope, uint4 (&outv)[PER / 8]) {
    const float inv = rms_inv(v);
#pragma unroll
    for (int c = 0; c < PER / 8; ++c)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = lane * 8 + 256 * c + k;
        v[c * 8 + k] *= inv * (w != nullptr ? __bfloat162float(w[i]) : 1.f);
        rb[i] = v[c * 8 + k];
      }
    __syncwarp();
#pragma unroll
    for (int c = 0; c < PER / 8; ++c) {
      float y[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = lane * 8 + 256 * c + k;
        float r = v[c * 8 + k];
        if (rope && i < rot) {
          if (i < half)
            r = r * cosp[i] - rb[i + half] * sinp[i];
          else
            r = r * cosp[i - half] + rb[i - half] * sinp[i - half];
        }
        y[k] = r;
      }
      outv[c] = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                           pack_bf16x2(y[6], y[7]));
    }
    __syncwarp();
  };

  float v[PER];
  uint4 outv[PER / 8];
  load(src, v);
  if (is_q) {
    norm_rope(v, qw, true, outv);
    __nv_bfloat16* dst = q_out + ((long)t * nq + h) * D;
#pragma unroll
    for (int c = 0; c < PER / 8; ++c) *reinterpret_cast<uint4*>(dst + lane * 8 + 256 * c) = outv[c];
    return;
  }
  const int slot = slots[t];
  int blk = slot >= 0 ? slot / PAGE : -1;
  if (blk >= 0 && !kcheck(blk < num_blocks, status)) blk = -1;
  float raw[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) raw[k] = v[k];
  norm_rope(v, kw, true, outv);
  if (blk >= 0) {
    __nv_bfloat16* dst = kv + (long)blk * block_stride + ((long)kh * PAGE + slot % PAGE) * D;
#pragma unroll
    for (int c = 0; c < PER / 8; ++c) *reinterpret_cast<uint4*>(dst + lane * 8 + 256 * c) = outv[c];
  }
  if (!k_eq_v) load(qkv + (long)t * ld + (long)(nq + nkv + kh) * D, raw);
  norm_rope(raw, nullptr, false, outv);
  if (blk >= 0) {
    __nv_bfloat16* dst = kv + (long)blk * block_stride + ((long)(nkv + kh) * PAGE + slot % PAGE) * D;
#pragma unroll
    for (int c = 0; c < PER / 8; ++c) *reinterpret_cast<uint4*>(dst + lane * 8 + 256 * c) = outv[c];
  }
}

// ---------------------------------------------------------------- residual norms
// One CTA (256 threads) per token row, H <= 8192, H % 8 == 0.
//   mode 0: x = a * in_scale                         (scaled embedding)
//   mode 1: x = (x + rmsnorm(a) * w_post) * out_scale (sandwich residual)
// then, when w_next is given, y = rmsnorm(x) * w_next from the stored bf16 x.
constexpr int kNormThreads = 256;
constexpr int kNormChunks = 4;  // 8-element chunks per thread

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) s += red[w];
  return s;
}

__global__ void __launch_bounds__(kNormThreads) residual_norm_kernel(
    const __nv_bfloat16* __restrict__ a, __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_post,
    const __nv_bfloat16* __restrict__ w_next, __nv_bfloat16* __restrict__ y, int H, float in_scale,
    float out_scale, float eps, int mode) {
  __shared__ float red[kNormThreads / 32];
  const long row = blockIdx.x;
  const int nch = H / 8;
  float av[kNormChunks][8];
  float inv_a = 1.f;
#pragma unroll
  for (int i = 0; i < kNormChunks; ++i) {
    const int c = threadIdx.x + kNormThreads * i;
    if (c < nch) {
      const uint4 u = *reinterpret_cast<const uint4*>(a + row * H + c * 8);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) av[i][k] = __bfloat162float(b[k]);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) av[i][k] = 0.f;
    }
  }
  if (mode == 1) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kNormChunks; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += av[i][k] * av[i][k];
    inv_a = rsqrtf(block_sum(ss, red) / H + eps);
  }
  float ss2 = 0.f;
#pragma unroll
  for (int i = 0; i < kNormChunks; ++i) {
    const int c = threadIdx.x + kNormThreads * i;
    if (c >= nch) continue;
    float xv[8];
    if (mode == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) xv[k] = av[i][k] * in_scale;
    } else {
      const uint4 u = *reinterpret_cast<const uint4*>(x + row * H + c * 8);
      const uint4 wu = *reinterpret_cast<const uint4*>(w_post + c * 8);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&u);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wu);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        xv[k] = (__bfloat162float(xb[k]) + av[i][k] * inv_a * __bfloat162float(wb[k])) * out_scale;
    }
    const uint4 st = make_uint4(pack_bf16x2(xv[0], xv[1]), pack_bf16x2(xv[2], xv[3]), pack_bf16x2(xv[4], xv[5]),
                                pack_bf16x2(xv[6], xv[7]));
    *reinterpret_cast<uint4*>(x + row * H + c * 8) = st;
    const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(&st);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      av[i][k] = __bfloat162float(sb[k]);  // the stored (rounded) x feeds the next norm
      ss2 += av[i][k] * av[i][k];
    }
  }
  if (w_next == nullptr) return;
  const float inv = rsqrtf(block_sum(ss2, red) / H + eps);
#pragma unroll
  for (int i = 0; i < kNormChunks; ++i) {
    const int c = threadIdx.x + kNormThreads * i;
    if (c >= nch) continue;
    const uint4 wu = *reinterpret_cast<const uint4*>(w_next + c * 8);
    const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wu);
    float yv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) yv[k] = av[i][k] * inv * __bfloat162float(wb[k]);
    *reinterpret_cast<uint4*>(y + row * H + c * 8) = make_uint4(
        pack_bf16x2(yv[0], yv[1]), pack_bf16x2(yv[2], yv[3]), pack_bf16x2(yv[4], yv[5]), pack_bf16x2(yv[6], yv[7]));
  }
}

// logits = cap * tanh(logits / cap), in place (bf16, 8 per thread)
__global__ void softcap_kernel(__nv_bfloat16* __restrict__ v, long n8, float cap) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    uint4 u = *reinterpret_cast<uint4*>(v + i * 8);
    __nv_bfloat16* b = reinterpret_cast<__nv_bfloat16*>(&u);
    float y[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) y[k] = cap * tanhf(__bfloat162float(b[k]) / cap);
    u = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
    *reinterpret_cast<uint4*>(v + i * 8) = u;
  }
}

template <int D, int ROWS, int STAGES>
void launch_wide(const WideArgs& a, dim3 grid, bool combine, cudaStream_t stream) {
  const int smem = Smem<D, ROWS, STAGES>::kTotal;
  static bool attr = false;  // first call per instantiation (host-serial launch path)
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(wide_attention_kernel<D, ROWS, STAGES>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr = true;
  }
  wide_attention_kernel<D, ROWS, STAGES><<<grid, kThreads, smem, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (combine) {
    wide_combine_kernel<D, ROWS><<<dim3(grid.x, grid.y), 256, 0, stream>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// query rows per CTA: decode rows of one KV head that fit 16 rows take the one-warp tile
inline int decode_rows(int64_t q_len, int64_t G) { return q_len * G <= 16 ? 16 : kRows; }

}  // namespace gemma

using gemma::WideArgs;

static WideArgs wide_common(const torch::Tensor& q, torch::Tensor& out, const torch::Tensor& kv_layer, int64_t nkv,
                            const torch::Tensor& block_table, int64_t window, double scale, double softcap,
                            const torch::Tensor& status) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.is_contiguous(),
              "wide attention: q [rows, nq, D] bf16 contiguous");
  TORCH_CHECK(out.sizes() == q.sizes() && out.scalar_type() == at::kBFloat16 && out.is_contiguous(),
              "wide attention: out like q");
  TORCH_CHECK(kv_layer.scalar_type() == at::kBFloat16 && kv_layer.dim() == 2 && kv_layer.stride(1) == 1,
              "wide attention: kv layer [NB, E] bf16");
  const int D = q.size(2);
  TORCH_CHECK(D == 256 || D == 384 || D == 512, "wide attention: head_dim 256, 384 or 512");
  TORCH_CHECK(q.size(1) % nkv == 0, "wide attention: q heads must be a multiple of KV heads");
  TORCH_CHECK(kv_layer.stride(0) >= 2 * nkv * gemma::PAGE * D && kv_layer.stride(0) % 8 == 0,
              "wide attention: block stride too small or not 16-byte aligned");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.stride(1) == 1, "wide attention: int32 table");
  WideArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.kv = reinterpret_cast<const __nv_bfloat16*>(kv_layer.data_ptr());
  a.block_stride = kv_layer.stride(0);
  a.nq = q.size(1);
  a.nkv = nkv;
  a.num_blocks = kv_layer.size(0);
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = block_table.stride(0);
  a.causal = 1;
  a.window = int(window);
  a.scale = float(scale);
  a.softcap = float(softcap);
  a.splits = 1;
  TORCH_CHECK(status.scalar_type() == at::kInt && status.is_cuda(), "wide attention: int32 status word");
  a.status = status.data_ptr<int>();
  return a;
}

static void launch_wide_any(const WideArgs& a, int D, int rows, dim3 grid, bool combine) {
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (rows == 16) {
    if (D == 256)
      gemma::launch_wide<256, 16, 4>(a, grid, combine, stream);
    else if (D == 384)
      gemma::launch_wide<384, 16, 4>(a, grid, combine, stream);
    else
      gemma::launch_wide<512, 16, 4>(a, grid, combine, stream);
  } else {
    if (D == 256)
      gemma::launch_wide<256, 64, 3>(a, grid, combine, stream);
    else if (D == 384)
      gemma::launch_wide<384, 64, 2>(a, grid, combine, stream);
    else
      gemma::launch_wide<512, 64, 2>(a, grid, combine, stream);
  }
}

int64_t wide_decode_splits(int64_t batch, int64_t nq, int64_t nkv, int64_t head_dim, int64_t q_len,
                           int64_t max_kv_len, int64_t window, int64_t num_sms) {
  const int64_t G = nq / nkv;
  const int rows = gemma::decode_rows(q_len, G);
  const int64_t ctas = batch * nkv * ((q_len * G + rows - 1) / rows) * (head_dim / gemma::kDC);
  int64_t keys = window > 0 ? std::min<int64_t>(window + q_len, max_kv_len) : max_kv_len;
  const int64_t tiles = std::max<int64_t>(1, (keys + gemma::kKeys - 1) / gemma::kKeys + 1);
  int64_t s = (2 * num_sms + ctas - 1) / std::max<int64_t>(ctas, 1);
  s = std::min<int64_t>({s, tiles, gemma::kMaxSplits});
  return std::max<int64_t>(s, 1);
}

int64_t wide_decode_workspace_numel(int64_t batch, int64_t nq, int64_t nkv, int64_t head_dim, int64_t q_len,
                                    int64_t splits) {
  const int64_t G = nq / nkv;
  const int rows = gemma::decode_rows(q_len, G);
  const int64_t gy = nkv * ((q_len * G + rows - 1) / rows) * (head_dim / gemma::kDC);
  return splits > 1 ? batch * gy * splits * rows * (gemma::kDC + 2) : 1;
}

void wide_decode_attention(const torch::Tensor& q, torch::Tensor& out, const torch::Tensor& kv_layer, int64_t nkv,
                           const torch::Tensor& block_table, const torch::Tensor& seq_lens, int64_t q_len,
                           int64_t window, double scale, double softcap, int64_t splits,
                           const c10::optional<torch::Tensor>& workspace, const torch::Tensor& status) {
  WideArgs a = wide_common(q, out, kv_layer, nkv, block_table, window, scale, softcap, status);
  const int D = q.size(2);
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt, "wide decode: seq_lens int32");
  const int B = seq_lens.size(0);
  TORCH_CHECK(q.size(0) == (int64_t)B * q_len && q_len >= 1 && q_len <= 16, "wide decode: q rows = B * q_len");
  TORCH_CHECK(block_table.size(0) >= B, "wide decode: block table rows");
  if (B == 0) return;
  TORCH_CHECK(splits >= 1 && splits <= gemma::kMaxSplits, "wide decode: splits in [1, 16]");
  a.seq_lens = seq_lens.data_ptr<int>();
  a.ql = int(q_len);
  a.prefill = 0;
  a.splits = int(splits);
  const int G = a.nq / a.nkv;
  const int rows = gemma::decode_rows(a.ql, G);
  const int gy = a.nkv * ((a.ql * G + rows - 1) / rows) * (D / gemma::kDC);
  if (splits > 1) {
    TORCH_CHECK(workspace.has_value() && workspace->scalar_type() == at::kFloat &&
                    workspace->numel() >= wide_decode_workspace_numel(B, a.nq, a.nkv, D, q_len, splits),
                "wide decode: workspace too small for the splits");
    a.part = workspace->data_ptr<float>();
  }
  const at::cuda::CUDAGuard g(q.device());
  launch_wide_any(a, D, rows, dim3(B, gy, int(splits)), splits > 1);
}

void wide_prefill_attention(const torch::Tensor& q, torch::Tensor& out, const torch::Tensor& kv_layer, int64_t nkv,
                            const torch::Tensor& block_table, const torch::Tensor& ctx_lens,
                            const torch::Tensor& cu_q, const torch::Tensor& tile_seq,
                            const torch::Tensor& tile_start, int64_t window, double scale, double softcap,
                            const torch::Tensor& status, bool causal) {
  WideArgs a = wide_common(q, out, kv_layer, nkv, block_table, window, scale, softcap, status);
  a.causal = causal ? 1 : 0;
  const int D = q.size(2);
  TORCH_CHECK(ctx_lens.scalar_type() == at::kInt && cu_q.scalar_type() == at::kInt &&
                  tile_seq.scalar_type() == at::kInt && tile_start.scalar_type() == at::kInt,
              "wide prefill: int32 metadata");
  const int NT = tile_seq.size(0);
  if (NT == 0 || q.size(0) == 0) return;
  a.cu_q = cu_q.data_ptr<int>();
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.tile_seq = tile_seq.data_ptr<int>();
  a.tile_start = tile_start.data_ptr<int>();
  a.prefill = 1;
  const at::cuda::CUDAGuard g(q.device());
  // 128-row scheduler tiles run as two 64-row halves (an empty half exits at once)
  launch_wide_any(a, D, gemma::kRows, dim3(NT, a.nq * (D / gemma::kDC), 2), false);
}

void gemma_qkv_write(const torch::Tensor& qkv, const torch::Tensor& positions, const torch::Tensor& slots,
                     const torch::Tensor& cos_sin, torch::Tensor& q_out, torch::Tensor& kv_layer, int64_t nq,
                     int64_t nkv, int64_t rot, const torch::Tensor& q_w, const torch::Tensor& k_w, double eps,
                     bool k_eq_v, const torch::Tensor& status) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1, "gemma qkv: [T, cols] bf16");
  TORCH_CHECK(q_out.scalar_type() == at::kBFloat16 && q_out.dim() == 3 && q_out.is_contiguous(),
              "gemma qkv: q_out [T, nq, D]");
  const int D = q_out.size(2);
  TORCH_CHECK(D == 256 || D == 512, "gemma qkv: head_dim 256 or 512");
  const int T = qkv.size(0);
  TORCH_CHECK(qkv.size(1) >= (nq + (k_eq_v ? 1 : 2) * nkv) * D && qkv.stride(0) % 8 == 0, "gemma qkv: columns");
  TORCH_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kInt, "gemma qkv: int64 / int32");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.dim() == 2 && cos_sin.size(1) == rot && rot % 2 == 0 &&
                  rot <= D,
              "gemma qkv: cos_sin [max_pos, rot] f32");
  TORCH_CHECK(q_w.numel() == D && k_w.numel() == D, "gemma qkv: q/k norm weights [D]");
  TORCH_CHECK(kv_layer.scalar_type() == at::kBFloat16 && kv_layer.stride(1) == 1 &&
                  kv_layer.stride(0) >= 2 * nkv * gemma::PAGE * D,
              "gemma qkv: kv layer [NB, E]");
  if (T == 0) return;
  const at::cuda::CUDAGuard g(qkv.device());
  const long items = (long)T * (nq + nkv);
  const int blocks = int((items + 7) / 8);
  auto st = at::cuda::getCurrentCUDAStream();
#define BLOOM_GEMMA_QKV(DD)                                                                                        \
  gemma::qkv_write_kernel<DD><<<blocks, 256, 0, st>>>(                                                             \
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), T, int(nq), int(nkv), int(rot),      \
      positions.data_ptr<int64_t>(), slots.data_ptr<int>(), cos_sin.data_ptr<float>(), int(cos_sin.size(0)),      \
      reinterpret_cast<const __nv_bfloat16*>(q_w.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k_w.data_ptr()), \
      float(eps), k_eq_v ? 1 : 0, reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),                              \
      reinterpret_cast<__nv_bfloat16*>(kv_layer.data_ptr()), kv_layer.stride(0), int(kv_layer.size(0)),             \
      status.data_ptr<int>())
  if (D == 256)
    BLOOM_GEMMA_QKV(256);
  else
    BLOOM_GEMMA_QKV(512);
#undef BLOOM_GEMMA_QKV
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void residual_norm(const torch::Tensor& a, torch::Tensor& x, const c10::optional<torch::Tensor>& w_post,
                   const c10::optional<torch::Tensor>& w_next, const c10::optional<torch::Tensor>& y,
                   double in_scale, double out_scale, double eps) {
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16 && a.is_contiguous() &&
                  x.is_contiguous() && a.sizes() == x.sizes() && a.dim() == 2,
              "residual_norm: a, x [T, H] bf16 contiguous");
  const int T = a.size(0), H = a.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * gemma::kNormThreads * gemma::kNormChunks, "residual_norm: H % 8 == 0, <= 8192");
  TORCH_CHECK(!w_post.has_value() || w_post->numel() == H, "residual_norm: w_post [H]");
  TORCH_CHECK(w_next.has_value() == y.has_value(), "residual_norm: w_next and y go together");
  if (y.has_value()) TORCH_CHECK(y->sizes() == a.sizes() && y->is_contiguous(), "residual_norm: y like a");
  if (T == 0) return;
  const at::cuda::CUDAGuard g(a.device());
  gemma::residual_norm_kernel<<<T, gemma::kNormThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), reinterpret_cast<__nv_bfloat16*>(x.data_ptr()),
      w_post.has_value() ? reinterpret_cast<const __nv_bfloat16*>(w_post->data_ptr()) : nullptr,
      w_next.has_value() ? reinterpret_cast<const __nv_bfloat16*>(w_next->data_ptr()) : nullptr,
      y.has_value() ? reinterpret_cast<__nv_bfloat16*>(y->data_ptr()) : nullptr, H, float(in_scale),
      float(out_scale), float(eps), w_post.has_value() ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void softcap_(torch::Tensor& v, double cap) {
  TORCH_CHECK(v.scalar_type() == at::kBFloat16 && v.is_contiguous() && v.numel() % 8 == 0,
              "softcap_: contiguous bf16, numel % 8 == 0");
  TORCH_CHECK(cap > 0, "softcap_: cap > 0");
  const long n8 = v.numel() / 8;
  if (n8 == 0) return;
  const at::cuda::CUDAGuard g(v.device());
  const int blocks = int(std::min<long>((n8 + 255) / 256, 148L * 8));
  gemma::softcap_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(v.data_ptr()), n8, float(cap));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
