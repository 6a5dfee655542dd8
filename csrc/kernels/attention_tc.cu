// Paged prefill attention on the 5th-generation tensor cores (tcgen05).
//
// One CTA = 128 query rows of one q head (a 128-row prefill tile); KV in
// 128-token tiles (8 pages) double-buffered through TMA.  Per KV tile:
//   S = Q K^T      tcgen05.mma M=128 N=128 K=128, S accumulates in TMEM
//   softmax        4 warps, thread t owns query row t: tcgen05.ld its S row,
//                  online max / sum in the log2 domain, P = exp2(S - m) as bf16
//                  into shared memory (the K-major A operand of the next MMA)
//   O += P V       tcgen05.mma M=128 N=128 K=128, O stays in TMEM; V is read
//                  as an MN-major B operand straight from the TMA tile
// The running max is lazy (FlashAttention-4 style): O and the row sum are
// rescaled only when a row's max grows by more than 8 (a factor 256 in the
// exp2 domain, safe in fp32), so TMEM read-modify-writes of O are rare.
//
// Shared memory layout of a K or V tile: two 16 KB regions (head dims 0-63 and
// 64-127) of 128 token rows x 128 bytes with the 128-byte swizzle; page p of
// the tile lands at rows 16p..16p+15 (one 2 KB TMA box per region), so token
// rows are uniformly 128 bytes apart across pages.
//
// S is double-buffered in TMEM and K and V have separate TMA rings, so the
// tensor cores compute S(j+1) = Q K(j+1)^T while the softmax warps work on
// tile j, and P(j) V(j) runs while the next softmax starts.
// Warp roles: warps 0-7 softmax and epilogue, two threads per query row
// (warps w and w+4 read the same TMEM lanes, columns 0-63 and 64-127; the row
// max and sum are combined through shared memory); warp 8 is the TMA producer
// and TMEM owner; warp 9 issues the MMAs.  Every wait is bounded (status bit +
// return).  Reference behaviour: causal GQA attention over the paged cache
// (scheduler/paged_cache.rs:565-748).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "bloom/common.cuh"
#include "bloom/ops.h"
#include "bloom/tma_host.h"

namespace bloom {
namespace attn_tc {

constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int kRows = 128;                 // query rows per CTA
constexpr int kKv = 128;                   // kv tokens per tile
constexpr int kRegion = kKv * 64 * 2;      // 16 KB: one 64-dim half of a K or V tile
constexpr int kQBytes = kRows * D * 2;     // 32 KB
constexpr int kPBytes = kRows * kKv * 2;   // 32 KB
constexpr int kTileBytes = 2 * kRegion;    // one K or V tile = 32 KB
constexpr int kStages = 2;                 // separate K and V rings of kStages tiles each
constexpr int kSoftmaxThreads = 256;      // two threads per query row (64 columns each)
constexpr int kThreads = kSoftmaxThreads + 64;  // + TMA producer warp + MMA warp
constexpr int kSmem = kQBytes + kPBytes + 2 * kStages * kTileBytes + 256 + 1024;
constexpr int kTmemCols = 512;             // S0 [0,128), S1 [128,256), O [256,384)
constexpr float kLazy = 8.f;               // rescale threshold (log2 units)

struct Args {
  const __nv_bfloat16* q;  // [T, nq, 128]
  __nv_bfloat16* out;      // [T, nq, 128]
  const int* block_table;
  int bt_stride;
  const int* ctx_lens;
  const int* cu_q;
  const int* tile_seq;
  const int* tile_start;   // first query row of a 128-row tile (local to the sequence)
  int nq, nkv;
  float scale_log2;
  int causal;
  int* status;
  int num_blocks;          // pages in the cache (index checks only)
  // optional per-CTA profile (CTA = blockIdx.y * gridDim.x + blockIdx.x, 16
  // words each, CTAs past trace_ctas skipped): [0] %globaltimer at entry,
  // [1] at exit, [2] clock64 cycles of the kv loop, [3..9] cycles of thread 0
  // per loop phase summed over kv tiles: S(j+1) issue incl. its K wait, first
  // barrier, S(j) wait, S load + row max, P V(j-1) wait, exp + P store +
  // barrier, P-ready signal; [10] kv tiles; MMA warp: [11] / [12] cycles
  // waiting for K / V tiles, [13] for Q and P, [14] for a free S buffer
  unsigned long long* trace;
  int trace_ctas;
};

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// MN-major operand (the contiguous dimension is N): 64-element atoms of 8 K-rows.
// lbo = byte stride between 64-element atoms along N, sbo = between 8-row groups along K.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}
__host__ __device__ constexpr uint32_t idesc_bf16_bmn(int M, int N) { return umma_idesc_bf16(M, N) | (1u << 16); }

__device__ __forceinline__ void named_sync_softmax() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// named barrier that also reports whether any softmax thread passed `pred`
__device__ __forceinline__ bool named_sync_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, 1, 256, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred))
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmKV, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sP = smem + kQBytes;
  uint8_t* sK = sP + kPBytes;                       // K ring
  uint8_t* sV = sK + kStages * kTileBytes;          // V ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages * kTileBytes);
  uint64_t* fullK = bars;           // [kStages]
  uint64_t* emptyK = bars + 2;
  uint64_t* fullV = bars + 4;
  uint64_t* emptyV = bars + 6;
  uint64_t* s_done = bars + 8;      // [2]: one per S buffer
  uint64_t* o_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint64_t* s_free = bars + 12;     // [2]: the softmax has read S buffer b (one arrival per softmax warp)
  uint64_t* p_ready = bars + 14;    // P of the current tile is in shared memory, O rescaled
  uint64_t* q_ready = bars + 15;    // the Q tile is in shared memory
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tile = blockIdx.x, h = blockIdx.y;
  const long cta = (long)blockIdx.y * gridDim.x + blockIdx.x;
  unsigned long long* tr = (a.trace != nullptr && cta < a.trace_ctas) ? a.trace + cta * 16 : nullptr;
  if (tr != nullptr && threadIdx.x == 0) tr[0] = globaltimer_ns();
  const int warp = warp_id(), lane = lane_id();
  const int G = a.nq / a.nkv;
  const int kh = h / G;
  const int s_idx = a.tile_seq[tile];
  const int row0 = a.tile_start[tile];
  const int q_begin = a.cu_q[s_idx];
  const int q_len = a.cu_q[s_idx + 1] - q_begin;
  const int ctx = a.ctx_lens[s_idx];
  const int* bt = a.block_table + (long)s_idx * a.bt_stride;
  const int n_pages = (ctx + PAGE - 1) / PAGE;
  const int last_row = min(row0 + kRows, q_len) - 1;
  const int kv_end = a.causal ? min(ctx, ctx - q_len + last_row + 1) : ctx;
  const int n_kt = (kv_end + kKv - 1) / kKv;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&fullK[s], 1);
      mbar_init(&emptyK[s], 1);
      mbar_init(&fullV[s], 1);
      mbar_init(&emptyV[s], 1);
    }
    mbar_init(&s_done[0], 1);
    mbar_init(&s_done[1], 1);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    mbar_init(&s_free[0], kSoftmaxThreads / 32);
    mbar_init(&s_free[1], kSoftmaxThreads / 32);
    mbar_init(p_ready, 1);
    mbar_init(q_ready, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tO = tmem_base + 256;  // S buffers at tmem_base + 128 * (j % 2)

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      bool ok = true;
      int issuedK = 0, issuedV = 0;
      // Block ids of a kv tile's 8 pages: independent loads issued together
      // (one memory latency per tile, not one per page); the next K tile's
      // ids are fetched right after its predecessor's copies are issued, so
      // their latency hides behind the ring waits.
      auto fetch_ids = [&](int jt, int (&ids)[kKv / PAGE]) {
#pragma unroll
        for (int pg = 0; pg < kKv / PAGE; ++pg) {
          const int page = jt * (kKv / PAGE) + pg;
          ids[pg] = __ldg(bt + (page < n_pages ? page : 0));
          if (!kcheck(ids[pg] >= 0 && ids[pg] < a.num_blocks, a.status)) ids[pg] = 0;
        }
      };
      auto load_tile = [&](const int (&ids)[kKv / PAGE], uint8_t* dst, uint64_t* bar, int kv) {
        mbar_arrive_expect_tx(bar, kTileBytes);
#pragma unroll
        for (int pg = 0; pg < kKv / PAGE; ++pg) {
          const int row = ((ids[pg] * 2 + kv) * a.nkv + kh) * PAGE;
          tma_load_2d(dst + pg * 2048, &tmKV, bar, 0, row);
          tma_load_2d(dst + kRegion + pg * 2048, &tmKV, bar, 64, row);
        }
      };
      int idsK[kKv / PAGE], idsV[kKv / PAGE];
      if (n_kt > 0) fetch_ids(0, idsK);
      // K and V rings advance independently: a K tile is requested as soon as
      // its slot is free (S of the tile two back done), without queueing
      // behind the V tile whose slot waits for an older P V; V never runs
      // ahead of K.  Bounded: no progress for kLocalWaitTimeoutNs -> error.
      uint64_t t_prog = globaltimer_ns();
      uint32_t spins = 0;
      while (ok && (issuedK < n_kt || issuedV < n_kt)) {
        bool progressed = false;
        if (issuedK < n_kt) {
          const int s = issuedK % kStages;
          if (mbar_try_wait(&emptyK[s], ((issuedK / kStages) & 1) ^ 1u)) {
            load_tile(idsK, sK + s * kTileBytes, &fullK[s], 0);
            ++issuedK;
            if (issuedK < n_kt) fetch_ids(issuedK, idsK);
            progressed = true;
          }
        }
        if (issuedV < issuedK) {
          const int s = issuedV % kStages;
          if (mbar_try_wait(&emptyV[s], ((issuedV / kStages) & 1) ^ 1u)) {
            fetch_ids(issuedV, idsV);  // the K tile of the same index read these ids: cache hits
            load_tile(idsV, sV + s * kTileBytes, &fullV[s], 1);
            ++issuedV;
            progressed = true;
          }
        }
        if (progressed) {
          t_prog = globaltimer_ns();
        } else if ((++spins & 31u) == 0) {
          if (*abort_flag) {
            ok = false;
          } else if (globaltimer_ns() - t_prog > kLocalWaitTimeoutNs) {
            *abort_flag = 1;
            atomicOr(a.status, kStatusAttnTimeout);
            ok = false;
          }
        }
      }
      if (!ok) {  // wait (bounded) for the loads already in flight before leaving
        for (int jt = max(0, issuedK - kStages); jt < issuedK; ++jt)
          mbar_drain(&fullK[jt % kStages], (jt / kStages) & 1);
        for (int jt = max(0, issuedV - kStages); jt < issuedV; ++jt)
          mbar_drain(&fullV[jt % kStages], (jt / kStages) & 1);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    // One thread issues every tcgen05.mma: S(j+1) = Q K(j+1)^T goes into the
    // free S buffer while the softmax of tile j runs, then O += P(j) V(j)
    // once the softmax has written P(j).  An MMA issue blocks its thread while
    // the tensor pipe drains its queue, so it lives in its own warp: the
    // softmax warps never wait on it.
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc_bf16(128, kKv);
      constexpr uint32_t idO = idesc_bf16_bmn(128, D);
      bool ok = true, issued_any = false;
      long long wK = 0, wV = 0, wP = 0, wF = 0;
      auto timed_wait = [&](uint64_t* bar, uint32_t par, long long& acc) -> bool {
        const long long tw = tr != nullptr ? clock64() : 0;
        const bool r = mbar_wait(bar, par, abort_flag, a.status, kStatusAttnTimeout);
        if (tr != nullptr) acc += clock64() - tw;
        return r;
      };
      auto issue_s = [&](int jt) -> bool {
        if (jt >= 2 && !timed_wait(&s_free[jt & 1], ((jt >> 1) - 1) & 1, wF)) return false;
        const int sk = jt % kStages;
        if (!timed_wait(&fullK[sk], (jt / kStages) & 1, wK)) return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(sK + sk * kTileBytes);
        const uint32_t qb = smem_u32(sQ);
        const uint32_t tS = tmem_base + 128u * static_cast<uint32_t>(jt & 1);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(qb + (kk >> 2) * (kRows * 128)) + 2 * (kk & 3);
          const uint64_t bd = umma_desc_sw128(kb + (kk >> 2) * kRegion) + 2 * (kk & 3);
          umma_f16(tS, ad, bd, idS, kk > 0 ? 1u : 0u);
        }
        issued_any = true;
        umma_commit(&s_done[jt & 1]);
        umma_commit(&emptyK[sk]);
        return true;
      };
      if (n_kt > 0) ok = timed_wait(q_ready, 0, wP) && issue_s(0);
      for (int j = 0; j < n_kt && ok; ++j) {
        if (j + 1 < n_kt && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        const int sv_ = j % kStages;
        if (!timed_wait(p_ready, j & 1, wP) || !timed_wait(&fullV[sv_], (j / kStages) & 1, wV)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t pb = smem_u32(sP);
        const uint32_t vb = smem_u32(sV + sv_ * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kKv / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(pb + (kk >> 2) * (kRows * 128)) + 2 * (kk & 3);
          const uint64_t bd = umma_desc_sw128_mn(vb + kk * 16 * 128, kRegion, 1024);
          umma_f16(tO, ad, bd, idO, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(o_done);
        umma_commit(&emptyV[sv_]);
      }
      if (!ok && issued_any) {  // let the tensor pipe finish what was issued before TMEM is freed
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
      if (tr != nullptr) {
        tr[11] = static_cast<unsigned long long>(wK);
        tr[12] = static_cast<unsigned long long>(wV);
        tr[13] = static_cast<unsigned long long>(wP);
        tr[14] = static_cast<unsigned long long>(wF);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax warps
    __shared__ float red_m[kSoftmaxThreads], red_l[kSoftmaxThreads];
    const int t = threadIdx.x & (kRows - 1);  // query row of the tile, = TMEM lane
    const int half = threadIdx.x >> 7;        // columns [64 * half, 64 * half + 64)
    const int cb = half * 64;
    const int lr = row0 + t;
    const bool valid = lr < q_len;
    // rows past the chunk keep a finite softmax (no masking) and are not stored
    const int qpos = valid ? (a.causal ? ctx - q_len + lr : ctx - 1) : ctx - 1;
    {  // this thread's half of the Q row -> shared memory, K-major SW128 (region = half)
      const uint4* src = reinterpret_cast<const uint4*>(a.q + ((long)(q_begin + (valid ? lr : 0)) * a.nq + h) * D);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = valid ? src[half * 8 + c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(sQ + half * (kRows * 128) + t * 128 + ((c ^ (t & 7)) << 4)) = v;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    named_sync_softmax();
    if (threadIdx.x == 0) mbar_arrive(q_ready);
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool failed = false;
    int j = 0;
    long long ph[7] = {0, 0, 0, 0, 0, 0, 0};
    long long tprev = clock64();
    const long long tloop = tprev;
    auto lap = [&](int k) {  // thread 0's time in phase k since the previous lap
      if (tr != nullptr && threadIdx.x == 0) {
        const long long t1 = clock64();
        ph[k] += t1 - tprev;
        tprev = t1;
      }
    };
    for (; j < n_kt; ++j) {
      lap(0);
      if (named_sync_or(failed)) {
        failed = true;
        break;
      }
      lap(1);
      if (!mbar_wait(&s_done[j & 1], (j >> 1) & 1, abort_flag, a.status, kStatusAttnTimeout)) failed = true;
      if (named_sync_or(failed)) {
        failed = true;
        break;
      }
      lap(2);
      tc_fence_after();
      // ---- this thread's 64 columns of its row
      float sv[64];
      const uint32_t sbase = tmem_base + 128u * static_cast<uint32_t>(j & 1) + lane_off + cb;
#pragma unroll
      for (int c = 0; c < 64; c += 16) {
        float v16[16];
        tmem_ld_32x32b_x16(sbase + c, v16);
        tmem_wait_ld();  // registers are valid only after the wait
#pragma unroll
        for (int q = 0; q < 16; ++q) sv[c + q] = v16[q];
      }
      tc_fence_before();  // S(j) is in registers: its TMEM buffer may take S(j + 2)
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[j & 1]);
      const int kv0 = j * kKv + cb;
      float mx = -INFINITY;
      if (kv0 + 63 <= qpos && kv0 + 63 < ctx) {  // the whole half is visible: no masking
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          sv[c] *= a.scale_log2;
          mx = fmaxf(mx, sv[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int idx = kv0 + c;
          float v = sv[c] * a.scale_log2;
          if (idx > qpos || idx >= ctx) v = -INFINITY;
          sv[c] = v;
          mx = fmaxf(mx, v);
        }
      }
      red_m[threadIdx.x] = mx;
      lap(3);
      // the previous P V must be done before P is rewritten and before O is rescaled
      if (j > 0 && !mbar_wait(o_done, (j - 1) & 1, abort_flag, a.status, kStatusAttnTimeout)) failed = true;
      if (named_sync_or(failed)) {
        failed = true;
        break;
      }
      lap(4);
      tc_fence_after();
      mx = fmaxf(mx, red_m[threadIdx.x ^ 128]);  // the row max over both halves
      const float m_new = fmaxf(m, mx);
      const bool grow = (m_new > m + kLazy) || j == 0;  // identical in both threads of a row
      const float alpha = (grow && j > 0) ? exp2f(m - m_new) : 1.f;
      if (__any_sync(0xffffffffu, grow && j > 0)) {  // warp-collective TMEM read-modify-write of O
#pragma unroll 1
        for (int c = 0; c < 64; c += 16) {
          float o16[16];
          tmem_ld_32x32b_x16(tO + lane_off + cb + c, o16);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 16; ++q) o16[q] *= alpha;
          tmem_st_32x32b_x16(tO + lane_off + cb + c, o16);
        }
        tmem_wait_st();
      }
      if (grow) {
        l *= alpha;
        m = m_new;
      }
      float ps = 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        float p8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          p8[q] = exp2f(sv[c + q] - m);
          ps += p8[q];
        }
        uint4 pk;
        pk.x = pack_bf16x2(p8[0], p8[1]);
        pk.y = pack_bf16x2(p8[2], p8[3]);
        pk.z = pack_bf16x2(p8[4], p8[5]);
        pk.w = pack_bf16x2(p8[6], p8[7]);
        const int chunk = c >> 3;
        *reinterpret_cast<uint4*>(sP + half * (kRows * 128) + t * 128 + ((chunk ^ (t & 7)) << 4)) = pk;
      }
      l += ps;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      named_sync_softmax();
      lap(5);
      // ---- the MMA warp may run O += P V
      if (threadIdx.x == 0) mbar_arrive(p_ready);
      lap(6);
    }
    if (tr != nullptr && threadIdx.x == 0) {
      tr[2] = static_cast<unsigned long long>(clock64() - tloop);
      for (int k = 0; k < 7; ++k) tr[3 + k] = static_cast<unsigned long long>(ph[k]);
      tr[10] = static_cast<unsigned long long>(n_kt);
    }
    if (!failed && n_kt > 0) {
      if (!mbar_wait(o_done, (n_kt - 1) & 1, abort_flag, a.status, kStatusAttnTimeout)) failed = true;
    }
    red_l[threadIdx.x] = l;
    if (named_sync_or(failed)) failed = true;
    if (!failed && n_kt > 0) {
      tc_fence_after();
      const float lt = l + red_l[threadIdx.x ^ 128];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      __nv_bfloat16* orow = a.out + ((long)(q_begin + (valid ? lr : 0)) * a.nq + h) * D + cb;
#pragma unroll 1
      for (int c = 0; c < 64; c += 16) {
        float o16[16];
        tmem_ld_32x32b_x16(tO + lane_off + cb + c, o16);
        tmem_wait_ld();
        if (valid) {
          uint4 w0, w1;
          w0.x = pack_bf16x2(o16[0] * inv, o16[1] * inv);
          w0.y = pack_bf16x2(o16[2] * inv, o16[3] * inv);
          w0.z = pack_bf16x2(o16[4] * inv, o16[5] * inv);
          w0.w = pack_bf16x2(o16[6] * inv, o16[7] * inv);
          w1.x = pack_bf16x2(o16[8] * inv, o16[9] * inv);
          w1.y = pack_bf16x2(o16[10] * inv, o16[11] * inv);
          w1.z = pack_bf16x2(o16[12] * inv, o16[13] * inv);
          w1.w = pack_bf16x2(o16[14] * inv, o16[15] * inv);
          *reinterpret_cast<uint4*>(orow + c) = w0;
          *reinterpret_cast<uint4*>(orow + c + 8) = w1;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (tr != nullptr && threadIdx.x == 0) tr[1] = globaltimer_ns();
}

}  // namespace attn_tc

// Per-CTA profile buffer of the next prefill launches (see Args::trace).
static unsigned long long* g_attn_tc_trace = nullptr;
static int g_attn_tc_trace_ctas = 0;

void attn_tc_set_trace(const c10::optional<torch::Tensor>& buf) {
  if (buf.has_value() && buf->defined()) {
    TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong, "attn trace: int64 CUDA tensor");
    g_attn_tc_trace = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
    g_attn_tc_trace_ctas = static_cast<int>(buf->numel() / 16);
  } else {
    g_attn_tc_trace = nullptr;
    g_attn_tc_trace_ctas = 0;
  }
}

void paged_prefill_attention_tc(const torch::Tensor& q, const torch::Tensor& kv_cache, int64_t layer,
                                const torch::Tensor& block_table, const torch::Tensor& ctx_lens,
                                const torch::Tensor& cu_seqlens_q, const torch::Tensor& tile_seq,
                                const torch::Tensor& tile_start, torch::Tensor& out, double scale, bool causal,
                                const torch::Tensor& status) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.size(-1) == attn_tc::D,
              "prefill_tc: q [T, nq, 128] bf16");
  TORCH_CHECK(kv_cache.dim() == 6 && kv_cache.size(5) == attn_tc::D && kv_cache.size(4) == attn_tc::PAGE &&
                  kv_cache.is_contiguous(),
              "prefill_tc: kv_cache [L, NB, 2, KVH, 16, 128]");
  const int n_tiles = tile_seq.size(0);
  if (n_tiles == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  attn_tc::Args a;
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
  a.trace = g_attn_tc_trace;
  a.trace_ctas = g_attn_tc_trace_ctas;
  const uint64_t rows = (uint64_t)kv_cache.size(1) * 2 * kv_cache.size(3) * attn_tc::PAGE;
  TORCH_CHECK(rows < (1ull << 31), "prefill_tc: kv_cache too many rows per layer for int32 TMA coordinates");
  const auto* base = reinterpret_cast<const __nv_bfloat16*>(kv_cache.data_ptr()) + layer * kv_cache.stride(0);
  const CUtensorMap tm = make_tmap_bf16_2d(base, attn_tc::D, rows, attn_tc::D * 2, 64, attn_tc::PAGE);
  static uint64_t configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((configured >> dev) & 1u)) {
    cudaFuncSetAttribute(attn_tc::prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_tc::kSmem);
    configured |= uint64_t(1) << dev;
  }
  attn_tc::prefill_tc_kernel<<<dim3(n_tiles, a.nq), attn_tc::kThreads, attn_tc::kSmem, stream>>>(tm, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bloom
