// Device-side building blocks shared by every sm_100a kernel in bloom_b200:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (UMMA + TMEM) wrappers,
// and the status word that kernels use to report a timed-out wait instead of
// hanging the GPU.
//
// Every wait in this file is bounded by a %globaltimer budget.  A wait that
// runs out sets a bit in the caller's status word and returns false; callers
// then stop issuing work, drain what they already issued (again bounded) and
// return, so the CUDA context stays usable and the host can read the status.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace bloom {

// Status bits written by kernels (host reads them through bloom_b200.ops.status()).
enum StatusBits : int {
  kStatusGemmTimeout = 1 << 0,
  kStatusAttnTimeout = 1 << 1,
  kStatusCommTimeout = 1 << 2,
  kStatusBadArgument = 1 << 3,
  kStatusMoeOverflow = 1 << 4,
  // a fused collective found its communicator poisoned by an earlier timeout
  // and did nothing (the host must fail the step and stop using it)
  kStatusCommPoisoned = 1 << 5,
  // an index read from a table (block id, cache slot, token id, expert row)
  // was out of range; only builds with -DBLOOM_KERNEL_CHECKS look
  kStatusIndexCheck = 1 << 6,
};

// Index checks compiled in by -DBLOOM_KERNEL_CHECKS (the bloom_b200._C_checked
// extension): kcheck(ok, status) records a failed check in the status word
// and returns ok, so the caller skips the access.  In the regular build it is
// the constant true and costs nothing.
#ifdef BLOOM_KERNEL_CHECKS
__device__ __forceinline__ bool kcheck(bool ok, int* status) {
  if (!ok && status != nullptr) atomicOr(status, kStatusIndexCheck);
  return ok;
}
#else
__device__ __forceinline__ constexpr bool kcheck(bool, int*) { return true; }
#endif

// Words of a rank's tensor-parallel flag block (bloom_b200.parallel.fused)
// that kernels outside comm.cu also touch: the poison word, and the counter
// and expectation of a deferred all-gather (see wait_deferred_rows).
constexpr int kFlagPoison = 18, kFlagDoneCount = 19, kFlagDoneExpect = 20;

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Consumer side of a deferred all-gather: a tensor-parallel collective that
// does not wait for its peers' rows leaves that wait to the kernel that reads
// them.  Every block of every rank adds 1 to this rank's done counter after
// its rows are stored here; the collective also raised the expectation by its
// number of blocks x ranks.  Waits (bounded) until the counter reaches the
// expectation (wrap-around safe).  A timeout poisons the communicator and
// sets kStatusCommTimeout; the caller goes on (the step is failed by the host).
__device__ __forceinline__ bool wait_deferred_rows(uint32_t* flags, uint64_t timeout_ns, int* status);

// Byte position of element i in an int8 KV page row stored in MMA fragment
// order: within each group of 16 the elements (2t, 2t+1, 2t+8, 2t+9) of
// thread-in-quad t are the four bytes at 4t (K rows: i = head dim; V rows,
// which are dim-major: i = token).
__host__ __device__ __forceinline__ int q8_perm16(int i) {
  return (i & ~15) | (((i & 7) >> 1) << 2) | (((i >> 3) & 1) << 1) | (i & 1);
}

// Local (same-GPU) pipeline waits never legitimately take this long.
constexpr uint64_t kLocalWaitTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  `abort` is a
// CTA-shared flag: once any role of the CTA gave up, the others stop waiting
// too.  On timeout the status bit is OR-ed into *status and false returned.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                          int status_bit, uint64_t timeout_ns = kLocalWaitTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0) {
      if (abort != nullptr && *abort) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (abort != nullptr) *abort = 1;
        if (status != nullptr) atomicOr(status, status_bit);
        return false;
      }
    }
  }
}

// Drain-only wait used on the abort path: no status update, short budget.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kLocalWaitTimeoutNs) return;
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// 2D tiled load, no multicast (multicast is never used in this code base:
// every kernel may run inside a multi-GPU process).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tm, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* tm, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 1D bulk copy global -> shared (addresses and size 16-byte aligned).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16/f16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05 op of this thread completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns: thread t gets lane (base_lane + t).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major operand tile stored as rows of
// 128 bytes with the 128-byte swizzle (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B and a 64 x bf16 inner box).  8-row groups are
// 1024 bytes apart; the tile base must be 1024-byte aligned.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);   // start address
  d |= static_cast<uint64_t>(1u) << 16;                      // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;                      // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                      // swizzle mode: 128B
  return d;
}

// Instruction descriptor: kind::f16, A=B=bf16, D=f32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4)                                  // D format f32
         | (1u << 7)                                // A bf16
         | (1u << 10)                               // B bf16
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// ---------------------------------------------------------------- misc math
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while the previous kernel of the
// stream is still running; griddep_wait() blocks until that kernel has
// completed and its memory is visible, so everything before it may only touch
// memory the previous kernel neither writes nor reads (weights).
// griddep_launch_dependents() lets the next such kernel start early.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ bool wait_deferred_rows(uint32_t* flags, uint64_t timeout_ns, int* status) {
  if (flags == nullptr) return true;
  volatile uint32_t* vf = flags;
  if (vf[kFlagPoison] != 0u) return true;  // the step fails anyway; do not wait
  const uint32_t expect = vf[kFlagDoneExpect];
  const uint64_t t0 = globaltimer_ns();
  while (static_cast<int>(ld_acquire_sys_u32(flags + kFlagDoneCount) - expect) < 0) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      vf[kFlagPoison] = 1u;
      __threadfence();
      atomicOr(status, kStatusCommTimeout);
      return false;
    }
  }
  return true;
}

}  // namespace bloom
