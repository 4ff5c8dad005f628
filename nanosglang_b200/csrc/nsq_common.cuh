// Shared device helpers for libnsq: mbarriers with bounded waits, TMA,
// tcgen05 (TMEM / UMMA), warp-level mma.sync, cluster DSMEM and the packed
// int4 / fp8 unpack primitives. sm_100a only.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/nsq.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "libnsq is written for sm_100a only"
#endif

namespace nsq {

// Device-side status word. A kernel whose bounded wait runs out records the
// first failure here and winds down instead of spinning forever.
struct DevStatus {
  unsigned int code;   // 0 = ok, else NSQ_EDEVICE_TIMEOUT
  unsigned int where;  // which wait gave up (kernel-specific tag)
  unsigned int block;  // linear block index that gave up
  unsigned int pad;
  unsigned long long wait_limit_ns;  // limit of the waits that report here; 0 = default
};

// Default upper bound for any single wait on an mbarrier (nanoseconds).
// Normal waits last microseconds; reaching this means a protocol bug, not a
// slow GPU. Waits that report to the status word use its wait_limit_ns when
// set; the wind-down waits (no status word) always use this bound.
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait. Returns false (after recording the failure and raising the
// CTA-wide abort flag) if the phase does not complete within the limit
// or if another thread of the CTA already aborted.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, DevStatus* st,
                                            uint32_t where, volatile int* abort_flag) {
  const unsigned long long t0 = globaltimer_ns();
  unsigned long long limit = kWaitTimeoutNs;
  if (st != nullptr) {
    const unsigned long long l = *reinterpret_cast<volatile unsigned long long*>(&st->wait_limit_ns);
    if (l != 0ull) limit = l;
  }
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer_ns() - t0 > limit) {
        if (st != nullptr && atomicCAS(&st->code, 0u, (unsigned)NSQ_EDEVICE_TIMEOUT) == 0u) {
          st->where = where;
          st->block = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
        }
        if (abort_flag != nullptr) *abort_flag = 1;
        __threadfence();
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, DevStatus* st,
                                          uint32_t where, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, st, where, abort_flag);
}

// ---------------------------------------------------------------------------
// TMA (tensor-map bulk copies, global -> shared, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Programmatic dependent launch controls (no-ops when launched without PDL).
__device__ __forceinline__ void pdl_wait_prior_grids() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue/commit, TMEM loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on `bar` once every tcgen05 op issued so far by the elected lane of
// this (converged) warp completes. The issuing warps run their loops
// converged; one lane (elect.sync) issues, the others keep the warp together.
__device__ __forceinline__ void tc_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, over one or two 64-column
// k-blocks (4 UMMAs of K = 16 each), issued back to back by the elected lane
// of a converged warp. A is read from tensor memory (M = 128 rows per CTA: row
// i in lane i, K pairs packed two per 32-bit column; k-block j at a + 32 j, +8
// columns per K = 16 step); B from the 128-byte-swizzled x tile of k-block j
// (descriptor b_j, +32 bytes per step). Only the first UMMA takes
// `accumulate`; the others accumulate. CG = 2: the paired form (each CTA's
// TMEM holds its 128 rows of A at the same address; B comes from both CTAs'
// shared memory, N / 2 rows each at the same offset; D lands in each CTA's
// TMEM, its 128 rows x N).
// Why one asm block with every operand in its own register: issued one per
// statement (a predicate set-up and the descriptor arithmetic between them,
// from a lone lane), a UMMA costs the issuing thread 100-130 cycles on B200,
// 3.5x the tensor time of a 128 x 64 x 16 step; issued this way a chain of
// them runs at 34 / 67 / 131 cycles for N = 64 / 128 / 256 (measured), the
// tensor pipe's own pace.
#define NSQ_UMMA_TS_PRE \
  "{\n\t.reg .pred e, p, t;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\t"
template <int CG, int KB>
__device__ __forceinline__ void umma_ts_kblocks_elect(uint32_t d, uint32_t a, uint64_t b0, uint64_t b1,
                                                      uint32_t idesc, uint32_t accumulate) {
  static_assert((CG == 1 || CG == 2) && (KB == 1 || KB == 2), "cta_group 1/2, one or two k-blocks");
#define NSQ_MMA1 "@e tcgen05.mma.cta_group::1.kind::f16 [%0], "
#define NSQ_MMA2 "@e tcgen05.mma.cta_group::2.kind::f16 [%0], "
  if constexpr (KB == 2) {
#define NSQ_X8(M)                                                                                   \
  NSQ_UMMA_TS_PRE "setp.ne.b32 p, %18, 0;\n\tsetp.eq.b32 t, %18, %18;\n\t"                          \
  M "[%1], %9, %17, p;\n\t" M "[%2], %10, %17, t;\n\t" M "[%3], %11, %17, t;\n\t"                  \
  M "[%4], %12, %17, t;\n\t" M "[%5], %13, %17, t;\n\t" M "[%6], %14, %17, t;\n\t"                 \
  M "[%7], %15, %17, t;\n\t" M "[%8], %16, %17, t;\n\t}"
#define NSQ_X8_ARGS                                                                                 \
  "r"(d), "r"(a), "r"(a + 8), "r"(a + 16), "r"(a + 24), "r"(a + 32), "r"(a + 40), "r"(a + 48),      \
      "r"(a + 56), "l"(b0), "l"(b0 + 2), "l"(b0 + 4), "l"(b0 + 6), "l"(b1), "l"(b1 + 2), "l"(b1 + 4), \
      "l"(b1 + 6), "r"(idesc), "r"(accumulate)
    if constexpr (CG == 1) {
      asm volatile(NSQ_X8(NSQ_MMA1)::NSQ_X8_ARGS : "memory");
    } else {
      asm volatile(NSQ_X8(NSQ_MMA2)::NSQ_X8_ARGS : "memory");
    }
#undef NSQ_X8
#undef NSQ_X8_ARGS
  } else {
    (void)b1;
#define NSQ_X4(M)                                                                          \
  NSQ_UMMA_TS_PRE "setp.ne.b32 p, %10, 0;\n\tsetp.eq.b32 t, %10, %10;\n\t"                 \
  M "[%1], %5, %9, p;\n\t" M "[%2], %6, %9, t;\n\t" M "[%3], %7, %9, t;\n\t" M "[%4], %8, %9, t;\n\t}"
#define NSQ_X4_ARGS                                                                              \
  "r"(d), "r"(a), "r"(a + 8), "r"(a + 16), "r"(a + 24), "l"(b0), "l"(b0 + 2), "l"(b0 + 4), "l"(b0 + 6), \
      "r"(idesc), "r"(accumulate)
    if constexpr (CG == 1) {
      asm volatile(NSQ_X4(NSQ_MMA1)::NSQ_X4_ARGS : "memory");
    } else {
      asm volatile(NSQ_X4(NSQ_MMA2)::NSQ_X4_ARGS : "memory");
    }
#undef NSQ_X4
#undef NSQ_X4_ARGS
  }
#undef NSQ_MMA1
#undef NSQ_MMA2
}
#undef NSQ_UMMA_TS_PRE

// 16 registers per thread -> 32 lanes x 16 consecutive 32-bit TMEM columns.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major tile written with the 128-byte
// swizzle (rows of 128 B, 8-row groups 1024 B apart; tile base 1024-aligned).
// Fields: start>>4 [0,14), LBO>>4 [16,30) (unused for swizzled K-major, 1),
// SBO>>4 [32,46), version 1 [46,48), layout SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A/B K-major.
// c_format [4,6)=1 (F32); a_format [7,10), b_format [10,13): 0 F16, 1 BF16;
// n_dim [17,23) = N>>3; m_dim [24,29) = M>>4.
__host__ __device__ constexpr uint32_t umma_idesc_f16(bool bf16, int m, int n) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// 16 lanes x 256 bits, 4 repetitions along the columns: thread t gets lanes
// base + t/4 and base + t/4 + 8, 32-bit columns 8j + 2(t%4) and 8j + 2(t%4) + 1
// in r[4j .. 4j+3] = {(lane, c), (lane, c+1), (lane+8, c), (lane+8, c+1)} --
// the m8n8 fragment layout of mma / ldmatrix / stmatrix.
__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// Four 8x8 b16 matrices from fragments, stored transposed: thread 8q + i gives
// the shared address of row i of matrix q (16 bytes).
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2,
                                                  uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0),
               "r"(r1), "r"(r2), "r"(r3)
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Paired-CTA (cta_group::2) forms: one UMMA spans the two CTAs of a cluster
// pair; the even CTA (rank 0) issues it and owns the barriers the pair syncs on.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// Arrive on the barrier at the same offset in every CTA of `cta_mask` once all
// tcgen05 ops issued so far by the elected lane of this (converged) warp complete.
__device__ __forceinline__ void tc_commit_pair_mc_elect(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
// Arrive on a barrier of another CTA of the cluster (default semantics). The
// paired prefill kernel's converters arrive here after tcgen05.wait::st and
// tcgen05.fence::before_thread_sync on the TMEM operand the pair's UMMA will
// read; its epilogue warps after their last tcgen05.ld of the accumulator.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// TMA store of a shared-memory tile (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier that also returns the AND of `pred` over the participating
// threads, so a group can leave a loop together when any member gave up.
__device__ __forceinline__ bool named_bar_all(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, %3, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------
// Warp-level MMA m16n8k16 (row.col), fp32 accumulate
// ---------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4],
                                          uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// ---------------------------------------------------------------------------
// Cluster / distributed shared memory
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Cluster barrier halves (not .aligned: callable where the warp diverged).
__device__ __forceinline__ void cluster_arrive_rel() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acq() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from this CTA's shared memory into another CTA's, counted on the barrier
// `bar_cluster` in the destination CTA.
__device__ __forceinline__ void bulk_copy_s2cluster(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                    uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ uint32_t dsmem_map(uint32_t smem_addr, uint32_t cta_rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(cta_rank));
  return r;
}
__device__ __forceinline__ float dsmem_ld_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// ---------------------------------------------------------------------------
// Shared-memory vector access
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                       uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// ---------------------------------------------------------------------------
// Packed unpack primitives
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;  // (a & b) | c
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Biased-integer construction: (magic | nibble) reads as magic_value + q
// exactly, because the nibble lands in the low mantissa bits whose weight is 1:
//   fp16 0x6400 = 1024.0 (ulp 1 on [1024, 2048)), bf16 0x4300 = 128.0 (ulp 1 on [128, 256)).
template <bool BF16>
struct Magic {
  static constexpr uint32_t kPair = BF16 ? 0x43004300u : 0x64006400u;
  static constexpr float kValue = BF16 ? 128.0f : 1024.0f;
};

// Word of 8 sequential nibbles (nibble i = column 8j+i) -> four packed pairs
// {magic+q_t, magic+q_{t+4}} for t = 0..3.
template <bool BF16>
__device__ __forceinline__ void unpack_nibble_pairs(uint32_t w, uint32_t (&e)[4]) {
  constexpr uint32_t M = Magic<BF16>::kPair;
  e[0] = lop3_and_or(w, 0x000F000Fu, M);
  e[1] = lop3_and_or(w >> 4, 0x000F000Fu, M);
  e[2] = lop3_and_or(w >> 8, 0x000F000Fu, M);
  e[3] = lop3_and_or(w >> 12, 0x000F000Fu, M);
}

// The A operands of the two m16n8k16 MMAs of one word of row g (wg) and the
// same word of row g + 8 (wh), written straight in fragment order:
//   a0 = {p0(wg), p0(wh), p1(wg), p1(wh)},  a1 = {p2(wg), p2(wh), p3(wg), p3(wh)}
// with p_t = {magic+q_t, magic+q_{t+4}} as in unpack_nibble_pairs.
template <bool BF16>
__device__ __forceinline__ void nibble_quads(uint32_t wg, uint32_t wh, uint32_t (&a0)[4],
                                             uint32_t (&a1)[4]) {
  constexpr uint32_t M = Magic<BF16>::kPair;
  a0[0] = lop3_and_or(wg, 0x000F000Fu, M);
  a0[1] = lop3_and_or(wh, 0x000F000Fu, M);
  a0[2] = lop3_and_or(wg >> 4, 0x000F000Fu, M);
  a0[3] = lop3_and_or(wh >> 4, 0x000F000Fu, M);
  a1[0] = lop3_and_or(wg >> 8, 0x000F000Fu, M);
  a1[1] = lop3_and_or(wh >> 8, 0x000F000Fu, M);
  a1[2] = lop3_and_or(wg >> 12, 0x000F000Fu, M);
  a1[3] = lop3_and_or(wh >> 12, 0x000F000Fu, M);
}

// Four e4m3 codes (one word, low byte first) -> two packed pairs of the MMA
// element type, exact, with integer ops plus one packed multiply per pair
// (no conversion-pipe instructions). The sign bit goes to bit 15 and the
// 7-bit exponent|mantissa field lands right below the target exponent field:
//   bf16: s | em << 4  reads as value * 2^-120,   fp16: s | em << 7  reads as value * 2^-8
// for every finite code, subnormals included (they land on subnormals of the
// target type); the packed multiply by 2^120 / 2^8 then restores the value
// exactly. (NaN codes are not preserved; quantised weights never hold them.)
template <bool BF16>
__device__ __forceinline__ void e4m3x4_to_pairs(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t em = w & 0x7F7F7F7Fu;
  const uint32_t sg = w & 0x80808080u;
  // per 16-bit lane: (sign byte << 8) | em byte
  const uint32_t t0 = prmt(em, sg, 0x5140);
  const uint32_t t1 = prmt(em, sg, 0x7362);
  constexpr uint32_t kMul = BF16 ? 15u : 127u;  // em + kMul*em = em << 4 (bf16) / << 7 (fp16)
  const uint32_t r0 = t0 + kMul * (t0 & 0x007F007Fu);
  const uint32_t r1 = t1 + kMul * (t1 & 0x007F007Fu);
  if constexpr (BF16) {
    const uint32_t kbits = 0x7B807B80u;  // {2^120, 2^120}
    const __nv_bfloat162 k = *reinterpret_cast<const __nv_bfloat162*>(&kbits);
    __nv_bfloat162 a = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&r0), k);
    __nv_bfloat162 b = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&r1), k);
    lo = *reinterpret_cast<uint32_t*>(&a);
    hi = *reinterpret_cast<uint32_t*>(&b);
  } else {
    const uint32_t kbits = 0x5C005C00u;  // {256, 256}
    const __half2 k = *reinterpret_cast<const __half2*>(&kbits);
    __half2 a = __hmul2(*reinterpret_cast<const __half2*>(&r0), k);
    __half2 b = __hmul2(*reinterpret_cast<const __half2*>(&r1), k);
    lo = *reinterpret_cast<uint32_t*>(&a);
    hi = *reinterpret_cast<uint32_t*>(&b);
  }
}

template <bool BF16>
__device__ __forceinline__ float elem_to_float(uint16_t bits) {
  if constexpr (BF16) {
    return __uint_as_float(static_cast<uint32_t>(bits) << 16);
  } else {
    return __half2float(__ushort_as_half(bits));
  }
}

template <bool BF16>
__device__ __forceinline__ uint16_t float_to_elem(float v) {
  if constexpr (BF16) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  } else {
    return __half_as_ushort(__float2half_rn(v));
  }
}

__device__ __forceinline__ float load_bias(const void* bias, int dtype, int n) {
  switch (dtype) {
    case NSQ_DTYPE_F16:
      return __half2float(reinterpret_cast<const __half*>(bias)[n]);
    case NSQ_DTYPE_BF16:
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
    case NSQ_DTYPE_F32:
      return reinterpret_cast<const float*>(bias)[n];
    default:
      return 0.0f;
  }
}

// n / d for 0 <= n < 2^31 with one multiply-high, one add and one shift: the
// invariant-divisor method of Granlund & Montgomery (PLDI 1994) with the
// 33-bit multiplier 2^32 + mul, l = ceil(log2 d), mul = floor(2^32 (2^l - d) / d) + 1.
struct FastDiv {
  uint32_t mul, shift;
};
__host__ __device__ inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while (l < 31 && (1u << l) < d) ++l;
  const uint64_t m = ((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1;
  return FastDiv{static_cast<uint32_t>(m), l};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, FastDiv f) {
  return (__umulhi(n, f.mul) + n) >> f.shift;
}

}  // namespace nsq
