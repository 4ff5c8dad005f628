// Tensor-core decode linear (M <= 32 tokens) for layers of at least 64 rows per
// SM: the tcgen05 UMMAs take the weight from the TMA-staged tiles (FP8) or from
// tensor memory, where four warps store the nibbles widened to bytes (AWQ), and
// x enters the tensor core as two narrow terms, so no CUDA-core instruction
// does arithmetic on a weight value (FP8) or more than widen nibbles (AWQ).
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152 and :49-52) for small batches on large layers
// (Llama-3-8B / Qwen2.5-72B gate, up, fused q/k/v). The reference dequantises
// the weight and calls cuBLAS.
//
// Why: the warp-MMA decode kernels spend their time converting weights on the
// CUDA cores (one conversion per two e4m3 codes on a 16-lane pipe; a lop3 and
// a subtract per two nibbles plus operand shuffles), and on B200 that, not
// HBM, set their pace on large layers. Here the tensor core takes the weight
// in its stored type:
//   FP8: kind::f8f6f4, A = e4m3 codes as stored, B = x as two e4m3 terms;
//   AWQ: kind::i8, A = nibbles widened to u8 (0..15, one lop3 per four), B = x
//        as two s8 terms; zero point and group scale applied per 128-column
//        k-block in the epilogue: s * (sum q x - z * sum x).
// x terms, per token and k-block of 128 columns (one power-of-two scale 2^e):
//   AWQ: x * 2^-e = T1 + T2 / 128, T1, T2 integers in [-64, 64] (max |x| of the
//        block maps into [32, 64)): 13 bits of the block's range, so every
//        element within 2^-4 of the block's largest keeps its bf16 precision;
//   FP8: x * 2^-e = T1 + T2 / 16, T1 = e4m3(x * 2^-e), T2 = e4m3 of the
//        remainder times 16 (max |x| maps into [128, 256)): about 8 significant
//        bits per element, an element's own bf16 precision, down to 2^-14 of
//        the block's largest.
// Integer products (AWQ) are exact; the accumulators are fp32 throughout.
//
// Work split: CTA i owns a block of weight rows, a multiple of 8 between 64 and
// 128 (TMEM lane = row; one TMA box of [rows x 128 B] per ring slot), and the
// whole K range: accumulators never leave the CTA, no split-K. One CTA per SM,
// or fewer CTAs of 64+ rows on smaller layers.
// Warp roles (FP8 448 threads, AWQ 576):
//   warp 0      TMA producer (one lane): one 128-byte chunk of every row per
//               ring slot -- an FP8 k-block, which is the UMMA A tile itself,
//               or two AWQ k-blocks of packed nibbles. Weights are static, so
//               it never waits for the previous kernel.
//   warp 1      TMEM owner and UMMA issuer: per k-block four UMMAs (M = 128,
//               N = 2 MP, K = 32; A from the ring slot or the tensor-memory
//               tile, B from shared memory) into one of four accumulators,
//               then commits that free the A tile, the x-term tile and fill
//               the accumulator.
//   warps 2-9   x terms, two groups of four warps taking alternate k-blocks:
//               x k-blocks by TMA, four ahead; per k-block and token the scale
//               2^e, T1 and T2 in the UMMA B layout (K-major, 128-byte
//               swizzle), and the per-token sums of the terms (AWQ zero point).
//   warps 10-13 epilogue: warp w reads TMEM sub-partition w % 4 (32 rows)
//               after every k-block and accumulates in registers.
//   warps 14-17 (AWQ) weight transfer: warp w takes TMEM sub-partition w % 4,
//               one weight row per lane: the row's 128 bytes of a ring slot
//               into registers (the slot is then free), nibbles widened to
//               bytes, tcgen05.st into one of four tensor-memory A tiles.
// Every wait is bounded. Measured performance and the variants that lost are
// in the design notes (tensor-core decode kernel).
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr int kTcM = 128;                  // UMMA M: weight rows per CTA tile (TMEM lanes)
constexpr int kTcWarpProd = 0;
constexpr int kTcWarpMma = 1;
constexpr int kTcWarpPrep0 = 2;
constexpr int kTcPrepWarps = 8;
constexpr int kTcXGroups = 2;  // x-term groups of four warps, alternating k-blocks
constexpr int kTcEpiWarps = 4;
constexpr int kTcXfrWarps = 4;  // weight transfer: one per TMEM sub-partition
constexpr int kTcND = 4;   // accumulators in TMEM (two at 64 token slots)
constexpr int kTcNB = 4;   // x-term tiles
constexpr int kTcNX = 8;   // per-token scalars of a k-block
constexpr int kTcNXR = 4;  // x k-blocks staged ahead of the x-term warps
constexpr int kTcNA = 4;  // AWQ tensor-memory A tiles

constexpr int kTcMaxNS = 12;  // weight ring slots (upper bound; the plan sizes the ring to shared memory)
constexpr int kTcSmemMax = 227 * 1024;

// A ring slot holds 128 bytes of every row: one FP8 k-block, or two AWQ
// k-blocks of packed nibbles. FP8: the UMMAs read A straight from the ring
// slot (shared memory); AWQ: transfer warps widen it into tensor memory and
// the UMMAs read A there.
// PRE: the x terms come precomputed (tc_xterm_kernel, once per launch instead
// of once per CTA): one warp copies them in by TMA in place of the eight
// x-term warps.
// Epilogue: four warps (one per TMEM sub-partition), or with PRE and 32+
// token slots eight, each taking half the token slots of its sub-partition.
template <int FMT, int MP, bool PRE>
struct TcCfg {
  static constexpr bool kTmemA = FMT == 0;
  static constexpr int kEpi0 = PRE ? kTcWarpPrep0 + 1 : kTcWarpPrep0 + kTcPrepWarps;  // first epilogue warp
  static constexpr int kEpiWarps = PRE && MP >= 32 ? 2 * kTcEpiWarps : kTcEpiWarps;
  static constexpr int kXfr0 = kEpi0 + kEpiWarps;                                     // first transfer warp
  static constexpr int kXfrGroups = 1;  // transfer groups of four warps taking alternate ring slots (two: no faster)
  static constexpr int kThreads = (kTmemA ? kXfr0 + kXfrGroups * kTcXfrWarps : kXfr0) * 32;
  static constexpr int kKPS = FMT == 0 ? 2 : 1;  // k-blocks per ring slot
};

// Tensor memory and occupancy of one instantiation. Accumulators at columns
// d * 2 MP (d < kND); AWQ: A tile t (t < kTcNA, 128 lanes x 128 bytes of
// widened weight) at kA + 32 t. Two CTAs per SM (112 KB of shared memory and
// at most 256 columns each, so that the next launch's CTA streams its weights
// while this one finishes) measured slower than one CTA with the full ring:
// FP8 4096 -> 14336 at M = 32 18.5 -> 22.7 us.
template <int FMT, int MP, bool PRE>
struct TcMem {
  static constexpr bool kPair = false;  // two CTAs per SM measured slower (a smaller weight ring): one
  static constexpr int kMinBlocks = kPair ? 2 : 1;
  static constexpr int kSmem = kPair ? 112 * 1024 : kTcSmemMax;  // dynamic shared memory, alignment slack included
  static constexpr int kND = MP == 64 ? 2 : kTcND;                // accumulators
  static constexpr uint32_t kA = kND * 2 * MP;                    // AWQ A tiles after the accumulators
  static constexpr uint32_t kUsed = kA + (FMT == 0 ? 32 * kTcNA : 0);
  static constexpr uint32_t kCols = kUsed <= 128 ? 128 : kUsed <= 256 ? 256 : 512;
  static_assert(!kPair || kCols <= 256, "two CTAs per SM share 512 columns");
};

// Fixed part of the shared-memory layout (after the weight ring, whose size
// the plan chooses): x-term tiles, x k-blocks (not with PRE), per-token
// scalars, barriers.
template <int MP, bool PRE>
struct TcFixed {
  static constexpr int kBBytes = 2 * MP * 128;  // x-term tile: 2 MP rows (T1 rows, then T2 rows) x 128 B
  static constexpr int kXBytes = MP * 256;      // one x k-block: two boxes of [MP tokens x 64 columns] 16-bit
  static constexpr int kNB = kTcNB;  // eight with precomputed terms measured no faster
  static constexpr int kB = 0;
  static constexpr int kX = kB + kNB * kBBytes;
  static constexpr int kXs = kX + (PRE ? 0 : kTcNXR * kXBytes);  // [NX][2][MP] fp32: scale 2^e, term sum (AWQ)
  static constexpr int kBar = kXs + kTcNX * 2 * MP * 4;
  static constexpr int kNumBars = 2 * kTcMaxNS + 2 * kTcNA + 2 * kNB + 2 * kTcND + 2 * kTcNX + kTcNXR + 1;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kBytes = ((kAbort + 4 + 1023) / 1024) * 1024;
  static_assert(kBBytes % 1024 == 0 && kXBytes % 1024 == 0, "tiles stay 1 KB aligned");
};

struct TcParams {
  const void* x;
  const __half* scales;  // AWQ [N, G]
  const __half* zeros;   // AWQ [N, G]
  const float* wscale;   // FP8 per-tensor scale (device)
  const void* bias;
  void* y;
  DevStatus* status;
  int M, K, N;
  int G, group_size;
  int bias_dtype;
  int rlo, nhi;  // weight rows per CTA: rlo + 8 for the first nhi CTAs, rlo for the others (multiples of 8)
  int nkb;       // k-blocks of 128 columns
  int tile;       // bytes of a ring slot: the tallest CTA's rows x 128 B
  int ns;         // weight ring slots (at shared-memory offset 0)
  int off_fixed;  // the fixed part (TcFixed)
  int sz_vec;     // AWQ: G % 8 == 0 and 16-byte aligned scales / zeros (eight groups per load)
  const float* xsg;  // PRE: per-k-block scalars [nkb][2][MP] (the terms: tensor map bmap)
};

// Instruction descriptor: AWQ kind::i8 (A u8, B s8, D s32), FP8 kind::f8f6f4
// (A, B e4m3, D f32); both operands K-major.
__host__ __device__ constexpr uint32_t tc_idesc(int fmt, int m, int n) {
  return (fmt == 0 ? ((2u << 4) | (0u << 7) | (1u << 10)) : ((1u << 4) | (0u << 7) | (0u << 10))) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// The four UMMAs of one k-block (K = 32 each), issued by the elected lane of a
// converged warp in one asm block; the first starts a fresh accumulator. B is
// the x-term tile (128-byte swizzle, +32 bytes = +2 descriptor units per
// step). A is either a shared-memory tile (descriptor, same stepping; FP8) or
// a tensor-memory tile at column ta (row i in lane i, 32 bytes = 8 columns per
// step, bytes in K order; AWQ).
// Cost (measured, Llama-3-8B gate at 16 tokens): with A in shared memory the
// four UMMAs of a k-block keep the issuer about 0.43 us with every barrier
// already passed (0.36 us with one UMMA instead of four, nearly the same at
// half the N), so reading the 128 A rows, not the MACs, costs; tcgen05.cp of
// the tile into tensor memory first is no faster (it reads the same rows).
// With A in tensor memory the UMMAs are cheap but the transfer warps' loads,
// stores and waits add about 0.6 us of latency per k-block: for FP8 that lost
// (19.9 us against 17.7), for AWQ, whose nibbles need the warps anyway, it won
// (22.7 us against 27.9, and 31.5 against 38.5 at 32 tokens).
#define NSQ_TC_UMMA4(KIND, A0, A1, A2, A3, ACON, ...)                                             \
  asm volatile(                                                                                  \
      "{\n\t.reg .pred e, p, t;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\t"              \
      "setp.ne.b32 p, %9, %9;\n\tsetp.eq.b32 t, %9, %9;\n\t"                                     \
      "@e tcgen05.mma.cta_group::1.kind::" KIND " [%0], " A0 ", %5, %9, p;\n\t"                 \
      "@e tcgen05.mma.cta_group::1.kind::" KIND " [%0], " A1 ", %6, %9, t;\n\t"                 \
      "@e tcgen05.mma.cta_group::1.kind::" KIND " [%0], " A2 ", %7, %9, t;\n\t"                 \
      "@e tcgen05.mma.cta_group::1.kind::" KIND " [%0], " A3 ", %8, %9, t;\n\t}" ::"r"(d),      \
      ACON(a), ACON(a + (__VA_ARGS__)), ACON(a + 2 * (__VA_ARGS__)), ACON(a + 3 * (__VA_ARGS__)), \
      "l"(b), "l"(b + 2), "l"(b + 4), "l"(b + 6), "r"(idesc)                                      \
      : "memory")
#define NSQ_TC_R(x) "r"(x)
#define NSQ_TC_L(x) "l"(x)
// A in shared memory (descriptor a)
__device__ __forceinline__ void tc_umma_ss_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc) {
  NSQ_TC_UMMA4("f8f6f4", "%1", "%2", "%3", "%4", NSQ_TC_L, 2);
}
// A in tensor memory (column a)
__device__ __forceinline__ void tc_umma_ts_i8(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
  NSQ_TC_UMMA4("i8", "[%1]", "[%2]", "[%3]", "[%4]", NSQ_TC_R, 8);
}
#undef NSQ_TC_UMMA4
#undef NSQ_TC_R
#undef NSQ_TC_L

// Three commits from the elected lane in one asm block: each barrier gets one
// arrival once every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void tc_commit3_elect(uint64_t* a, uint64_t* b, uint64_t* c) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%1];\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%2];\n\t}" ::"r"(smem_u32(a)),
      "r"(smem_u32(b)), "r"(smem_u32(c))
      : "memory");
}

// Non-blocking probe of three barrier phases in one asm block (the three
// reads overlap): true if all three have completed. The callers fall back to
// the bounded waits one by one when it returns false.
// Why: the UMMA issuer's three blocking waits in a row cost it about 0.1 us
// per k-block even with every phase long completed (measured: the FP8 gate of
// Llama-3-8B at 16 tokens went from 21.2 to 18.0 us with this probe first).
__device__ __forceinline__ bool mbar_test3(uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb, uint64_t* c,
                                           uint32_t pc) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p, q, r;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 q, [%3], %4;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 r, [%5], %6;\n\t"
      "and.pred p, p, q;\n\tand.pred p, p, r;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(a)), "r"(pa), "r"(smem_u32(b)), "r"(pb), "r"(smem_u32(c)), "r"(pc)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of one barrier phase.
__device__ __forceinline__ bool mbar_test1(uint64_t* a, uint32_t pa) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(a)), "r"(pa)
      : "memory");
  return ok != 0;
}

// One rank-3 TMA box into shared memory (no multicast), completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// One contiguous global -> shared copy (no multicast), completing on `bar`;
// both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// bytes 0 of a, b, c, d -> one word (a in the low byte)
__device__ __forceinline__ uint32_t pack_b0(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return prmt(prmt(a, b, 0x5140u), prmt(c, d, 0x5140u), 0x5410u);
}

// two floats -> two e4m3 codes (hi in the upper byte), round to nearest, saturating
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// two e4m3 codes (low byte first) -> their two values
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t codes16) {
  uint32_t h;
  asm("{\n\t.reg .b16 c;\n\tcvt.u16.u32 c, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, c;\n\t}" : "=r"(h) : "r"(codes16));
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// The x terms of one token's EPT columns of a k-block (this thread's share;
// the token's TPT threads are adjacent lanes and reduce the block's largest
// |x| and the term sums by shuffles): term bytes o1 (T1) and o2 (T2) in the A
// operand's column order, the scale sc = 2^e and (AWQ) sx = 2^e times the
// term sum (the zero point's factor in the epilogue).
template <int FMT, bool BF16, int EPT, int TPT>
__device__ __forceinline__ void tc_x_terms(const uint4 (&v)[EPT / 8], uint32_t (&o1)[EPT / 4], uint32_t (&o2)[EPT / 4],
                                           float& sc, float& sx) {
  float f[EPT];
#pragma unroll
  for (int i = 0; i < EPT / 8; ++i) {
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      f[8 * i + 2 * e] = elem_to_float<BF16>((uint16_t)(w[e] & 0xFFFFu));
      f[8 * i + 2 * e + 1] = elem_to_float<BF16>((uint16_t)(w[e] >> 16));
    }
  }
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < EPT; ++i) mx = fmaxf(mx, fabsf(f[i]));
#pragma unroll
  for (int m = 1; m < TPT; m <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
  const int E = (__float_as_int(mx) >> 23) & 0xFF;  // biased exponent of the block's largest |x|
  sc = 0.f;
  sx = 0.f;
  if constexpr (FMT == 0) {
    // x * 2^-e in [-64, 64): e = E - 127 - 5; blocks below 2^-119 count as zero
    const bool nz = E >= 12;
    const float inv = nz ? __int_as_float((259 - E) << 23) : 0.f;
    sc = nz ? __int_as_float((E - 5) << 23) : 0.f;
    constexpr float kRnd = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer, kept in the low bits
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int g = 0; g < EPT / 8; ++g) {
      uint32_t b1[8], b2[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float a1 = fmaf(f[8 * g + i], inv, kRnd);
        const float t1 = a1 - kRnd;
        const float rr = fmaf(f[8 * g + i], inv, -t1);
        const float a2 = fmaf(rr, 128.0f, kRnd);
        s1 += t1;
        s2 += a2 - kRnd;
        b1[i] = __float_as_uint(a1);  // low byte: the integer, two's complement
        b2[i] = __float_as_uint(a2);
      }
      // widened weight bytes of one 32-bit word: columns 0,2,4,6 then 1,3,5,7
      o1[2 * g] = pack_b0(b1[0], b1[2], b1[4], b1[6]);
      o1[2 * g + 1] = pack_b0(b1[1], b1[3], b1[5], b1[7]);
      o2[2 * g] = pack_b0(b2[0], b2[2], b2[4], b2[6]);
      o2[2 * g + 1] = pack_b0(b2[1], b2[3], b2[5], b2[7]);
    }
#pragma unroll
    for (int m = 1; m < TPT; m <<= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, m);
      s2 += __shfl_xor_sync(0xffffffffu, s2, m);
    }
    sx = s1 + s2 * 0.0078125f;
  } else {
    // x * 2^-e with its largest in [128, 256): e = E - 127 - 7; blocks below 2^-115 count as zero
    const bool nz = E >= 12;
    const float inv = nz ? __int_as_float((261 - E) << 23) : 0.f;
    sc = nz ? __int_as_float((E - 7) << 23) : 0.f;
#pragma unroll
    for (int i = 0; i < EPT; i += 4) {
      const float x0 = f[i] * inv, x1 = f[i + 1] * inv, x2 = f[i + 2] * inv, x3 = f[i + 3] * inv;
      const uint32_t c01 = f32x2_to_e4m3x2(x1, x0), c23 = f32x2_to_e4m3x2(x3, x2);
      const float2 v01 = e4m3x2_to_f32x2(c01), v23 = e4m3x2_to_f32x2(c23);
      const uint32_t d01 = f32x2_to_e4m3x2((x1 - v01.y) * 16.0f, (x0 - v01.x) * 16.0f);
      const uint32_t d23 = f32x2_to_e4m3x2((x3 - v23.y) * 16.0f, (x2 - v23.x) * 16.0f);
      o1[i / 4] = c01 | (c23 << 16);
      o2[i / 4] = d01 | (d23 << 16);
    }
  }
  // an infinite or NaN x makes the token's outputs NaN, as the reference's
  // matmul would (the terms of such a block are meaningless)
  if (E == 255) sc = __int_as_float(0x7FC00000);
  if constexpr (FMT == 0) sx *= sc;
}

template <int FMT, bool BF16, int MP, bool PRE>
__global__ void __launch_bounds__(TcCfg<FMT, MP, PRE>::kThreads, (TcMem<FMT, MP, PRE>::kMinBlocks))
    decode_tc_kernel(const __grid_constant__ CUtensorMap wmap_lo, const __grid_constant__ CUtensorMap wmap_hi,
                     const __grid_constant__ CUtensorMap xmap, const TcParams p) {
  using F = TcFixed<MP, PRE>;
  using C = TcCfg<FMT, MP, PRE>;
  using T = TcMem<FMT, MP, PRE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* fx = smem + p.off_fixed;
  uint64_t* bars = reinterpret_cast<uint64_t*>(fx + F::kBar);
  // Weight ring (one box of 128 bytes of every row per slot, filled by TMA;
  // slots `tile` bytes apart, the tallest CTA's rows): wfull / wempty (the
  // four transfer warps have the slot in registers). Tensor-memory A tiles:
  // afull (four transfer warps stored) / aempty (their UMMAs finished).
  // bfull / bempty: x-term tiles. dfull: an accumulator's UMMAs finished;
  // dempty: its four readers are done. xsfull / xsempty: the per-token
  // scalars of a k-block.
  uint64_t* wfull = bars;
  uint64_t* wempty = wfull + kTcMaxNS;
  uint64_t* afull = wempty + kTcMaxNS;
  uint64_t* aempty = afull + kTcNA;
  uint64_t* bfull = aempty + kTcNA;
  uint64_t* bempty = bfull + F::kNB;
  uint64_t* dfull = bempty + F::kNB;
  uint64_t* dempty = dfull + kTcND;
  uint64_t* xsfull = dempty + kTcND;
  uint64_t* xsempty = xsfull + kTcNX;
  uint64_t* xfull = xsempty + kTcNX;
  uint64_t* mdone = xfull + kTcNXR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fx + F::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(fx + F::kAbort);
  float* xs = reinterpret_cast<float*>(fx + F::kXs);
  constexpr int KPS = C::kKPS;
  const int NS = p.ns;
  const uint32_t tile = (uint32_t)p.tile;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i_cta = (int)blockIdx.x;
  const int rows = i_cta < p.nhi ? p.rlo + 8 : p.rlo;      // this CTA's rows (multiple of 8)
  const int r0 = i_cta * p.rlo + 8 * min(i_cta, p.nhi);
  const int rvalid = min(rows, p.N - r0);
  const CUtensorMap* wmap = i_cta < p.nhi ? &wmap_hi : &wmap_lo;
  const uint32_t ctile = (uint32_t)rows * 128u;  // bytes one TMA box of this CTA's rows lands
  const int nkb = p.nkb;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], C::kTmemA ? kTcXfrWarps : 1);
    }
    for (int i = 0; i < kTcNA; ++i) {
      mbar_init(&afull[i], kTcXfrWarps);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < F::kNB; ++i) {
      mbar_init(&bfull[i], 1);
      mbar_init(&bempty[i], 1);
    }
    for (int i = 0; i < kTcND; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], C::kEpiWarps);
    }
    for (int i = 0; i < kTcNX; ++i) {
      mbar_init(&xsfull[i], 1);
      mbar_init(&xsempty[i], C::kEpiWarps);
    }
    for (int i = 0; i < kTcNXR; ++i) mbar_init(&xfull[i], 1);
    mbar_init(mdone, 1);
    fence_barrier_init();
  }
  if (warp == kTcWarpMma) {
    tmem_alloc(tmem_slot, T::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  bool ok = true;

  if (warp == kTcWarpProd) {
    // ---------------- producer ----------------
    if (lane == 0) {
      // Slot st: the box [rows][128 B] of 128-byte chunk st of every row (one
      // FP8 k-block, or two AWQ k-blocks of packed nibbles). Chunks past the
      // row read zeros; their k-blocks are never used.
      tma_prefetch_desc(wmap);
      const int nst = (nkb + KPS - 1) / KPS;
      uint8_t* ring = smem;
      int st = 0;
      for (; st < nst; ++st) {
        const int slot = st % NS;
        if (st >= NS && !(ok = mbar_wait(&wempty[slot], ((st / NS) - 1) & 1, p.status, 80, abort_flag))) break;
        mbar_arrive_expect_tx(&wfull[slot], ctile);
        tma_load_2d(ring + (size_t)slot * tile, wmap, &wfull[slot], st * 32, r0);
      }
      if (!ok) {  // copies in flight land before the CTA can exit
        for (int j = (st > NS ? st - NS : 0); j < st; ++j) mbar_wait(&wfull[j % NS], (j / NS) & 1, nullptr, 0, nullptr);
      }
    }
  } else if (warp == kTcWarpMma) {
    // ---------------- UMMA issuer (whole warp, converged) ----------------
    const uint32_t idesc = tc_idesc(FMT, kTcM, 2 * MP);
    for (int b = 0; b < nkb; ++b) {
      const int s = b % F::kNB, d = b % T::kND;  // x-term tile, accumulator
      // the A tile: FP8 ring slot b % ns; AWQ tensor-memory tile b % kTcNA
      const int a = FMT == 1 ? b % NS : b % kTcNA;
      uint64_t* abar = FMT == 1 ? &wfull[a] : &afull[a];
      const uint32_t apar = FMT == 1 ? ((b / NS) & 1) : ((b / kTcNA) & 1);
      const uint32_t bpar = (b / F::kNB) & 1;
      const uint32_t dpar = ((b / T::kND) - 1) & 1;  // accumulator d free again (k-block b - T::kND read out)
      // the A tile, the x-term tile and the accumulator
      const bool ready = __all_sync(
          0xffffffffu, mbar_test3(abar, apar, &bfull[s], bpar, b >= T::kND ? &dempty[d] : &bfull[s], b >= T::kND ? dpar : bpar));
      if (!ready) {
        ok = __all_sync(0xffffffffu, mbar_wait(abar, apar, p.status, FMT == 1 ? 81 : 82, abort_flag));
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bfull[s], bpar, p.status, 83, abort_flag));
        if (ok && b >= T::kND) ok = __all_sync(0xffffffffu, mbar_wait(&dempty[d], dpar, p.status, 84, abort_flag));
        if (!ok) break;
      }
      tc_fence_after();
      const uint64_t bdesc = sw128_kmajor_desc(smem_u32(fx + F::kB + s * F::kBBytes));
      const uint32_t dt = tmem_base + (uint32_t)(d * 2 * MP);
      if constexpr (FMT == 1) {
        tc_umma_ss_f8(dt, sw128_kmajor_desc(smem_u32(smem) + (uint32_t)a * tile), bdesc, idesc);
        tc_commit3_elect(&wempty[a], &bempty[s], &dfull[d]);
      } else {
        tc_umma_ts_i8(dt, tmem_base + T::kA + 32u * (uint32_t)a, bdesc, idesc);
        tc_commit3_elect(&aempty[a], &bempty[s], &dfull[d]);
      }
    }
    // every UMMA issued has finished before TMEM is released
    tc_commit_elect(mdone);
    mbar_wait(mdone, 0, nullptr, 0, nullptr);
  } else if (warp < C::kEpi0 && PRE) {
    // ---------------- x terms by TMA (precomputed) ----------------
    // xmap covers the terms [nkb x 2 MP rows][128 B]: one box of a k-block's
    // 2 MP rows lands as the x-term tile (128-byte swizzle); its scalars
    // [2][MP] fp32 follow by one bulk copy.
    if (lane == 0) {
      tma_prefetch_desc(&xmap);
      pdl_wait_prior_grids();  // the terms are written by the previous kernel
      int b = 0;
      for (; b < nkb; ++b) {
        const int s = b % F::kNB, xsl = b % kTcNX;
        if (b >= F::kNB && !(ok = mbar_wait(&bempty[s], ((b / F::kNB) - 1) & 1, p.status, 85, abort_flag))) break;
        if (b >= kTcNX && !(ok = mbar_wait(&xsempty[xsl], ((b / kTcNX) - 1) & 1, p.status, 86, abort_flag))) break;
        mbar_arrive_expect_tx(&bfull[s], (uint32_t)F::kBBytes);
        tma_load_2d(fx + F::kB + s * F::kBBytes, &xmap, &bfull[s], 0, b * 2 * MP);
        mbar_arrive_expect_tx(&xsfull[xsl], (uint32_t)(2 * MP * 4));
        bulk_load_1d(xs + xsl * 2 * MP, p.xsg + (size_t)b * 2 * MP, 2 * MP * 4, &xsfull[xsl]);
      }
      if (!ok) {  // copies in flight land before the CTA can exit
        for (int j = (b > F::kNB ? b - F::kNB : 0); j < b; ++j)
          mbar_wait(&bfull[j % F::kNB], (j / F::kNB) & 1, nullptr, 0, nullptr);
        for (int j = (b > kTcNX ? b - kTcNX : 0); j < b; ++j)
          mbar_wait(&xsfull[j % kTcNX], (j / kTcNX) & 1, nullptr, 0, nullptr);
      }
    }
  } else if (warp < C::kEpi0) {
    if constexpr (!PRE) {
    // ---------------- x terms ----------------
    pdl_wait_prior_grids();  // x is written by the previous kernel
    constexpr int kGT = kTcPrepWarps / kTcXGroups * 32;  // threads of a group
    constexpr int TPT = kGT / MP;                        // threads per token
    constexpr int EPT = 128 / TPT;                       // columns per thread: one or two 16-byte chunks of a term row
    static_assert(EPT == 16 || EPT == 32, "16 or 32 token slots");
    static_assert(kTcNXR % kTcXGroups == 0 && kTcNB % kTcXGroups == 0 && kTcNX % kTcXGroups == 0, "group slots");
    const int grp = (threadIdx.x - kTcWarpPrep0 * 32) / kGT;  // this group takes k-blocks grp, grp + 2, ...
    const int t = threadIdx.x - kTcWarpPrep0 * 32 - grp * kGT;
    const int tok = t / TPT, part = t - (t / TPT) * TPT;
    // x k-blocks arrive by TMA, kTcNXR ahead: [2 boxes][MP tokens][64 columns]
    // (tokens past M are zero-filled)
    int xissued = 0;
    auto issue_x = [&](int b) {
      const int slot = b % kTcNXR;
      mbar_arrive_expect_tx(&xfull[slot], (uint32_t)F::kXBytes);
      tma_load_3d(fx + F::kX + slot * F::kXBytes, &xmap, &xfull[slot], 0, 0, b * 2);
      ++xissued;
    };
    if (t == 0) {
      tma_prefetch_desc(&xmap);
      for (int b = grp; b < nkb && b < kTcNXR; b += kTcXGroups) issue_x(b);
    }
    const int xc0 = part * EPT;  // first column of this thread within the k-block
    const uint32_t xsrc0 = (uint32_t)((xc0 >> 6) * (F::kXBytes / 2) + tok * 128 + (xc0 & 63) * 2);
    for (int b = grp; b < nkb; b += kTcXGroups) {
      const int s = b % F::kNB, xsl = b % kTcNX, xr = b % kTcNXR;
      const uint32_t xpar = (b / kTcNXR) & 1;
      // the x-term tile and the scalar slot free, the x k-block landed
      if (!mbar_test3(b >= F::kNB ? &bempty[s] : &xfull[xr], b >= F::kNB ? (((b / F::kNB) - 1) & 1) : xpar,
                      b >= kTcNX ? &xsempty[xsl] : &xfull[xr], b >= kTcNX ? (((b / kTcNX) - 1) & 1) : xpar, &xfull[xr],
                      xpar)) {
        if (b >= F::kNB && !(ok = mbar_wait(&bempty[s], ((b / F::kNB) - 1) & 1, p.status, 85, abort_flag))) break;
        if (b >= kTcNX && !(ok = mbar_wait(&xsempty[xsl], ((b / kTcNX) - 1) & 1, p.status, 86, abort_flag))) break;
        if (!(ok = mbar_wait(&xfull[xr], xpar, p.status, 91, abort_flag))) break;
      }
      const uint32_t xsrc = smem_u32(fx + F::kX + xr * F::kXBytes) + xsrc0;
      uint4 v[EPT / 8];
#pragma unroll
      for (int i = 0; i < EPT / 8; ++i) v[i] = lds128(xsrc + 16 * i);
      uint32_t o1[EPT / 4], o2[EPT / 4];  // term bytes, in the A operand's column order
      float sc, sx;
      tc_x_terms<FMT, BF16, EPT, TPT>(v, o1, o2, sc, sx);
      // term rows tok (T1) and MP + tok (T2) of the x-term tile
      const uint32_t bt = smem_u32(fx + F::kB + s * F::kBBytes);
#pragma unroll
      for (int cc = 0; cc < EPT / 16; ++cc) {
        const int chunk = part * (EPT / 16) + cc;
        const int ra = tok, rb = MP + tok;
        sts128(bt + ra * 128 + ((chunk ^ (ra & 7)) << 4), o1[4 * cc], o1[4 * cc + 1], o1[4 * cc + 2], o1[4 * cc + 3]);
        sts128(bt + rb * 128 + ((chunk ^ (rb & 7)) << 4), o2[4 * cc], o2[4 * cc + 1], o2[4 * cc + 2], o2[4 * cc + 3]);
      }
      if (part == 0) {
        xs[(xsl * 2) * MP + tok] = sc;
        xs[(xsl * 2 + 1) * MP + tok] = sx;
      }
      // one proxy fence orders this thread's x reads before the slot's next
      // copy and its term stores before the UMMAs that read them
      fence_proxy_async_smem();
      named_bar_sync(5 + grp, kGT);
      if (t == 0) {
        mbar_arrive(&bfull[s]);
        mbar_arrive(&xsfull[xsl]);
        if (b + kTcNXR < nkb) issue_x(b + kTcNXR);
      }
    }
    if (t == 0 && !ok) {
      // x copies in flight land before the CTA can exit: this group's i-th
      // copy is of k-block grp + i * kTcXGroups; the last kTcNXR / kTcXGroups
      // may not have been waited for
      for (int i = xissued - kTcNXR / kTcXGroups; i < xissued; ++i) {
        if (i < 0) continue;
        const int bb = grp + i * kTcXGroups;
        mbar_wait(&xfull[bb % kTcNXR], (bb / kTcNXR) & 1, nullptr, 0, nullptr);
      }
    }
    }
  } else if (warp < C::kXfr0) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;  // TMEM sub-partition: rows 32 q .. 32 q + 31
    constexpr int MPE = MP * kTcEpiWarps / C::kEpiWarps;  // token slots of this warp
    const int t0 = (warp - C::kEpi0) / kTcEpiWarps * MPE;  // its first
    const int row = q * 32 + lane;
    const bool rv = row < rvalid;
    const int n = r0 + row;
    const uint32_t tq = tmem_base + ((uint32_t)(q * 32) << 16);
    float acc[MPE];
#pragma unroll
    for (int i = 0; i < MPE; ++i) acc[i] = 0.f;
    const unsigned short* sc16 = reinterpret_cast<const unsigned short*>(p.scales);
    const unsigned short* zr16 = reinterpret_cast<const unsigned short*>(p.zeros);
    // AWQ: (scale, zero point) of this row for k-block b (0 past K or for rows past N)
    auto load_sz = [&](int b) -> uint32_t {
      if (FMT != 0 || !rv || b >= nkb) return 0u;
      const int64_t off = (int64_t)n * p.G + (b * 128) / p.group_size;
      return (uint32_t)__ldg(sc16 + off) | ((uint32_t)__ldg(zr16 + off) << 16);
    };
    // Either eight groups' scales and zero points per 16-byte load (p.sz_vec:
    // G % 8 == 0, 16-byte aligned rows), the next eight loaded when the
    // current eight start; or one (scale, zero) per k-block, four ahead.
    const bool vec = FMT == 0 && p.sz_vec && rv;
    const int kpg = FMT == 0 ? p.group_size / 128 : 1;  // k-blocks per group
    const uint4* srow = reinterpret_cast<const uint4*>(sc16 + (int64_t)n * p.G);
    const uint4* zrow = reinterpret_cast<const uint4*>(zr16 + (int64_t)n * p.G);
    const uint4 kZero4 = make_uint4(0u, 0u, 0u, 0u);
    uint4 s_cur = kZero4, z_cur = kZero4, s_nxt = kZero4, z_nxt = kZero4;
    int cur_c = 0;
    if (vec) {
      s_cur = __ldg(srow), z_cur = __ldg(zrow);
      if (p.G > 8) s_nxt = __ldg(srow + 1), z_nxt = __ldg(zrow + 1);
    }
    // four k-blocks ahead (a global load's latency is about two k-blocks' time)
    uint32_t sz0 = 0u, sz1 = 0u, sz2 = 0u, sz3 = 0u;
    if (!vec) sz0 = load_sz(0), sz1 = load_sz(1), sz2 = load_sz(2), sz3 = load_sz(3);
    for (int b = 0; b < nkb; ++b) {
      const int d = b % T::kND, xsl = b % kTcNX;
      uint32_t sz;
      if (vec) {
        const int gi = b / kpg, c = gi >> 3, j = gi & 7;
        if (c != cur_c) {
          s_cur = s_nxt, z_cur = z_nxt, cur_c = c;
          if (8 * (c + 1) < p.G) s_nxt = __ldg(srow + c + 1), z_nxt = __ldg(zrow + c + 1);
        }
        const uint32_t sw = j < 4 ? (j < 2 ? s_cur.x : s_cur.y) : (j < 6 ? s_cur.z : s_cur.w);
        const uint32_t zw = j < 4 ? (j < 2 ? z_cur.x : z_cur.y) : (j < 6 ? z_cur.z : z_cur.w);
        sz = (j & 1) ? ((sw >> 16) | (zw & 0xFFFF0000u)) : ((sw & 0xFFFFu) | (zw << 16));
      } else {
        sz = sz0;
        sz0 = sz1, sz1 = sz2, sz2 = sz3, sz3 = load_sz(b + 4);
      }
      // the accumulator and the k-block's scalars
      if (!mbar_test3(&dfull[d], (b / T::kND) & 1, &xsfull[xsl], (b / kTcNX) & 1, &xsfull[xsl], (b / kTcNX) & 1)) {
        if (!(ok = mbar_wait(&dfull[d], (b / T::kND) & 1, p.status, 87, abort_flag))) break;
        if (!(ok = mbar_wait(&xsfull[xsl], (b / kTcNX) & 1, p.status, 88, abort_flag))) break;
      }
      tc_fence_after();
      const float s = __half2float(__ushort_as_half((unsigned short)(sz & 0xFFFFu)));
      const float z = __half2float(__ushort_as_half((unsigned short)(sz >> 16)));
      // AWQ: y += s 2^e (D1 + D2 / 128) - s z 2^e (S1 + S2 / 128), with 2^e and
      // 2^e (S1 + S2 / 128) the k-block's two scalars of the token
      const float u = s * 0.0078125f, w = -s * z;
      const float4* xsc4 = reinterpret_cast<const float4*>(xs + (xsl * 2) * MP + t0);
      const float4* xsx4 = reinterpret_cast<const float4*>(xs + (xsl * 2 + 1) * MP + t0);
#pragma unroll
      for (int th = 0; th < MPE; th += 16) {
        uint32_t ra[16], rb[16];
        tmem_ld_32x32b_x16(tq + (uint32_t)(d * 2 * MP + t0 + th), ra);
        tmem_ld_32x32b_x16(tq + (uint32_t)(d * 2 * MP + MP + t0 + th), rb);
        float sc4[16], sx4[16];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 cv = xsc4[th / 4 + q4];
          sc4[4 * q4] = cv.x, sc4[4 * q4 + 1] = cv.y, sc4[4 * q4 + 2] = cv.z, sc4[4 * q4 + 3] = cv.w;
          if constexpr (FMT == 0) {
            const float4 xv = xsx4[th / 4 + q4];
            sx4[4 * q4] = xv.x, sx4[4 * q4 + 1] = xv.y, sx4[4 * q4 + 2] = xv.z, sx4[4 * q4 + 3] = xv.w;
          }
        }
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float scl = sc4[i];
          if constexpr (FMT == 0) {
            const float v = (float)((int)ra[i] * 128 + (int)rb[i]);
            acc[th + i] = fmaf(scl, u * v, fmaf(w, sx4[i], acc[th + i]));
          } else {
            acc[th + i] = fmaf(__uint_as_float(ra[i]), scl, fmaf(__uint_as_float(rb[i]), scl * 0.0625f, acc[th + i]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&dempty[d]);
        mbar_arrive(&xsempty[xsl]);
      }
    }
    if (rv && ok) {
      const float ws = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
      const float bn = p.bias_dtype != NSQ_DTYPE_NONE ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
      uint16_t* y = static_cast<uint16_t*>(p.y);
#pragma unroll
      for (int i = 0; i < MPE; ++i) {
        if (t0 + i < p.M) {
          const float v = acc[i] * ws + bn;
          y[(int64_t)(t0 + i) * p.N + n] = float_to_elem<BF16>(v);
        }
      }
    }
  } else if constexpr (C::kTmemA) {
    // ---------------- AWQ weight transfer: ring slot -> tensor-memory A tiles ----------------
    // Lane i of warp w holds weight row 32 (w % 4) + i (its TMEM lane). A ring
    // slot is two k-blocks; the row's 128 bytes are 16-byte chunks c at
    // ((c ^ (row & 7)) << 4) (128-byte swizzle), k-block h = chunks 4h .. 4h + 3.
    // Chunk rc of a k-block (32 columns of nibbles) becomes columns
    // 8 rc .. 8 rc + 7 of its A tile: per word the bytes of nibbles 0,2,4,6
    // (w & 0x0F0F0F0F), then 1,3,5,7 ((w >> 4) & 0x0F0F0F0F), the order the x
    // terms are packed in. Rows past the CTA's store zeros (their accumulator
    // lanes are never read). Per slot: all loads, both k-blocks' stores, one
    // tcgen05.wait::st.
    // With two groups, group g takes ring slots g, g + 2, ... (k-blocks 4i + 2g
    // and 4i + 2g + 1: A tiles 2g and 2g + 1).
    const int q = warp & 3;
    static_assert(C::kXfrGroups == 1 || (kTcNA == 4 && KPS == 2), "two groups: A tiles 0-1 and 2-3");
    const int grp = (warp - C::kXfr0) / kTcXfrWarps;
    const int row = q * 32 + lane;
    const bool rin = row < rows;
    const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16);  // this warp's 32 lanes
    const int nst = (nkb + KPS - 1) / KPS;
    for (int st = grp; st < nst && ok; st += C::kXfrGroups) {
      const int rs = st % NS, b0 = KPS * st, nb = min(KPS, nkb - b0);
      const uint32_t wpar = (st / NS) & 1;
      if (!__all_sync(0xffffffffu, mbar_test1(&wfull[rs], wpar))) {
        ok = __all_sync(0xffffffffu, mbar_wait(&wfull[rs], wpar, p.status, 89, abort_flag));
        if (!ok) break;
      }
      const uint32_t src = smem_u32(smem) + (uint32_t)rs * tile + (uint32_t)row * 128u;
      uint4 w[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) w[c] = rin ? lds128(src + ((c ^ (row & 7)) << 4)) : make_uint4(0u, 0u, 0u, 0u);
      fence_proxy_async_smem();  // these reads precede the slot's next TMA write
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[rs]);
      // the UMMAs of k-block b - kTcNA have read tile b % kTcNA
      for (int j = 0; j < nb; ++j) {
        const int b = b0 + j;
        if (b < kTcNA) continue;
        const uint32_t apar = ((b / kTcNA) - 1) & 1;
        if (!__all_sync(0xffffffffu, mbar_test1(&aempty[b % kTcNA], apar))) {
          ok = __all_sync(0xffffffffu, mbar_wait(&aempty[b % kTcNA], apar, p.status, 90, abort_flag));
          if (!ok) break;
        }
      }
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < KPS; ++h) {
        if (h >= nb) break;
        uint32_t v0[16], v1[16];
#pragma unroll
        for (int rc = 0; rc < 4; ++rc) {
          const uint4 u = w[4 * h + rc];
          uint32_t* o = rc < 2 ? v0 + 8 * rc : v1 + 8 * (rc - 2);
          o[0] = u.x & 0x0F0F0F0Fu, o[1] = (u.x >> 4) & 0x0F0F0F0Fu;
          o[2] = u.y & 0x0F0F0F0Fu, o[3] = (u.y >> 4) & 0x0F0F0F0Fu;
          o[4] = u.z & 0x0F0F0F0Fu, o[5] = (u.z >> 4) & 0x0F0F0F0Fu;
          o[6] = u.w & 0x0F0F0F0Fu, o[7] = (u.w >> 4) & 0x0F0F0F0Fu;
        }
        const uint32_t ta = tl + T::kA + 32u * (uint32_t)((b0 + h) % kTcNA);
        tmem_st_32x32b_x16(ta, v0);
        tmem_st_32x32b_x16(ta + 16, v1);
      }
      tmem_st_wait();
      tc_fence_before();  // the stores precede the UMMAs that the arrivals release
      __syncwarp();
      if (lane == 0) {
        for (int j = 0; j < nb; ++j) mbar_arrive(&afull[(b0 + j) % kTcNA]);
      }
    }
  }
  __syncthreads();
  if (warp == kTcWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, T::kCols);
  }
}

// The x terms of one launch, once (one CTA per k-block, eight adjacent
// threads per token slot, 16 columns each): the x-term tile of k-block b as rows
// [b * 2 MP, b * 2 MP + 2 MP) of 128 bytes (T1 rows of the MP token slots,
// then their T2 rows; unswizzled, the tensor map swizzles on the way in) and
// its scalars xsg[b][0][tok] = 2^e, xsg[b][1][tok] = term sum (AWQ). Token
// slots past M get zero terms.
template <int FMT, bool BF16, int MP>
__global__ void __launch_bounds__(MP * 8) tc_xterm_kernel(const void* x, int M, int K, uint8_t* xt, float* xsg) {
  pdl_launch_dependents();
  pdl_wait_prior_grids();  // x is written by the previous kernel
  constexpr int TPT = 8, EPT = 128 / TPT;
  const int b = (int)blockIdx.x, t = (int)threadIdx.x;
  const int tok = t / TPT, part = t - (t / TPT) * TPT;
  uint4 v[EPT / 8];
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + (int64_t)tok * K + b * 128 +
                                                    part * EPT);
#pragma unroll
  for (int i = 0; i < EPT / 8; ++i) v[i] = tok < M ? __ldg(src + i) : make_uint4(0u, 0u, 0u, 0u);
  uint32_t o1[EPT / 4], o2[EPT / 4];
  float sc, sx;
  tc_x_terms<FMT, BF16, EPT, TPT>(v, o1, o2, sc, sx);
  uint4* rows = reinterpret_cast<uint4*>(xt + (int64_t)b * 2 * MP * 128);
#pragma unroll
  for (int cc = 0; cc < EPT / 16; ++cc) {
    const int chunk = part * (EPT / 16) + cc;
    rows[tok * 8 + chunk] = make_uint4(o1[4 * cc], o1[4 * cc + 1], o1[4 * cc + 2], o1[4 * cc + 3]);
    rows[(MP + tok) * 8 + chunk] = make_uint4(o2[4 * cc], o2[4 * cc + 1], o2[4 * cc + 2], o2[4 * cc + 3]);
  }
  if (part == 0) {
    xsg[(int64_t)b * 2 * MP + tok] = sc;
    xsg[(int64_t)b * 2 * MP + MP + tok] = sx;
  }
}

template <int FMT, bool BF16, int MP>
cudaError_t launch_xterm(const void* x, int M, int K, uint8_t* xt, float* xsg, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(K / 128, 1, 1);
  cfg.blockDim = dim3(MP * 8, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    na = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, tc_xterm_kernel<FMT, BF16, MP>, x, M, K, xt, xsg);
}

template <int FMT, bool BF16, int MP, bool PRE>
cudaError_t launch_tc(const CUtensorMap& wlo, const CUtensorMap& whi, const CUtensorMap& xmap, const TcParams& p,
                      int grid, cudaStream_t stream) {
  auto kern = decode_tc_kernel<FMT, BF16, MP, PRE>;
  static std::atomic<bool> configured{false};
  if (!configured.load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TcMem<FMT, MP, PRE>::kSmem);
    if (e != cudaSuccess) return e;
    configured.store(true);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(TcCfg<FMT, MP, PRE>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)p.off_fixed + TcFixed<MP, PRE>::kBytes + 1024;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    na = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, wlo, whi, xmap, p);
}

template <int FMT, bool BF16>
cudaError_t dispatch_tc(int mp, bool pre, const CUtensorMap& wlo, const CUtensorMap& whi, const CUtensorMap& xmap,
                        const TcParams& p, int grid, const void* x, uint8_t* xt, cudaStream_t s) {
  if (pre) {
    float* xsg = const_cast<float*>(p.xsg);
    cudaError_t e = mp == 16   ? launch_xterm<FMT, BF16, 16>(x, p.M, p.K, xt, xsg, s)
                    : mp == 32 ? launch_xterm<FMT, BF16, 32>(x, p.M, p.K, xt, xsg, s)
                               : launch_xterm<FMT, BF16, 64>(x, p.M, p.K, xt, xsg, s);
    if (e != cudaSuccess) return e;
    return mp == 16   ? launch_tc<FMT, BF16, 16, true>(wlo, whi, xmap, p, grid, s)
           : mp == 32 ? launch_tc<FMT, BF16, 32, true>(wlo, whi, xmap, p, grid, s)
                      : launch_tc<FMT, BF16, 64, true>(wlo, whi, xmap, p, grid, s);
  }
  if (mp == 64) return cudaErrorInvalidValue;  // 64 token slots only with precomputed terms
  return mp == 16 ? launch_tc<FMT, BF16, 16, false>(wlo, whi, xmap, p, grid, s)
                  : launch_tc<FMT, BF16, 32, false>(wlo, whi, xmap, p, grid, s);
}

}  // namespace

namespace {
// Rows per CTA in multiples of 8 (so every k-block tile of a stage stays on a
// 1 KB swizzle boundary): rlo for most CTAs, rlo + 8 for the first nhi.
bool tc_rows(const LinearArgs& a, int* rlo, int* nhi, int* grid) {
  if (a.M < 1 || a.M > 64 || a.K % 128 != 0 || a.K < 256) return false;
  if (a.fmt == 0 && (a.K % 256 != 0 || a.group_size % 128 != 0 || a.K % a.group_size != 0)) return false;
  const int sms = num_sms();
  const int g8 = (a.N + 7) / 8;
  // one CTA per SM, or fewer on smaller layers so that a CTA keeps >= 64 rows
  const int c = g8 / 8 < sms ? (g8 / 8 > 0 ? g8 / 8 : 1) : sms;
  const int base = g8 / c, rem = g8 - base * c;
  *rlo = 8 * base;
  *nhi = rem;
  *grid = c;
  return *rlo >= 64 && *rlo + (rem > 0 ? 8 : 0) <= kTcM;
}
}  // namespace

// Rows of the tallest CTA for the tensor-core decode kernel, 0 if it does not apply.
int decode_tc_rows(const LinearArgs& a) {
  int rlo, nhi, grid;
  if (!tc_rows(a, &rlo, &nhi, &grid)) return 0;
  return rlo + (nhi > 0 ? 8 : 0);
}

// token slots of a launch: 16, 32 or 64 (64 only with precomputed x terms)
static int tc_slots(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : 64; }

size_t decode_tc_workspace_bytes(const LinearArgs& a) {
  const int64_t nkb = a.K / 128, rows = nkb * 2 * tc_slots(a.M);
  return (size_t)(rows * 128 + rows * 4);
}

int run_decode_tc_linear(const LinearArgs& a, cudaStream_t stream) {
  int rlo, nhi, grid;
  if (!tc_rows(a, &rlo, &nhi, &grid)) return NSQ_ENOTSUP;
  const int rmax = rlo + (nhi > 0 ? 8 : 0);
  const int mp = tc_slots(a.M);
  // with a workspace, the x terms are computed once by tc_xterm_kernel: the
  // terms [nkb x 2 mp rows][128 B], then the scalars [nkb][2][mp] fp32
  const bool pre = a.ws != nullptr && a.ws_bytes >= decode_tc_workspace_bytes(a) && ((uintptr_t)a.ws & 15) == 0;
  uint8_t* xt = static_cast<uint8_t*>(a.ws);
  if (mp == 64 && !pre) return NSQ_ENOTSUP;
  TcParams p{};
  p.x = a.x;
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.zeros = reinterpret_cast<const __half*>(a.zeros);
  p.wscale = a.wscale;
  p.bias = a.bias;
  p.y = a.y;
  p.status = device_status_ptr();
  p.M = a.M;
  p.K = a.K;
  p.N = a.N;
  p.group_size = a.fmt == 0 ? a.group_size : 0;
  p.G = a.fmt == 0 ? a.K / a.group_size : 0;
  p.sz_vec = a.fmt == 0 && p.G % 8 == 0 && ((uintptr_t)a.scales & 15) == 0 && ((uintptr_t)a.zeros & 15) == 0;
  p.bias_dtype = a.bias ? a.bias_dtype : NSQ_DTYPE_NONE;
  p.rlo = rlo;
  p.nhi = nhi;
  p.nkb = a.K / 128;
  // Shared memory: the weight ring (sized to what is left, at most kTcMaxNS
  // slots of the tallest CTA's rows x 128 B), then the fixed part.
  p.tile = rmax * 128;
  const int fixed = pre ? (mp == 16 ? TcFixed<16, true>::kBytes : mp == 32 ? TcFixed<32, true>::kBytes
                                                                        : TcFixed<64, true>::kBytes)
                        : (mp == 16 ? TcFixed<16, false>::kBytes : TcFixed<32, false>::kBytes);
  const int room = kTcSmemMax - 1024 - fixed;
  p.ns = room / p.tile;
  if (p.ns > kTcMaxNS) p.ns = kTcMaxNS;
  p.off_fixed = p.ns * p.tile;
  if (p.ns < 4) return NSQ_ENOTSUP;
  // weights as 32-bit words [N rows x K/8 (AWQ) or K/4 (FP8)], boxes of
  // [rows of the CTA x 32 words = 128 B], 128-byte swizzle
  const uint64_t row_bytes = a.fmt == 0 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  CUtensorMap wmap_lo, wmap_hi;
  CUresult cr = encode_tensor_map_2d(&wmap_lo, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq), row_bytes / 4,
                                     (uint64_t)a.N, row_bytes, 32, (uint32_t)rlo, CU_TENSOR_MAP_SWIZZLE_128B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  cr = encode_tensor_map_2d(&wmap_hi, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq), row_bytes / 4,
                            (uint64_t)a.N, row_bytes, 32, (uint32_t)rmax, CU_TENSOR_MAP_SWIZZLE_128B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  CUtensorMap xmap;
  if (pre) {
    // the precomputed terms as 32-bit words [nkb * 2 mp rows x 32 words], one
    // box of [2 mp rows x 128 B] per k-block, 128-byte swizzle
    const uint64_t trows = (uint64_t)p.nkb * 2 * mp;
    p.xsg = reinterpret_cast<const float*>(xt + trows * 128);
    cr = encode_tensor_map_2d(&xmap, CU_TENSOR_MAP_DATA_TYPE_INT32, xt, 32, trows, 128, 32, (uint32_t)(2 * mp),
                              CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    // x, rank 3: [64-column halves of a k-block][tokens][64 columns] 16-bit,
    // one box of [2][mp][64] per k-block (tokens past M read as zero)
    cr = encode_tensor_map_3d(&xmap, a.x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              const_cast<void*>(a.x), 64, (uint64_t)a.M, (uint64_t)a.K / 64, (uint64_t)a.K * 2, 128,
                              64, (uint32_t)mp, 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  cudaError_t e;
  if (a.fmt == 0) {
    e = a.x_bf16 ? dispatch_tc<0, true>(mp, pre, wmap_lo, wmap_hi, xmap, p, grid, a.x, xt, stream)
                 : dispatch_tc<0, false>(mp, pre, wmap_lo, wmap_hi, xmap, p, grid, a.x, xt, stream);
  } else {
    e = a.x_bf16 ? dispatch_tc<1, true>(mp, pre, wmap_lo, wmap_hi, xmap, p, grid, a.x, xt, stream)
                 : dispatch_tc<1, false>(mp, pre, wmap_lo, wmap_hi, xmap, p, grid, a.x, xt, stream);
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // namespace nsq
