// Row-streaming decode linear (M <= 32 tokens): every CTA owns a contiguous
// block of output rows and streams its weight rows through a shared-memory
// ring, 256 bytes of every row per stage, while its warps consume the stages
// already landed. HBM-bound on the weight bytes.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152 and :49-52) for small batches, and serves the fused
// projections (q/k/v as one launch over the three weights; gate/up as one
// launch whose epilogue applies SiLU(gate) * up, the MLP of
// nano_sglang/model/causal_lm.py:482).
//
// Why this shape (measured on B200 with a pure TMA ring, 148 CTAs): stages of
// 28-64 KB stream at 5.7-6.3 TB/s whatever the length of the row runs (256 B
// or 1 KB per row), stages of 16 KB at 3-4 TB/s. A stage here is the CTA's
// rows x 256 B: two boxes of [rows x 128 B] (128-byte swizzle, so the eight
// rows a fragment load touches fall in eight bank groups) plus the matching
// x columns, [tokens x 64] boxes with the same swizzle. The rows of a CTA are
// fixed for the whole launch, so each warp keeps its accumulators in
// registers across all K stages; no global workspace, no second pass.
//
// Roles: consumer warps (R row groups of 16 rows x KW warps per row group,
// KW splitting every stage's four pieces) and one producer warp whose
// elected lane keeps the ring full. Weights are static: the first stages'
// weight boxes are requested before griddepcontrol.wait, x only after it.
//
// AWQ arithmetic is the one of the other decode kernels: a word of eight
// sequential nibbles becomes four pairs {magic+q_t, magic+q_{t+4}} with one
// lop3 each and x pairs are built to match with prmt; integer zero points are
// subtracted in the packed domain (exact), any other zero point is folded per
// 128-column piece through per-token sums of x: y += s (sum (magic+q) x -
// (magic+z) sum x). FP8: integer-only e4m3 -> MMA type, per-tensor scale in
// the epilogue. Every wait is bounded (nsq_common.cuh).
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"
#include "nsq_tmem_operand.cuh"

namespace nsq {

namespace {

constexpr int kMaxR = 15;   // row groups per CTA
constexpr int kMaxCW = 15;  // consumer warps (+ the producer: 512 threads, so up to 128 registers each)
constexpr int kThreadsRows = (kMaxCW + 1) * 32;
constexpr int kRowsSmem = 200 * 1024;
constexpr int kRedStrideR = 17;  // fp32 per token of a partial 16-row tile (conflict-free)

template <int FMT>
struct RowsFmt;
template <>
struct RowsFmt<0> {  // AWQ: 256 B of a row = 512 columns = 4 pieces of 128 (one scale group slice each)
  static constexpr int kSK = 512;
  static constexpr int kPieceK = 128;
};
template <>
struct RowsFmt<1> {  // FP8: 256 B of a row = 256 columns = 4 pieces of 64
  static constexpr int kSK = 256;
  static constexpr int kPieceK = 64;
};

struct RowsSeg {
  const __half* scales;  // AWQ [n, G]
  const __half* zeros;   // AWQ [n, G]
  const float* wscale;   // FP8 per-tensor scale (device)
  const void* bias;      // [n] or null
  int n;                 // output rows of this weight (features)
  int ycol;              // first column of y it writes (mode 0)
  int cta0;              // first CTA serving it (mode 0)
  int rbase, rrem;       // row groups of its i-th CTA: rbase + (i < rrem)
};

struct RowsParams {
  const void* x;
  void* y;
  DevStatus* status;
  int M, K, ldy;
  int G, group_size;  // AWQ
  int nstage, nst;    // K stages, ring depth
  int R, KW;          // row groups per CTA (most), warps per row group
  int bias_dtype;
  int mode;           // 0: y[:, seg] = x W_seg^T; 1: y = SiLU(x Wg^T) * (x Wu^T), seg 0 gate, seg 1 up
  int small_group;    // AWQ groups of 32 / 64 columns: dequantise before the MMA
  int nsegs;
  RowsSeg seg[3];
  int rows_half;      // smem rows of one weight half-box region (16 R)
  int stage_bytes;    // smem bytes of one stage (weights + x)
  int xoff;           // offset of the x boxes inside a stage
  int off_red, off_xs, off_bar;
};

// Weight maps: [2 * seg] = box of (16 or 8) * rbase rows, [2 * seg + 1] = one
// row group (16 or 8 rows); both 32 x int32 = 128 B wide, 128-byte swizzle.
struct RowsMaps {
  CUtensorMap m[6];
};

template <bool BF16>
__device__ __forceinline__ uint32_t rows_hsub2(uint32_t a, uint32_t b) {
  if constexpr (BF16) {
    __nv_bfloat162 r = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  } else {
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t rows_pair(float v) {
  if constexpr (BF16) {
    __nv_bfloat162 b = __floats2bfloat162_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&b);
  } else {
    __half2 h = __floats2half2_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// address of 16-byte chunk q of row `row` in a 128-byte-swizzled box region
__device__ __forceinline__ uint32_t sw128(uint32_t base, int row, int q) {
  return base + (uint32_t)row * 128u + ((uint32_t)(q ^ (row & 7)) << 4);
}

// Two e4m3 codes (low byte first) -> f16x2, exact (every e4m3 value is an
// fp16 value), with the hardware conversion.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t codes16) {
  uint32_t d;
  asm("{\n\t.reg .b16 c;\n\tcvt.u16.u32 c, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, c;\n\t}" : "=r"(d) : "r"(codes16));
  return d;
}

// bf16 pair -> fp16 pair of the values times 2^-8, rounded to nearest. Exact
// for |x| in [2^-6, 2^24); smaller values keep the fp16 subnormal precision,
// which only they lose (their products are below 2^-6 of the weight's).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2_scaled(uint32_t v) {
  const float lo = __uint_as_float(v << 16) * 0.00390625f;
  const float hi = __uint_as_float(v & 0xFFFF0000u) * 0.00390625f;
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <bool BF16>
__device__ __forceinline__ float chunk_sum8(const uint4& v) {
  const uint32_t r[4] = {v.x, v.y, v.z, v.w};
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) s += elem_to_float<BF16>((uint16_t)(r[e] & 0xFFFFu)) + elem_to_float<BF16>((uint16_t)(r[e] >> 16));
  return s;
}

template <int FMT, bool BF16, int MT, int KW>
__global__ void __launch_bounds__(kThreadsRows, 1) decode_rows_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                       const __grid_constant__ RowsMaps maps,
                                                                       const RowsParams p) {
  using F = RowsFmt<FMT>;
  constexpr int MPAD = MT * 8;
  constexpr int kXBoxes = F::kSK / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* fullw = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* fullx = fullw + p.nst;
  uint64_t* empty = fullx + p.nst;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + p.nst);
  int* int_z_flag = const_cast<int*>(reinterpret_cast<volatile int*>(empty + p.nst) + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncw = p.R * KW;  // consumer warps; the producer is warp ncw
  const int cta = blockIdx.x;

  // this CTA's weight segment and row groups
  int si = 0;
  if (p.mode == 0) {
    while (si + 1 < p.nsegs && cta >= p.seg[si + 1].cta0) ++si;
  }
  const RowsSeg& S = p.seg[si];
  const int li = cta - S.cta0;
  const int Rc = S.rbase + (li < S.rrem ? 1 : 0);
  const int rg0 = li * S.rbase + (li < S.rrem ? li : S.rrem);
  // mode 0: rows [16 rg0, 16 (rg0 + Rc)) of weight si; mode 1: features
  // [8 rg0, 8 (rg0 + Rc)) of gate (seg 0) and up (seg 1)
  const int rowpg = p.mode == 0 ? 16 : 8;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nst; ++i) {
      mbar_init(&fullw[i], 1);
      mbar_init(&fullx[i], 1);
      mbar_init(&empty[i], ncw);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  bool ok = true;
  if (warp == ncw) {
    // ---------------- producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&xmap);
      const int nwt = p.mode == 0 ? 1 : 2;  // weights read by this CTA
      auto issue_w = [&](int s, int slot) {
        uint32_t bytes = 0;
        for (int t = 0; t < nwt; ++t) bytes += (uint32_t)(Rc * rowpg) * 128u * 2u;
        mbar_arrive_expect_tx(&fullw[slot], bytes);
        for (int t = 0; t < nwt; ++t) {
          const int sg = p.mode == 0 ? si : t;
          // mode 0: rows at smem row 0; mode 1: gate rows at 0, up rows at 8 R
          const int srow0 = t * 8 * p.R;
          for (int h = 0; h < 2; ++h) {
            const int c0 = s * 64 + h * 32;  // int32 column of this 128-byte half
            uint8_t* dst = smem + (size_t)slot * p.stage_bytes + (size_t)h * p.rows_half * 128 + (size_t)srow0 * 128;
            tma_load_2d(dst, &maps.m[2 * sg], &fullw[slot], c0, rg0 * rowpg);
            if (Rc > S.rbase) {
              tma_load_2d(dst + (size_t)S.rbase * rowpg * 128, &maps.m[2 * sg + 1], &fullw[slot], c0,
                          (rg0 + S.rbase) * rowpg);
            }
          }
        }
      };
      auto issue_x = [&](int s, int slot) {
        mbar_arrive_expect_tx(&fullx[slot], (uint32_t)(kXBoxes * MPAD * 128));
        uint8_t* dst = smem + (size_t)slot * p.stage_bytes + p.xoff;
        for (int b = 0; b < kXBoxes; ++b) tma_load_2d(dst + b * MPAD * 128, &xmap, &fullx[slot], s * F::kSK + b * 64, 0);
      };
      const int pre = p.nstage < p.nst ? p.nstage : p.nst;
      for (int s = 0; s < pre; ++s) issue_w(s, s);
      int issued_w = pre, issued_x = 0;
      pdl_wait_prior_grids();  // x may be written by the previous kernel
      for (int s = 0; s < p.nstage; ++s) {
        const int slot = s % p.nst;
        if (s >= p.nst) {
          // the consumers released the slot, and its previous copies landed
          // (they did unless a consumer gave up), so no two loads of a slot overlap
          const uint32_t prev = ((s / p.nst) - 1) & 1;
          if (!(ok = mbar_wait(&empty[slot], prev, p.status, 70, abort_flag))) break;
          if (!(ok = mbar_wait(&fullw[slot], prev, p.status, 73, abort_flag))) break;
          if (!(ok = mbar_wait(&fullx[slot], prev, p.status, 74, abort_flag))) break;
          issue_w(s, slot);
          ++issued_w;
        }
        issue_x(s, slot);
        ++issued_x;
      }
      // the producer leaves only once every copy it requested has landed, so
      // nothing is in flight into this CTA's shared memory when it exits
      for (int j = (issued_w > p.nst ? issued_w - p.nst : 0); j < issued_w; ++j) {
        mbar_wait(&fullw[j % p.nst], (j / p.nst) & 1, nullptr, 0, nullptr);
      }
      for (int j = (issued_x > p.nst ? issued_x - p.nst : 0); j < issued_x; ++j) {
        mbar_wait(&fullx[j % p.nst], (j / p.nst) & 1, nullptr, 0, nullptr);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int r = warp / KW;  // row group within the CTA
  const int kw = warp - r * KW;
  const bool active = r < Rc;
  const int g = lane >> 2, c = lane & 3;
  // smem rows of this thread's two fragment rows (g and g + 8 of the 16)
  int srow_a, srow_b;
  int n_a, n_b;                 // weight rows (global, within their weight) of those fragment rows
  const RowsSeg& Sa = S;
  const RowsSeg& Sb = p.mode == 0 ? S : p.seg[1];
  // Fragment row g reads weight row pg = {0,4,1,5,2,6,3,7}[g] of its eight:
  // the four lanes of g = 2i and of g = 2i + 1 (one phase of a 16-byte shared
  // load) then read rows whose 128-byte swizzle patterns differ by 4, i.e.
  // opposite halves of the bank space (conflict-free). Outputs follow pg.
  const int pg = (g >> 1) | ((g & 1) << 2);
  if (p.mode == 0) {
    srow_a = 16 * r + pg;
    srow_b = srow_a + 8;
    n_a = 16 * (rg0 + r) + pg;
    n_b = n_a + 8;
  } else {
    srow_a = 8 * r + pg;
    srow_b = 8 * p.R + 8 * r + pg;
    n_a = 8 * (rg0 + r) + pg;
    n_b = n_a;
  }

  // AWQ: are all zero points of this CTA integers the MMA type holds exactly
  // (what the reference quantiser writes)? Then q - z is formed exactly in
  // the packed domain; otherwise the zero point is folded through sums of x.
  bool int_z = true;
  if constexpr (FMT == 0) {
    constexpr float kZMax = BF16 ? 127.0f : 1023.0f;
    const int nw = p.mode == 0 ? 1 : 2;
    const int rows = Rc * rowpg;
    const int total = nw * rows * p.G;
    const int nthr = ncw * 32;
    for (int idx = threadIdx.x; idx < total; idx += nthr) {
      const int t = idx / (rows * p.G);
      const int rem = idx - t * rows * p.G;
      const int rr = rem / p.G;
      const int gg = rem - rr * p.G;
      const RowsSeg& W = p.mode == 0 ? S : p.seg[t];
      const int n = rg0 * rowpg + rr;
      if (n < W.n) {
        const float z = __half2float(W.zeros[(int64_t)n * p.G + gg]);
        int_z = int_z && z == rintf(z) && fabsf(z) <= kZMax;
      }
    }
    if (threadIdx.x == 0) *int_z_flag = 1;
    named_bar_sync(1, ncw * 32);
    if (!int_z) atomicAnd(int_z_flag, 0);
    named_bar_sync(1, ncw * 32);
    int_z = *reinterpret_cast<volatile int*>(int_z_flag) != 0;
  }
  const bool va = n_a < Sa.n, vb = n_b < Sb.n;

  float acc[MT][4];
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) acc[jt][0] = acc[jt][1] = acc[jt][2] = acc[jt][3] = 0.f;

  const unsigned short* sca = reinterpret_cast<const unsigned short*>(Sa.scales);
  const unsigned short* zra = reinterpret_cast<const unsigned short*>(Sa.zeros);
  const unsigned short* scb = reinterpret_cast<const unsigned short*>(Sb.scales);
  const unsigned short* zrb = reinterpret_cast<const unsigned short*>(Sb.zeros);
  constexpr float kMagic = Magic<BF16>::kValue;

  // Per-thread shared-memory offsets inside a stage, the same for every stage:
  // the weight chunks of this warp's pieces (two rows each), the row of token
  // g in the first x box of each piece, and the swizzled 16-byte chunk of each
  // x load within its row (AWQ: chunk (4c + i) of the piece's 128 columns,
  // box 2j + c / 2; FP8: chunk 2c + h of box j). Token 8 jt + g lies jt KB
  // further (8 rows of 128 B).
  constexpr int NJ = 4 / KW;
  uint32_t woff_a[NJ], woff_b[NJ], xoff_j[NJ];
#pragma unroll
  for (int jj = 0; jj < NJ; ++jj) {
    const int j = kw + jj * KW;
    const int half = j >> 1, cq = ((j & 1) << 2) + c;
    woff_a[jj] = (uint32_t)(half * p.rows_half * 128 + srow_a * 128 + ((cq ^ (srow_a & 7)) << 4));
    woff_b[jj] = (uint32_t)(half * p.rows_half * 128 + srow_b * 128 + ((cq ^ (srow_b & 7)) << 4));
    const int box = FMT == 0 ? 2 * j + (c >> 1) : j;
    xoff_j[jj] = (uint32_t)(p.xoff + box * MPAD * 128 + g * 128);
  }
  uint32_t xq[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = FMT == 0 ? ((4 * c + i) & 7) : ((2 * c + i) & 7);
    xq[i] = (uint32_t)((q ^ g) << 4);
  }

  // AWQ: this thread's (scale, zero point) pairs of a stage's pieces, as fp16
  // bits {scale | zero << 16} per row; the next stage's are loaded while the
  // current one computes, so their latency hides behind a whole stage
  uint32_t nsz_a[4], nsz_b[4];
  auto load_sz = [&](int st) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      nsz_a[j] = nsz_b[j] = 0u;
      const int kk = st * F::kSK + j * F::kPieceK;
      if (FMT == 0 && active && st < p.nstage && (j % KW) == kw && kk < p.K) {
        // this thread's 32 columns of the piece lie in one group for groups of
        // 32, 64 and multiples of 128
        const int gi = (p.small_group ? kk + 32 * c : kk) / p.group_size;
        if (va) nsz_a[j] = (uint32_t)__ldg(sca + (int64_t)n_a * p.G + gi) | ((uint32_t)__ldg(zra + (int64_t)n_a * p.G + gi) << 16);
        if (vb) nsz_b[j] = (uint32_t)__ldg(scb + (int64_t)n_b * p.G + gi) | ((uint32_t)__ldg(zrb + (int64_t)n_b * p.G + gi) << 16);
      }
    }
  };
  if constexpr (FMT == 0) load_sz(0);

  for (int s = 0; s < p.nstage; ++s) {
    const int slot = s % p.nst;
    const uint32_t ph = (s / p.nst) & 1;
    float sa[4], za[4], sb[4], zb[4];
    if constexpr (FMT == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sa[j] = __half2float(__ushort_as_half((unsigned short)(nsz_a[j] & 0xFFFFu)));
        za[j] = __half2float(__ushort_as_half((unsigned short)(nsz_a[j] >> 16)));
        sb[j] = __half2float(__ushort_as_half((unsigned short)(nsz_b[j] & 0xFFFFu)));
        zb[j] = __half2float(__ushort_as_half((unsigned short)(nsz_b[j] >> 16)));
      }
      load_sz(s + 1);
    }
    if (ok) ok = mbar_wait(&fullw[slot], ph, p.status, 71, abort_flag);
    if (ok) ok = mbar_wait(&fullx[slot], ph, p.status, 72, abort_flag);
    if constexpr (FMT == 1 && BF16) {
      // FP8 runs the MMA in fp16: the e4m3 codes convert with one hardware
      // instruction per pair (the integer route to bf16 takes five). The
      // stage's bf16 x is rewritten in place as fp16 of x * 2^-8 (scaled back
      // in the epilogue), every 16-byte chunk once by one consumer thread.
      if (ok) {
        const uint32_t xb = smem_u32(smem + (size_t)slot * p.stage_bytes + p.xoff);
        constexpr int kChunks = kXBoxes * MPAD * 8;
        for (int i = threadIdx.x; i < kChunks; i += ncw * 32) {
          const uint4 v = lds128(xb + i * 16);
          sts128(xb + i * 16, bf16x2_to_f16x2_scaled(v.x), bf16x2_to_f16x2_scaled(v.y),
                 bf16x2_to_f16x2_scaled(v.z), bf16x2_to_f16x2_scaled(v.w));
        }
      }
      // every consumer warp passes here once per stage, aborted or not
      named_bar_sync(3, ncw * 32);
    }
    if (ok && active) {
      const uint32_t sbase = smem_u32(smem + (size_t)slot * p.stage_bytes);
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) {
        const int j = kw + jj * KW;
        const uint4 wa = lds128(sbase + woff_a[jj]);
        const uint4 wbv = lds128(sbase + woff_b[jj]);
        const uint32_t wg[4] = {wa.x, wa.y, wa.z, wa.w};
        const uint32_t wh[4] = {wbv.x, wbv.y, wbv.z, wbv.w};
        const uint32_t xrow = sbase + xoff_j[jj];  // this thread's x row (token g) in the piece's first box
        if constexpr (FMT == 0) {
          if (p.small_group) {
            // groups of 32 / 64: every thread's columns carry their own scale,
            // so the weights are dequantised before the MMA (as the prefill
            // converters do) and accumulate straight into acc
            const TsRowDq<BF16> rpa = ts_row_dq<BF16>(sa[j], za[j]);
            const TsRowDq<BF16> rpb = ts_row_dq<BF16>(sb[j], zb[j]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t eg[4], eh[4];
              unpack_nibble_pairs<BF16>(wg[i], eg);
              unpack_nibble_pairs<BF16>(wh[i], eh);
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                eg[t] = ts_dq2<BF16>(eg[t], rpa);
                eh[t] = ts_dq2<BF16>(eh[t], rpb);
              }
              const uint32_t a0[4] = {eg[0], eh[0], eg[1], eh[1]};
              const uint32_t a1[4] = {eg[2], eh[2], eg[3], eh[3]};
#pragma unroll
              for (int jt = 0; jt < MT; ++jt) {
                const uint4 v = lds128(xrow + xq[i] + jt * 1024);
                mma_16816<BF16>(acc[jt], a0, prmt(v.x, v.z, 0x5410), prmt(v.x, v.z, 0x7632));
                mma_16816<BF16>(acc[jt], a1, prmt(v.y, v.w, 0x5410), prmt(v.y, v.w, 0x7632));
              }
            }
            continue;
          }
          float part[MT][4];
#pragma unroll
          for (int jt = 0; jt < MT; ++jt) part[jt][0] = part[jt][1] = part[jt][2] = part[jt][3] = 0.f;
          const uint32_t zpa = rows_pair<BF16>(kMagic + za[j]);
          const uint32_t zpb = rows_pair<BF16>(kMagic + zb[j]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t eg[4], eh[4];
            unpack_nibble_pairs<BF16>(wg[i], eg);
            unpack_nibble_pairs<BF16>(wh[i], eh);
            if (int_z) {
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                eg[t] = rows_hsub2<BF16>(eg[t], zpa);
                eh[t] = rows_hsub2<BF16>(eh[t], zpb);
              }
            }
            const uint32_t a0[4] = {eg[0], eh[0], eg[1], eh[1]};
            const uint32_t a1[4] = {eg[2], eh[2], eg[3], eh[3]};
#pragma unroll
            for (int jt = 0; jt < MT; ++jt) {
              const uint4 v = lds128(xrow + xq[i] + jt * 1024);
              mma_16816<BF16>(part[jt], a0, prmt(v.x, v.z, 0x5410), prmt(v.x, v.z, 0x7632));
              mma_16816<BF16>(part[jt], a1, prmt(v.y, v.w, 0x5410), prmt(v.y, v.w, 0x7632));
            }
          }
          if (int_z) {
#pragma unroll
            for (int jt = 0; jt < MT; ++jt) {
              acc[jt][0] = fmaf(sa[j], part[jt][0], acc[jt][0]);
              acc[jt][1] = fmaf(sa[j], part[jt][1], acc[jt][1]);
              acc[jt][2] = fmaf(sb[j], part[jt][2], acc[jt][2]);
              acc[jt][3] = fmaf(sb[j], part[jt][3], acc[jt][3]);
            }
          } else {
            // per-token sums of the piece's x: the 8 lanes with this c split
            // the 16 chunks of each of its two tokens, then reduce over g
            const uint32_t xbase = sbase + p.xoff;
#pragma unroll
            for (int jt = 0; jt < MT; ++jt) {
              float xs0 = 0.f, xs1 = 0.f;
#pragma unroll
              for (int q2 = 0; q2 < 2; ++q2) {
                const int chunk = 2 * g + q2;  // 0..15 over the piece's 128 columns
                const int kk = j * 128 + chunk * 8;
                const uint32_t xb = xbase + (uint32_t)((kk >> 6) * MPAD * 128);
                xs0 += chunk_sum8<BF16>(lds128(sw128(xb, 8 * jt + 2 * c, (kk >> 3) & 7)));
                xs1 += chunk_sum8<BF16>(lds128(sw128(xb, 8 * jt + 2 * c + 1, (kk >> 3) & 7)));
              }
#pragma unroll
              for (int m = 4; m < 32; m <<= 1) {
                xs0 += __shfl_xor_sync(0xffffffffu, xs0, m);
                xs1 += __shfl_xor_sync(0xffffffffu, xs1, m);
              }
              const float zba = kMagic + za[j], zbb = kMagic + zb[j];
              acc[jt][0] = fmaf(sa[j], fmaf(-zba, xs0, part[jt][0]), acc[jt][0]);
              acc[jt][1] = fmaf(sa[j], fmaf(-zba, xs1, part[jt][1]), acc[jt][1]);
              acc[jt][2] = fmaf(sb[j], fmaf(-zbb, xs0, part[jt][2]), acc[jt][2]);
              acc[jt][3] = fmaf(sb[j], fmaf(-zbb, xs1, part[jt][3]), acc[jt][3]);
            }
          }
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 xv[MT];
#pragma unroll
            for (int jt = 0; jt < MT; ++jt) xv[jt] = lds128(xrow + xq[h] + jt * 1024);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const uint32_t wgu = wg[2 * h + u], whu = wh[2 * h + u];
              const uint32_t a[4] = {e4m3x2_to_f16x2(wgu & 0xFFFFu), e4m3x2_to_f16x2(whu & 0xFFFFu),
                                     e4m3x2_to_f16x2(wgu >> 16), e4m3x2_to_f16x2(whu >> 16)};
#pragma unroll
              for (int jt = 0; jt < MT; ++jt) mma_16816<false>(acc[jt], a, u ? xv[jt].z : xv[jt].x, u ? xv[jt].w : xv[jt].y);
            }
          }
        }
      }
    }
    // the stage's smem may be refilled once every consumer warp is done with it
    // (FP8: this thread's in-place x stores precede the next copy into the slot)
    if constexpr (FMT == 1 && BF16) fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  // ---------------- epilogue ----------------
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  if (KW > 1) {
    if (active && kw > 0) {
      float* dst = red + (size_t)((r * (KW - 1) + kw - 1) * MPAD) * kRedStrideR;
#pragma unroll
      for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          dst[(8 * jt + 2 * c + (e & 1)) * kRedStrideR + g + 8 * (e >> 1)] = acc[jt][e];
        }
      }
    }
    named_bar_sync(2, ncw * 32);
    if (active && kw == 0) {
      for (int q = 1; q < KW; ++q) {
        const float* src = red + (size_t)((r * (KW - 1) + q - 1) * MPAD) * kRedStrideR;
#pragma unroll
        for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[jt][e] += src[(8 * jt + 2 * c + (e & 1)) * kRedStrideR + g + 8 * (e >> 1)];
        }
      }
    }
  }
  if (active && kw == 0) {
    constexpr float kXScale = (FMT == 1 && BF16) ? 256.0f : 1.0f;  // undo the 2^-8 of the fp16 x
    const float ws_a = (FMT == 1) ? __ldg(Sa.wscale) * kXScale : 1.0f;
    const float ws_b = (FMT == 1) ? __ldg(Sb.wscale) * kXScale : 1.0f;
    float ba = 0.f, bb = 0.f;
    if (p.bias_dtype != NSQ_DTYPE_NONE) {
      if (va && Sa.bias) ba = load_bias(Sa.bias, p.bias_dtype, n_a);
      if (vb && Sb.bias) bb = load_bias(Sb.bias, p.bias_dtype, n_b);
    }
    uint16_t* y = static_cast<uint16_t*>(p.y);
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const int tok = 8 * jt + 2 * c + e2;
        if (tok >= p.M) continue;
        const float va_ = fmaf(acc[jt][e2], ws_a, ba);
        const float vb_ = fmaf(acc[jt][2 + e2], ws_b, bb);
        if (p.mode == 0) {
          if (va) y[(int64_t)tok * p.ldy + S.ycol + n_a] = float_to_elem<BF16>(va_);
          if (vb) y[(int64_t)tok * p.ldy + S.ycol + n_b] = float_to_elem<BF16>(vb_);
        } else if (va) {
          const float silu = va_ / (1.0f + __expf(-va_));
          y[(int64_t)tok * p.ldy + n_a] = float_to_elem<BF16>(silu * vb_);
        }
      }
    }
  }
}

template <int FMT, bool BF16, int MT, int KW>
cudaError_t launch_rows(const CUtensorMap& xmap, const RowsMaps& maps, const RowsParams& p, int grid, size_t smem,
                        cudaStream_t stream) {
  auto kern = decode_rows_kernel<FMT, BF16, MT, KW>;
  static std::atomic<bool> configured{false};
  if (!configured.load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowsSmem + 1024);
    if (e != cudaSuccess) return e;
    configured.store(true);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3((p.R * p.KW + 1) * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
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
  return cudaLaunchKernelEx(&cfg, kern, xmap, maps, p);
}

template <int FMT, bool BF16, int KW>
cudaError_t dispatch_rows_mt(int mt, const CUtensorMap& xmap, const RowsMaps& maps, const RowsParams& p, int grid,
                             size_t smem, cudaStream_t s) {
  switch (mt) {
    case 1: return launch_rows<FMT, BF16, 1, KW>(xmap, maps, p, grid, smem, s);
    case 2: return launch_rows<FMT, BF16, 2, KW>(xmap, maps, p, grid, smem, s);
    case 3: return launch_rows<FMT, BF16, 3, KW>(xmap, maps, p, grid, smem, s);
    default: return launch_rows<FMT, BF16, 4, KW>(xmap, maps, p, grid, smem, s);
  }
}

template <int FMT, bool BF16>
cudaError_t dispatch_rows(int mt, const CUtensorMap& xmap, const RowsMaps& maps, const RowsParams& p, int grid,
                          size_t smem, cudaStream_t s) {
  switch (p.KW) {
    case 1: return dispatch_rows_mt<FMT, BF16, 1>(mt, xmap, maps, p, grid, smem, s);
    case 2: return dispatch_rows_mt<FMT, BF16, 2>(mt, xmap, maps, p, grid, smem, s);
    default: return dispatch_rows_mt<FMT, BF16, 4>(mt, xmap, maps, p, grid, smem, s);
  }
}

}  // namespace

// Plan and launch over 1..3 weights (segments) sharing x. mode 0: weight i
// writes y columns [ycol_i, ycol_i + n_i); mode 1: w[0] = gate, w[1] = up,
// y[:, :n] = SiLU(x gate^T) * (x up^T).
int run_decode_rows(const RowsLaunch& L, cudaStream_t stream) {
  const int M = L.M, K = L.K;
  if (M <= 0 || M > 32 || L.nw < 1 || L.nw > 3 || (L.mode == 1 && L.nw != 2)) return NSQ_ENOTSUP;
  if (L.fmt == 0 && !(L.group_size == 32 || L.group_size == 64 || L.group_size % 128 == 0)) return NSQ_ENOTSUP;
  const int mt = (M + 7) / 8;
  const int mpad = mt * 8;
  const int rowpg = L.mode == 0 ? 16 : 8;
  const int sms = num_sms();
  // row groups per weight (mode 1: both weights share the feature groups)
  int rgs[3] = {0, 0, 0}, total = 0;
  const int nseg = L.mode == 0 ? L.nw : 1;
  for (int i = 0; i < nseg; ++i) {
    rgs[i] = (L.w[i].n + rowpg - 1) / rowpg;
    total += rgs[i];
  }
  if (total == 0) return NSQ_OK;
  int R = (total + sms - 1) / sms;
  if (R < 1) R = 1;
  if (R > kMaxR) R = kMaxR;
  RowsParams p{};
  int cta = 0, rmax = 0;
  for (int i = 0; i < nseg; ++i) {
    const int ctas = (rgs[i] + R - 1) / R;
    RowsSeg& sg = p.seg[i];
    sg.cta0 = cta;
    sg.rbase = rgs[i] / ctas;
    sg.rrem = rgs[i] - sg.rbase * ctas;
    const int rm = sg.rbase + (sg.rrem > 0 ? 1 : 0);
    rmax = rm > rmax ? rm : rmax;
    cta += ctas;
  }
  if (L.mode == 1) p.seg[1] = p.seg[0];  // up shares gate's row groups
  const int grid = cta;
  p.R = rmax;
  p.KW = rmax <= 3 ? 4 : (rmax <= 7 ? 2 : 1);  // R * KW <= 15 consumer warps
  p.nsegs = L.nw;
  for (int i = 0; i < L.nw; ++i) {
    RowsSeg& sg = p.seg[i];
    sg.scales = reinterpret_cast<const __half*>(L.w[i].scales);
    sg.zeros = reinterpret_cast<const __half*>(L.w[i].zeros);
    sg.wscale = L.w[i].wscale;
    sg.bias = L.w[i].bias;
    sg.n = L.w[i].n;
    sg.ycol = L.w[i].ycol;
  }
  constexpr int kSKa = 512, kSKf = 256;
  const int SK = L.fmt == 0 ? kSKa : kSKf;
  p.x = L.x;
  p.y = L.y;
  p.status = device_status_ptr();
  p.M = M;
  p.K = K;
  p.ldy = L.ldy;
  p.G = L.fmt == 0 ? (K + L.group_size - 1) / L.group_size : 0;
  p.group_size = L.group_size;
  p.nstage = (K + SK - 1) / SK;
  p.bias_dtype = L.bias_dtype;
  p.mode = L.mode;
  p.small_group = L.fmt == 0 && L.group_size < 128 ? 1 : 0;
  p.rows_half = 16 * p.R;
  const int wbytes = 2 * p.rows_half * 128;
  p.xoff = wbytes;
  p.stage_bytes = wbytes + (SK / 64) * mpad * 128;
  const int red_bytes = p.KW > 1 ? p.R * (p.KW - 1) * mpad * kRedStrideR * 4 : 0;
  const int fixed = ((red_bytes + 1023) & ~1023) + 1024;  // reduction tiles + barriers
  int nst = (kRowsSmem - fixed) / p.stage_bytes;
  if (nst > p.nstage) nst = p.nstage;
  if (nst > 6) nst = 6;
  if (nst < 1) return NSQ_ENOTSUP;
  p.nst = nst;
  p.off_red = nst * p.stage_bytes;
  p.off_bar = p.off_red + ((red_bytes + 1023) & ~1023);
  const size_t smem = (size_t)p.off_bar + 3 * nst * 8 + 16 + 1024;

  CUtensorMap xmap;
  CUresult cr = encode_tensor_map_2d(&xmap, L.x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                     const_cast<void*>(L.x), (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, 64, mpad,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  RowsMaps maps{};
  const uint64_t row_bytes = L.fmt == 0 ? (uint64_t)K / 2 : (uint64_t)K;
  for (int i = 0; i < L.nw; ++i) {
    const RowsSeg& sg = p.seg[i];
    const uint32_t main_rows = (uint32_t)(sg.rbase * rowpg);
    cr = encode_tensor_map_2d(&maps.m[2 * i], CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(L.w[i].w), row_bytes / 4,
                              (uint64_t)sg.n, row_bytes, 32, main_rows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
    cr = encode_tensor_map_2d(&maps.m[2 * i + 1], CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(L.w[i].w),
                              row_bytes / 4, (uint64_t)sg.n, row_bytes, 32, (uint32_t)rowpg, CU_TENSOR_MAP_SWIZZLE_128B);
    if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  }
  cudaError_t e;
  if (L.fmt == 0) {
    e = L.x_bf16 ? dispatch_rows<0, true>(mt, xmap, maps, p, grid, smem, stream)
                 : dispatch_rows<0, false>(mt, xmap, maps, p, grid, smem, stream);
  } else {
    e = L.x_bf16 ? dispatch_rows<1, true>(mt, xmap, maps, p, grid, smem, stream)
                 : dispatch_rows<1, false>(mt, xmap, maps, p, grid, smem, stream);
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

int run_decode_rows_linear(const LinearArgs& a, cudaStream_t stream) {
  RowsLaunch L{};
  L.fmt = a.fmt;
  L.x = a.x;
  L.x_bf16 = a.x_bf16;
  L.M = a.M;
  L.K = a.K;
  L.y = a.y;
  L.ldy = a.N;
  L.group_size = a.group_size;
  L.bias_dtype = a.bias ? a.bias_dtype : NSQ_DTYPE_NONE;
  L.mode = 0;
  L.nw = 1;
  L.w[0] = RowsWeight{a.wq, a.scales, a.zeros, a.wscale, a.bias, a.N, 0};
  return run_decode_rows(L, stream);
}

}  // namespace nsq
