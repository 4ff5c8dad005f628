// Prefill-regime quantized linear on a CTA pair with the dequantised weight
// in tensor memory: y^T = W_deq . x^T with one tcgen05.mma.cta_group::2 of
// 256 weight rows x 256 tokens x 16 per step. The main large-M path.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152, :49-52) for prefill-sized batches.
//
// Each CTA of the pair converts its own 128 weight rows straight into its own
// TMEM (A operand, same address in both CTAs) and stages its own 128 tokens of
// x in shared memory (B operand, N split over the pair); the accumulator of
// each CTA holds its 128 weight rows x all 256 tokens. Per CTA and 64-column
// k-block, shared memory carries 16 KB of x and the packed weight tile (TMA
// writes, the converters' read and the tensor core's x read: ~48 KB against
// 512 cycles of MMA), and the conversion of a weight row is shared by 256
// tokens.
//
// Warp roles (both CTAs, 576 threads each):
//   warp 0        TMA producer: x tile [128 tokens x 64] (128-byte swizzle)
//                 and this CTA's packed weight tile [128 rows x 64 columns],
//                 KPS of each per stage, NS-stage ring, completion on this
//                 CTA's own barrier.
//   warp 1        TMEM allocation (512 columns, paired); in the even CTA it
//                 runs the issue loop converged, and one elected lane issues
//                 each stage's 8 UMMAs as one block and the multicast commits.
//   warps 2..9    converters: warp w serves TMEM sub-partition w % 4 (32
//                 weight rows, one per lane) and half (w - 2) / 4 of the 64
//                 columns; tcgen05.st into an NS-stage TMEM operand ring, then
//                 each warp arrives on the even CTA's operand barrier (a hop
//                 through one forwarding warp per CTA measured ~5% slower).
//   warps 10..17  epilogue: two warps per TMEM sub-partition (128 tokens
//                 each), tcgen05.ld of the accumulator (lane = output feature,
//                 column = token), scale (FP8), bias, rounding into a staged
//                 [tokens][features] tile, TMA stores of y.
// A stage holds KPS k-blocks, so each round of barrier operations in the UMMA
// issuer (a wait and a commit, ~300 cycles in which the tensor pipe drains on
// B200) covers 8 UMMAs. The single accumulator (256 columns) leaves the other
// 256 TMEM columns to the operand ring; the UMMAs of the next tile start once
// both CTAs' epilogues have drained theirs into shared memory, and the y
// stores overlap them. Every wait is bounded; no TMA multicast.
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"
#include "nsq_tmem_operand.cuh"

namespace nsq {

namespace {

constexpr int BWC = 128;  // weight rows per CTA (TMEM lanes); the pair tile is 256
constexpr int BTP = 256;  // tokens per pair tile (UMMA N); 128 per CTA
constexpr int BK = 64;
constexpr int KPS = 2;    // k-blocks per stage: one barrier round per 8 UMMAs (one issue block)
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpConv0 = 2;
constexpr int kConvWarps = 8;
constexpr int kWarpEpi0 = kWarpConv0 + kConvWarps;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = BTP;  // operand stages start after the accumulator
constexpr int kXBytes = (BTP / 2) * BK * 2;  // one k-block of x: 16 KB per CTA

// Stages (x + packed weight in shared memory, operand in TMEM): 4. The staged
// y tile holds all 256 tokens of a tile (AWQ, 64 KB) or 128 of them (FP8,
// 32 KB, drained in two rounds), so that 4 stages fit beside it: with 3 the
// refill of a stage (TMA, conversion, arrival: ~2.5 k cycles) outruns the
// ring at every tile start.
constexpr int NS = 4;
__host__ __device__ constexpr int ts2_stage_rounds(int fmt) { return fmt == 1 ? 2 : 1; }

template <int FMT, bool STAGED>
struct Ts2Smem {
  static constexpr int kRounds = ts2_stage_rounds(FMT);
  static constexpr int kTokRound = BTP / kRounds;  // tokens staged per round
  static_assert(kTmemA + NS * KPS * 32 <= kTmemCols, "tensor memory budget");
  static constexpr int kWcBytes = FMT == 0 ? BWC * BK / 2 : BWC * BK;
  static constexpr int kX = 0;                          // [NS][KPS] x tiles
  static constexpr int kWc = kX + NS * KPS * kXBytes;   // [NS][KPS] packed weight tiles
  static constexpr int kY = kWc + NS * KPS * kWcBytes;  // staged y tile: 2 x [256 tokens][64 features]
  static constexpr int kYHalfBytes = kTokRound * 64 * 2;
  static constexpr int kBar = kY + (STAGED ? 2 * kYHalfBytes : 0);
  // full_w[NS], full_x[NS], read_w[NS], full_a[NS], mma_done[NS], full_acc, empty_acc
  static constexpr int kNumBars = 5 * NS + 2;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kTotal = kAbort + 4;
  static constexpr int kAlloc = kTotal + 1024;
  static_assert(kAlloc <= 227 * 1024, "shared memory per CTA");
  static_assert(kY % 1024 == 0, "staged y tile stays 1 KB aligned (128-byte swizzle)");
};

struct Ts2Params {
  const __half* scales;
  const __half* zeros;
  const float* wscale;
  const void* bias;
  void* y;
  DevStatus* status;
  int M, K, N;
  int group_size, G;
  int bias_dtype;
  int num_w_tiles, num_t_tiles, num_kb;  // w tiles of 256 rows, t tiles of 256 tokens
  int wt_fast;  // unit order: weight tile fastest (1) or token tile fastest (0)
  int num_st;                            // stages per tile: ceil(num_kb / KPS)
};

// Weight tile and token tile of work unit u. Weight tile fastest when x is
// the larger operand: the pairs that run at the same time then share their x
// tiles (each read once from DRAM, the other readers hit L2) and the smaller
// weight stays in L2 across waves; token tile fastest otherwise.
__device__ __forceinline__ void ts2_unit(const Ts2Params& p, int u, int& wt, int& tt) {
  if (p.wt_fast) {
    tt = u / p.num_w_tiles;
    wt = u - tt * p.num_w_tiles;
  } else {
    wt = u / p.num_t_tiles;
    tt = u - wt * p.num_t_tiles;
  }
}

// tokens of pair tile tt given to the UMMA (N): all 256, or the remainder
// rounded up to 32 (paired N is a multiple of 32; x rows past M read as zero)
__device__ __forceinline__ int ts2_n_eff(int M, int tt) {
  const int rem = M - tt * BTP;
  return rem >= BTP ? BTP : ((rem + 31) & ~31);
}

template <int FMT, bool BF16, bool STAGED>
__global__ void __launch_bounds__(kThreads, 1) prefill_ts2_kernel(
    const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
    const __grid_constant__ CUtensorMap ymap, const Ts2Params p) {
  using L = Ts2Smem<FMT, STAGED>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  // Per stage s (both CTAs unless noted): full_w / full_x (this CTA's packed
  // weight / x bytes landed), read_w (this CTA's converters read the packed
  // weight), full_a (even CTA: every converter warp of both CTAs wrote its
  // part of the TMEM operand and saw its CTA's full_x, so full_a implies both
  // x tiles landed), mma_done (multicast commit: frees the x tile and the TMEM
  // operand in both CTAs).
  uint64_t* full_w = bars;
  uint64_t* full_x = bars + NS;
  uint64_t* read_w = bars + 2 * NS;
  uint64_t* full_a = bars + 3 * NS;
  uint64_t* mma_done = bars + 4 * NS;
  uint64_t* full_acc = bars + 5 * NS;
  uint64_t* empty_acc = full_acc + 1;  // even CTA: every epilogue warp of both CTAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = blockIdx.x >> 1;
  const int ncl = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full_w[i], 1);
      mbar_init(&full_x[i], 1);
      mbar_init(&read_w[i], kConvWarps);
      mbar_init(&full_a[i], 2 * kConvWarps);
      mbar_init(&mma_done[i], 1);
    }
    mbar_init(full_acc, 1);
    mbar_init(empty_acc, 2 * kEpiWarps);
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers and TMEM exist before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The weights (packed tiles, scales, zero points, bias) are static: their
  // loads and the conversion into TMEM may run before the previous kernel on
  // the stream finishes. The producer waits for it before its x loads, the
  // epilogue before its stores.

  const int num_units = p.num_w_tiles * p.num_t_tiles;  // ordered by ts2_unit
  bool ok = true;

  if (warp == kWarpTma) {
    if (lane == 0) {
      tma_prefetch_desc(&xmap);
      tma_prefetch_desc(&wmap);
      // packed weight tiles of a stage: k-blocks kb0 .. kb0+nk-1 of weight tile wt
      auto load_w = [&](int wt, int kb0, int nk, int s) {
        mbar_arrive_expect_tx(&full_w[s], (uint32_t)nk * L::kWcBytes);
        for (int i = 0; i < nk; ++i) {
          const int kb = kb0 + i;
          tma_load_2d(smem + L::kWc + (s * KPS + i) * L::kWcBytes, &wmap, &full_w[s],
                      FMT == 0 ? kb * (BK / 8) : kb * BK, wt * (2 * BWC) + (int)rank * BWC);
        }
      };
      // the first NS stages' weights before the previous kernel finishes
      int pre = 0;
      for (int u = cid; u < num_units && pre < NS; u += ncl) {
        for (int st = 0; st < p.num_st && pre < NS; ++st, ++pre) {
          const int kb0 = st * KPS;
          int wt, tt;
          ts2_unit(p, u, wt, tt);
          load_w(wt, kb0, p.num_kb - kb0 < KPS ? p.num_kb - kb0 : KPS, pre);
        }
      }
      pdl_wait_prior_grids();
      int it = 0;
      for (int u = cid; u < num_units && ok; u += ncl) {
        int wt, tt;
        ts2_unit(p, u, wt, tt);
        // this CTA's tokens: the second half of the UMMA's N starts at n_eff / 2
        const int tok0 = tt * BTP + (int)rank * (ts2_n_eff(p.M, tt) >> 1);
        for (int st = 0; st < p.num_st; ++st, ++it) {
          const int s = it % NS;
          const uint32_t ph = ((it / NS) & 1) ^ 1;  // previous use of the stage
          const int kb0 = st * KPS;
          const int nk = p.num_kb - kb0 < KPS ? p.num_kb - kb0 : KPS;
          if (it >= pre) {
            // a reuse of the stage: the converters are done with its packed
            // tiles, the UMMAs with its x tiles and TMEM operand
            if (!(ok = mbar_wait(&read_w[s], ph, p.status, 150, abort_flag))) break;
            if (!(ok = mbar_wait(&mma_done[s], ph, p.status, 151, abort_flag))) break;
            load_w(wt, kb0, nk, s);
          }
          mbar_arrive_expect_tx(&full_x[s], (uint32_t)nk * kXBytes);
          for (int i = 0; i < nk; ++i) {
            tma_load_2d(smem + L::kX + (s * KPS + i) * kXBytes, &xmap, &full_x[s], (kb0 + i) * BK, tok0);
          }
        }
      }
      if (!ok) {  // let in-flight copies land before the CTA can exit
        const int last = it > pre ? it : pre;
        for (int j = (last > NS ? last - NS : 0); j < last; ++j) {
          mbar_wait(&full_w[j % NS], (j / NS) & 1, nullptr, 0, nullptr);
          if (j < it) mbar_wait(&full_x[j % NS], (j / NS) & 1, nullptr, 0, nullptr);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // Even CTA: the whole warp runs the loop (every lane waits on the
    // barriers, so the warp stays converged); one elected lane issues the
    // UMMAs of a stage as one block and the multicast commits.
    if (leader) {
      int it = 0, tcount = 0;
      for (int u = cid; u < num_units && ok; u += ncl, ++tcount) {
        int wt, tt;
        ts2_unit(p, u, wt, tt);
        const uint32_t idesc = umma_idesc_f16(BF16, 2 * BWC, ts2_n_eff(p.M, tt));
        ok = __all_sync(0xffffffffu, mbar_wait(empty_acc, (tcount & 1) ^ 1, p.status, 152, abort_flag));
        if (!ok) break;
        tc_fence_after();
        for (int st = 0; st < p.num_st; ++st, ++it) {
          const int s = it % NS;
          ok = __all_sync(0xffffffffu, mbar_wait(&full_a[s], (it / NS) & 1, p.status, 153, abort_flag));
          if (!ok) break;
          tc_fence_after();
          // A: the stage's TMEM operand (32 columns per k-block); B: its x tiles
          const uint32_t a = tmem_base + kTmemA + s * KPS * 32;
          const uint64_t b0 = sw128_kmajor_desc(smem_u32(smem + L::kX + s * KPS * kXBytes));
          const uint32_t acc_in = st > 0 ? 1u : 0u;
          if (p.num_kb - st * KPS >= 2) {
            const uint64_t b1 = sw128_kmajor_desc(smem_u32(smem + L::kX + (s * KPS + 1) * kXBytes));
            umma_ts_kblocks_elect<2, 2>(tmem_base, a, b0, b1, idesc, acc_in);
          } else {
            umma_ts_kblocks_elect<2, 1>(tmem_base, a, b0, 0, idesc, acc_in);
          }
          tc_commit_pair_mc_elect(&mma_done[s], 0x3);
        }
        if (!ok) break;
        tc_commit_pair_mc_elect(full_acc, 0x3);
      }
    }
  } else if (warp < kWarpEpi0) {
    // ---------------- converters: packed weight -> TMEM operand ----------------
    const int sub = warp & 3;                   // TMEM sub-partition = 32 weight rows
    const int half = (warp - kWarpConv0) >> 2;  // 32-column half of the k-block
    const int row = sub * 32 + lane;            // weight row within this CTA's 128
    const uint32_t a_lane = tmem_base + ((uint32_t)(sub * 32) << 16) + kTmemA + half * 16;
    const uint32_t full_a_leader0 = dsmem_map(smem_u32(&full_a[0]), 0);
    // AWQ: (scale, zero) of this thread's row, in the order of use, loaded
    // three groups ahead into a register ring
    const unsigned short* sc16 = reinterpret_cast<const unsigned short*>(p.scales);
    const unsigned short* zr16 = reinterpret_cast<const unsigned short*>(p.zeros);
    int pu = cid, pg = 0;
    auto load_sz = [&]() -> uint32_t {
      uint32_t v = 0;
      if (pu < num_units) {
        int pwt, ptt;
        ts2_unit(p, pu, pwt, ptt);
        const int n = pwt * (2 * BWC) + (int)rank * BWC + row;
        if (n < p.N) {
          const int64_t off = (int64_t)n * p.G + pg;
          v = (uint32_t)__ldg(sc16 + off) | ((uint32_t)__ldg(zr16 + off) << 16);
        }
        if (++pg == p.G) {
          pg = 0;
          pu += ncl;
        }
      }
      return v;
    };
    uint32_t sz0 = 0, sz1 = 0, sz2 = 0;
    if constexpr (FMT == 0) {
      sz0 = load_sz();
      sz1 = load_sz();
      sz2 = load_sz();
    }
    TsRowDq<BF16> rp{};
    int it = 0;
    for (int u = cid; u < num_units && ok; u += ncl) {
      for (int st = 0; st < p.num_st; ++st, ++it) {
        const int s = it % NS;
        const uint32_t ph = (it / NS) & 1;
        if (!(ok = mbar_wait(&full_w[s], ph, p.status, 155, abort_flag))) break;
        // the TMEM operand stage is free once the UMMAs of its previous use finished
        if (!(ok = mbar_wait(&mma_done[s], ph ^ 1, p.status, 156, abort_flag))) break;
        tc_fence_after();
        const int nk = p.num_kb - st * KPS < KPS ? p.num_kb - st * KPS : KPS;
#pragma unroll
        for (int i = 0; i < KPS; ++i) {
          if (i < nk) {
            if constexpr (FMT == 0) {
              if (((st * KPS + i) * BK) % p.group_size == 0) {  // a new group (k-block 0 included)
                rp = ts_row_dq_packed<BF16>(sz0);
                sz0 = sz1;
                sz1 = sz2;
                sz2 = load_sz();
              }
            }
            uint32_t o[16];
            ts_convert_k32<FMT, BF16>(smem_u32(smem + L::kWc + (s * KPS + i) * L::kWcBytes), row, half, rp, o);
            tmem_st_32x32b_x16(a_lane + (s * KPS + i) * 32, o);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&read_w[s]);
        tmem_st_wait();
        tc_fence_before();
        // the operand is ready; the UMMAs also need this CTA's x tiles
        if (!(ok = mbar_wait(&full_x[s], ph, p.status, 158, abort_flag))) break;
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(full_a_leader0 + s * 8);
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> staged tile -> TMA store ----------------
    pdl_wait_prior_grids();  // y may alias memory the previous kernel still used
    // STAGED: the accumulator is drained into shared memory (bf16/fp16, two
    // 128-byte-swizzled [tokens][64 features] halves; all 256 tokens at once,
    // or 128 per round for FP8) and released as soon as the last round is in
    // shared memory; the TMA stores overlap the next tile's UMMAs. The drain
    // reads TMEM in the 16x256b shape (the m8n8 fragment layout) and writes 8
    // tokens x 8 features per stmatrix.trans, so the transpose costs no
    // shuffles. Else (N % 8 != 0: no 16-byte row pitch for a tensor map) the
    // lanes store y directly.
    const int sub = warp & 3;
    const int chalf = (warp - kWarpEpi0) >> 2;  // which half of the tokens (of a round) this warp drains
    const int etid = threadIdx.x - kWarpEpi0 * 32;
    const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
    const bool has_bias = p.bias_dtype != NSQ_DTYPE_NONE;
    const uint32_t empty_acc_leader = dsmem_map(smem_u32(empty_acc), 0);
    uint16_t* y = static_cast<uint16_t*>(p.y);
    // staged tile half of this warp's 32 features (sub / 2); stmatrix row
    // addresses: thread 8q + i writes row i (a token) of matrix q (features
    // 8q .. 8q+7 of the warp) = 16-byte chunk (sub & 1) * 4 + q of the row
    const uint32_t ystage = smem_u32(smem + L::kY + (sub >> 1) * L::kYHalfBytes);
    const uint32_t ychunk = (uint32_t)((sub & 1) * 4 + (lane >> 3));
    const int g = lane >> 2;  // fragment row: features g, g + 8 of each 16-lane half
    int tcount = 0;
    for (int u = cid; u < num_units && ok; u += ncl, ++tcount) {
      int wt, tt;
      ts2_unit(p, u, wt, tt);
      ok = mbar_wait(full_acc, tcount & 1, p.status, 157, abort_flag);
      if (!named_bar_all(1, kEpiWarps * 32, ok)) {  // leave together if anyone gave up
        ok = false;
        break;
      }
      tc_fence_after();
      const int n = wt * (2 * BWC) + (int)rank * BWC + sub * 32 + lane;  // this lane's output feature
      const float bn = (has_bias && n < p.N) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
      const uint32_t taddr = tmem_base + ((uint32_t)(sub * 32) << 16) + chalf * 128;
      const int m0 = tt * BTP + chalf * 128;  // accumulator column c holds token tt * 256 + c
      if constexpr (STAGED) {
        // bias of the fragment rows this thread holds: features 16h + g (+ 8)
        float bf[4] = {0.f, 0.f, 0.f, 0.f};
        if (has_bias) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int nq = wt * (2 * BWC) + (int)rank * BWC + sub * 32 + 8 * q + g;
            bf[q] = nq < p.N ? load_bias(p.bias, p.bias_dtype, nq) : 0.f;
          }
        }
        // rounds of kTokRound tokens; this warp drains kTokRound / 2 of them
        constexpr int kWarpTok = L::kTokRound / 2;
#pragma unroll 1
        for (int rd = 0; rd < L::kRounds; ++rd) {
          // the previous stores have read the staged tile
          if (etid == 0) bulk_wait_group_read<0>();
          named_bar_sync(1, kEpiWarps * 32);
          const int col0 = rd * L::kTokRound + chalf * kWarpTok;  // accumulator column = token in the tile
          // two 32-token chunks per TMEM wait (tcgen05.wait::ld waits for every
          // load in flight, so batching, not prefetching, hides its latency)
          auto stage_chunk = [&](const uint32_t (&r0)[16], const uint32_t (&r1)[16], int c) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              auto v = [&](uint32_t x, float b) {
                return has_bias ? fmaf(__uint_as_float(x), wscale, b) : __uint_as_float(x) * wscale;
              };
              const uint32_t m0w = ts_pack2<BF16>(v(r0[4 * j], bf[0]), v(r0[4 * j + 1], bf[0]));
              const uint32_t m1w = ts_pack2<BF16>(v(r0[4 * j + 2], bf[1]), v(r0[4 * j + 3], bf[1]));
              const uint32_t m2w = ts_pack2<BF16>(v(r1[4 * j], bf[2]), v(r1[4 * j + 1], bf[2]));
              const uint32_t m3w = ts_pack2<BF16>(v(r1[4 * j + 2], bf[3]), v(r1[4 * j + 3], bf[3]));
              const uint32_t t = (uint32_t)(chalf * kWarpTok + c * 32 + 8 * j + (lane & 7));  // staged row
              stmatrix_x4_trans(ystage + t * 128 + ((ychunk ^ (t & 7)) << 4), m0w, m1w, m2w, m3w);
            }
          };
          const int nc_all = kWarpTok / 32;
          int nc = (p.M - (tt * BTP + col0) + 31) / 32;
          nc = nc < nc_all ? nc : nc_all;
#pragma unroll 1
          for (int c = 0; c < nc; c += 2) {
            // the accumulator's 32 lanes of this warp as two 16-lane fragment
            // halves, 32 token columns each chunk, then 4 transposed 8x8
            // stores per 8 tokens
            uint32_t a0[16], a1[16], b0[16], b1[16];
            const uint32_t tcol = tmem_base + ((uint32_t)(sub * 32) << 16) + col0 + c * 32;
            tmem_ld_16x256b_x4(tcol, a0);
            tmem_ld_16x256b_x4(tcol + (16u << 16), a1);
            if (c + 1 < nc) {
              tmem_ld_16x256b_x4(tcol + 32, b0);
              tmem_ld_16x256b_x4(tcol + (16u << 16) + 32, b1);
            }
            tmem_ld_wait();
            stage_chunk(a0, a1, c);
            if (c + 1 < nc) stage_chunk(b0, b1, c + 1);
          }
          if (rd == L::kRounds - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(empty_acc_leader);  // the accumulator is free
          }
          fence_proxy_async_smem();
          named_bar_sync(1, kEpiWarps * 32);
          if (etid == 0) {
            for (int h = 0; h < 2; ++h) {
              const int f0 = wt * (2 * BWC) + (int)rank * BWC + h * 64;
              if (f0 < p.N) tma_store_2d(&ymap, smem + L::kY + h * L::kYHalfBytes, f0, tt * BTP + rd * L::kTokRound);
            }
            bulk_commit_group();
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < 4 && m0 + c * 32 < p.M; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          tmem_ld_wait();
          ts_store_tokens<BF16, 32>(y, p.M, p.N, n, m0 + c * 32, r, wscale, has_bias, bn, lane);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(empty_acc_leader);
      }
    }
    if (STAGED && etid == 0) bulk_wait_group<0>();  // the staged tiles are written out
  }

  pdl_launch_dependents();
  __syncthreads();
  tc_fence_before();
  cluster_sync_all();  // the pair is done with both CTAs' TMEM and barriers
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <int FMT, bool BF16, bool STAGED>
cudaError_t launch_ts2(const CUtensorMap& xmap, const CUtensorMap& wmap, const CUtensorMap& ymap,
                       const Ts2Params& p, int grid, cudaStream_t stream) {
  using L = Ts2Smem<FMT, STAGED>;
  auto kern = prefill_ts2_kernel<FMT, BF16, STAGED>;
  static std::atomic<bool> configured{false};
  if (!configured.load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    configured.store(true);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeClusterDimension;
  attrs[na].val.clusterDim.x = 2;
  attrs[na].val.clusterDim.y = 1;
  attrs[na].val.clusterDim.z = 1;
  ++na;
  if (pdl_enabled()) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, xmap, wmap, ymap, p);
}

}  // namespace

int run_prefill_ts2_linear(const LinearArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0) return NSQ_OK;
  CUtensorMap xmap, wmap;
  CUresult cr = encode_tensor_map_2d(
      &xmap, a.x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
      const_cast<void*>(a.x), (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2, BK, BTP / 2,
      CU_TENSOR_MAP_SWIZZLE_128B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  if (a.fmt == 0) {
    cr = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                              (uint64_t)a.K / 8, (uint64_t)a.N, (uint64_t)a.K / 2, BK / 8, BWC,
                              CU_TENSOR_MAP_SWIZZLE_32B);
  } else {
    cr = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<void*>(a.wq),
                              (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, BK, BWC,
                              CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  // y: [M][N] in the activation dtype, stored as [tokens][64 features] boxes
  // from the staged tile when N % 8 == 0 (16-byte row pitch for the tensor map)
  CUtensorMap ymap = xmap;
  const int num_st = ((a.K + BK - 1) / BK + KPS - 1) / KPS;
  const bool staged = (a.N % 8) == 0;
  if (staged) {
    cr = encode_tensor_map_2d(&ymap, a.x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              a.y, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.N * 2, 64,
                              (uint32_t)(BTP / ts2_stage_rounds(a.fmt)), CU_TENSOR_MAP_SWIZZLE_128B);
    if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  }
  Ts2Params p{};
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.zeros = reinterpret_cast<const __half*>(a.zeros);
  p.wscale = a.wscale;
  p.bias = a.bias;
  p.y = a.y;
  p.status = device_status_ptr();
  p.M = a.M;
  p.K = a.K;
  p.N = a.N;
  p.group_size = a.group_size;
  p.G = a.fmt == 0 ? (a.K + a.group_size - 1) / a.group_size : 0;
  p.bias_dtype = a.bias ? a.bias_dtype : NSQ_DTYPE_NONE;
  p.num_w_tiles = (a.N + 2 * BWC - 1) / (2 * BWC);
  p.num_t_tiles = (a.M + BTP - 1) / BTP;
  // x larger than the packed weight (e.g. down at M = 8192: 80 MB of x for
  // 4.4 MB of weight): weight tile fastest
  const int64_t w_bytes = (int64_t)a.N * (a.fmt == 0 ? a.K / 2 : a.K);
  p.wt_fast = (int64_t)a.M * a.K * 2 > w_bytes ? 1 : 0;
  p.num_kb = (a.K + BK - 1) / BK;
  p.num_st = num_st;
  const int units = p.num_w_tiles * p.num_t_tiles;
  const int pairs = num_sms() / 2;
  const int grid = 2 * (units < pairs ? units : pairs);
  cudaError_t e;
  if (a.fmt == 0) {
    if (staged) {
      e = a.x_bf16 ? launch_ts2<0, true, true>(xmap, wmap, ymap, p, grid, stream)
                   : launch_ts2<0, false, true>(xmap, wmap, ymap, p, grid, stream);
    } else {
      e = a.x_bf16 ? launch_ts2<0, true, false>(xmap, wmap, ymap, p, grid, stream)
                   : launch_ts2<0, false, false>(xmap, wmap, ymap, p, grid, stream);
    }
  } else {
    if (staged) {
      e = a.x_bf16 ? launch_ts2<1, true, true>(xmap, wmap, ymap, p, grid, stream)
                   : launch_ts2<1, false, true>(xmap, wmap, ymap, p, grid, stream);
    } else {
      e = a.x_bf16 ? launch_ts2<1, true, false>(xmap, wmap, ymap, p, grid, stream)
                   : launch_ts2<1, false, false>(xmap, wmap, ymap, p, grid, stream);
    }
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // namespace nsq
