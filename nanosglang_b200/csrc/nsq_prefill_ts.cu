// Prefill-regime quantized linear, one CTA per 128 weight rows, with the
// dequantised weight tile held in tensor memory: y^T = W_deq . x^T on
// tcgen05, A operand (128 weight rows) read from TMEM, B operand (the token
// tile of x, 64 or 128 tokens) from shared memory.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152, :49-52) for prefill-sized problems too small to
// fill the GPU with the paired kernel's 256 x 256 tiles: small outputs (q/k/v
// at M = 128 .. 1024, k/v at M = 8192) and long-K layers with few tiles
// (down at M <= 1024), whose K range is then split over the CTAs of a
// thread-block cluster.
//
// Why TMEM for the weight: with both operands in shared memory, a 64-column
// K step moves the converted weight through shared memory twice more than the
// tensor core needs; here the converters write it from registers straight
// into tensor memory (tcgen05.st) and shared memory carries only x and the
// packed weight.
//
// Warp roles, 448 threads:
//   warp 0        TMA producer: per stage KPS x tiles [BT tokens x 64]
//                 (128-byte swizzle) and KPS packed weight tiles [128 rows x
//                 64 columns] of the reference layout, NS-stage ring.
//   warp 1        TMEM allocation; runs the issue loop converged, and one
//                 elected lane issues each stage's 8 UMMAs (128 x BT x 16, A
//                 from TMEM) as one block; one barrier wait and one commit per
//                 stage: each barrier operation in the issuer opens a bubble
//                 of a few hundred cycles in the tensor pipe on B200.
//   warps 2..9    converters: warp w serves TMEM sub-partition w % 4 (32 weight
//                 rows, one per lane) and half (w - 2) / 4 of each k-block;
//                 int4 with zero point and group scale (AWQ) or e4m3 (FP8) ->
//                 MMA element type -> tcgen05.st into the TMEM operand ring.
//   warps 10..13  epilogue: tcgen05.ld of the accumulator (lane = output
//                 feature, column = token), per-tensor scale (FP8), bias,
//                 rounding, stores of feature pairs exchanged between lanes.
// Without a K split the accumulators are double-buffered (the epilogue of tile
// i overlaps the main loop of tile i + 1). With a K split of ks CTAs per tile
// (a cluster), every CTA owns BT / ks token columns of the tile: after its
// main loop it stages its other fp32 columns in its own idle x ring and sends
// them with one bulk shared-to-shared copy per owner into the owner's idle x
// ring (counted on the owner's transaction barrier, once the owner signalled
// that its UMMAs are done), and sums the partials of its own columns in rank
// order, so the result does not depend on timing.
// Every wait is bounded.
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"
#include "nsq_tmem_operand.cuh"

namespace nsq {

namespace {

constexpr int BW = 128;  // weight rows per tile (UMMA M, TMEM lanes)
constexpr int BK = 64;   // columns per k-block
constexpr int KPS = 2;   // k-blocks per stage (the UMMA issue block covers two)
constexpr int NS = 4;    // stages
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpConv0 = 2;
constexpr int kConvWarps = 8;
constexpr int kWarpEpi0 = kWarpConv0 + kConvWarps;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;
constexpr int kMinSmem = 120 * 1024;  // keeps one CTA (and one TMEM owner) per SM
constexpr int kXChunk = 16;           // token columns per exchanged chunk (split K)

template <int FMT>
struct TsFmt;
template <>
struct TsFmt<0> {  // AWQ: 128 rows x 8 words (32 B per row), 32-byte swizzle
  static constexpr int kWcBytes = BW * BK / 2;
};
template <>
struct TsFmt<1> {  // FP8: 128 rows x 64 B, 64-byte swizzle
  static constexpr int kWcBytes = BW * BK;
};

template <int BT>
struct TsTmem {
  static constexpr uint32_t kAcc = 0;         // 2 accumulators of BT columns
  static constexpr uint32_t kA = 2 * BT;      // NS operand stages of KPS x 32 columns
  static constexpr uint32_t kUsed = kA + NS * KPS * 32;
  static constexpr uint32_t kCols = kUsed <= 256 ? 256 : 512;
  static_assert(kUsed <= 512, "tensor memory budget");
};

template <int FMT, int BT>
struct TsSmem {
  static constexpr int kXBytes = BT * BK * 2;               // one k-block of x
  static constexpr int kX = 0;                              // [NS][KPS] x tiles
  static constexpr int kWc = kX + NS * KPS * kXBytes;       // [NS][KPS] packed weight tiles
  static constexpr int kBar = kWc + NS * KPS * TsFmt<FMT>::kWcBytes;
  // full_w[NS], full_x[NS], read_w[NS], full_a[NS], mma_done[NS], full_acc[2], empty_acc[2],
  // recv, peers_free, peers_received
  static constexpr int kNumBars = 5 * NS + 7;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kTotal = kAbort + 4;
  static constexpr int kNeed = kTotal + 1024;  // room to align the base to 1 KB
  static constexpr int kAlloc = kNeed > kMinSmem ? kNeed : kMinSmem;
  static_assert(kXBytes % 1024 == 0, "x stages stay 1 KB aligned");
  static_assert(kAlloc <= 227 * 1024, "shared memory per CTA");
  // split K: the receive slots of all ranks and the staged partials of the
  // other owners (together less than 2 x BW x BT fp32) fit in the x ring
  static_assert(kWc - kX >= 2 * BW * BT * 4, "split-K receive and staging slots");
};

struct TsParams {
  const __half* scales;
  const __half* zeros;
  const float* wscale;
  const void* bias;
  void* y;
  DevStatus* status;
  int M, K, N;
  int group_size, G;
  int bias_dtype;
  int num_w_tiles, num_t_tiles, num_kb;
  int ksplit;  // CTAs per tile along K = cluster size (1: no split)
};

// Offset of 16-byte unit u of row r in a split-K receive slot whose rows hold
// `units` units (4 per 16-column chunk): XOR-swizzled so that the eight rows a
// quarter-warp stores hit eight different bank groups.
__device__ __forceinline__ uint32_t ts_slot_unit(uint32_t u, uint32_t r, uint32_t units) {
  if (units >= 8) return ((u & ~7u) | ((u & 7u) ^ (r & 7u))) << 4;
  return (u ^ ((r >> 1) & 3u)) << 4;  // 64-byte rows: two rows per 128 bytes
}

template <int FMT, bool BF16, int BT>
__global__ void __launch_bounds__(kThreads, 1) prefill_ts_kernel(
    const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
    const TsParams p) {
  using L = TsSmem<FMT, BT>;
  using TM = TsTmem<BT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  // Per stage s: full_w / full_x (TMA bytes of the packed weight / of x
  // landed), read_w (the converters read the packed weight), full_a (the
  // converters wrote the TMEM operand and saw full_x), mma_done (the UMMAs of
  // the stage finished: frees both the x tiles and the TMEM operand).
  uint64_t* full_w = bars;
  uint64_t* full_x = bars + NS;
  uint64_t* read_w = bars + 2 * NS;
  uint64_t* full_a = bars + 3 * NS;
  uint64_t* mma_done = bars + 4 * NS;
  uint64_t* full_acc = bars + 5 * NS;
  uint64_t* empty_acc = full_acc + 2;
  // split K: the other ranks' partial columns landed here (recv); every
  // other rank's receive slots are free (peers_free); every other rank
  // received this CTA's partials, so their source tiles were read (peers_received)
  uint64_t* recv = full_acc + 4;
  uint64_t* peers_free = full_acc + 5;
  uint64_t* peers_received = full_acc + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KS = p.ksplit;
  const int cpo = (BT / kXChunk) / KS;  // exchanged chunks owned per rank

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full_w[i], 1);
      mbar_init(&full_x[i], 1);
      mbar_init(&read_w[i], kConvWarps);
      mbar_init(&full_a[i], kConvWarps);
      mbar_init(&mma_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full_acc[i], 1);
      mbar_init(&empty_acc[i], kEpiWarps);
    }
    mbar_init(recv, 1);
    if (KS > 1) {
      mbar_init(peers_free, KS - 1);
      mbar_init(peers_received, KS - 1);
    }
    fence_barrier_init();
    if (KS > 1) mbar_arrive_expect_tx(recv, (uint32_t)((KS - 1) * BW * cpo * kXChunk * 4));
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, TM::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // split K: this CTA's barriers are initialised; every thread waits for the
  // other ranks' arrivals before its first remote operation (or at its end)
  if (KS > 1) cluster_arrive_rel();

  // The weights (packed tiles, scales, zero points, bias) are static: their
  // loads and the conversion into TMEM may run before the previous kernel on
  // the stream finishes. Everything that touches x or y waits for it first
  // (pdl_wait_prior_grids in the producer before its x loads and in the
  // epilogue before its stores).

  // work units: (tile, K range), token tile fastest; a split tile is one cluster
  const int num_units = p.num_w_tiles * p.num_t_tiles * KS;
  auto unit_tile = [&](int u, int& wt, int& tt) {
    const int tile = u / KS;
    wt = tile / p.num_t_tiles;
    tt = tile - wt * p.num_t_tiles;
  };
  auto unit_kb = [&](int u, int& lo, int& hi) {  // k-blocks [lo, hi) of unit u
    const int ks = u % KS;
    lo = (int)(((int64_t)ks * p.num_kb) / KS);
    hi = (int)(((int64_t)(ks + 1) * p.num_kb) / KS);
  };
  bool ok = true;

  if (warp == kWarpTma) {
    if (lane == 0) {
      tma_prefetch_desc(&xmap);
      tma_prefetch_desc(&wmap);
      // packed weight tiles of stage it (k-blocks kb0 .. kb0+nk-1 of unit u)
      auto load_w = [&](int u, int kb0, int nk, int s) {
        int wt, tt;
        unit_tile(u, wt, tt);
        mbar_arrive_expect_tx(&full_w[s], (uint32_t)nk * TsFmt<FMT>::kWcBytes);
        for (int i = 0; i < nk; ++i) {
          const int kb = kb0 + i;
          tma_load_2d(smem + L::kWc + (s * KPS + i) * TsFmt<FMT>::kWcBytes, &wmap, &full_w[s],
                      FMT == 0 ? kb * (BK / 8) : kb * BK, wt * BW);
        }
      };
      // the first NS stages' weights before the previous kernel finishes
      int pre = 0;
      for (int u = blockIdx.x; u < num_units && pre < NS; u += gridDim.x) {
        int lo, hi;
        unit_kb(u, lo, hi);
        for (int kb0 = lo; kb0 < hi && pre < NS; kb0 += KPS, ++pre) {
          load_w(u, kb0, hi - kb0 < KPS ? hi - kb0 : KPS, pre);
        }
      }
      pdl_wait_prior_grids();
      int it = 0;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int wt, tt, lo, hi;
        unit_tile(u, wt, tt);
        unit_kb(u, lo, hi);
        for (int kb0 = lo; kb0 < hi; kb0 += KPS, ++it) {
          const int s = it % NS;
          const uint32_t ph = ((it / NS) & 1) ^ 1;  // previous use of the stage
          const int nk = hi - kb0 < KPS ? hi - kb0 : KPS;
          if (it >= pre) {
            // a reuse of the stage: the converters are done with its packed
            // tiles, the UMMAs with its x tiles and TMEM operand
            if (!(ok = mbar_wait(&read_w[s], ph, p.status, 50, abort_flag))) break;
            if (!(ok = mbar_wait(&mma_done[s], ph, p.status, 57, abort_flag))) break;
            load_w(u, kb0, nk, s);
          }
          mbar_arrive_expect_tx(&full_x[s], (uint32_t)nk * L::kXBytes);
          for (int i = 0; i < nk; ++i) {
            tma_load_2d(smem + L::kX + (s * KPS + i) * L::kXBytes, &xmap, &full_x[s], (kb0 + i) * BK, tt * BT);
          }
        }
      }
      // let in-flight copies land before the CTA can exit
      if (!ok) {
        const int last = it > pre ? it : pre;
        for (int j = (last > NS ? last - NS : 0); j < last; ++j) {
          mbar_wait(&full_w[j % NS], (j / NS) & 1, nullptr, 0, nullptr);
          if (j < it) mbar_wait(&full_x[j % NS], (j / NS) & 1, nullptr, 0, nullptr);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // The whole warp runs the loop (every lane waits on the barriers, so the
    // warp stays converged); one elected lane issues the UMMAs of a stage as
    // one block and the commits.
    int it = 0, tcount = 0;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++tcount) {
      int wt, tt, lo, hi;
      unit_tile(u, wt, tt);
      unit_kb(u, lo, hi);
      // UMMA N: the tile's tokens rounded up to 16 (the x rows past M are
      // zero-filled by TMA; their accumulator columns are never stored)
      int n_eff = p.M - tt * BT;
      n_eff = n_eff > BT ? BT : ((n_eff + 15) & ~15);
      const uint32_t idesc = umma_idesc_f16(BF16, BW, n_eff);
      const int acc = tcount & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&empty_acc[acc], ((tcount >> 1) & 1) ^ 1, p.status, 51, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t d = tmem_base + TM::kAcc + acc * BT;
      for (int kb0 = lo; kb0 < hi; kb0 += KPS, ++it) {
        const int s = it % NS;
        ok = __all_sync(0xffffffffu, mbar_wait(&full_a[s], (it / NS) & 1, p.status, 53, abort_flag));
        if (!ok) break;
        tc_fence_after();
        // A: the stage's TMEM operand (32 columns per k-block); B: its x tiles
        const uint32_t a = tmem_base + TM::kA + s * KPS * 32;
        const uint64_t b0 = sw128_kmajor_desc(smem_u32(smem + L::kX + s * KPS * L::kXBytes));
        const uint32_t acc_in = kb0 > lo ? 1u : 0u;
        if (hi - kb0 >= 2) {
          const uint64_t b1 = sw128_kmajor_desc(smem_u32(smem + L::kX + (s * KPS + 1) * L::kXBytes));
          umma_ts_kblocks_elect<1, 2>(d, a, b0, b1, idesc, acc_in);
        } else {
          umma_ts_kblocks_elect<1, 1>(d, a, b0, 0, idesc, acc_in);
        }
        tc_commit_elect(&mma_done[s]);
      }
      if (!ok) break;
      tc_commit_elect(&full_acc[acc]);
    }
  } else if (warp < kWarpEpi0) {
    // ---------------- converters: packed weight -> TMEM operand ----------------
    const int sub = warp & 3;                   // TMEM sub-partition = 32 weight rows
    const int half = (warp - kWarpConv0) >> 2;  // 32-column half of each k-block
    const int row = sub * 32 + lane;            // weight row within the tile
    const uint32_t a_lane = tmem_base + ((uint32_t)(sub * 32) << 16) + TM::kA + half * 16;
    // AWQ: the (scale, zero) pairs this thread needs, in the order it needs
    // them -- (unit, group) for its row -- loaded three groups ahead into a
    // register ring so their latency hides behind whole groups of k-blocks
    const unsigned short* sc16 = reinterpret_cast<const unsigned short*>(p.scales);
    const unsigned short* zr16 = reinterpret_cast<const unsigned short*>(p.zeros);
    // Groups of 32 columns: this thread's 32 columns of k-block kb are group
    // 2 kb + half, so it walks every other group; larger groups span whole
    // k-blocks and both halves share them.
    const int gstep = p.group_size < BK ? BK / p.group_size : 1;
    int pu = blockIdx.x, pg = 0, pg_hi = 0;
    auto unit_groups = [&](int u, int& glo, int& ghi) {
      int lo, hi;
      unit_kb(u, lo, hi);
      if (gstep > 1) {
        glo = lo * gstep + (half * 32) / p.group_size;
        ghi = hi * gstep;
      } else {
        glo = (lo * BK) / p.group_size;
        ghi = hi > lo ? ((hi - 1) * BK) / p.group_size + 1 : glo;
      }
    };
    if (pu < num_units) unit_groups(pu, pg, pg_hi);
    auto load_sz = [&]() -> uint32_t {
      uint32_t v = 0;
      while (pu < num_units && pg >= pg_hi) {
        pu += gridDim.x;
        if (pu < num_units) unit_groups(pu, pg, pg_hi);
      }
      if (pu < num_units) {
        int wt, tt;
        unit_tile(pu, wt, tt);
        const int n = wt * BW + row;
        if (n < p.N && pg < p.G) {  // (a half past K in the last k-block has no group)
          const int64_t off = (int64_t)n * p.G + pg;
          v = (uint32_t)__ldg(sc16 + off) | ((uint32_t)__ldg(zr16 + off) << 16);
        }
        pg += gstep;
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
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int lo, hi;
      unit_kb(u, lo, hi);
      for (int kb0 = lo; kb0 < hi; kb0 += KPS, ++it) {
        const int s = it % NS;
        const uint32_t ph = (it / NS) & 1;
        if (!(ok = mbar_wait(&full_w[s], ph, p.status, 54, abort_flag))) break;
        // the TMEM operand stage is free once the UMMAs of its previous use finished
        if (!(ok = mbar_wait(&mma_done[s], ph ^ 1, p.status, 55, abort_flag))) break;
        tc_fence_after();
        const int nk = hi - kb0 < KPS ? hi - kb0 : KPS;
#pragma unroll
        for (int i = 0; i < KPS; ++i) {
          if (i < nk) {
            const int kb = kb0 + i;
            if constexpr (FMT == 0) {
              if (kb == lo || (kb * BK) % p.group_size == 0) {  // a new group
                rp = ts_row_dq_packed<BF16>(sz0);
                sz0 = sz1;
                sz1 = sz2;
                sz2 = load_sz();
              }
            }
            uint32_t o[16];
            ts_convert_k32<FMT, BF16>(smem_u32(smem + L::kWc + (s * KPS + i) * TsFmt<FMT>::kWcBytes), row,
                                      half, rp, o);
            tmem_st_32x32b_x16(a_lane + (s * KPS + i) * 32, o);
          }
        }
        // the packed tiles are consumed (the x tiles of the stage are freed by
        // the UMMAs' commit)
        __syncwarp();
        if (lane == 0) mbar_arrive(&read_w[s]);
        tmem_st_wait();
        tc_fence_before();
        // the operand is ready; the UMMAs also need the stage's x tiles
        if (!(ok = mbar_wait(&full_x[s], ph, p.status, 59, abort_flag))) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> y ----------------
    pdl_wait_prior_grids();  // y may alias memory the previous kernel still used
    const int sub = warp & 3;
    const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
    const bool has_bias = p.bias_dtype != NSQ_DTYPE_NONE;
    uint16_t* y = static_cast<uint16_t*>(p.y);
    int tcount = 0;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++tcount) {
      int wt, tt;
      unit_tile(u, wt, tt);
      const int acc = tcount & 1;
      if (!(ok = mbar_wait(&full_acc[acc], (tcount >> 1) & 1, p.status, 56, abort_flag))) break;
      tc_fence_after();
      if (KS > 1) break;  // split K: the accumulator stays in TMEM for the exchange below
      const int n = wt * BW + sub * 32 + lane;  // this thread's output feature
      const float bn = (has_bias && n < p.N) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
      const uint32_t taddr = tmem_base + ((uint32_t)(sub * 32) << 16) + TM::kAcc + acc * BT;
      const int m0 = tt * BT;
      // two 32-token chunks per TMEM wait (tcgen05.wait::ld waits for every
      // load in flight, so batching the loads, not prefetching, hides them)
      const int nc = (p.M - m0 + 31) / 32 < BT / 32 ? (p.M - m0 + 31) / 32 : BT / 32;
#pragma unroll 1
      for (int c = 0; c < nc; c += 2) {
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(taddr + c * 32, ra);
        if (c + 1 < nc) tmem_ld_32x32b_x32(taddr + (c + 1) * 32, rb);
        tmem_ld_wait();
        ts_store_tokens<BF16, 32>(y, p.M, p.N, n, m0 + c * 32, ra, wscale, has_bias, bn, lane);
        if (c + 1 < nc) ts_store_tokens<BF16, 32>(y, p.M, p.N, n, m0 + (c + 1) * 32, rb, wscale, has_bias, bn, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_acc[acc]);
    }
  }

  if (KS > 1) {
    // The exchange. Each rank owns cpo 16-column chunks of the tile: its own
    // partial of them goes straight into its receive slot `me`; its partials
    // of every other owner's chunks are staged locally in that owner's slot
    // layout and sent with one bulk shared-to-shared copy per owner, counted
    // on the owner's recv barrier, once the owner said that its receive
    // slots (its x ring) are free. Receivers sum the KS slots in rank order
    // (the result does not depend on timing) and then tell every sender that
    // its staged tiles were read.
    // The first four 16-column chunks of the accumulator go to registers first
    // (one TMEM wait).
    constexpr int kBatch = 4;
    uint32_t rb[kBatch][16];
    const uint32_t taddr0 = tmem_base + ((uint32_t)((warp & 3) * 32) << 16);  // accumulator 0
    if (warp >= kWarpEpi0) {
      if (ok) {
#pragma unroll
        for (int i = 0; i < kBatch; ++i) tmem_ld_32x32b_x16(taddr0 + i * kXChunk, rb[i]);
        tmem_ld_wait();
      }
      cluster_wait_acq();  // every rank's barriers are initialised
    }
    if (warp >= kWarpEpi0 && ok) {
      const uint32_t me = cluster_ctarank();
      const int etid = threadIdx.x - kWarpEpi0 * 32;
      const int sub = warp & 3;
      const int r_in = sub * 32 + lane;  // this thread's row (output feature) of the tile
      int wt, tt;
      unit_tile(blockIdx.x, wt, tt);
      const uint32_t units = (uint32_t)cpo * 4;  // 16-byte units per slot row
      const uint32_t slot_bytes = (uint32_t)BW * units * 16;
      const uint32_t row_off = (uint32_t)r_in * units * 16;
      // receive slots q = 0..KS-1 at the start of the (idle) x ring, then the
      // staged partials of the other owners (o < me at o, o > me at o - 1)
      const uint32_t xbase = smem_u32(smem + L::kX);
      const uint32_t stage0 = xbase + (uint32_t)KS * slot_bytes;
      auto stage_of = [&](uint32_t o) { return stage0 + (o < me ? o : o - 1) * slot_bytes; };
      // this CTA's UMMAs are done: its receive slots are free for the others
      if (etid == 0) {
        for (uint32_t q = 0; q < (uint32_t)KS; ++q) {
          if (q != me) mbar_arrive_cluster(dsmem_map(smem_u32(peers_free), q));
        }
      }
      auto put = [&](const uint32_t (&r)[16], int c) {
        const uint32_t owner = (uint32_t)(c / cpo);
        const int lc = c - (int)owner * cpo;
        const uint32_t dst = (owner == me ? xbase + me * slot_bytes : stage_of(owner)) + row_off;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sts128(dst + ts_slot_unit((uint32_t)(lc * 4 + j), (uint32_t)r_in, units), r[4 * j], r[4 * j + 1],
                 r[4 * j + 2], r[4 * j + 3]);
        }
      };
#pragma unroll
      for (int c0 = 0; c0 < BT / kXChunk; c0 += kBatch) {
        if (c0 > 0) {  // later batches (128-token tiles): load, then one wait
#pragma unroll
          for (int i = 0; i < kBatch; ++i) tmem_ld_32x32b_x16(taddr0 + (c0 + i) * kXChunk, rb[i]);
          tmem_ld_wait();
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) put(rb[i], c0 + i);
      }
      fence_proxy_async_smem();           // the staged tiles are read by bulk copies
      named_bar_sync(3, kEpiWarps * 32);  // every partial is in place
      if (etid == 0 && mbar_wait(peers_free, 0, p.status, 60, nullptr)) {
        const uint32_t rbar = smem_u32(recv);
        for (uint32_t q = 0; q < (uint32_t)KS; ++q) {
          if (q != me) {
            bulk_copy_s2cluster(dsmem_map(xbase + me * slot_bytes, q), stage_of(q), slot_bytes, dsmem_map(rbar, q));
          }
        }
      }
      if (mbar_wait(recv, 0, p.status, 58, nullptr)) {
        if (etid == 0) {  // the senders' staged tiles are read
          for (uint32_t q = 0; q < (uint32_t)KS; ++q) {
            if (q != me) mbar_arrive_cluster(dsmem_map(smem_u32(peers_received), q));
          }
        }
        const int n = wt * BW + r_in;
        const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
        const bool has_bias = p.bias_dtype != NSQ_DTYPE_NONE;
        const float bn = (has_bias && n < p.N) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
        const uint32_t base = xbase + row_off;
#pragma unroll 1
        for (int lc = 0; lc < cpo; ++lc) {
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
          for (int q = 0; q < KS; ++q) {  // rank order: the sum does not depend on timing
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 w =
                  lds128(base + q * slot_bytes + ts_slot_unit((uint32_t)(lc * 4 + j), (uint32_t)r_in, units));
              v[4 * j] += __uint_as_float(w.x);
              v[4 * j + 1] += __uint_as_float(w.y);
              v[4 * j + 2] += __uint_as_float(w.z);
              v[4 * j + 3] += __uint_as_float(w.w);
            }
          }
          uint32_t rr[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) rr[i] = __float_as_uint(v[i]);
          ts_store_tokens<BF16, 16>(static_cast<uint16_t*>(p.y), p.M, p.N, n, tt * BT + ((int)me * cpo + lc) * kXChunk,
                                    rr, wscale, has_bias, bn, lane);
        }
        // the CTA leaves only after the other ranks read its staged tiles
        if (etid == 0) mbar_wait(peers_received, 0, p.status, 61, nullptr);
      }
      tc_fence_before();  // the TMEM reads above precede the deallocation
    }
    if (warp == kWarpEpi0 && lane == 0) {
      // Every way out of the exchange passes here. After a wait that ran out
      // (in the main loop or in the exchange above) the other ranks may still
      // arrive on this CTA's barriers and copy into its shared memory: let
      // those land (bounded) before the CTA can leave. When the exchange
      // completed, all three phases are already complete and these waits
      // return at once.
      mbar_wait(peers_free, 0, nullptr, 0, nullptr);
      mbar_wait(recv, 0, nullptr, 0, nullptr);
      mbar_wait(peers_received, 0, nullptr, 0, nullptr);
    }
    if (warp < kWarpEpi0) cluster_wait_acq();
    // No CTA of the cluster exits while another one may still address its
    // shared memory: every rank reaches this barrier (all waits above are
    // bounded) only after its own remote operations were issued and the
    // ones aimed at it landed or were given up on.
    cluster_arrive_rel();
    cluster_wait_acq();
  }

  pdl_launch_dependents();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TM::kCols);
  }
}

template <int FMT, bool BF16, int BT>
cudaError_t launch_ts(const CUtensorMap& xmap, const CUtensorMap& wmap, const TsParams& p, int grid,
                      cudaStream_t stream) {
  using L = TsSmem<FMT, BT>;
  auto kern = prefill_ts_kernel<FMT, BF16, BT>;
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
  if (p.ksplit > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = p.ksplit;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl_enabled()) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, xmap, wmap, p);
}

template <int BT>
int run_ts(const LinearArgs& a, int ksplit, cudaStream_t stream) {
  CUtensorMap xmap, wmap;
  CUresult cr = encode_tensor_map_2d(
      &xmap, a.x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
      const_cast<void*>(a.x), (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2, BK, BT,
      CU_TENSOR_MAP_SWIZZLE_128B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  if (a.fmt == 0) {
    cr = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                              (uint64_t)a.K / 8, (uint64_t)a.N, (uint64_t)a.K / 2, BK / 8, BW,
                              CU_TENSOR_MAP_SWIZZLE_32B);
  } else {
    cr = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<void*>(a.wq),
                              (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, BK, BW,
                              CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  TsParams p{};
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
  p.num_w_tiles = (a.N + BW - 1) / BW;
  p.num_t_tiles = (a.M + BT - 1) / BT;
  p.num_kb = (a.K + BK - 1) / BK;
  // every rank of a split needs a non-empty K range
  p.ksplit = ksplit > 1 && ksplit <= p.num_kb && (BT / kXChunk) % ksplit == 0 ? ksplit : 1;
  const int tiles = p.num_w_tiles * p.num_t_tiles;
  const int sms = num_sms();
  // a split launch runs one tile per cluster; the plan keeps it within one wave
  const int grid = p.ksplit > 1 ? tiles * p.ksplit : (tiles < sms ? tiles : sms);
  cudaError_t e;
  if (a.fmt == 0) {
    e = a.x_bf16 ? launch_ts<0, true, BT>(xmap, wmap, p, grid, stream)
                 : launch_ts<0, false, BT>(xmap, wmap, p, grid, stream);
  } else {
    e = a.x_bf16 ? launch_ts<1, true, BT>(xmap, wmap, p, grid, stream)
                 : launch_ts<1, false, BT>(xmap, wmap, p, grid, stream);
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // namespace

TsPlan prefill_ts_plan(int fmt, int64_t M, int64_t K, int64_t N) {
  // The one-CTA kernel serves problems that CTA pairs of 256 x 256 tiles
  // would leave mostly idle: outputs of at most 2^20 elements, or pair tiles
  // covering less than a quarter of the SMs. The token tile and K split
  // minimise rounds x (k-blocks per CTA x c + f + exchange) us, the exchange
  // of a split costing ~1 us for 64-token tiles and 2.5 + 0.3 ks us for
  // 128-token tiles, with c = 0.28 / f = 5.7 for FP8 and c = 0.52 / f = 6.2
  // for AWQ (its converters do twice the work per k-block). For AWQ the
  // paired kernel, ~4.5 + 1.1 us per two-k-block stage when its tiles fit one
  // wave, is taken when cheaper. All constants are fits of forced plans timed
  // on B200 over the Qwen2.5-0.5B and Llama-3-8B shapes at M = 128 / 1024. At
  // least 2 k-blocks per CTA.
  TsPlan best{0, 1};
  // decode-sized batches (M <= 64) take the one-CTA kernel with 64-token tiles
  const bool decode = M <= kDecodeMaxM;
  const int64_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
  const int sms = num_sms();
  if (!decode && M * N > ((int64_t)1 << 20) && pair_tiles * 4 > sms) return best;
  const int64_t kb = (K + BK - 1) / BK;
  const int64_t wt = (N + BW - 1) / BW;
  const double c = fmt == 0 ? 0.52 : 0.28;
  const double f = fmt == 0 ? 6.2 : 5.7;
  double best_cost = 0.0;
  for (int bt : {64, 128}) {
    if (decode && bt == 128) break;
    const int64_t units = wt * ((M + bt - 1) / bt);
    for (int ks = 1; ks <= bt / kXChunk; ks *= 2) {
      if (ks > 1 && (units * ks > sms || (kb + ks - 1) / ks < 2)) break;
      const int64_t rounds = (units * ks + sms - 1) / sms;
      const double exchange = ks == 1 ? 0.0 : (bt == 64 ? 1.0 : 2.5 + 0.3 * ks);
      const double cost = (double)rounds * ((double)((kb + ks - 1) / ks) * c + f + exchange);
      if (best.tokens_per_tile == 0 || cost < best_cost) {
        best = TsPlan{bt, ks};
        best_cost = cost;
      }
    }
  }
  if (!decode && fmt == 0 && pair_tiles * 2 <= sms && 4.5 + 1.1 * (double)((kb + 1) / 2) < best_cost) {
    return TsPlan{0, 1};
  }
  return best;
}

int run_prefill_ts_linear(const LinearArgs& a, TsPlan plan, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0) return NSQ_OK;
  switch (plan.tokens_per_tile) {
    case 64: return run_ts<64>(a, plan.ksplit, stream);
    case 128: return run_ts<128>(a, plan.ksplit, stream);
    default: return NSQ_ENOTSUP;
  }
}

}  // namespace nsq
