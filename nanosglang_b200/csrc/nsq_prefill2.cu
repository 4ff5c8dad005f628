// Prefill-regime quantized linear on a CTA pair (tcgen05 cta_group::2): the
// main large-M path (M > 128).
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152, :49-52) for prefill-sized batches. One UMMA of
// 256 tokens x 256 output features x 16 spans the two CTAs of a cluster:
// each CTA stages its own 128 tokens of x and converts only its own 128 rows
// of the packed weight, so the int4/e4m3 -> bf16/fp16 conversion (the cost
// of fusing dequantisation into the GEMM) is paid once per 256 tokens
// instead of once per 128, and each SM's shared memory feeds half of B.
//
// Warp roles (both CTAs of the pair, 448 threads each):
//   warp 0        TMA producer: x tile [128 x 64] (128-byte swizzle; completion
//                 counted on the even CTA's barrier) and this CTA's packed
//                 weight tile [128 rows x 64 columns] of the reference layout
//                 (own barrier), 6-stage ring.
//   warp 1        TMEM allocation (512 columns = 2 accumulators, paired);
//                 in the even CTA, lane 0 issues the 256x256x16 UMMAs and the
//                 commits that release stages in both CTAs.
//   warps 2..9    converters, two threads per weight row (32 columns each):
//                 AWQ int4 with zero point and group scale, or e4m3, into the
//                 UMMA 128-byte-swizzled K-major layout (3-stage ring).
//   warps 10..13  epilogue: tcgen05.ld of this CTA's 128 accumulator lanes,
//                 scale (FP8) + bias, bf16/fp16 rounding, staged through a
//                 64-byte-swizzled tile and written with TMA stores.
// The accumulator is double-buffered so the epilogue of tile i overlaps the
// main loop of tile i+1. Every wait is bounded; no TMA multicast is used.
#include <atomic>
#include <type_traits>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr int BMC = 128;  // tokens per CTA (TMEM lanes); the pair tile is 256
constexpr int BN = 256;   // output features per pair tile (UMMA N)
constexpr int BNC = 128;  // weight rows converted per CTA
constexpr int BK = 64;
constexpr int NL = 6;  // load stages
constexpr int NB = 3;  // converted-weight stages
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpConv0 = 2;
constexpr int kConvWarps = 8;
constexpr int kWarpEpi0 = kWarpConv0 + kConvWarps;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 2 * BN;
constexpr int kXTileBytes = BMC * BK * 2;  // 16 KB
constexpr int kBTileBytes = BNC * BK * 2;  // 16 KB
constexpr int kYChunkCols = 32;
constexpr int kYStageBytes = BMC * kYChunkCols * 2;  // 8 KB

template <int FMT>
struct PairFmt;
template <>
struct PairFmt<0> {  // AWQ: 128 rows x 8 words (32 B per row), 32-byte swizzle
  static constexpr int kWcBytes = BNC * BK / 2;
  static constexpr int kRowBytes = 32;
};
template <>
struct PairFmt<1> {  // FP8: 128 rows x 64 B, 64-byte swizzle
  static constexpr int kWcBytes = BNC * BK;
  static constexpr int kRowBytes = 64;
};

struct PairParams {
  const __half* scales;
  const __half* zeros;
  const float* wscale;
  const void* bias;
  DevStatus* status;
  int M, K, N;
  int group_size, G;
  int bias_dtype;
  int num_m_tiles, num_n_tiles, num_kb;  // m tiles of 256 tokens
};

template <int FMT>
struct PairSmem {
  static constexpr int kX = 0;
  static constexpr int kB = kX + NL * kXTileBytes;
  static constexpr int kWc = kB + NB * kBTileBytes;
  static constexpr int kY = kWc + NL * PairFmt<FMT>::kWcBytes;
  static constexpr int kBias = kY + 2 * kYStageBytes;
  static constexpr int kBar = kBias + BN * 4;
  // full_x[NL], full_w[NL], empty_l[NL], full_b[NB], empty_b[NB], full_acc[2], empty_acc[2]
  static constexpr int kNumBars = 3 * NL + 2 * NB + 4;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kTotal = kAbort + 4;
  static constexpr int kAlloc = kTotal + 1024;
  static_assert(kY % 1024 == 0, "staging tile must stay 1 KB aligned");
};

template <bool BF16>
struct RowDq {  // per-row AWQ dequant constants in the MMA element type
  uint32_t s2, zb2, magic2, c2;
  bool exact;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2f(float v) {
  if constexpr (BF16) {
    __nv_bfloat162 b = __floats2bfloat162_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&b);
  } else {
    __half2 h = __floats2half2_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <bool BF16>
__device__ __forceinline__ RowDq<BF16> row_dq(float s, float z) {
  RowDq<BF16> r;
  constexpr float kZMax = BF16 ? 127.0f : 1023.0f;
  r.exact = (z == rintf(z)) && fabsf(z) <= kZMax;
  r.s2 = pack2f<BF16>(s);
  r.zb2 = pack2f<BF16>(Magic<BF16>::kValue + z);
  r.magic2 = pack2f<BF16>(Magic<BF16>::kValue);
  r.c2 = pack2f<BF16>(-z * s);
  return r;
}

template <bool BF16>
__device__ __forceinline__ uint32_t dq_pair(uint32_t e, const RowDq<BF16>& rp) {
  using T2 = typename std::conditional<BF16, __nv_bfloat162, __half2>::type;
  const T2 ev = *reinterpret_cast<const T2*>(&e);
  const T2 s = *reinterpret_cast<const T2*>(&rp.s2);
  T2 o;
  if (rp.exact) {
    o = __hmul2(__hsub2(ev, *reinterpret_cast<const T2*>(&rp.zb2)), s);
  } else {
    o = __hfma2(__hsub2(ev, *reinterpret_cast<const T2*>(&rp.magic2)), s, *reinterpret_cast<const T2*>(&rp.c2));
  }
  return *reinterpret_cast<uint32_t*>(&o);
}

// Four packed words (32 columns of one weight row) -> four 16-byte chunks of
// the 128-byte-swizzled UMMA row: (q - z) * s per element.
template <bool BF16, bool EXACT>
__device__ __forceinline__ void awq_words_to_b(const uint32_t (&words)[4], const RowDq<BF16>& rp,
                                               uint32_t brow, int half, int row) {
  using T2 = typename std::conditional<BF16, __nv_bfloat162, __half2>::type;
  const T2 s = *reinterpret_cast<const T2*>(&rp.s2);
  const T2 zb = *reinterpret_cast<const T2*>(&rp.zb2);
  const T2 mg = *reinterpret_cast<const T2*>(&rp.magic2);
  const T2 c = *reinterpret_cast<const T2*>(&rp.c2);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t e[4];
    unpack_nibble_pairs<BF16>(words[j], e);
    // e[t] = {q_t, q_{t+4}} -> in-order pairs {q0,q1},{q2,q3},{q4,q5},{q6,q7}
    uint32_t in[4] = {prmt(e[0], e[1], 0x5410), prmt(e[2], e[3], 0x5410), prmt(e[0], e[1], 0x7632),
                      prmt(e[2], e[3], 0x7632)};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const T2 ev = *reinterpret_cast<const T2*>(&in[t]);
      T2 r;
      if constexpr (EXACT) {
        r = __hmul2(__hsub2(ev, zb), s);
      } else {
        r = __hfma2(__hsub2(ev, mg), s, c);
      }
      o[t] = *reinterpret_cast<uint32_t*>(&r);
    }
    const int w = 4 * half + j;
    sts128(brow + ((w ^ (row & 7)) << 4), o[0], o[1], o[2], o[3]);
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_out(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <int FMT, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) prefill_pair_kernel(
    const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
    const __grid_constant__ CUtensorMap ymap, const PairParams p) {
  using L = PairSmem<FMT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* full_x = bars;
  uint64_t* full_w = bars + NL;
  uint64_t* empty_l = bars + 2 * NL;
  uint64_t* full_b = bars + 3 * NL;
  uint64_t* empty_b = full_b + NB;
  uint64_t* full_acc = empty_b + NB;
  uint64_t* empty_acc = full_acc + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbort);
  float* bias_s = reinterpret_cast<float*>(smem + L::kBias);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = blockIdx.x >> 1;
  const int ncl = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < NL; ++i) {
      mbar_init(&full_x[i], 1);
      mbar_init(&full_w[i], 1);
      mbar_init(&empty_l[i], 2);  // this CTA's converter group + the UMMA commit
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&full_b[i], 2);   // one arrival per CTA's converter group
      mbar_init(&empty_b[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full_acc[i], 1);
      mbar_init(&empty_acc[i], 2 * kEpiWarps);
    }
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

  pdl_wait_prior_grids();

  const int num_tiles = p.num_m_tiles * p.num_n_tiles;
  bool ok = true;

  if (warp == kWarpTma) {
    if (lane == 0) {
      tma_prefetch_desc(&xmap);
      tma_prefetch_desc(&wmap);
      int it = 0;
      for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
        const int mt = tile / p.num_n_tiles;
        const int nt = tile - mt * p.num_n_tiles;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const int s = it % NL;
          const uint32_t r = it / NL;
          if (!(ok = mbar_wait(&empty_l[s], (r & 1) ^ 1, p.status, 110, abort_flag))) break;
          if (leader) mbar_arrive_expect_tx(&full_x[s], 2 * kXTileBytes);
          tma_load_2d_pair(smem + L::kX + s * kXTileBytes, &xmap, dsmem_map(smem_u32(&full_x[s]), 0),
                           kb * BK, mt * (2 * BMC) + rank * BMC);
          mbar_arrive_expect_tx(&full_w[s], PairFmt<FMT>::kWcBytes);
          tma_load_2d(smem + L::kWc + s * PairFmt<FMT>::kWcBytes, &wmap, &full_w[s],
                      FMT == 0 ? kb * (BK / 8) : kb * BK, nt * BN + rank * BNC);
        }
      }
      if (!ok) {  // let this CTA's in-flight weight copies land before exiting
        for (int j = (it > NL ? it - NL : 0); j < it; ++j) {
          mbar_wait(&full_w[j % NL], (j / NL) & 1, nullptr, 0, nullptr);
        }
      }
    }
  } else if (warp == kWarpMma) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BF16, 2 * BMC, BN);
      int it_l = 0, it_b = 0, tcount = 0;
      for (int tile = cid; tile < num_tiles && ok; tile += ncl, ++tcount) {
        const int acc = tcount & 1;
        const uint32_t ar = tcount >> 1;
        if (!(ok = mbar_wait(&empty_acc[acc], (ar & 1) ^ 1, p.status, 120, abort_flag))) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it_l, ++it_b) {
          const int sl = it_l % NL, sb = it_b % NB;
          if (!(ok = mbar_wait(&full_x[sl], (it_l / NL) & 1, p.status, 121, abort_flag))) break;
          if (!(ok = mbar_wait(&full_b[sb], (it_b / NB) & 1, p.status, 122, abort_flag))) break;
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(smem + L::kX + sl * kXTileBytes));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(smem + L::kB + sb * kBTileBytes));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            umma_f16_pair(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit_pair_mc(&empty_l[sl], 0x3);
          tc_commit_pair_mc(&empty_b[sb], 0x3);
        }
        if (!ok) break;
        tc_commit_pair_mc(&full_acc[acc], 0x3);
      }
    }
  } else if (warp < kWarpEpi0) {
    // ---------------- converters: two threads per weight row ----------------
    const int tc = threadIdx.x - kWarpConv0 * 32;  // 0..255
    const int row = tc >> 1;                       // 0..127
    const int half = tc & 1;                       // columns [32*half, 32*half + 32)
    int it_l = 0, it_b = 0;
    RowDq<BF16> rp{};
    const unsigned short* sc16 = reinterpret_cast<const unsigned short*>(p.scales);
    const unsigned short* zr16 = reinterpret_cast<const unsigned short*>(p.zeros);
    auto fetch_sz = [&](int tile, int kb, unsigned short& s16, unsigned short& z16) {
      s16 = 0;
      z16 = 0;
      if (tile < num_tiles) {
        const int n = (tile % p.num_n_tiles) * BN + rank * BNC + row;
        if (n < p.N) {
          const int64_t off = (int64_t)n * p.G + (kb * BK) / p.group_size;
          s16 = __ldg(sc16 + off);
          z16 = __ldg(zr16 + off);
        }
      }
    };
    unsigned short cur_s = 0, cur_z = 0;
    if constexpr (FMT == 0) fetch_sz(cid, 0, cur_s, cur_z);
    const uint32_t full_b_leader0 = dsmem_map(smem_u32(&full_b[0]), 0);
    for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
      for (int kb = 0; kb < p.num_kb; ++kb, ++it_l, ++it_b) {
        const int sl = it_l % NL, sb = it_b % NB;
        if constexpr (FMT == 0) {
          unsigned short nxt_s, nxt_z;
          if (kb + 1 < p.num_kb) {
            fetch_sz(tile, kb + 1, nxt_s, nxt_z);
          } else {
            fetch_sz(tile + ncl, 0, nxt_s, nxt_z);
          }
          if (kb == 0 || (kb * BK) % p.group_size == 0) {
            rp = row_dq<BF16>(__half2float(__ushort_as_half(cur_s)), __half2float(__ushort_as_half(cur_z)));
          }
          cur_s = nxt_s;
          cur_z = nxt_z;
        }
        bool got = mbar_wait(&full_w[sl], (it_l / NL) & 1, p.status, 130, abort_flag);
        got = got && mbar_wait(&empty_b[sb], ((it_b / NB) & 1) ^ 1, p.status, 131, abort_flag);
        if (got) {
          const uint32_t wc = smem_u32(smem + L::kWc + sl * PairFmt<FMT>::kWcBytes) + row * PairFmt<FMT>::kRowBytes;
          const uint32_t brow = smem_u32(smem + L::kB + sb * kBTileBytes) + row * 128;
          if constexpr (FMT == 0) {
            // 32-byte swizzle: 16-byte chunk c of row r sits at c ^ ((r >> 2) & 1)
            const uint4 v = lds128(wc + ((half ^ ((row >> 2) & 1)) << 4));
            const uint32_t words[4] = {v.x, v.y, v.z, v.w};
            // the exact/general choice is per row and group: branch once, not per pair
            if (rp.exact) {
              awq_words_to_b<BF16, true>(words, rp, brow, half, row);
            } else {
              awq_words_to_b<BF16, false>(words, rp, brow, half, row);
            }
          } else {
            // 64-byte swizzle: 16-byte chunk c of row r sits at c ^ ((r >> 1) & 3)
  #pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int cch = 2 * half + u;
              const uint4 v = lds128(wc + ((cch ^ ((row >> 1) & 3)) << 4));
              uint32_t o0, o1, o2, o3, o4, o5, o6, o7;
              e4m3x4_to_pairs<BF16>(v.x, o0, o1);
              e4m3x4_to_pairs<BF16>(v.y, o2, o3);
              e4m3x4_to_pairs<BF16>(v.z, o4, o5);
              e4m3x4_to_pairs<BF16>(v.w, o6, o7);
              sts128(brow + (((2 * cch) ^ (row & 7)) << 4), o0, o1, o2, o3);
              sts128(brow + (((2 * cch + 1) ^ (row & 7)) << 4), o4, o5, o6, o7);
            }
          }
        }
        // every converter thread publishes its writes to the async proxy, the
        // group syncs locally, and one thread signals the pair's UMMA issuer
        // (a single cluster-scope release per CTA and k-block)
        fence_proxy_async_smem();
        if (!named_bar_all(2, kConvWarps * 32, got)) {  // leave together if anyone gave up
          ok = false;
          break;
        }
        if (tc == 0) {
          mbar_arrive_cluster(full_b_leader0 + sb * 8);
          mbar_arrive(&empty_l[sl]);
        }
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> staged TMA store ----------------
    const int sub = warp & 3;                       // TMEM sub-partition
    const int etid = threadIdx.x - kWarpEpi0 * 32;  // 0..127
    const int rloc = sub * 32 + lane;               // accumulator lane = token within the CTA
    const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
    const bool has_bias = p.bias_dtype != NSQ_DTYPE_NONE;
    const uint32_t empty_acc_leader0 = dsmem_map(smem_u32(&empty_acc[0]), 0);
    int tcount = 0;
    for (int tile = cid; tile < num_tiles && ok; tile += ncl, ++tcount) {
      const int mt = tile / p.num_n_tiles;
      const int nt = tile - mt * p.num_n_tiles;
      const int acc = tcount & 1;
      const uint32_t ar = tcount >> 1;
      if (has_bias) {
        named_bar_sync(1, kEpiWarps * 32);  // everyone is done with the previous tile's bias
        for (int i = etid; i < BN; i += kEpiWarps * 32) {
          const int n = nt * BN + i;
          bias_s[i] = n < p.N ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
        }
        named_bar_sync(1, kEpiWarps * 32);
      }
      ok = mbar_wait(&full_acc[acc], ar & 1, p.status, 140, abort_flag);
      if (!named_bar_all(1, kEpiWarps * 32, ok)) {  // leave together if anyone gave up
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(sub * 32) << 16) + acc * BN;
      const int m_cta = mt * (2 * BMC) + rank * BMC;
#pragma unroll 1
      for (int cc = 0; cc < BN / kYChunkCols; ++cc) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + cc * 32, r);
        tmem_ld_wait();
        uint32_t o[16];
        if (has_bias) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 b = *reinterpret_cast<const float2*>(&bias_s[cc * 32 + 2 * i]);
            o[i] = pack_out<BF16>(fmaf(__uint_as_float(r[2 * i]), wscale, b.x),
                                  fmaf(__uint_as_float(r[2 * i + 1]), wscale, b.y));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            o[i] = pack_out<BF16>(__uint_as_float(r[2 * i]) * wscale, __uint_as_float(r[2 * i + 1]) * wscale);
          }
        }
        uint8_t* ys = smem + L::kY + (cc & 1) * kYStageBytes;
        if (etid == 0) bulk_wait_group_read<1>();  // the store that last used this buffer has read it
        named_bar_sync(1, kEpiWarps * 32);
        const uint32_t yrow = smem_u32(ys) + rloc * 64;
        const int sw = (rloc >> 1) & 3;  // 64-byte swizzle
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          sts128(yrow + ((v ^ sw) << 4), o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
        }
        fence_proxy_async_smem();
        named_bar_sync(1, kEpiWarps * 32);
        if (etid == 0) {
          tma_store_2d(&ymap, ys, nt * BN + cc * kYChunkCols, m_cta);
          bulk_commit_group();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(empty_acc_leader0 + acc * 8);
    }
    if (etid == 0) bulk_wait_group<0>();
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

template <int FMT, bool BF16>
cudaError_t launch_pair(const CUtensorMap& xmap, const CUtensorMap& wmap, const CUtensorMap& ymap,
                        const PairParams& p, int grid, cudaStream_t stream) {
  using L = PairSmem<FMT>;
  auto kern = prefill_pair_kernel<FMT, BF16>;
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

bool pair_prefill_supported(const LinearArgs& a) {
  // TMA stores need 16-byte row pitch for y; tiny M is better served unpaired
  return a.M > 128 && (a.N % 8) == 0;
}

int run_prefill_pair_linear(const LinearArgs& a, cudaStream_t stream) {
  const CUtensorMapDataType act =
      a.x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap xmap, wmap, ymap;
  CUresult cr = encode_tensor_map_2d(&xmap, act, const_cast<void*>(a.x), (uint64_t)a.K, (uint64_t)a.M,
                                     (uint64_t)a.K * 2, BK, BMC, CU_TENSOR_MAP_SWIZZLE_128B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  if (a.fmt == 0) {
    cr = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                              (uint64_t)a.K / 8, (uint64_t)a.N, (uint64_t)a.K / 2, BK / 8, BNC,
                              CU_TENSOR_MAP_SWIZZLE_32B);
  } else {
    cr = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<void*>(a.wq),
                              (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, BK, BNC,
                              CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  cr = encode_tensor_map_2d(&ymap, act, a.y, (uint64_t)a.N, (uint64_t)a.M, (uint64_t)a.N * 2, kYChunkCols,
                            BMC, CU_TENSOR_MAP_SWIZZLE_64B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  PairParams p{};
  p.scales = reinterpret_cast<const __half*>(a.scales);
  p.zeros = reinterpret_cast<const __half*>(a.zeros);
  p.wscale = a.wscale;
  p.bias = a.bias;
  p.status = device_status_ptr();
  p.M = a.M;
  p.K = a.K;
  p.N = a.N;
  p.group_size = a.group_size;
  p.G = a.fmt == 0 ? (a.K + a.group_size - 1) / a.group_size : 0;
  p.bias_dtype = a.bias ? a.bias_dtype : NSQ_DTYPE_NONE;
  p.num_m_tiles = (a.M + 2 * BMC - 1) / (2 * BMC);
  p.num_n_tiles = (a.N + BN - 1) / BN;
  p.num_kb = (a.K + BK - 1) / BK;
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int pairs = num_sms() / 2;
  const int grid = 2 * (tiles < pairs ? tiles : pairs);
  cudaError_t e;
  if (a.fmt == 0) {
    e = a.x_bf16 ? launch_pair<0, true>(xmap, wmap, ymap, p, grid, stream)
                 : launch_pair<0, false>(xmap, wmap, ymap, p, grid, stream);
  } else {
    e = a.x_bf16 ? launch_pair<1, true>(xmap, wmap, ymap, p, grid, stream)
                 : launch_pair<1, false>(xmap, wmap, ymap, p, grid, stream);
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // namespace nsq
