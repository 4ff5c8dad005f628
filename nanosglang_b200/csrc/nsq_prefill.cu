// Prefill-regime quantized linear (any M; used for M > 64): a dense
// contraction on the 5th-generation tensor cores.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152, :49-52), whose reference path materialises the
// whole dequantised weight in HBM and then calls cuBLAS.
//
// Persistent, warp-specialised kernel, one 128-token x 256-feature output
// tile at a time per CTA, fp32 accumulators in tensor memory:
//   warp 0        TMA producer: x tile [128 x 64] (128-byte swizzle) and the
//                 packed weight tile [256 rows x 64 columns] of the reference
//                 layout into an NS-stage ring (shared with the converted tiles).
//   warp 1        tcgen05.mma issuer (one thread), 128x256x16 kind::f16 steps;
//                 also owns the 512-column TMEM allocation (2 accumulators).
//   warps 2..9    converters: one weight row per thread; unpack int4 (AWQ,
//                 zero point and group scale applied) or e4m3 (FP8) into the
//                 MMA element type, written in the UMMA 128-byte-swizzled
//                 K-major layout.
//   warps 10..13  epilogue: tcgen05.ld of the finished accumulator, per-tensor
//                 scale (FP8), bias, rounding to the activation dtype, store.
// The accumulator is double-buffered so the epilogue of tile i overlaps the
// main loop of tile i+1. The UMMA issuer waits on one barrier and commits one
// per k-block (each barrier operation in its loop delays the next UMMA).
// Every mbarrier wait is bounded.
//
// Split-K (problems whose tiles leave most SMs idle, e.g. M = 128): the K
// range of a tile is split over the `ksplit` CTAs of a thread-block cluster
// (one tile per cluster). After the main loops (cluster barrier) every CTA
// owns 256 / ksplit output columns: it sends the other columns of its fp32
// accumulator straight into their owners' shared memory (st.async counted on
// the owner's transaction barrier; the idle operand rings hold the slots),
// then sums the ksplit partials of its own columns in rank order, so the
// result does not depend on timing, and stores them.
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr int BM = 128;  // tokens per tile (UMMA M, TMEM lanes)
constexpr int BN = 256;  // output features per tile (UMMA N, TMEM columns)
constexpr int BK = 64;   // columns per k-block (one 128-byte swizzle row of 16-bit)
constexpr int NS = 3;    // stages (x tile, packed weight tile, converted weight tile)
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpConv0 = 2;
constexpr int kConvWarps = 8;
constexpr int kWarpEpi0 = kWarpConv0 + kConvWarps;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 2 * BN;
constexpr int kXTileBytes = BM * BK * 2;  // 16 KB
constexpr int kBTileBytes = BN * BK * 2;  // 32 KB

template <int FMT>
struct PreFmt;
template <>
struct PreFmt<0> {  // AWQ: 256 rows x 8 words (32 B per row), 32-byte swizzle
  static constexpr int kWcBytes = BN * BK / 2;
  static constexpr int kRowBytes = 32;
};
template <>
struct PreFmt<1> {  // FP8: 256 rows x 64 B, 64-byte swizzle
  static constexpr int kWcBytes = BN * BK;
  static constexpr int kRowBytes = 64;
};

struct PrefillParams {
  const __half* scales;
  const __half* zeros;
  const float* wscale;
  const void* bias;
  void* y;
  DevStatus* status;
  int M, K, N;
  int group_size, G;
  int bias_dtype;
  int num_m_tiles, num_n_tiles, num_kb;
  int ksplit;           // CTAs per tile along K = cluster size (1: no split)
};

template <int FMT>
struct Smem {
  static constexpr int kX = 0;
  static constexpr int kB = kX + NS * kXTileBytes;
  static constexpr int kWc = kB + NS * kBTileBytes;
  static constexpr int kBar = kWc + NS * PreFmt<FMT>::kWcBytes;
  // barriers: full_l[NS], read_w[NS], full_b[NS], mma_done[NS], full_acc[2], empty_acc[2]
  static constexpr int kNumBars = 4 * NS + 4;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kRecvBar = kAbort + 4;  // split-K: partial tiles received (8-byte aligned)
  static constexpr int kTotal = kRecvBar + 8;
  static constexpr int kAlloc = kTotal + 1024;  // room to align the base to 1 KB
  static_assert(kAlloc <= 227 * 1024, "shared memory per CTA");
  // split-K receives up to 128 KB of partial tiles at kX (x and B rings)
  static_assert(kWc - kX >= 128 * 1024, "split-K receive slots");
};

// Per-row dequant parameters for one AWQ group, in the MMA element type.
template <bool BF16>
struct AwqRowParams {
  uint32_t s2;      // {s, s}
  uint32_t zb2;     // {magic + z, magic + z}      (exact path)
  uint32_t magic2;  // {magic, magic}              (general path)
  uint32_t c2;      // {-z*s, -z*s}                (general path)
  bool exact;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float v) {
  if constexpr (BF16) {
    __nv_bfloat162 b = __floats2bfloat162_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&b);
  } else {
    __half2 h = __floats2half2_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2_rn(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <bool BF16>
__device__ __forceinline__ AwqRowParams<BF16> awq_row_params(float s, float z) {
  AwqRowParams<BF16> r;
  constexpr float kMagic = Magic<BF16>::kValue;
  constexpr float kZMax = BF16 ? 127.0f : 1023.0f;
  r.exact = (z == rintf(z)) && fabsf(z) <= kZMax;
  if constexpr (BF16) {
    r.s2 = pack2<true>(s);
  } else {
    r.s2 = pack2<false>(s);  // s is an fp16 value: exact
  }
  r.zb2 = pack2<BF16>(kMagic + z);
  r.magic2 = pack2<BF16>(kMagic);
  r.c2 = pack2<BF16>(-z * s);
  return r;
}

template <bool BF16>
__device__ __forceinline__ uint32_t dq2(uint32_t e, const AwqRowParams<BF16>& rp) {
  if constexpr (BF16) {
    const __nv_bfloat162 ev = *reinterpret_cast<const __nv_bfloat162*>(&e);
    const __nv_bfloat162 s = *reinterpret_cast<const __nv_bfloat162*>(&rp.s2);
    __nv_bfloat162 o;
    if (rp.exact) {
      o = __hmul2(__hsub2(ev, *reinterpret_cast<const __nv_bfloat162*>(&rp.zb2)), s);
    } else {
      o = __hfma2(__hsub2(ev, *reinterpret_cast<const __nv_bfloat162*>(&rp.magic2)), s,
                  *reinterpret_cast<const __nv_bfloat162*>(&rp.c2));
    }
    return *reinterpret_cast<uint32_t*>(&o);
  } else {
    const __half2 ev = *reinterpret_cast<const __half2*>(&e);
    const __half2 s = *reinterpret_cast<const __half2*>(&rp.s2);
    __half2 o;
    if (rp.exact) {
      o = __hmul2(__hsub2(ev, *reinterpret_cast<const __half2*>(&rp.zb2)), s);
    } else {
      o = __hfma2(__hsub2(ev, *reinterpret_cast<const __half2*>(&rp.magic2)), s,
                  *reinterpret_cast<const __half2*>(&rp.c2));
    }
    return *reinterpret_cast<uint32_t*>(&o);
  }
}

// Scale, bias, round and store the 32 values of columns nb .. nb+31 of row m
// (a warp stores 32 consecutive rows; lane i loads the bias of column nb + i).
template <bool BF16>
__device__ __forceinline__ void store_chunk(const PrefillParams& p, const float (&v)[32], int m, int nb,
                                            float wscale, int lane) {
  uint32_t o[16];
  if (p.bias_dtype != NSQ_DTYPE_NONE) {
    const float bl = (nb + lane < p.N) ? load_bias(p.bias, p.bias_dtype, nb + lane) : 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float b0 = __shfl_sync(0xffffffffu, bl, 2 * i);
      const float b1 = __shfl_sync(0xffffffffu, bl, 2 * i + 1);
      o[i] = pack2_rn<BF16>(fmaf(v[2 * i], wscale, b0), fmaf(v[2 * i + 1], wscale, b1));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = pack2_rn<BF16>(v[2 * i] * wscale, v[2 * i + 1] * wscale);
  }
  if (m < p.M) {
    uint16_t* dst = static_cast<uint16_t*>(p.y) + (int64_t)m * p.N + nb;
    if ((p.N & 7) == 0 && nb + 32 <= p.N) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (nb + i < p.N) dst[i] = static_cast<uint16_t>(o[i >> 1] >> (16 * (i & 1)));
      }
    }
  }
}

template <int FMT, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) prefill_linear_kernel(
    const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
    const PrefillParams p) {
  using L = Smem<FMT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  // Per stage s: full_l (TMA bytes of x and the packed weight), read_w (the
  // converters read the packed weight), full_b (the converters wrote B;
  // implies full_l), mma_done (the UMMAs of the stage finished: frees x and B).
  uint64_t* full_l = bars;
  uint64_t* read_w = bars + NS;
  uint64_t* full_b = bars + 2 * NS;
  uint64_t* mma_done = bars + 3 * NS;
  uint64_t* full_acc = bars + 4 * NS;
  uint64_t* empty_acc = full_acc + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full_l[i], 1);
      mbar_init(&read_w[i], kConvWarps);
      mbar_init(&full_b[i], kConvWarps);
      mbar_init(&mma_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full_acc[i], 1);
      mbar_init(&empty_acc[i], kEpiWarps);
    }
    if (p.ksplit > 1) {
      // the other CTAs of the cluster send (ksplit - 1) slices of 128 rows x
      // 256 / ksplit fp32 columns into this CTA
      uint64_t* rbar = reinterpret_cast<uint64_t*>(smem + L::kRecvBar);
      mbar_init(rbar, 1);
      fence_barrier_init();
      mbar_arrive_expect_tx(rbar, (uint32_t)((p.ksplit - 1) * BM * (BN / p.ksplit) * 4));
    }
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // everything below may read what the previous kernel on the stream wrote
  pdl_wait_prior_grids();

  const int num_tiles = p.num_m_tiles * p.num_n_tiles;
  const int num_units = num_tiles * p.ksplit;  // (tile, K range) pairs
  // k-blocks [lo, hi) of unit u
  auto unit_kb = [&](int u, int& lo, int& hi) {
    const int ks = u % p.ksplit;
    lo = (int)(((int64_t)ks * p.num_kb) / p.ksplit);
    hi = (int)(((int64_t)(ks + 1) * p.num_kb) / p.ksplit);
  };
  bool ok = true;

  if (warp == kWarpTma) {
    if (lane == 0) {
      tma_prefetch_desc(&xmap);
      tma_prefetch_desc(&wmap);
      int it = 0;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int tile = u / p.ksplit;
        const int mt = tile / p.num_n_tiles;
        const int nt = tile - mt * p.num_n_tiles;
        int kb_lo, kb_hi;
        unit_kb(u, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
          const int s = it % NS;
          const uint32_t ph = ((it / NS) & 1) ^ 1;  // previous use of the stage
          if (!(ok = mbar_wait(&read_w[s], ph, p.status, 10, abort_flag))) break;
          if (!(ok = mbar_wait(&mma_done[s], ph, p.status, 11, abort_flag))) break;
          mbar_arrive_expect_tx(&full_l[s], kXTileBytes + PreFmt<FMT>::kWcBytes);
          tma_load_2d(smem + L::kX + s * kXTileBytes, &xmap, &full_l[s], kb * BK, mt * BM);
          tma_load_2d(smem + L::kWc + s * PreFmt<FMT>::kWcBytes, &wmap, &full_l[s],
                      FMT == 0 ? kb * (BK / 8) : kb * BK, nt * BN);
        }
      }
      // let in-flight copies land before the CTA can exit
      if (!ok) {
        const int last = it;
        for (int j = (last > NS ? last - NS : 0); j < last; ++j) {
          mbar_wait(&full_l[j % NS], (j / NS) & 1, nullptr, 0, nullptr);
        }
      }
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BF16, BM, BN);
      int it = 0, tcount = 0;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++tcount) {
        const int acc = tcount & 1;
        const uint32_t ar = tcount >> 1;
        if (!(ok = mbar_wait(&empty_acc[acc], (ar & 1) ^ 1, p.status, 20, abort_flag))) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        int kb_lo, kb_hi;
        unit_kb(u, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
          const int s = it % NS;
          if (!(ok = mbar_wait(&full_b[s], (it / NS) & 1, p.status, 22, abort_flag))) break;
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(smem + L::kX + s * kXTileBytes));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(smem + L::kB + s * kBTileBytes));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // +32 bytes along K inside the swizzled row = +2 in the address field
            umma_f16(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > kb_lo || kk > 0) ? 1u : 0u);
          }
          tc_commit(&mma_done[s]);
        }
        if (!ok) break;
        tc_commit(&full_acc[acc]);
      }
    }
  } else if (warp < kWarpEpi0) {
    // ---------------- converters: one weight row per thread ----------------
    const int row = (warp - kWarpConv0) * 32 + lane;  // 0..255
    int it = 0;
    AwqRowParams<BF16> rp{};
    // AWQ: raw fp16 (scale, zero) of the k-block about to be converted, loaded
    // one k-block ahead so the global-load latency hides behind a conversion
    const unsigned short* sc16 = reinterpret_cast<const unsigned short*>(p.scales);
    const unsigned short* zr16 = reinterpret_cast<const unsigned short*>(p.zeros);
    auto fetch_sz = [&](int u, int kb, unsigned short& s16, unsigned short& z16) {
      s16 = 0;
      z16 = 0;
      if (u < num_units) {
        const int n = ((u / p.ksplit) % p.num_n_tiles) * BN + row;
        if (n < p.N) {
          const int64_t off = (int64_t)n * p.G + (kb * BK) / p.group_size;
          s16 = __ldg(sc16 + off);
          z16 = __ldg(zr16 + off);
        }
      }
    };
    unsigned short cur_s = 0, cur_z = 0;
    if constexpr (FMT == 0) {
      int lo0, hi0;
      unit_kb(blockIdx.x, lo0, hi0);
      fetch_sz(blockIdx.x, lo0, cur_s, cur_z);
    }
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int kb_lo, kb_hi;
      unit_kb(u, kb_lo, kb_hi);
      for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
        const int s = it % NS;
        const uint32_t ph = (it / NS) & 1;
        if constexpr (FMT == 0) {
          unsigned short nxt_s, nxt_z;
          if (kb + 1 < kb_hi) {
            fetch_sz(u, kb + 1, nxt_s, nxt_z);
          } else {
            int lo1, hi1;
            unit_kb(u + gridDim.x, lo1, hi1);
            fetch_sz(u + gridDim.x, lo1, nxt_s, nxt_z);
          }
          if (kb == kb_lo || (kb * BK) % p.group_size == 0) {
            rp = awq_row_params<BF16>(__half2float(__ushort_as_half(cur_s)),
                                      __half2float(__ushort_as_half(cur_z)));
          }
          cur_s = nxt_s;
          cur_z = nxt_z;
        }
        if (!(ok = mbar_wait(&full_l[s], ph, p.status, 30, abort_flag))) break;
        if (!(ok = mbar_wait(&mma_done[s], ph ^ 1, p.status, 31, abort_flag))) break;
        const uint32_t wc = smem_u32(smem + L::kWc + s * PreFmt<FMT>::kWcBytes) +
                            row * PreFmt<FMT>::kRowBytes;
        const uint32_t brow = smem_u32(smem + L::kB + s * kBTileBytes) + row * 128;
        if constexpr (FMT == 0) {
          // 32-byte swizzle: 16-byte chunk c of row r sits at c ^ ((r >> 2) & 1)
          const uint32_t sw = (row >> 2) & 1;
          const uint4 v0 = lds128(wc + ((0 ^ sw) << 4));
          const uint4 v1 = lds128(wc + ((1 ^ sw) << 4));
          const uint32_t words[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            uint32_t e[4];
            unpack_nibble_pairs<BF16>(words[w], e);
            // e[t] = {q_t, q_{t+4}}  ->  in-order pairs {q0,q1},{q2,q3},{q4,q5},{q6,q7}
            const uint32_t o0 = dq2<BF16>(prmt(e[0], e[1], 0x5410), rp);
            const uint32_t o1 = dq2<BF16>(prmt(e[2], e[3], 0x5410), rp);
            const uint32_t o2 = dq2<BF16>(prmt(e[0], e[1], 0x7632), rp);
            const uint32_t o3 = dq2<BF16>(prmt(e[2], e[3], 0x7632), rp);
            sts128(brow + ((w ^ (row & 7)) << 4), o0, o1, o2, o3);
          }
        } else {
          // 64-byte swizzle: 16-byte chunk c of row r sits at c ^ ((r >> 1) & 3)
          const uint32_t sw = (row >> 1) & 3;
#pragma unroll
          for (int cch = 0; cch < 4; ++cch) {
            const uint4 v = lds128(wc + ((cch ^ sw) << 4));
            uint32_t o0, o1, o2, o3, o4, o5, o6, o7;
            e4m3x4_to_pairs<BF16>(v.x, o0, o1);
            e4m3x4_to_pairs<BF16>(v.y, o2, o3);
            e4m3x4_to_pairs<BF16>(v.z, o4, o5);
            e4m3x4_to_pairs<BF16>(v.w, o6, o7);
            sts128(brow + (((2 * cch) ^ (row & 7)) << 4), o0, o1, o2, o3);
            sts128(brow + (((2 * cch + 1) ^ (row & 7)) << 4), o4, o5, o6, o7);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&read_w[s]);
          mbar_arrive(&full_b[s]);
        }
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> y ----------------
    const int sub = warp & 3;  // TMEM sub-partition this warp may access
    const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
    int tcount = 0;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++tcount) {
      const int tile = u / p.ksplit;
      const int mt = tile / p.num_n_tiles;
      const int nt = tile - mt * p.num_n_tiles;
      const int acc = tcount & 1;
      const uint32_t ar = tcount >> 1;
      if (!(ok = mbar_wait(&full_acc[acc], ar & 1, p.status, 40, abort_flag))) break;
      tc_fence_after();
      const int m = mt * BM + sub * 32 + lane;
      const uint32_t taddr = tmem_base + ((uint32_t)(sub * 32) << 16) + acc * BN;
      if (p.ksplit == 1) {
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + cc * 32, r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          store_chunk<BF16>(p, v, m, nt * BN + cc * 32, wscale, lane);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_acc[acc]);
        continue;
      }
      // split-K: the accumulator stays in TMEM for the exchange below
      break;
    }
  }

  if (p.ksplit > 1) {
    // every CTA of the cluster is done with its main loop: all operand rings
    // are free to receive the partial tiles
    __syncwarp();
    cluster_arrive_rel();
    cluster_wait_acq();
    if (warp >= kWarpEpi0 && ok) {
      const int KS = p.ksplit;
      const int me = (int)cluster_ctarank();
      const int cpo = (BN / 32) / KS;               // 32-column chunks owned per CTA
      const int sub = warp & 3;
      const int r_in = sub * 32 + lane;             // this thread's row of the tile
      const int tile = blockIdx.x / KS;
      const int mt = tile / p.num_n_tiles;
      const int nt = tile - mt * p.num_n_tiles;
      const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
      uint64_t* rbar = reinterpret_cast<uint64_t*>(smem + L::kRecvBar);
      // slot q (partial of rank q) of an owner: [128 rows][cpo * 8 units of
      // 16 B], unit u of row r at (u & ~7) | ((u & 7) ^ (r & 7))
      const uint32_t slot_bytes = BM * cpo * 128;
      const uint32_t row_off = (uint32_t)r_in * cpo * 128;
      const uint32_t taddr = tmem_base + ((uint32_t)(sub * 32) << 16);  // accumulator 0
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + cc * 32, r);
        tmem_ld_wait();
        const int owner = cc / cpo, lc = cc - owner * cpo;
        const uint32_t local = smem_u32(smem + L::kX) + me * slot_bytes + row_off;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t u = (uint32_t)(lc * 8 + j);
          const uint32_t off = (((u & ~7u) | ((u & 7u) ^ (uint32_t)(r_in & 7))) << 4);
          if (owner == me) {
            sts128(local + off, r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
          } else {
            st_async_f32x4(dsmem_map(local + off, (uint32_t)owner), __uint_as_float(r[4 * j]),
                           __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                           __uint_as_float(r[4 * j + 3]), dsmem_map(smem_u32(rbar), (uint32_t)owner));
          }
        }
      }
      named_bar_sync(3, kEpiWarps * 32);  // this CTA's own slot is written
      if (mbar_wait(rbar, 0, p.status, 41, nullptr)) {
        const int m = mt * BM + r_in;
        const uint32_t base = smem_u32(smem + L::kX) + row_off;
#pragma unroll 1
        for (int lc = 0; lc < cpo; ++lc) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
          for (int q = 0; q < KS; ++q) {  // rank order: the sum does not depend on timing
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t u = (uint32_t)(lc * 8 + j);
              const uint4 w = lds128(base + q * slot_bytes + ((((u & ~7u) | ((u & 7u) ^ (uint32_t)(r_in & 7)))) << 4));
              v[4 * j] += __uint_as_float(w.x);
              v[4 * j + 1] += __uint_as_float(w.y);
              v[4 * j + 2] += __uint_as_float(w.z);
              v[4 * j + 3] += __uint_as_float(w.w);
            }
          }
          store_chunk<BF16>(p, v, m, nt * BN + (me * cpo + lc) * 32, wscale, lane);
        }
      }
      tc_fence_before();  // the TMEM reads above precede the deallocation
    }
  }

  pdl_launch_dependents();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int FMT, bool BF16>
cudaError_t launch_t(const CUtensorMap& xmap, const CUtensorMap& wmap, const PrefillParams& p, int grid,
                     cudaStream_t stream) {
  using L = Smem<FMT>;
  auto kern = prefill_linear_kernel<FMT, BF16>;
  static std::atomic<bool> configured{false};
  if (!configured.load()) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
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

}  // namespace

int prefill_split_factor(int64_t M, int64_t K, int64_t N) {
  // clusters of 2, 4 or 8 CTAs along K, one tile each, when the tiles alone
  // would leave at least half of the SMs idle and K is long enough for the
  // shorter main loops to pay for the exchange (measured on B200: K = 4864
  // gains 1.4-2.2x at M = 128 / 1024, K = 896 loses)
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int64_t kb = (K + BK - 1) / BK;
  const int sms = num_sms();
  if (M <= kDecodeMaxM || tiles * 2 > sms || kb < 32) return 1;
  int ks = 8;
  while (ks > 1 && (tiles * ks > sms || ks > kb)) ks >>= 1;
  return ks;
}

int run_prefill_linear(const LinearArgs& a, cudaStream_t stream) {
  CUtensorMap xmap, wmap;
  CUresult cr = encode_tensor_map_2d(
      &xmap, a.x_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
      const_cast<void*>(a.x), (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2, BK, BM,
      CU_TENSOR_MAP_SWIZZLE_128B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  if (a.fmt == 0) {
    cr = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                              (uint64_t)a.K / 8, (uint64_t)a.N, (uint64_t)a.K / 2, BK / 8, BN,
                              CU_TENSOR_MAP_SWIZZLE_32B);
  } else {
    cr = encode_tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<void*>(a.wq),
                              (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, BK, BN,
                              CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  PrefillParams p{};
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
  p.num_m_tiles = (a.M + BM - 1) / BM;
  p.num_n_tiles = (a.N + BN - 1) / BN;
  p.num_kb = (a.K + BK - 1) / BK;
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int sms = num_sms();
  int grid = tiles < sms ? tiles : sms;
  // split K over a cluster when the tiles leave most SMs idle: one tile per
  // cluster, one K range per CTA (the operand rings are free at the end)
  p.ksplit = prefill_split_factor(a.M, a.K, a.N);
  if (p.ksplit > 1) grid = tiles * p.ksplit;
  cudaError_t e;
  if (a.fmt == 0) {
    e = a.x_bf16 ? launch_t<0, true>(xmap, wmap, p, grid, stream)
                 : launch_t<0, false>(xmap, wmap, p, grid, stream);
  } else {
    e = a.x_bf16 ? launch_t<1, true>(xmap, wmap, p, grid, stream)
                 : launch_t<1, false>(xmap, wmap, p, grid, stream);
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // namespace nsq
