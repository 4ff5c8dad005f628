// Streaming decode linear (M <= 64 tokens) for weights larger than one wave
// of CTAs can hold on chip: persistent CTAs (one per SM) each own a contiguous
// range of output rows and stream their weight rows through a shared-memory
// ring, K stage by K stage, while the warps consume the previous stages.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152 and :49-52) for small batches on large layers
// (e.g. Llama-3-8B gate/up/down). The reference dequantises the weight and
// calls cuBLAS.
//
// Roles in a CTA (12 consumer warps + 1 producer warp):
//   producer: one lane requests stage after stage of the CTA's weight rows
//     with TMA, two boxes of (rows x 128 B) per stage straight from the
//     reference layout, written with the 128-byte swizzle; a stage is reused
//     once all 12 consumer warps have released it (mbarrier ring);
//   consumers: stage the scales / zero points of their rows once (AWQ); then
//     per stage: read the next stage's x with every load in flight, compute
//     the current stage with mma.sync m16n8k16 (weight rows = MMA M, tokens =
//     MMA N), release the stage, and store the next x (permuted into the MMA
//     operand order for AWQ, with per-piece sums) into the other x buffer.
//     A row group of 16 rows belongs to 1, 2 or 4 warps that split each stage's
//     pieces; their partial tiles meet in shared memory at the end.
// AWQ arithmetic is the one of the single-wave kernel, with the zero point
// folded through per-piece sums of x:
//   y += s * (sum_k (magic+q_k) x_k - (magic+z) * sum_k x_k).
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr int kCWarps = 12;                    // consumer warps (13 warps: 128 registers each)
constexpr int kCThreads = kCWarps * 32;
constexpr int kSThreads = kCThreads + 32;      // + the producer warp
constexpr int kMaxRGS = kCWarps;               // row groups per CTA (one warp each at least)
constexpr int kMaxStages = 8;                  // depth of the weight ring
constexpr int kSmemMaxS = 200 * 1024;
constexpr int kSzBudget = 40 * 1024;           // staged scales + zero points (AWQ)

template <int FMT>
struct StreamFmt;
template <>
struct StreamFmt<0> {  // AWQ: a piece is 128 columns = 64 B of a weight row
  static constexpr int kPieceK = 128;
  static constexpr int kChunks = 16;  // 16-byte chunks of x per token per piece
};
template <>
struct StreamFmt<1> {  // FP8: a piece is 64 columns = 64 B of a weight row
  static constexpr int kPieceK = 64;
  static constexpr int kChunks = 8;
};

struct StreamParams {
  const void* x;
  const __half* scales;
  const __half* zeros;
  const float* wscale;
  const void* bias;
  void* y;
  DevStatus* status;
  int M, K, N;
  int G;             // AWQ groups per row
  FastDiv gpp;       // AWQ pieces per group
  int NG, P;         // row groups of 16 in N, pieces in K
  int C;             // CTAs
  int ppst;          // pieces per stage (2 or 4)
  int nst;           // ring depth
  int nstage;        // stages over K
  int kw;            // warps per row group (1, 2 or 4)
  int xrs;           // bytes per token row of an x buffer
  int rs;            // fp32 stride of a token row of the partial tile
  int bias_dtype;
  int stage_bytes;   // weight bytes of one stage for the tallest CTA
  FastDiv divC[1];   // 4-chunk items per x row of a stage
  int off_x, off_xsum, off_sz, off_bar;
};

template <int FMT>
__device__ __forceinline__ int xpos_s(int qq, int t) {
  if constexpr (FMT == 0) {
    return qq ^ ((qq >> 3) & 1) ^ ((t & 1) << 1);
  } else {
    return qq ^ (t & 1);
  }
}

__device__ __forceinline__ uint4 ldg128_cg(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <bool BF16>
__device__ __forceinline__ float chunk_sum_s(const uint4& v) {
  if constexpr (BF16) {
    return ((__uint_as_float(v.x << 16) + __uint_as_float(v.x & 0xFFFF0000u)) +
            (__uint_as_float(v.y << 16) + __uint_as_float(v.y & 0xFFFF0000u))) +
           ((__uint_as_float(v.z << 16) + __uint_as_float(v.z & 0xFFFF0000u)) +
            (__uint_as_float(v.w << 16) + __uint_as_float(v.w & 0xFFFF0000u)));
  } else {
    const uint32_t r[4] = {v.x, v.y, v.z, v.w};
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r[e]));
      s += f.x + f.y;
    }
    return s;
  }
}

// x[:, stage s] of this CTA in items of 4 chunks (64 B of one token row):
// every load of a stage is issued first, the stores come after the MMAs.
// NX items per consumer thread (2 only for AWQ beyond 32 tokens).
template <int NX>
struct XStage {
  uint4 v[NX][4];
  int t[NX], q0[NX];
  bool valid[NX];
};

template <int FMT, int MPAD, int NX>
__device__ __forceinline__ void x_load(const StreamParams& p, int s, int tid, XStage<NX>& xs) {
  using F = StreamFmt<FMT>;
  const int cpr4 = p.ppst * F::kChunks / 4;
  const uint16_t* x = static_cast<const uint16_t*>(p.x);
#pragma unroll
  for (int n = 0; n < NX; ++n) {
    const int it = tid + n * kCThreads;
    xs.t[n] = (int)fdiv((uint32_t)it, p.divC[0]);
    xs.q0[n] = 4 * (it - xs.t[n] * cpr4);
    xs.valid[n] = it < MPAD * cpr4;
    const int k = s * p.ppst * F::kPieceK + 8 * xs.q0[n];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      xs.v[n][e] = make_uint4(0u, 0u, 0u, 0u);
      if (xs.valid[n] && xs.t[n] < p.M && k + 8 * e < p.K) {
        xs.v[n][e] = ldg128_cg(x + (int64_t)xs.t[n] * p.K + k + 8 * e);
      }
    }
  }
}

template <int FMT, bool BF16, int NX>
__device__ __forceinline__ void x_store(const StreamParams& p, uint32_t xbuf, float* xsum,
                                        const XStage<NX>& xs) {
#pragma unroll
  for (int n = 0; n < NX; ++n) {
    const uint32_t row = xbuf + xs.t[n] * p.xrs;
    if constexpr (FMT == 0) {
      if (xs.valid[n]) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint4& v = xs.v[n][e];
          sts128(row + xpos_s<0>(xs.q0[n] + e, xs.t[n]) * 16, prmt(v.x, v.z, 0x5410),
                 prmt(v.x, v.z, 0x7632), prmt(v.y, v.w, 0x5410), prmt(v.y, v.w, 0x7632));
        }
      }
      // the 4 items of one (token, piece) sit on 4 consecutive lanes
      float sm = (chunk_sum_s<BF16>(xs.v[n][0]) + chunk_sum_s<BF16>(xs.v[n][1])) +
                 (chunk_sum_s<BF16>(xs.v[n][2]) + chunk_sum_s<BF16>(xs.v[n][3]));
      sm += __shfl_xor_sync(0xffffffffu, sm, 1);
      sm += __shfl_xor_sync(0xffffffffu, sm, 2);
      if (xs.valid[n] && (xs.q0[n] & 15) == 0) xsum[xs.t[n] * 4 + (xs.q0[n] >> 4)] = sm;
    } else {
      if (xs.valid[n]) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          sts128(row + xpos_s<1>(xs.q0[n] + e, xs.t[n]) * 16, xs.v[n][e].x, xs.v[n][e].y, xs.v[n][e].z,
                 xs.v[n][e].w);
        }
      }
    }
  }
}

template <int FMT, bool BF16, int MT>
__global__ void __launch_bounds__(kSThreads, 1) decode_stream_kernel(
    const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
    const StreamParams p) {
  using F = StreamFmt<FMT>;
  constexpr int MPAD = MT * 8;
  constexpr int NX = (FMT == 0 && MT > 4) ? 2 : 1;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  // this CTA's row groups [rg0, rg0 + RGc)
  const int rg0 = (int)(((int64_t)blockIdx.x * p.NG) / p.C);
  const int RGc = (int)(((int64_t)(blockIdx.x + 1) * p.NG) / p.C) - rg0;
  const int R = 16 * RGc;
  const int n0 = 16 * rg0;
  const int RGhi = (p.NG + p.C - 1) / p.C;
  const CUtensorMap* map = (RGc == RGhi) ? &map_hi : &map_lo;
  const int box_bytes = R * 128;  // one box: all rows x 128 B

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* empty = full + kMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMaxStages);
  float* xsum = reinterpret_cast<float*>(smem + p.off_xsum);  // [2][MPAD][4]
  const uint32_t xbuf0 = smem_u32(smem + p.off_x);
  const int xbuf_bytes = MPAD * p.xrs;

  if (tid == 0) {
    for (int i = 0; i < p.nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kCWarps) {
    // ---------------- producer: the weight ring ----------------
    if (lane == 0) {
      tma_prefetch_desc(map);
      const int kword_stage = p.ppst * 16;  // 32-bit words of a row per stage
      for (int s = 0; s < p.nstage; ++s) {
        const int slot = s % p.nst;
        const uint32_t ph = (uint32_t)(s / p.nst) & 1u;
        if (!mbar_wait(&empty[slot], ph ^ 1u, p.status, 0x41, abort_flag)) break;
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(p.ppst * 64 * R));
        uint8_t* dst = smem + slot * p.stage_bytes;
        for (int h = 0; h < p.ppst / 2; ++h) {
          tma_load_2d(dst + h * box_bytes, map, &full[slot], s * kword_stage + h * 32, n0);
        }
      }
    }
    pdl_launch_dependents();
    return;
  }

  // ---------------- consumers ----------------
  // A slot is (pair of row groups, piece of a stage): the two row groups share
  // every x fragment the slot loads. The CTA has ceil(RGc / 2) * ppst slots and
  // warp w owns slots w, w + 12, ... (at most SMAX, each with accumulators that
  // live across the stages), so all warps work whatever the row count.
  constexpr int SMAX = MT <= 2 ? 2 : 1;
  const int ppst = p.ppst;
  const int lpp = ppst == 4 ? 2 : 1;  // log2(ppst)
  const int nslots = ((RGc + 1) >> 1) * ppst;
  const int G = p.G;

  // scales and biased zero points of this CTA's rows as fp32 pairs, staged
  // once (weights: before the wait)
  const float2* szp = reinterpret_cast<const float2*>(smem + p.off_sz);  // [R][G]
  if constexpr (FMT == 0) {
    // the CTA's rows are one contiguous block of R * G halves in each table;
    // 8 entries (16 B) per load, every load of the block in flight at once
    const int total8 = (R * G) >> 3;          // R is a multiple of 16
    const int valid8 = (min(R, p.N - n0) * G) >> 3;  // entries of rows < N (G * rows % 8 == 0 below)
    const uint4* s_src = reinterpret_cast<const uint4*>(p.scales + (int64_t)n0 * G);
    const uint4* z_src = reinterpret_cast<const uint4*>(p.zeros + (int64_t)n0 * G);
    float4* sd = reinterpret_cast<float4*>(smem + p.off_sz);
    constexpr int kU = 4;
    for (int base = 0; base < total8; base += kCThreads * kU) {
      uint4 sv[kU], zv[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = base + tid + u * kCThreads;
        sv[u] = make_uint4(0u, 0u, 0u, 0u);
        zv[u] = sv[u];
        if (i < valid8) {
          sv[u] = __ldg(s_src + i);
          zv[u] = __ldg(z_src + i);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = base + tid + u * kCThreads;
        if (i < total8) {
          const uint32_t sw[4] = {sv[u].x, sv[u].y, sv[u].z, sv[u].w};
          const uint32_t zw[4] = {zv[u].x, zv[u].y, zv[u].z, zv[u].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 sf = __half22float2(*reinterpret_cast<const __half2*>(&sw[e]));
            const float2 zf = __half22float2(*reinterpret_cast<const __half2*>(&zw[e]));
            sd[4 * i + e] = make_float4(sf.x, Magic<BF16>::kValue + zf.x, sf.y, Magic<BF16>::kValue + zf.y);
          }
        }
      }
    }
  }
  float wscale = 1.0f;
  if constexpr (FMT == 1) {
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(wscale) : "l"(p.wscale));
  }

  float acc[SMAX][2][MT][4];
#pragma unroll
  for (int k = 0; k < SMAX; ++k)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int jt = 0; jt < MT; ++jt) acc[k][h][jt][0] = acc[k][h][jt][1] = acc[k][h][jt][2] = acc[k][h][jt][3] = 0.f;

  // per-thread fragment addresses in x buffer 0 for token tile jt, chunk i of a piece
  uint32_t xa[MT][4];
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t off = FMT == 0 ? xpos_s<0>(4 * c + i, g) * 16 : xpos_s<1>(2 * c + (i & 1), g) * 16;
      xa[jt][i] = xbuf0 + (8 * jt + g) * p.xrs + off;
    }
  }
  // per-slot weight offset inside a stage: rows 32 rp + g (+ 8, + 16, + 24) of
  // box jj / 2, piece jj & 1 of the 128 B, 128-byte swizzle (chunk ^ row % 8)
  uint32_t woff[SMAX];
#pragma unroll
  for (int k = 0; k < SMAX; ++k) {
    const int q = warp + k * kCWarps;
    const int rp = q >> lpp, jj = q & (ppst - 1);
    woff[k] = (uint32_t)((jj >> 1) * box_bytes + (32 * rp + g) * 128 + (((4 * (jj & 1) + c) ^ (g & 7)) * 16));
  }

  // x (produced by the previous kernel) for stage 0
  pdl_wait_prior_grids();
  {
    XStage<NX> xs;
    x_load<FMT, MPAD, NX>(p, 0, tid, xs);
    x_store<FMT, BF16, NX>(p, xbuf0, xsum, xs);
  }
  named_bar_sync(1, kCThreads);

  bool ok = true;
  for (int s = 0; s < p.nstage; ++s) {
    const int slot = s % p.nst;
    const uint32_t ph = (uint32_t)(s / p.nst) & 1u;
    const uint32_t xbo = (s & 1) * xbuf_bytes;  // offset of this stage's x buffer
    const float* xsm = xsum + (s & 1) * MPAD * 4;
    const int valid = min(ppst, p.P - s * ppst);  // pieces of this stage inside K
    // next stage's x: loads in flight during this stage's MMAs
    XStage<NX> xs;
    const bool more = s + 1 < p.nstage;
    if (more) x_load<FMT, MPAD, NX>(p, s + 1, tid, xs);
    if (ok) ok = mbar_wait(&full[slot], ph, p.status, 0x42, abort_flag);
    const uint32_t wst = smem_u32(smem + slot * p.stage_bytes);
#pragma unroll
    for (int k = 0; k < SMAX; ++k) {
      const int q = warp + k * kCWarps;
      const int rp = q >> lpp, jj = q & (ppst - 1);
      if (!ok || q >= nslots || jj >= valid) continue;
      const bool two = 2 * rp + 1 < RGc;  // the pair's second row group exists
      const uint32_t wrow = wst + woff[k];
      const uint4 w0 = lds128(wrow);              // row 32 rp + g
      const uint4 w1 = lds128(wrow + 8 * 128);    // + 8
      uint4 w2 = make_uint4(0u, 0u, 0u, 0u), w3 = w2;
      if (two) {
        w2 = lds128(wrow + 16 * 128);             // + 16
        w3 = lds128(wrow + 24 * 128);             // + 24
      }
      const uint32_t wA[4] = {w0.x, w0.y, w0.z, w0.w}, wB[4] = {w1.x, w1.y, w1.z, w1.w};
      const uint32_t wC[4] = {w2.x, w2.y, w2.z, w2.w}, wD[4] = {w3.x, w3.y, w3.z, w3.w};
      const uint32_t xp = xbo + (uint32_t)jj * (F::kChunks * 16);
      if constexpr (FMT == 0) {
        const int grp = (int)fdiv((uint32_t)(s * ppst + jj), p.gpp);
        const float2* sz0 = szp + (32 * rp + g) * G + grp;
        const float2 sa = sz0[0], sb = sz0[8 * G];  // (scale, magic + zero) of rows g, g + 8
        float2 sc2 = make_float2(0.f, 0.f), sd2 = sc2;
        if (two) {
          sc2 = sz0[16 * G];
          sd2 = sz0[24 * G];
        }
        float part[2][MT][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int jt = 0; jt < MT; ++jt) part[h][jt][0] = part[h][jt][1] = part[h][jt][2] = part[h][jt][3] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t a0[4], a1[4], b0[4], b1[4];
          nibble_quads<BF16>(wA[i], wB[i], a0, a1);
          nibble_quads<BF16>(wC[i], wD[i], b0, b1);
#pragma unroll
          for (int jt = 0; jt < MT; ++jt) {
            const uint4 xv = lds128(xa[jt][i] + xp);
            mma_16816<BF16>(part[0][jt], a0, xv.x, xv.y);
            mma_16816<BF16>(part[0][jt], a1, xv.z, xv.w);
            mma_16816<BF16>(part[1][jt], b0, xv.x, xv.y);
            mma_16816<BF16>(part[1][jt], b1, xv.z, xv.w);
          }
        }
#pragma unroll
        for (int jt = 0; jt < MT; ++jt) {
          const float x0 = xsm[(8 * jt + 2 * c) * 4 + jj];
          const float x1 = xsm[(8 * jt + 2 * c + 1) * 4 + jj];
          acc[k][0][jt][0] = fmaf(sa.x, fmaf(-sa.y, x0, part[0][jt][0]), acc[k][0][jt][0]);
          acc[k][0][jt][1] = fmaf(sa.x, fmaf(-sa.y, x1, part[0][jt][1]), acc[k][0][jt][1]);
          acc[k][0][jt][2] = fmaf(sb.x, fmaf(-sb.y, x0, part[0][jt][2]), acc[k][0][jt][2]);
          acc[k][0][jt][3] = fmaf(sb.x, fmaf(-sb.y, x1, part[0][jt][3]), acc[k][0][jt][3]);
          acc[k][1][jt][0] = fmaf(sc2.x, fmaf(-sc2.y, x0, part[1][jt][0]), acc[k][1][jt][0]);
          acc[k][1][jt][1] = fmaf(sc2.x, fmaf(-sc2.y, x1, part[1][jt][1]), acc[k][1][jt][1]);
          acc[k][1][jt][2] = fmaf(sd2.x, fmaf(-sd2.y, x0, part[1][jt][2]), acc[k][1][jt][2]);
          acc[k][1][jt][3] = fmaf(sd2.x, fmaf(-sd2.y, x1, part[1][jt][3]), acc[k][1][jt][3]);
        }
      } else {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint4 xv[MT];
#pragma unroll
          for (int jt = 0; jt < MT; ++jt) xv[jt] = lds128(xa[jt][hh] + xp);
#pragma unroll
          for (int uu = 0; uu < 2; ++uu) {
            const int sidx = 2 * hh + uu;
            uint32_t a[4], b[4];
            e4m3x4_to_pairs<BF16>(wA[sidx], a[0], a[2]);
            e4m3x4_to_pairs<BF16>(wB[sidx], a[1], a[3]);
            e4m3x4_to_pairs<BF16>(wC[sidx], b[0], b[2]);
            e4m3x4_to_pairs<BF16>(wD[sidx], b[1], b[3]);
#pragma unroll
            for (int jt = 0; jt < MT; ++jt) {
              mma_16816<BF16>(acc[k][0][jt], a, uu ? xv[jt].z : xv[jt].x, uu ? xv[jt].w : xv[jt].y);
              mma_16816<BF16>(acc[k][1][jt], b, uu ? xv[jt].z : xv[jt].x, uu ? xv[jt].w : xv[jt].y);
            }
          }
        }
      }
    }
    // this warp is done with the stage's weights
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (more) x_store<FMT, BF16, NX>(p, xbuf0 + ((s + 1) & 1) * xbuf_bytes, xsum + ((s + 1) & 1) * MPAD * 4, xs);
    named_bar_sync(1, kCThreads);  // next x visible; this x free for stage s + 2
  }

  // ---------------- epilogue: slots of a row group meet in shared memory ----------------
  uint16_t* y = static_cast<uint16_t*>(p.y);
  const bool has_bias = p.bias_dtype != NSQ_DTYPE_NONE;
  float* red = reinterpret_cast<float*>(smem + p.off_x);  // the x buffers are free now
  for (int i = tid; i < MPAD * p.rs; i += kCThreads) red[i] = 0.f;
  named_bar_sync(1, kCThreads);
#pragma unroll
  for (int k = 0; k < SMAX; ++k) {
    const int q = warp + k * kCWarps;
    if (q >= nslots) continue;
    const int rp = q >> lpp;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (2 * rp + h >= RGc) continue;
      const int rowg = 32 * rp + 16 * h + g;
#pragma unroll
      for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = 8 * jt + 2 * c + (e & 1);
          if (tok < p.M) atomicAdd(&red[tok * p.rs + rowg + 8 * (e >> 1)], acc[k][h][jt][e]);
        }
      }
    }
  }
  named_bar_sync(1, kCThreads);
  for (int tok = 0; tok < p.M; ++tok) {
    for (int row = tid; row < R; row += kCThreads) {
      const int n = n0 + row;
      if (n < p.N) {
        const float b = has_bias ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
        y[(int64_t)tok * p.N + n] = float_to_elem<BF16>(fmaf(red[tok * p.rs + row], wscale, b));
      }
    }
  }
  // after an abort, let the weight copies in flight land before the CTA exits
  if (!ok && tid == 0) {
    for (int i = 0; i < p.nst; ++i) mbar_wait(&full[i], 0, nullptr, 0, nullptr);
  }
}

}  // namespace

struct StreamPlan {
  bool ok;
  int C, ppst, nst, nstage, kw, xrs, rs, stage_bytes, rg_hi, rg_lo;
  size_t smem;
  int off_x, off_xsum, off_sz, off_bar;
};

StreamPlan plan_decode_stream(int fmt, int M, int K, int N, int group_size) {
  StreamPlan pl{};
  pl.ok = false;
  const int PK = fmt == 0 ? 128 : 64;
  const int mpad = ((M + 7) / 8) * 8;
  const int P = (K + PK - 1) / PK;
  const int NG = (N + 15) / 16;
  const int C = NG < num_sms() ? NG : num_sms();
  const int rg_hi = (NG + C - 1) / C;
  if (rg_hi > kMaxRGS) return pl;
  pl.C = C;
  pl.rg_hi = rg_hi;
  pl.rg_lo = NG / C;
  // pieces per stage: x items of a stage (4 chunks each) stay within one
  // (AWQ beyond 32 tokens: two) per consumer thread
  pl.ppst = fmt == 0 ? (mpad <= 24 ? 4 : 2) : (mpad <= 32 ? 4 : 2);
  // every (row group, piece of a stage) slot needs a warp slot
  const int mt = mpad / 8;
  if (mt > 4) return pl;  // beyond 32 tokens the accumulators no longer fit in registers
  const int smax = mt <= 2 ? 2 : 1;
  if (((rg_hi + 1) / 2) * pl.ppst > kCWarps * smax) return pl;
  pl.kw = 1;
  pl.nstage = (P + pl.ppst - 1) / pl.ppst;
  const int R = 16 * rg_hi;
  pl.stage_bytes = ((R * pl.ppst * 64 + 1023) / 1024) * 1024;
  pl.xrs = pl.ppst * PK * 2;
  pl.rs = R + ((4 - R % 32) + 32) % 32;
  const size_t xbytes = (size_t)2 * mpad * pl.xrs;
  const size_t red_bytes = (size_t)mpad * pl.rs * 4;
  const size_t xreg = xbytes > red_bytes ? xbytes : red_bytes;
  const int G = fmt == 0 ? (K + group_size - 1) / group_size : 0;
  const size_t szb = fmt == 0 ? (size_t)R * G * 8 : 0;  // (scale, magic + zero) as fp32 pairs
  if (szb > (size_t)kSzBudget) return pl;
  const size_t fixed = xreg + (size_t)2 * mpad * 4 * 4 + szb + 2 * kMaxStages * 8 + 16 + 3 * 128;
  int nst = (int)(((size_t)kSmemMaxS - fixed) / (size_t)pl.stage_bytes);
  if (nst > kMaxStages) nst = kMaxStages;
  if (nst > pl.nstage) nst = pl.nstage;
  if (nst < 2 && pl.nstage >= 2) return pl;
  if (nst < 1) return pl;
  pl.nst = nst;
  size_t off = (size_t)nst * pl.stage_bytes;
  pl.off_x = (int)off;
  off += xreg;
  off = (off + 15) & ~(size_t)15;
  pl.off_xsum = (int)off;
  off += (size_t)2 * mpad * 4 * 4;
  pl.off_sz = (int)off;
  off += szb;
  off = (off + 7) & ~(size_t)7;
  pl.off_bar = (int)off;
  off += (size_t)2 * kMaxStages * 8 + 16;
  pl.smem = off;
  if (pl.smem > (size_t)kSmemMaxS) return pl;
  pl.ok = true;
  return pl;
}

namespace {

template <int FMT, bool BF16, int MT>
cudaError_t launch_stream(const CUtensorMap& hi, const CUtensorMap& lo, const StreamParams& p,
                          const StreamPlan& pl, cudaStream_t stream) {
  auto kern = decode_stream_kernel<FMT, BF16, MT>;
  static std::atomic<bool> configured{false};
  if (!configured.load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMaxS);
    if (e != cudaSuccess) return e;
    configured.store(true);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.C, 1, 1);
  cfg.blockDim = dim3(kSThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  int na = 0;
  if (pdl_enabled()) {
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    na = 1;
  }
  cfg.attrs = &attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, hi, lo, p);
}

template <int FMT, bool BF16>
cudaError_t dispatch_stream(int mt, const CUtensorMap& hi, const CUtensorMap& lo,
                            const StreamParams& p, const StreamPlan& pl, cudaStream_t s) {
  switch (mt) {
    case 1: return launch_stream<FMT, BF16, 1>(hi, lo, p, pl, s);
    case 2: return launch_stream<FMT, BF16, 2>(hi, lo, p, pl, s);
    case 3: return launch_stream<FMT, BF16, 3>(hi, lo, p, pl, s);
    case 4: return launch_stream<FMT, BF16, 4>(hi, lo, p, pl, s);
    case 5: return launch_stream<FMT, BF16, 5>(hi, lo, p, pl, s);
    case 6: return launch_stream<FMT, BF16, 6>(hi, lo, p, pl, s);
    case 7: return launch_stream<FMT, BF16, 7>(hi, lo, p, pl, s);
    default: return launch_stream<FMT, BF16, 8>(hi, lo, p, pl, s);
  }
}

}  // namespace

int run_decode_stream_linear(const LinearArgs& a, cudaStream_t stream) {
  if (a.fmt == 0 && a.group_size % 128 != 0) return NSQ_ENOTSUP;
  const StreamPlan pl = plan_decode_stream(a.fmt, a.M, a.K, a.N, a.group_size);
  if (!pl.ok) return NSQ_ENOTSUP;
  if (a.fmt == 0) {
    // the scale / zero-point tables are read 16 bytes at a time
    const int G = (a.K + a.group_size - 1) / a.group_size;
    if ((reinterpret_cast<uintptr_t>(a.scales) & 15) || (reinterpret_cast<uintptr_t>(a.zeros) & 15) ||
        (G * (a.N % 16)) % 8 != 0) {
      return NSQ_ENOTSUP;
    }
  }
  // the weight as rows of 32-bit words, boxes of 32 words (128 B) x all rows of
  // a CTA, 128-byte swizzle; one map per CTA height (they differ by one group)
  const uint64_t row_bytes = a.fmt == 0 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  CUtensorMap hi, lo;
  CUresult cr = encode_tensor_map_2d(&hi, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                                     row_bytes / 4, (uint64_t)a.N, row_bytes, 32, 16 * pl.rg_hi,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  lo = hi;
  if (pl.rg_lo != pl.rg_hi && pl.rg_lo > 0) {
    cr = encode_tensor_map_2d(&lo, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                              row_bytes / 4, (uint64_t)a.N, row_bytes, 32, 16 * pl.rg_lo,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  }
  StreamParams p{};
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
  p.G = a.fmt == 0 ? (a.K + a.group_size - 1) / a.group_size : 0;
  p.gpp = make_fastdiv(a.fmt == 0 ? (uint32_t)(a.group_size / 128) : 1u);
  p.NG = (a.N + 15) / 16;
  p.P = a.fmt == 0 ? (a.K + 127) / 128 : (a.K + 63) / 64;
  p.C = pl.C;
  p.ppst = pl.ppst;
  p.nst = pl.nst;
  p.nstage = pl.nstage;
  p.kw = pl.kw;
  p.xrs = pl.xrs;
  p.rs = pl.rs;
  p.bias_dtype = a.bias ? a.bias_dtype : NSQ_DTYPE_NONE;
  p.stage_bytes = pl.stage_bytes;
  p.divC[0] = make_fastdiv((uint32_t)(pl.ppst * (a.fmt == 0 ? 16 : 8) / 4));
  p.off_x = pl.off_x;
  p.off_xsum = pl.off_xsum;
  p.off_sz = pl.off_sz;
  p.off_bar = pl.off_bar;
  const int mt = (a.M + 7) / 8;
  cudaError_t e;
  if (a.fmt == 0) {
    e = a.x_bf16 ? dispatch_stream<0, true>(mt, hi, lo, p, pl, stream)
                 : dispatch_stream<0, false>(mt, hi, lo, p, pl, stream);
  } else {
    e = a.x_bf16 ? dispatch_stream<1, true>(mt, hi, lo, p, pl, stream)
                 : dispatch_stream<1, false>(mt, hi, lo, p, pl, stream);
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // namespace nsq
