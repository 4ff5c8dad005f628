// Single-wave decode linear (M <= 64 tokens) for weights that fit on chip in
// one wave of CTAs: at most one CTA per SM, so the next linear on the stream
// always finds room to start (programmatic launch) while this one finishes.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152 and :49-52) for small batches; the reference
// dequantises the whole weight and calls cuBLAS.
//
// What a CTA does, in order:
//   before the previous kernel has finished (nothing it reads is produced there):
//     * warp 0 initialises one barrier per row group of 16 rows and requests
//       the CTA's whole weight slice with TMA, one box of 16 rows x 64 B per
//       (row group, piece), straight from the reference layout (qweight
//       [N, K/8] int32, weight_fp8 [N, K] viewed as 32-bit words);
//     * the next kernel on the stream is released;
//     * AWQ scales / biased zero points, bias and the fp8 scale are staged,
//       and the CTA decides whether every zero point is an integer;
//   after it (griddepcontrol.wait):
//     * x[:, K slice] is read (four 16-byte loads in flight per thread),
//       permuted into the MMA operand order (AWQ), XOR-swizzled into shared
//       memory, and summed per 128-column piece only when a zero point is
//       not an integer;
//     * work units (16 rows x one piece) are spread evenly over the warps;
//       each runs mma.sync m16n8k16 with the weight rows as the MMA M dimension
//       and the tokens as N (swap-AB), so 1..64 tokens cost 1..8 n-tiles;
//     * partial tiles meet in shared memory; when K is split over a cluster,
//       every CTA pushes the rows another CTA owns straight into that CTA's
//       shared memory (st.async with a transaction-count barrier) and stores
//       only its own rows.
//
// AWQ arithmetic: a word of 8 sequential nibbles becomes four packed pairs
// {magic+q_t, magic+q_{t+4}} with one lop3 each (magic = 128 for bf16, 1024 for
// fp16; exact), and x is stored pre-permuted into the same pair order.
//   integer zero points (what the reference quantiser produces): one packed
//     subtraction of {magic+z, magic+z} gives q - z exactly, and each piece's
//     MMA sum is scaled by its group's scale in fp32;
//   any other zero point: y += s * (sum_k (magic+q_k) x_k - (magic+z) sum_k x_k).
// FP8: e4m3 pairs convert exactly to the MMA type; the per-tensor scale is
// applied once in the epilogue.
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr int kMaxRG = 64;             // row groups (one barrier each) per CTA
constexpr int kSmemMax = 112 * 1024;   // two CTAs per SM: this launch and the next one
constexpr int kWBudget = 80 * 1024;    // weight slice held in shared memory
constexpr int kXBudget = 40 * 1024;    // x slice held in shared memory
constexpr int kBoxBytes = 16 * 64;     // one (row group, piece) box

// FP8 up to 16 tokens: 16 warps (more warps hide the MMA and shared-memory
// latencies) in 64 registers; otherwise 8 warps in 128 registers (the AWQ
// unit needs them: fewer registers spill). Two CTAs per SM either way.
template <int FMT, int MT>
struct WaveThreads {
  static constexpr int kThreads = (MT <= 2 && FMT == 1) ? 512 : 256;
  static constexpr int kWarps = kThreads / 32;
};

template <int FMT>
struct WaveFmt;
template <>
struct WaveFmt<0> {  // AWQ: a piece is 128 columns = 64 B of one weight row = one scale group slice
  static constexpr int kPieceK = 128;
  static constexpr int kChunks = 16;  // 16-byte chunks of x per token per piece
  static constexpr int kSteps = 8;    // k16 MMA steps per piece
};
template <>
struct WaveFmt<1> {  // FP8: a piece is 64 columns = 64 B of one weight row
  static constexpr int kPieceK = 64;
  static constexpr int kChunks = 8;
  static constexpr int kSteps = 4;
};

struct WaveParams {
  const void* x;
  const __half* scales;
  const __half* zeros;
  const float* wscale;
  const void* bias;
  void* y;
  DevStatus* status;
  int M, K, N;
  int G;             // AWQ: groups per row
  FastDiv gpp;       // AWQ: pieces per group
  int NG, P;         // row groups of 16 in N, pieces in K
  int RG, Pc;        // row groups and pieces per CTA
  int rs;            // fp32 stride of a token row of the partial tile
  int xrs;           // bytes per token row of staged x
  int recv_rows;     // rows of a receive slot (cluster split)
  int bias_dtype;
  // divisors precomputed on the host, [0] for a full tile / K slice, [1] for
  // the last (shorter) one: rows R, row pairs R/2, 4-chunk items per x row,
  // and the quads of rows a cluster rank owns (floor / ceil of R/4/S)
  FastDiv divR[2], divR2[2], divC[2], divQ[2][2];
  int off_x, off_xsum, off_sz, off_bias, off_red, off_recv, off_bar;
};

// Position of 16-byte chunk qq of token row t in staged x. AWQ: bit 0 takes
// bit 3 of qq and bit 1 the token parity; FP8: bit 0 takes the token parity.
// Either way the eight lanes of a quarter warp hit eight different 16-byte
// bank groups at every fragment load.
template <int FMT>
__device__ __forceinline__ int xpos(int qq, int t) {
  if constexpr (FMT == 0) {
    return qq ^ ((qq >> 3) & 1) ^ ((t & 1) << 1);
  } else {
    return qq ^ (t & 1);
  }
}

__device__ __forceinline__ uint4 ldg128(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 16-byte store into another CTA's shared memory, counted on its barrier.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, const float4& v,
                                            uint32_t cluster_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          cluster_addr),
      "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(cluster_bar)
      : "memory");
}

// Sum of the 8 elements of a 16-byte chunk (fp32).
template <bool BF16>
__device__ __forceinline__ float chunk_sum(const uint4& v) {
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

template <bool BF16>
__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
  if constexpr (BF16) {
    __nv_bfloat162 r = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                               *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  } else {
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_pair(float v) {
  if constexpr (BF16) {
    __nv_bfloat162 b = __floats2bfloat162_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&b);
  } else {
    __half2 h = __floats2half2_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Rows [lo, hi) of the CTA's tile owned by cluster rank q (multiples of 4).
__device__ __forceinline__ void owner_rows(int q, int S, int R, int& lo, int& hi) {
  const int r4 = R >> 2;
  lo = 4 * ((q * r4) / S);
  hi = 4 * (((q + 1) * r4) / S);
}

struct UnitCtx {
  uint32_t wbase;   // shared address of this thread's first weight chunk (unit 0)
  uint32_t xr[8];   // shared address of token row 8jt + g of staged x
  uint32_t xoff[4]; // per-thread chunk offsets inside a piece
  const float* sz;  // scales [Pa][R], biased zero points at + Pc * R
  const float* xsum;
  int R, Pc, Pa;
};

// The units [u, u1) of one warp, row group by row group, accumulated into
// the partial tile with shared-memory atomics.
template <int FMT, bool BF16, int MT, bool INT_Z>
__device__ __forceinline__ bool run_units(const UnitCtx& cx, const WaveParams& p, uint64_t* wbar,
                                          volatile int* abort_flag, float* red, int u, int u1,
                                          int g, int c) {
  using F = WaveFmt<FMT>;
  bool ok = true;
  int rg = u / cx.Pa;
  int j = u - rg * cx.Pa;
  while (u < u1) {
    if (ok) ok = mbar_wait(&wbar[rg], 0, p.status, 0x31, abort_flag);
    float acc[MT][4];
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) acc[jt][0] = acc[jt][1] = acc[jt][2] = acc[jt][3] = 0.f;
    const int jend = min(cx.Pa, j + (u1 - u));
    if (ok) {
      for (; j < jend; ++j, ++u) {
        const uint32_t wt = cx.wbase + (uint32_t)u * kBoxBytes;
        const uint4 wa = lds128(wt);             // row g
        const uint4 wb = lds128(wt + 8 * 64);    // row g + 8
        const uint32_t wg[4] = {wa.x, wa.y, wa.z, wa.w};
        const uint32_t wh[4] = {wb.x, wb.y, wb.z, wb.w};
        const uint32_t xp = (uint32_t)j * (F::kChunks * 16);
        if constexpr (FMT == 0) {
          const float* szj = cx.sz + j * cx.R + 16 * rg + g;
          const float s0 = szj[0], s1 = szj[8];
          const float zb0 = szj[cx.Pc * cx.R], zb1 = szj[cx.Pc * cx.R + 8];
          uint32_t z2g = 0, z2h = 0;
          if constexpr (INT_Z) {
            z2g = pack_pair<BF16>(zb0);
            z2h = pack_pair<BF16>(zb1);
          }
          float part[MT][4];
#pragma unroll
          for (int jt = 0; jt < MT; ++jt) part[jt][0] = part[jt][1] = part[jt][2] = part[jt][3] = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t eg[4], eh[4];
            unpack_nibble_pairs<BF16>(wg[i], eg);
            unpack_nibble_pairs<BF16>(wh[i], eh);
            if constexpr (INT_Z) {
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                eg[t] = hsub2_bits<BF16>(eg[t], z2g);
                eh[t] = hsub2_bits<BF16>(eh[t], z2h);
              }
            }
            const uint32_t a0[4] = {eg[0], eh[0], eg[1], eh[1]};
            const uint32_t a1[4] = {eg[2], eh[2], eg[3], eh[3]};
#pragma unroll
            for (int jt = 0; jt < MT; ++jt) {
              // x[8jt+g][128j + 32c + 8i .. +7] as pairs (x_t, x_t+4)
              const uint4 xv = lds128(cx.xr[jt] + xp + cx.xoff[i]);
              mma_16816<BF16>(part[jt], a0, xv.x, xv.y);
              mma_16816<BF16>(part[jt], a1, xv.z, xv.w);
            }
          }
#pragma unroll
          for (int jt = 0; jt < MT; ++jt) {
            if constexpr (INT_Z) {
              acc[jt][0] = fmaf(s0, part[jt][0], acc[jt][0]);
              acc[jt][1] = fmaf(s0, part[jt][1], acc[jt][1]);
              acc[jt][2] = fmaf(s1, part[jt][2], acc[jt][2]);
              acc[jt][3] = fmaf(s1, part[jt][3], acc[jt][3]);
            } else {
              const float xa = cx.xsum[(8 * jt + 2 * c) * cx.Pc + j];
              const float xb = cx.xsum[(8 * jt + 2 * c + 1) * cx.Pc + j];
              acc[jt][0] = fmaf(s0, fmaf(-zb0, xa, part[jt][0]), acc[jt][0]);
              acc[jt][1] = fmaf(s0, fmaf(-zb0, xb, part[jt][1]), acc[jt][1]);
              acc[jt][2] = fmaf(s1, fmaf(-zb1, xa, part[jt][2]), acc[jt][2]);
              acc[jt][3] = fmaf(s1, fmaf(-zb1, xb, part[jt][3]), acc[jt][3]);
            }
          }
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 xv[MT];
#pragma unroll
            for (int jt = 0; jt < MT; ++jt) {
              // x[8jt+g][64j + 16c + 8h .. +7]
              xv[jt] = lds128(cx.xr[jt] + xp + cx.xoff[h]);
            }
#pragma unroll
            for (int uu = 0; uu < 2; ++uu) {
              const int s = 2 * h + uu;
              uint32_t a[4];
              e4m3x4_to_pairs<BF16>(wg[s], a[0], a[2]);
              e4m3x4_to_pairs<BF16>(wh[s], a[1], a[3]);
#pragma unroll
              for (int jt = 0; jt < MT; ++jt) {
                mma_16816<BF16>(acc[jt], a, uu ? xv[jt].z : xv[jt].x, uu ? xv[jt].w : xv[jt].y);
              }
            }
          }
        }
      }
    } else {
      u += jend - j;
    }
    // this row group's share -> the partial tile [token][row]
    float* dst = red + 16 * rg + g;
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = 8 * jt + 2 * c + (e & 1);
        if (tok < p.M) atomicAdd(dst + tok * p.rs + 8 * (e >> 1), acc[jt][e]);
      }
    }
    ++rg;
    j = 0;
  }
  return ok;
}

template <int FMT, bool BF16, int MT>
__global__ void __launch_bounds__(WaveThreads<FMT, MT>::kThreads, 2) decode_wave_kernel(
    const __grid_constant__ CUtensorMap wmap, const WaveParams p) {
  using F = WaveFmt<FMT>;
  constexpr int MPAD = MT * 8;
  constexpr int NT = WaveThreads<FMT, MT>::kThreads;
  constexpr int NW = WaveThreads<FMT, MT>::kWarps;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int S = gridDim.x;                // cluster = the K split
  const int rank = blockIdx.x;            // rank in the cluster (cluster dims = (S, 1, 1))
  const int rg0 = blockIdx.y * p.RG;
  const int RGa = min(p.RG, p.NG - rg0);  // row groups of this CTA
  const int R = 16 * RGa;
  const int n0 = 16 * rg0;
  const int pc0 = rank * p.Pc;            // first piece of this CTA
  const int Pa = min(p.Pc, p.P - pc0);    // pieces of this CTA
  const int k0 = pc0 * F::kPieceK;

  uint64_t* wbar = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* rbar = wbar + kMaxRG;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(wbar + kMaxRG + 1);
  const uint32_t xbuf = smem_u32(smem + p.off_x);
  float* xsum = reinterpret_cast<float*>(smem + p.off_xsum);
  float* sz = reinterpret_cast<float*>(smem + p.off_sz);
  float* biasf = reinterpret_cast<float*>(smem + p.off_bias);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  float* recv = reinterpret_cast<float*>(smem + p.off_recv);

  // ---- 1. weight requests: one lane per row group, one box per piece ----
  if (warp == 0) {
    const int kword0 = (FMT == 0 ? k0 / 2 : k0) / 4;
    for (int rg = lane; rg < RGa; rg += 32) {
      uint64_t* bar = &wbar[rg];
      mbar_init(bar, 1);
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar, (uint32_t)(Pa * kBoxBytes));
      uint8_t* dst = smem + rg * Pa * kBoxBytes;
      for (int j = 0; j < Pa; ++j) {
        tma_load_2d(dst + j * kBoxBytes, &wmap, bar, kword0 + 16 * j, n0 + 16 * rg);
      }
    }
  }
  // the receive barrier of the cluster split expects every peer's rows of ours
  int own_lo = 0, own_hi = R;
  if (S > 1) owner_rows(rank, S, R, own_lo, own_hi);
  if (tid == 32) {
    *abort_flag = 0;
    if (S > 1) {
      mbar_init(rbar, 1);
      fence_barrier_init();
      mbar_arrive_expect_tx(rbar, (uint32_t)((S - 1) * p.M * (own_hi - own_lo) * 4));
    }
  }
  // the next kernel on the stream may start its own weight loads now
  pdl_launch_dependents();
  // Kernel parameters live in the constant bank, whose cache is cold for every
  // launch; a field first read after the wait would cost a memory round trip
  // there. Read every 16 bytes of the parameter block now.
  if (warp == 1) {
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(&p);
    const int nw = (int)(sizeof(WaveParams) / 4);
    uint32_t acc = 0;
    for (int i = 4 * lane; i < nw; i += 128) acc ^= pw[i];
    asm volatile("" ::"r"(acc));
  }

  // ---- 2. everything else that does not depend on the previous kernel ----
  {
    float4* r4 = reinterpret_cast<float4*>(red);
    for (int i = tid; i < MPAD * p.rs / 4; i += NT) r4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  bool all_int = true;
  if constexpr (FMT == 0) {
    // scale and biased zero point per (piece, row): sz[j][row], sz[Pc + j][row]
    constexpr float kMagic = Magic<BF16>::kValue;
    constexpr float kZMax = BF16 ? 127.0f : 1023.0f;  // magic + z stays exact
    const FastDiv divR = p.divR[RGa == p.RG ? 0 : 1];
    const int total = Pa * R;
    for (int base = 0; base < total; base += NT * 2) {
      __half sv[2], zv[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int idx = base + tid + NT * u;
        const int j = (int)fdiv((uint32_t)idx, divR), row = idx - j * R;
        const int n = n0 + row;
        sv[u] = __float2half(0.f);
        zv[u] = __float2half(0.f);
        if (idx < total && n < p.N) {
          const int64_t off = (int64_t)n * p.G + (int)fdiv((uint32_t)(pc0 + j), p.gpp);
          sv[u] = p.scales[off];
          zv[u] = p.zeros[off];
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int idx = base + tid + NT * u;
        if (idx < total) {
          const float zf = __half2float(zv[u]);
          sz[idx] = __half2float(sv[u]);
          sz[p.Pc * R + idx] = kMagic + zf;
          all_int = all_int && zf == rintf(zf) && zf >= 0.f && zf <= kZMax;
        }
      }
    }
  }
  if (p.bias_dtype != NSQ_DTYPE_NONE) {
    for (int row = tid; row < R; row += NT) {
      const int n = n0 + row;
      biasf[row] = n < p.N ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
    }
  }
  // (the fp8 scale is a weight: read it now, not after the wait)
  float wscale = 1.0f;
  if constexpr (FMT == 1) {
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(wscale) : "l"(p.wscale));
  }
  // barriers initialised, partial tile zeroed, staging visible; the integer
  // zero-point decision is CTA-wide
  const bool int_z = __syncthreads_and(all_int ? 1 : 0) != 0;
  if (S > 1) cluster_arrive_release();  // receive barriers are ready for the peers

  // ---- 3. x slice (produced by the previous kernel) ----
  pdl_wait_prior_grids();
  {
    const int cpr4 = Pa * F::kChunks / 4;  // items of 4 chunks per token row
    const FastDiv divc = p.divC[Pa == p.Pc ? 0 : 1];
    const int items = MPAD * cpr4;
    const uint16_t* x = static_cast<const uint16_t*>(p.x);
    for (int base = 0; base < items; base += NT) {
      const int it = base + tid;
      const int t = (int)fdiv((uint32_t)it, divc), q0 = 4 * (it - t * cpr4);
      const int k = k0 + 8 * q0;
      const bool valid = it < items;
      uint4 v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[e] = make_uint4(0u, 0u, 0u, 0u);
        if (valid && t < p.M && k + 8 * e < p.K) v[e] = ldg128(x + (int64_t)t * p.K + k + 8 * e);
      }
      const uint32_t row = xbuf + t * p.xrs;
      if constexpr (FMT == 0) {
        if (valid) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // pairs (x_t, x_t+4) to match the nibble pairs
            sts128(row + xpos<0>(q0 + e, t) * 16, prmt(v[e].x, v[e].z, 0x5410),
                   prmt(v[e].x, v[e].z, 0x7632), prmt(v[e].y, v[e].w, 0x5410),
                   prmt(v[e].y, v[e].w, 0x7632));
          }
        }
        if (!int_z) {  // CTA-uniform: per-piece sums over 4 consecutive lanes
          float s = (chunk_sum<BF16>(v[0]) + chunk_sum<BF16>(v[1])) +
                    (chunk_sum<BF16>(v[2]) + chunk_sum<BF16>(v[3]));
          s += __shfl_xor_sync(0xffffffffu, s, 1);
          s += __shfl_xor_sync(0xffffffffu, s, 2);
          if (valid && (q0 & 15) == 0) xsum[t * p.Pc + (q0 >> 4)] = s;
        }
      } else {
        if (valid) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            sts128(row + xpos<1>(q0 + e, t) * 16, v[e].x, v[e].y, v[e].z, v[e].w);
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- 4. work units (row group, piece), spread evenly over the warps ----
  bool ok = true;
  {
    const int U = RGa * Pa;
    const int u0 = (warp * U) / NW, u1 = ((warp + 1) * U) / NW;
    UnitCtx cx;
    cx.wbase = smem_u32(smem) + g * 64 + c * 16;
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) cx.xr[jt] = xbuf + (8 * jt + g) * p.xrs;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (FMT == 0) {
        cx.xoff[i] = xpos<0>(4 * c + i, g) * 16;        // x[t][32c + 8i .. +7] within a piece
      } else {
        cx.xoff[i] = xpos<1>(2 * c + (i & 1), g) * 16;  // x[t][16c + 8h .. +7], h = i & 1
      }
    }
    cx.sz = sz;
    cx.xsum = xsum;
    cx.R = R;
    cx.Pc = p.Pc;
    cx.Pa = Pa;
    if (u0 < u1) {
      if (FMT == 1 || int_z) {
        ok = run_units<FMT, BF16, MT, true>(cx, p, wbar, abort_flag, red, u0, u1, g, c);
      } else {
        ok = run_units<FMT, BF16, MT, false>(cx, p, wbar, abort_flag, red, u0, u1, g, c);
      }
    }
  }
  __syncthreads();

  // ---- 5. epilogue ----
  uint16_t* y = static_cast<uint16_t*>(p.y);
  const bool has_bias = p.bias_dtype != NSQ_DTYPE_NONE;
  if (S == 1) {
    // two adjacent rows per thread (one 32-bit store when N is even)
    const int R2 = R >> 1;
    const FastDiv div2 = p.divR2[RGa == p.RG ? 0 : 1];
    const bool pairs = (p.N & 1) == 0;
    for (int idx = tid; idx < p.M * R2; idx += NT) {
      const int tok = (int)fdiv((uint32_t)idx, div2), row = 2 * (idx - tok * R2);
      const int n = n0 + row;
      const float2 a = *reinterpret_cast<const float2*>(&red[tok * p.rs + row]);
      const float v0 = fmaf(a.x, wscale, has_bias ? biasf[row] : 0.f);
      const float v1 = fmaf(a.y, wscale, has_bias ? biasf[row + 1] : 0.f);
      uint16_t* dst = y + (int64_t)tok * p.N + n;
      if (pairs && n + 1 < p.N) {
        *reinterpret_cast<uint32_t*>(dst) =
            (uint32_t)float_to_elem<BF16>(v0) | ((uint32_t)float_to_elem<BF16>(v1) << 16);
      } else {
        if (n < p.N) dst[0] = float_to_elem<BF16>(v0);
        if (n + 1 < p.N) dst[1] = float_to_elem<BF16>(v1);
      }
    }
  } else {
    cluster_wait_acquire();  // every peer's receive barrier is initialised
    // push the rows each peer owns into its receive slot for this rank
    for (int q = 0; q < S; ++q) {
      if (q == rank) continue;
      int lo, hi;
      owner_rows(q, S, R, lo, hi);
      const int nq4 = (hi - lo) >> 2;
      if (nq4 == 0) continue;
      const FastDiv divq = p.divQ[RGa == p.RG ? 0 : 1][nq4 == (R >> 2) / S ? 0 : 1];
      const int slot = rank < q ? rank : rank - 1;
      const uint32_t rbase = dsmem_map(smem_u32(recv + (size_t)slot * MPAD * p.recv_rows), q);
      const uint32_t rb = dsmem_map(smem_u32(rbar), q);
      for (int i = tid; i < p.M * nq4; i += NT) {
        const int tok = (int)fdiv((uint32_t)i, divq), q4 = i - tok * nq4;
        const float4 v = *reinterpret_cast<const float4*>(&red[tok * p.rs + lo + 4 * q4]);
        st_async_v4(rbase + (uint32_t)((tok * p.recv_rows + 4 * q4) * 4), v, rb);
      }
    }
    // own rows, four at a time: this CTA's partial plus every peer's
    const bool got = mbar_wait(rbar, 0, p.status, 0x32, nullptr);
    const int nq4 = (own_hi - own_lo) >> 2;
    if (got && nq4 > 0) {
      const FastDiv divo = p.divQ[RGa == p.RG ? 0 : 1][nq4 == (R >> 2) / S ? 0 : 1];
      const bool quads = (p.N & 3) == 0;
      for (int idx = tid; idx < p.M * nq4; idx += NT) {
        const int tok = (int)fdiv((uint32_t)idx, divo), q4 = idx - tok * nq4;
        const int row = own_lo + 4 * q4;
        const int n = n0 + row;
        float4 v = *reinterpret_cast<const float4*>(&red[tok * p.rs + row]);
        for (int s = 0; s < S - 1; ++s) {
          const float4 r =
              *reinterpret_cast<const float4*>(&recv[((size_t)s * MPAD + tok) * p.recv_rows + 4 * q4]);
          v.x += r.x;
          v.y += r.y;
          v.z += r.z;
          v.w += r.w;
        }
        const float o[4] = {fmaf(v.x, wscale, has_bias ? biasf[row] : 0.f),
                            fmaf(v.y, wscale, has_bias ? biasf[row + 1] : 0.f),
                            fmaf(v.z, wscale, has_bias ? biasf[row + 2] : 0.f),
                            fmaf(v.w, wscale, has_bias ? biasf[row + 3] : 0.f)};
        uint16_t* dst = y + (int64_t)tok * p.N + n;
        if (quads && n + 3 < p.N) {
          *reinterpret_cast<uint2*>(dst) =
              make_uint2((uint32_t)float_to_elem<BF16>(o[0]) | ((uint32_t)float_to_elem<BF16>(o[1]) << 16),
                         (uint32_t)float_to_elem<BF16>(o[2]) | ((uint32_t)float_to_elem<BF16>(o[3]) << 16));
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (n + e < p.N) dst[e] = float_to_elem<BF16>(o[e]);
          }
        }
      }
    }
  }

  // after an abort, let the weight copies land before the CTA exits
  if (!__syncthreads_and(ok ? 1 : 0) && warp == 0) {
    for (int rg = lane; rg < RGa; rg += 32) mbar_wait(&wbar[rg], 0, nullptr, 0, nullptr);
  }
}

}  // namespace

struct WavePlan {
  bool ok;
  int S, RG, Pc, tiles, rs, xrs, recv_rows, warps;
  size_t smem;
  int off_x, off_xsum, off_sz, off_bias, off_red, off_recv, off_bar;
};

namespace {

// Clusters of `s` CTAs that fit at once (cached per device and size).
int max_active_clusters(int s);

template <int FMT>
WavePlan make_wave_plan(int M, int K, int N) {
  using F = WaveFmt<FMT>;
  WavePlan best{};
  best.ok = false;
  const int sms = num_sms();
  const int mpad = ((M + 7) / 8) * 8;
  const int nwarps = (mpad <= 16 && FMT == 1) ? 16 : 8;
  const int P = (K + F::kPieceK - 1) / F::kPieceK;
  const int NG = (N + 15) / 16;
  double best_cost = 1e30;
  for (int S = 1; S <= 8; S *= 2) {
    if (S > P) break;
    const int Pc = (P + S - 1) / S;
    if ((P + Pc - 1) / Pc != S) continue;  // every rank gets at least one piece
    const size_t xbytes = (size_t)mpad * Pc * F::kPieceK * 2;
    if (xbytes > (size_t)kXBudget) continue;
    const int per_wave = sms / S;  // row tiles that fit beside each other
    if (per_wave < 1) continue;
    const int RG = (NG + per_wave - 1) / per_wave;
    const int tiles = (NG + RG - 1) / RG;
    const size_t wbytes = (size_t)RG * Pc * kBoxBytes;
    if (wbytes > (size_t)kWBudget || RG > kMaxRG) continue;
    if (S > 1 && max_active_clusters(S) < tiles) continue;
    WavePlan pl{};
    pl.S = S;
    pl.RG = RG;
    pl.Pc = Pc;
    pl.tiles = tiles;
    pl.warps = nwarps;
    const int R = 16 * RG;
    pl.rs = R + ((4 - R % 32) + 32) % 32;  // rs = 4 (mod 32): conflict-free fragment flushes
    pl.xrs = Pc * F::kPieceK * 2;
    pl.recv_rows = S > 1 ? 4 * (((R / 4) + S - 1) / S) : 0;
    size_t off = wbytes;
    off = (off + 127) & ~(size_t)127;
    pl.off_x = (int)off;
    off += xbytes;
    pl.off_xsum = (int)off;
    off += FMT == 0 ? (size_t)mpad * Pc * 4 : 0;
    pl.off_sz = (int)off;
    off += FMT == 0 ? (size_t)2 * Pc * R * 4 : 0;
    pl.off_bias = (int)off;
    off += (size_t)R * 4;
    off = (off + 15) & ~(size_t)15;
    pl.off_red = (int)off;
    off += (size_t)mpad * pl.rs * 4;
    pl.off_recv = (int)off;
    off += S > 1 ? (size_t)(S - 1) * mpad * pl.recv_rows * 4 : 0;
    off = (off + 7) & ~(size_t)7;
    pl.off_bar = (int)off;
    off += (size_t)(kMaxRG + 1) * 8 + 16;
    pl.smem = off;
    if (pl.smem > (size_t)kSmemMax) continue;
    // estimated time after the previous kernel finishes (us): x reads, the
    // tensor-pipe time of the busiest SM or the longest warp, the cluster
    // exchange (m16n8k16 = 4096 flop; mma.sync sustains about 1900
    // flop/clk/SM; a unit costs a warp about 30 cycles per k16 step)
    const double units = (double)RG * Pc;
    const double mma_cycles = units * F::kSteps * (mpad / 8) * 4096.0 / 1900.0;
    const double warp_serial = (double)((RG * Pc + nwarps - 1) / nwarps) * F::kSteps * 30.0;
    const double cost = 0.05 + (double)xbytes / 78000.0 +
                        (mma_cycles > warp_serial ? mma_cycles : warp_serial) / 1900.0 +
                        (S > 1 ? 0.25 + (double)mpad * R * 4 / 200000.0 : 0.0);
    if (cost < best_cost) {
      best_cost = cost;
      best = pl;
      best.ok = true;
    }
  }
  return best;
}

template <int FMT, bool BF16, int MT>
cudaError_t launch_wave(const CUtensorMap& map, const WaveParams& p, const WavePlan& pl,
                        cudaStream_t stream) {
  auto kern = decode_wave_kernel<FMT, BF16, MT>;
  static std::atomic<bool> configured{false};
  if (!configured.load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
    if (e != cudaSuccess) return e;
    configured.store(true);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.S, pl.tiles, 1);
  cfg.blockDim = dim3(WaveThreads<FMT, MT>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (pl.S > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = pl.S;
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
  return cudaLaunchKernelEx(&cfg, kern, map, p);
}

template <int FMT, bool BF16>
cudaError_t dispatch_wave(int mt, const CUtensorMap& map, const WaveParams& p, const WavePlan& pl,
                          cudaStream_t s) {
  switch (mt) {
    case 1: return launch_wave<FMT, BF16, 1>(map, p, pl, s);
    case 2: return launch_wave<FMT, BF16, 2>(map, p, pl, s);
    case 3: return launch_wave<FMT, BF16, 3>(map, p, pl, s);
    case 4: return launch_wave<FMT, BF16, 4>(map, p, pl, s);
    case 5: return launch_wave<FMT, BF16, 5>(map, p, pl, s);
    case 6: return launch_wave<FMT, BF16, 6>(map, p, pl, s);
    case 7: return launch_wave<FMT, BF16, 7>(map, p, pl, s);
    default: return launch_wave<FMT, BF16, 8>(map, p, pl, s);
  }
}

int max_active_clusters(int s) {
  constexpr int kMaxDev = 64;
  static std::atomic<int> cache[kMaxDev][4];  // 0 = unknown, else value + 1
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 0;
  const int slot = s == 2 ? 0 : s == 4 ? 1 : s == 8 ? 2 : 3;
  const int cached = cache[dev][slot].load();
  if (cached > 0) return cached - 1;
  auto kern = decode_wave_kernel<1, true, 1>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(s, 1, 1);
  cfg.blockDim = dim3(WaveThreads<1, 1>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemMax;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = s;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[dev][slot].store(n + 1);
  return n;
}

}  // namespace

WavePlan plan_decode_wave(int fmt, int M, int K, int N) {
  return fmt == 0 ? make_wave_plan<0>(M, K, N) : make_wave_plan<1>(M, K, N);
}

int run_decode_wave_linear(const LinearArgs& a, cudaStream_t stream) {
  if (a.fmt == 0 && a.group_size % 128 != 0) return NSQ_ENOTSUP;
  const WavePlan pl = plan_decode_wave(a.fmt, a.M, a.K, a.N);
  if (!pl.ok) return NSQ_ENOTSUP;
  CUtensorMap map;
  const uint64_t row_bytes = a.fmt == 0 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  CUresult cr = encode_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                                     row_bytes / 4, (uint64_t)a.N, row_bytes, 16, 16,
                                     CU_TENSOR_MAP_SWIZZLE_NONE);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  WaveParams p{};
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
  p.RG = pl.RG;
  p.Pc = pl.Pc;
  p.rs = pl.rs;
  p.xrs = pl.xrs;
  p.recv_rows = pl.recv_rows;
  p.bias_dtype = a.bias ? a.bias_dtype : NSQ_DTYPE_NONE;
  p.off_x = pl.off_x;
  p.off_xsum = pl.off_xsum;
  p.off_sz = pl.off_sz;
  p.off_bias = pl.off_bias;
  p.off_red = pl.off_red;
  p.off_recv = pl.off_recv;
  p.off_bar = pl.off_bar;
  {
    const int rg_last = p.NG - (pl.tiles - 1) * pl.RG;
    const int pc_last = p.P - (pl.S - 1) * pl.Pc;
    const int chunks = a.fmt == 0 ? 16 : 8;
    const int rgs[2] = {pl.RG, rg_last};
    for (int v = 0; v < 2; ++v) {
      const uint32_t r = 16u * (uint32_t)rgs[v];
      p.divR[v] = make_fastdiv(r);
      p.divR2[v] = make_fastdiv(r / 2);
      const uint32_t q_lo = (r / 4) / (uint32_t)pl.S, q_hi = (r / 4 + pl.S - 1) / (uint32_t)pl.S;
      p.divQ[v][0] = make_fastdiv(q_lo > 0 ? q_lo : 1u);
      p.divQ[v][1] = make_fastdiv(q_hi > 0 ? q_hi : 1u);
    }
    p.divC[0] = make_fastdiv((uint32_t)(pl.Pc * chunks / 4));
    p.divC[1] = make_fastdiv((uint32_t)(pc_last * chunks / 4));
  }
  const int mt = (a.M + 7) / 8;
  cudaError_t e;
  if (a.fmt == 0) {
    e = a.x_bf16 ? dispatch_wave<0, true>(mt, map, p, pl, stream)
                 : dispatch_wave<0, false>(mt, map, p, pl, stream);
  } else {
    e = a.x_bf16 ? dispatch_wave<1, true>(mt, map, p, pl, stream)
                 : dispatch_wave<1, false>(mt, map, p, pl, stream);
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // namespace nsq
