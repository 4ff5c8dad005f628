// Decode-regime quantized linear (M <= 64 tokens): HBM-bound on weight bytes.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152 and :49-52) for small batches. The reference
// dequantises the whole weight and calls cuBLAS; here the packed weight is
// streamed once from HBM and consumed in registers.
//
// Design (swap-AB skinny GEMM on the warp-level tensor path):
//   * W rows (output features) form the MMA M dimension (16 per warp), tokens
//     form MMA N (8 per n-tile), so M = 1..64 tokens costs 1..8 n-tiles.
//   * CTA = 4 row groups of 16 rows (64 output rows) x a K slice, with 1-2
//     warps per row group splitting that slice. The whole weight slice of each
//     row group is requested at once as a few large TMA boxes (up to 16 rows x
//     1 KB) straight from the reference layout (qweight [N, K/8] int32 or
//     weight_fp8 [N, K] viewed as 32-bit words); no repacked copy of the
//     weight exists. The issuing lane initialises its group's barriers itself,
//     so the loads leave before anything else happens, and the next kernel on
//     the stream is released (programmatic launch) right after.
//   * x is copied with cp.async (all copies in flight at once, edges
//     zero-filled) into an XOR-swizzled layout that makes every fragment load
//     conflict-free.
//   * AWQ: a word of 8 sequential nibbles becomes four packed pairs
//     {magic+q_t, magic+q_{t+4}} with one lop3 each (magic = 128 for bf16,
//     1024 for fp16; exact). The matching pairs of x are built with prmt.
//     When every zero point of the CTA is an integer the MMA type represents
//     exactly with the magic bias (the reference quantiser always produces
//     those), one packed subtraction gives the exact (q - z); otherwise the
//     zero point is applied per 128-column piece in fp32 from per-token sums
//     of x: y += s * (sum (magic+q) x - (magic+z) * sum x).
//   * FP8: e4m3 pairs convert exactly to the MMA type; the per-tensor scale
//     is applied once in the epilogue.
//   * K is split over a thread-block cluster of up to 8 CTAs only when there
//     are too few row tiles to cover the SMs; partial tiles are reduced
//     through distributed shared memory (no global workspace). Unsplit CTAs
//     store straight from registers.
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr int kRowWarps = 4;       // row groups of 16 rows per CTA
constexpr int kMaxKGroups = 2;     // warps per row group splitting K (intra-CTA split-K)
constexpr int kMaxThreads = kRowWarps * kMaxKGroups * 32;
constexpr int kRows = 64;          // output rows per CTA
constexpr int kMaxSlabs = 16;      // TMA boxes per row group (one barrier each)
constexpr int kSlabRowMax = 1024;  // bytes per row of one TMA box (256 x 32-bit)
constexpr int kWBudget = 96 * 1024;  // bytes of weight slice per CTA held in shared memory
constexpr int kRedStride = 68;     // fp32 per token row of the partial tile (conflict-free)
constexpr int kMaxSmem = 200 * 1024;
constexpr int kXBudget = 48 * 1024;  // bytes for x staging buffers

template <int FMT>
struct DecFmt;
template <>
struct DecFmt<0> {  // AWQ: piece = 128 columns = 64 B per weight row
  static constexpr int kPieceK = 128;
  static constexpr int kChunksPerPiece = 16;
};
template <>
struct DecFmt<1> {  // FP8: piece = 64 columns = 64 B per weight row
  static constexpr int kPieceK = 64;
  static constexpr int kChunksPerPiece = 8;
};

struct DecodeParams {
  const void* x;
  const __half* scales;
  const __half* zeros;
  const float* wscale;
  const void* bias;
  void* y;
  DevStatus* status;
  int M, K, N;
  int group_size, G;
  int k_split;  // columns per CTA (multiple of the piece width)
  int pmax;     // pieces per CTA (k_split / piece)
  int kw;       // k-groups of warps inside the CTA (blockDim = 128 * kw)
  int nslab;    // TMA boxes per row group
  int slab_row; // bytes per row of one box (multiple of 64)
  int pps;      // pieces per box
  int ppc;      // pieces per x staging chunk
  int xrs;      // bytes per token row of an x buffer (ppc * piece * 2)
  int bias_dtype;
  int withhold;  // test hook: row group 0 of every CTA skips its first weight box
  int off_x, off_xsum, off_sz, off_red, off_redk, off_bar, off_abort;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Position of 16-byte chunk qq (counted along the chunk's columns) of token t.
// AWQ: XOR bit 0 with bit 3 of qq and bit 1 with the token parity; FP8: XOR
// bit 0 with the token parity. Both stay inside one piece.
template <int FMT>
__device__ __forceinline__ int x_swz(int qq, int t) {
  if constexpr (FMT == 0) {
    return qq ^ ((qq >> 3) & 1) ^ ((t & 1) << 1);
  } else {
    return qq ^ (t & 1);
  }
}

// Issue (without waiting) the copies of x[:, kc0 : kc0 + np*PK) into an x
// buffer; rows past M and columns past K are zero-filled by the copy itself.
template <int FMT, int MPAD>
__device__ __forceinline__ void issue_x_copy(const DecodeParams& p, uint32_t xbuf, int kc0, int np,
                                             int tid) {
  using F = DecFmt<FMT>;
  const int cpr = np * F::kChunksPerPiece;  // 16-byte chunks per token row
  const int total = MPAD * cpr;
  const uint16_t* x = static_cast<const uint16_t*>(p.x);
  // (t, q) of chunk idx, advanced by the stride instead of divided each time
  // (this loop runs after the wait, on the launch's critical path)
  const int nthr = blockDim.x;
  const int dt = nthr / cpr, dq = nthr - dt * cpr;
  int t = tid / cpr, q = tid - (tid / cpr) * cpr;
  for (int idx = tid; idx < total; idx += nthr) {
    const int k = kc0 + q * 8;
    const bool valid = t < p.M && k < p.K;
    const uint16_t* src = valid ? x + (int64_t)t * p.K + k : x;
    cp_async16(xbuf + t * p.xrs + x_swz<FMT>(q, t) * 16, src, valid ? 16u : 0u);
    t += dt;
    q += dq;
    if (q >= cpr) {
      q -= cpr;
      ++t;
    }
  }
}

// AWQ general path: per-token sums of x over each 128-column piece (fp32).
template <bool BF16, int MPAD>
__device__ __forceinline__ void piece_sums(const DecodeParams& p, uint32_t xbuf, float* xsum, int np,
                                           int tid) {
  constexpr int CPP = DecFmt<0>::kChunksPerPiece;
  const int total = np * MPAD * CPP;
  for (int base = 0; base < total; base += blockDim.x) {
    const int item = base + tid;
    const bool valid = item < total;
    const int q = item % CPP;
    const int pt = item / CPP;  // jl * MPAD + t
    const int t = pt % MPAD;
    const int jl = pt / MPAD;
    float s = 0.f;
    if (valid) {
      const uint4 v = lds128(xbuf + t * p.xrs + x_swz<0>(jl * CPP + q, t) * 16);
      const uint32_t r[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s += elem_to_float<BF16>(static_cast<uint16_t>(r[i] & 0xFFFFu));
        s += elem_to_float<BF16>(static_cast<uint16_t>(r[i] >> 16));
      }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 8);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (valid && q == 0) xsum[pt] = s;
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

// One 128-column piece of one warp's 16 rows (AWQ). INT_Z: exact integer zero
// points subtracted in the packed domain; else the fp32 fold with x sums.
template <bool BF16, int MT, bool INT_Z>
__device__ __forceinline__ void awq_piece(float (&acc)[MT][4], const uint4& wa, const uint4& wb,
                                          uint32_t xrow0, int xrs, const float* xs, float s0, float zb0,
                                          float s1, float zb1, int g, int c) {
  // two accumulator sets (first and second k16 step of each word), so the
  // MMA dependency chains are 4 long instead of 8 (up to 32 tokens)
  float part[MT][4], part2[MT][4];
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) {
    part[jt][0] = part[jt][1] = part[jt][2] = part[jt][3] = 0.f;
    part2[jt][0] = part2[jt][1] = part2[jt][2] = part2[jt][3] = 0.f;
  }
  const uint32_t wg[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t wh[4] = {wb.x, wb.y, wb.z, wb.w};
  uint32_t z2g = 0, z2h = 0;
  if constexpr (INT_Z) {
    z2g = pack_pair<BF16>(zb0);
    z2h = pack_pair<BF16>(zb1);
  }
  const int m = (c >> 1) | ((g & 1) << 1);  // swizzle of this thread's chunks
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
      // x[8jt+g][32c + 8i .. +7] -> pairs (x_t, x_{t+4})
      const uint4 v = lds128(xrow0 + (8 * jt + g) * xrs + (4 * c + (i ^ m)) * 16);
      const uint32_t p0 = prmt(v.x, v.z, 0x5410), p1 = prmt(v.x, v.z, 0x7632);
      const uint32_t p2 = prmt(v.y, v.w, 0x5410), p3 = prmt(v.y, v.w, 0x7632);
      mma_16816<BF16>(part[jt], a0, p0, p1);
      if constexpr (MT <= 4) {
        mma_16816<BF16>(part2[jt], a1, p2, p3);
      } else {  // more token tiles already give independent chains; keep registers
        mma_16816<BF16>(part[jt], a1, p2, p3);
      }
    }
  }
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) part[jt][e] += part2[jt][e];
    if constexpr (INT_Z) {
      acc[jt][0] = fmaf(s0, part[jt][0], acc[jt][0]);
      acc[jt][1] = fmaf(s0, part[jt][1], acc[jt][1]);
      acc[jt][2] = fmaf(s1, part[jt][2], acc[jt][2]);
      acc[jt][3] = fmaf(s1, part[jt][3], acc[jt][3]);
    } else {
      const float xa = xs[8 * jt + 2 * c], xb = xs[8 * jt + 2 * c + 1];
      acc[jt][0] = fmaf(s0, fmaf(-zb0, xa, part[jt][0]), acc[jt][0]);
      acc[jt][1] = fmaf(s0, fmaf(-zb0, xb, part[jt][1]), acc[jt][1]);
      acc[jt][2] = fmaf(s1, fmaf(-zb1, xa, part[jt][2]), acc[jt][2]);
      acc[jt][3] = fmaf(s1, fmaf(-zb1, xb, part[jt][3]), acc[jt][3]);
    }
  }
}

template <bool BF16, int MT>
__device__ __forceinline__ void fp8_piece(float (&acc)[MT][4], const uint4& wa, const uint4& wb,
                                          uint32_t xrow0, int xrs, int g, int c) {
  const uint32_t wg[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t wh[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint4 xv[MT];
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) {
      // x[8jt+g][16c + 8h .. +7]
      xv[jt] = lds128(xrow0 + (8 * jt + g) * xrs + (2 * c + (h ^ (g & 1))) * 16);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int s = 2 * h + u;
      uint32_t a[4];
      e4m3x4_to_pairs<BF16>(wg[s], a[0], a[2]);
      e4m3x4_to_pairs<BF16>(wh[s], a[1], a[3]);
#pragma unroll
      for (int jt = 0; jt < MT; ++jt) {
        mma_16816<BF16>(acc[jt], a, u ? xv[jt].z : xv[jt].x, u ? xv[jt].w : xv[jt].y);
      }
    }
  }
}

// KWMAX: the most warps per row group the instantiation is launched with.
template <int FMT, bool BF16, int MT, int KWMAX>
__global__ void __launch_bounds__(kRowWarps * KWMAX * 32, 2) decode_linear_kernel(
    const __grid_constant__ CUtensorMap wmap, const DecodeParams p) {
  using F = DecFmt<FMT>;
  constexpr int MPAD = MT * 8;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nthreads = blockDim.x;
  const int rg = warp & (kRowWarps - 1);  // which 16 of the 64 rows
  const int kg = warp / kRowWarps;        // which k-group (pieces kg, kg+kw, ...)
  const int kw = p.kw;
  const int g = lane >> 2, c = lane & 3;
  const int rank = blockIdx.x;  // split-K rank == rank in the cluster
  const int S = gridDim.x;
  const int n0 = blockIdx.y * kRows;
  const int k_begin = rank * p.k_split;
  const int k_end = min(p.K, k_begin + p.k_split);
  const int P = (k_end - k_begin + F::kPieceK - 1) / F::kPieceK;
  const int nslab_used = (P + p.pps - 1) / p.pps;
  const int group_bytes = 16 * p.slab_row * p.nslab;  // shared memory of one row group

  const uint32_t wgroup = smem_u32(smem) + rg * group_bytes;
  const uint32_t xbuf0 = smem_u32(smem + p.off_x);
  float* xsum = reinterpret_cast<float*>(smem + p.off_xsum);
  float* sz = reinterpret_cast<float*>(smem + p.off_sz);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  float* redk = reinterpret_cast<float*>(smem + p.off_redk);
  uint64_t* sbar = reinterpret_cast<uint64_t*>(smem + p.off_bar) + rg * kMaxSlabs;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.off_abort);
  const int xbuf_bytes = MPAD * p.xrs;

  // the first warp of each row group initialises that group's barriers and
  // requests the group's whole weight slice before anything else
  if (kg == 0 && lane == 0) {
    for (int sl = 0; sl < nslab_used; ++sl) mbar_init(&sbar[sl], 1);
    fence_proxy_async_smem();
    const int kbytes = FMT == 0 ? k_begin / 2 : k_begin;  // byte offset of the slice in a row
    // (test hook: with p.withhold, row group 0 never requests its first box,
    // so its waits run out and the CTA winds down through the abort path;
    // nothing is in flight for the box that was never requested)
    for (int sl = (p.withhold && rg == 0) ? 1 : 0; sl < nslab_used; ++sl) {
      mbar_arrive_expect_tx(&sbar[sl], 16 * p.slab_row);
      tma_load_2d(smem + rg * group_bytes + sl * 16 * p.slab_row, &wmap, &sbar[sl],
                  (kbytes + sl * p.slab_row) / 4, n0 + 16 * rg);
    }
  }
  if (tid == 0) *abort_flag = 0;
  // the next kernel on the stream may launch now and start its own weight
  // loads; it still waits for this grid before it reads anything we write
  pdl_launch_dependents();

  bool int_zeros = true;
  if constexpr (FMT == 0) {
    // per-piece scale and biased zero point of this CTA's 64 rows (fp32);
    // loads are batched so their latencies overlap
    constexpr float kZMax = BF16 ? 127.0f : 1023.0f;
    const int total = P * kRows;
    bool all_int = true;
    for (int base = 0; base < total; base += nthreads * 8) {
      float sv[8], zv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int idx = base + tid + nthreads * u;
        const int j = idx / kRows, r = idx % kRows;
        const int n = n0 + r;
        sv[u] = 0.f;
        zv[u] = 0.f;
        if (idx < total && n < p.N) {
          const int64_t off = (int64_t)n * p.G + (k_begin + j * F::kPieceK) / p.group_size;
          sv[u] = __half2float(p.scales[off]);
          zv[u] = __half2float(p.zeros[off]);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int idx = base + tid + nthreads * u;
        if (idx < total) {
          const int j = idx / kRows, r = idx % kRows;
          sz[j * kRows + r] = sv[u];
          sz[(p.pmax + j) * kRows + r] = Magic<BF16>::kValue + zv[u];
          all_int = all_int && (zv[u] == rintf(zv[u])) && fabsf(zv[u]) <= kZMax;
        }
      }
    }
    int_zeros = all_int;  // combined across the CTA at the first barrier below
  }

  // x (and bias) may be produced by the previous kernel on the stream
  pdl_wait_prior_grids();

  float acc[MT][4];
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) acc[jt][0] = acc[jt][1] = acc[jt][2] = acc[jt][3] = 0.f;

  bool ok = true;
  const int nchunks = (P + p.ppc - 1) / p.ppc;
  // x chunks double-buffered: the copy of chunk ch+1 flies while chunk ch computes
  issue_x_copy<FMT, MPAD>(p, xbuf0, k_begin, min(P, p.ppc), tid);
  cp_async_commit();
  for (int ch = 0; ch < nchunks; ++ch) {
    const int j0 = ch * p.ppc;
    const int j1 = min(P, j0 + p.ppc);
    const uint32_t xb = xbuf0 + (ch & 1) * xbuf_bytes;
    if (ch + 1 < nchunks) {
      const int n1 = min(P, j1 + p.ppc) - j1;
      issue_x_copy<FMT, MPAD>(p, xbuf0 + ((ch + 1) & 1) * xbuf_bytes, k_begin + j1 * F::kPieceK, n1, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    if (ch == 0) {
      // chunk 0 landed for every thread; scale/zero staging is visible and
      // the integer-zero-point decision is made CTA-wide
      int_zeros = __syncthreads_and(int_zeros ? 1 : 0) != 0;
    } else {
      __syncthreads();  // chunk ch landed for every thread
    }
    if constexpr (FMT == 0) {
      if (!int_zeros) {
        piece_sums<BF16, MPAD>(p, xb, xsum, j1 - j0, tid);
        __syncthreads();
      }
    }
    // this warp's pieces in [j0, j1): j == kg (mod kw)
    for (int j = j0 + ((kg - j0 % kw) + kw) % kw; j < j1; j += kw) {
      const int sl = j / p.pps;
      if (ok) ok = mbar_wait(&sbar[sl], 0, p.status, 1, abort_flag);
      if (ok) {
        const uint32_t wt = wgroup + sl * 16 * p.slab_row + (j - sl * p.pps) * 64;
        const uint4 wa = lds128(wt + g * p.slab_row + c * 16);
        const uint4 wb = lds128(wt + (g + 8) * p.slab_row + c * 16);
        const int jl = j - j0;
        const uint32_t xrow0 = xb + jl * F::kPieceK * 2;
        if constexpr (FMT == 0) {
          const int r0 = 16 * rg + g;
          const float s0 = sz[j * kRows + r0], s1 = sz[j * kRows + r0 + 8];
          const float zb0 = sz[(p.pmax + j) * kRows + r0], zb1 = sz[(p.pmax + j) * kRows + r0 + 8];
          if (int_zeros) {
            awq_piece<BF16, MT, true>(acc, wa, wb, xrow0, p.xrs, nullptr, s0, zb0, s1, zb1, g, c);
          } else {
            awq_piece<BF16, MT, false>(acc, wa, wb, xrow0, p.xrs, xsum + jl * MPAD, s0, zb0, s1, zb1, g, c);
          }
        } else {
          fp8_piece<BF16, MT>(acc, wa, wb, xrow0, p.xrs, g, c);
        }
      }
    }
    if (ch + 1 < nchunks) __syncthreads();  // every warp is done with this x buffer
  }

  // k-groups 1.. hand their partial sums to k-group 0 through shared memory
  if (kw > 1) {
    if (kg > 0) {
      float* dst = redk + (size_t)(kg - 1) * MPAD * kRedStride;
#pragma unroll
      for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = 8 * jt + 2 * c + (e & 1);
          const int row = 16 * rg + g + 8 * (e >> 1);
          dst[tok * kRedStride + row] = acc[jt][e];
        }
      }
    }
    __syncthreads();
    if (kg == 0) {
      for (int q = 1; q < kw; ++q) {
        const float* src = redk + (size_t)(q - 1) * MPAD * kRedStride;
#pragma unroll
        for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = 8 * jt + 2 * c + (e & 1);
            const int row = 16 * rg + g + 8 * (e >> 1);
            acc[jt][e] += src[tok * kRedStride + row];
          }
        }
      }
    }
  }

  const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
  uint16_t* y = static_cast<uint16_t*>(p.y);
  if (S == 1) {
    // unsplit: scale, bias and store straight from the accumulators
    if (kg == 0) {
      const int ra = n0 + 16 * rg + g, rb = ra + 8;
      float ba = 0.f, bb = 0.f;
      if (p.bias_dtype != NSQ_DTYPE_NONE) {
        if (ra < p.N) ba = load_bias(p.bias, p.bias_dtype, ra);
        if (rb < p.N) bb = load_bias(p.bias, p.bias_dtype, rb);
      }
#pragma unroll
      for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = 8 * jt + 2 * c + (e & 1);
          const int n = (e >> 1) ? rb : ra;
          if (tok < p.M && n < p.N) {
            y[(int64_t)tok * p.N + n] = float_to_elem<BF16>(fmaf(acc[jt][e], wscale, (e >> 1) ? bb : ba));
          }
        }
      }
    }
  } else {
    // partial tile -> shared memory [token][row], reduced across the cluster
    if (kg == 0) {
#pragma unroll
      for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = 8 * jt + 2 * c + (e & 1);
          const int row = 16 * rg + g + 8 * (e >> 1);
          red[tok * kRedStride + row] = acc[jt][e];
        }
      }
    }
    cluster_sync_all();
    const int E = p.M * kRows;
    const int per = (E + S - 1) / S;
    const int e0 = rank * per;
    const int e1 = min(E, e0 + per);
    for (int e = e0 + tid; e < e1; e += nthreads) {
      const int tok = e / kRows, row = e % kRows;
      const int n = n0 + row;
      if (n >= p.N) continue;
      const uint32_t la = smem_u32(&red[tok * kRedStride + row]);
      float v = 0.f;
      for (int r = 0; r < S; ++r) v += (r == rank) ? red[tok * kRedStride + row] : dsmem_ld_f32(dsmem_map(la, r));
      v *= wscale;
      if (p.bias_dtype != NSQ_DTYPE_NONE) v += load_bias(p.bias, p.bias_dtype, n);
      y[(int64_t)tok * p.N + n] = float_to_elem<BF16>(v);
    }
    cluster_sync_all();
  }

  // after an abort, let this group's copies land before the CTA exits
  if (!ok && kg == 0 && lane == 0) {
    for (int sl = 0; sl < nslab_used; ++sl) mbar_wait(&sbar[sl], 0, nullptr, 0, nullptr);
  }
}

struct Plan {
  bool ok;
  int S, k_split, pmax, kw, nslab, slab_row, pps, ppc, xrs;
  size_t smem;
  int off_x, off_xsum, off_sz, off_red, off_redk, off_bar, off_abort;
};

template <int FMT>
Plan make_plan(int M, int K, int N) {
  using F = DecFmt<FMT>;
  constexpr int kPieceRowBytes = 64;  // one piece of one weight row in shared memory
  Plan pl{};
  const int mpad = ((M + 7) / 8) * 8;
  const int pieces = (K + F::kPieceK - 1) / F::kPieceK;
  const int rt = (N + kRows - 1) / kRows;
  const int sms = num_sms();
  // split K across the CTAs of a cluster only as far as needed to put a CTA
  // on every SM, and far enough that a CTA's weight slice fits on chip
  int S = (sms + rt - 1) / rt;
  S = S < 1 ? 1 : S;
  const int min_s = (int)(((size_t)pieces * kPieceRowBytes * kRows + kWBudget - 1) / kWBudget);
  S = S < min_s ? min_s : S;
  S = S > 8 ? 8 : S;  // portable cluster size
  S = S > pieces ? pieces : S;
  int per = (pieces + S - 1) / S;
  S = (pieces + per - 1) / per;
  pl.ok = (size_t)per * kPieceRowBytes * kRows <= (size_t)kWBudget && (FMT != 0 || per <= 64);
  pl.S = S;
  pl.pmax = per;
  pl.k_split = per * F::kPieceK;
  // boxes of equal width covering the slice with little overhang
  const int row_bytes = per * kPieceRowBytes;
  int nslab = (row_bytes + kSlabRowMax - 1) / kSlabRowMax;
  int slab_pieces = (per + nslab - 1) / nslab;
  nslab = (per + slab_pieces - 1) / slab_pieces;
  pl.pps = slab_pieces;
  pl.slab_row = slab_pieces * kPieceRowBytes;
  pl.nslab = nslab;
  if (nslab > kMaxSlabs) pl.ok = false;
  // two warps per row group when each can keep at least two pieces
  // (four warps per row group, 64 registers each, measured slower on B200:
  // config 0 6.3 -> 7.4 us per linear)
  pl.kw = per >= 4 ? 2 : 1;
  // x staging: one buffer for the whole slice if it fits, else two chunk buffers
  const int piece_token_bytes = F::kPieceK * 2;
  int nbuf;
  if ((size_t)per * piece_token_bytes * mpad <= (size_t)kXBudget) {
    pl.ppc = per;
    nbuf = 1;
  } else {
    int ppc = kXBudget / (2 * mpad * piece_token_bytes);
    pl.ppc = ppc < 1 ? 1 : ppc;
    nbuf = 2;
  }
  pl.xrs = pl.ppc * piece_token_bytes;
  size_t off = (size_t)kRowWarps * 16 * pl.slab_row * pl.nslab;
  off = (off + 127) & ~(size_t)127;
  pl.off_x = (int)off;
  off += (size_t)nbuf * mpad * pl.xrs;
  pl.off_xsum = (int)off;
  off += (FMT == 0) ? (size_t)mpad * pl.ppc * 4 : 0;
  pl.off_sz = (int)off;
  off += (FMT == 0) ? (size_t)2 * per * kRows * 4 : 0;
  off = (off + 15) & ~(size_t)15;
  pl.off_red = (int)off;
  off += (S > 1) ? (size_t)mpad * kRedStride * 4 : 0;
  pl.off_redk = (int)off;
  off += (size_t)(pl.kw - 1) * mpad * kRedStride * 4;
  off = (off + 7) & ~(size_t)7;
  pl.off_bar = (int)off;
  off += (size_t)kRowWarps * kMaxSlabs * 8;
  pl.off_abort = (int)off;
  off += 16;
  pl.smem = off;
  if (pl.smem > (size_t)kMaxSmem) pl.ok = false;
  return pl;
}

template <int FMT, bool BF16, int MT, int KWMAX>
cudaError_t launch_t(const CUtensorMap& map, const DecodeParams& p, const Plan& pl,
                     cudaStream_t stream) {
  auto kern = decode_linear_kernel<FMT, BF16, MT, KWMAX>;
  if (pl.kw > KWMAX) return cudaErrorInvalidValue;
  // one fixed cap for every plan, set on first use (a warm-up call before any
  // graph capture takes care of it)
  static std::atomic<bool> configured{false};
  if (!configured.load()) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kMaxSmem);
    if (e != cudaSuccess) return e;
    configured.store(true);
  }
  if (pl.smem > (size_t)kMaxSmem) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.S, (p.N + kRows - 1) / kRows, 1);
  cfg.blockDim = dim3(kRowWarps * pl.kw * 32, 1, 1);
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
cudaError_t dispatch_mt(int mt, const CUtensorMap& map, const DecodeParams& p, const Plan& pl,
                        cudaStream_t s) {
  switch (mt) {
    case 1: return launch_t<FMT, BF16, 1, 2>(map, p, pl, s);
    case 2: return launch_t<FMT, BF16, 2, 2>(map, p, pl, s);
    case 3: return launch_t<FMT, BF16, 3, 2>(map, p, pl, s);
    case 4: return launch_t<FMT, BF16, 4, 2>(map, p, pl, s);
    case 5: return launch_t<FMT, BF16, 5, 2>(map, p, pl, s);
    case 6: return launch_t<FMT, BF16, 6, 2>(map, p, pl, s);
    case 7: return launch_t<FMT, BF16, 7, 2>(map, p, pl, s);
    default: return launch_t<FMT, BF16, 8, 2>(map, p, pl, s);
  }
}

}  // namespace

int decode_linear_ctas(const LinearArgs& a) {
  const Plan pl = a.fmt == 0 ? make_plan<0>(a.M, a.K, a.N) : make_plan<1>(a.M, a.K, a.N);
  return pl.ok ? pl.S * ((a.N + kRows - 1) / kRows) : -1;
}

int run_decode_linear(const LinearArgs& a, cudaStream_t stream) {
  const int mt = (a.M + 7) / 8;
  Plan pl = a.fmt == 0 ? make_plan<0>(a.M, a.K, a.N) : make_plan<1>(a.M, a.K, a.N);
  if (!pl.ok) return NSQ_ENOTSUP;
  // both formats viewed as rows of 32-bit words: qweight [N, K/8] int32,
  // weight_fp8 [N, K] as [N, K/4]; one box = slab_row bytes x 16 rows
  CUtensorMap map;
  const uint64_t row_bytes = a.fmt == 0 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  CUresult cr = encode_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                                     row_bytes / 4, (uint64_t)a.N, row_bytes, pl.slab_row / 4, 16,
                                     CU_TENSOR_MAP_SWIZZLE_NONE);
  if (cr != CUDA_SUCCESS) return NSQ_ECUDA;
  DecodeParams p{};
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
  p.group_size = a.group_size;
  p.G = a.fmt == 0 ? (a.K + a.group_size - 1) / a.group_size : 0;
  p.k_split = pl.k_split;
  p.pmax = pl.pmax;
  p.kw = pl.kw;
  p.nslab = pl.nslab;
  p.slab_row = pl.slab_row;
  p.pps = pl.pps;
  p.ppc = pl.ppc;
  p.xrs = pl.xrs;
  p.bias_dtype = a.bias ? a.bias_dtype : NSQ_DTYPE_NONE;
  p.withhold = test_withhold() ? 1 : 0;
  p.off_x = pl.off_x;
  p.off_xsum = pl.off_xsum;
  p.off_sz = pl.off_sz;
  p.off_red = pl.off_red;
  p.off_redk = pl.off_redk;
  p.off_bar = pl.off_bar;
  p.off_abort = pl.off_abort;
  cudaError_t e;
  if (a.fmt == 0) {
    e = a.x_bf16 ? dispatch_mt<0, true>(mt, map, p, pl, stream)
                 : dispatch_mt<0, false>(mt, map, p, pl, stream);
  } else {
    e = a.x_bf16 ? dispatch_mt<1, true>(mt, map, p, pl, stream)
                 : dispatch_mt<1, false>(mt, map, p, pl, stream);
  }
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // namespace nsq
