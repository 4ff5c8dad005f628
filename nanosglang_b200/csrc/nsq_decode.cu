// Decode-regime quantized linear (M <= 64 tokens): HBM-bound on weight bytes.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152 and :49-52) for small batches. The reference
// dequantises the whole weight and calls cuBLAS; here the packed weight is
// streamed once from HBM and consumed in registers.
//
// Design (swap-AB skinny GEMM on the legacy tensor path):
//   * W rows (output features) form the MMA M dimension (16 per warp), tokens
//     form MMA N (8 per n-tile), so M = 1..64 tokens costs 1..8 n-tiles.
//   * CTA = 4 warps = 64 output rows x a K slice. Each warp streams its own
//     16-row strip through a private 8-deep ring of 1 KB TMA tiles taken
//     straight from the reference layout (qweight [N, K/8] int32 or
//     weight_fp8 [N, K] uint8) -- no repacked copy of the weight exists.
//   * AWQ: a 32-bit word of 8 sequential nibbles becomes four packed pairs
//     {magic+q_t, magic+q_{t+4}} with one lop3 each (magic = 128 for bf16,
//     1024 for fp16, exact). The K permutation this implies is applied to x
//     once per CTA while x is staged into shared memory. Zero points and
//     scales are applied per 128-column piece in fp32:
//        y += s * (sum_k (magic+q) x_k - (magic+z) * sum_k x_k),
//     which is exact algebra for any fp16 zero point.
//   * FP8: e4m3 pairs convert exactly to the MMA type; the per-tensor scale
//     is applied once in the epilogue.
//   * K is split over a thread-block cluster of up to 8 CTAs; partial tiles
//     are reduced through distributed shared memory (no global workspace),
//     then bias is added and y is stored coalesced.
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr int kWarps = 4;
constexpr int kRows = 64;          // output rows per CTA
constexpr int kNst = 8;            // TMA ring depth per warp
constexpr int kStageBytes = 1024;  // 16 rows x 64 B
constexpr int kRedStride = 68;     // fp32 per token row of the partial tile (conflict-free)

template <int FMT>
struct DecFmt;
template <>
struct DecFmt<0> {  // AWQ: piece = 128 columns = 64 B per row
  static constexpr int kPieceK = 128;
  static constexpr int kXRowBytes = 320;  // 256 B of permuted x + 64 B pad per token
  static constexpr int kChunksPerPiece = 16;
};
template <>
struct DecFmt<1> {  // FP8: piece = 64 columns = 64 B per row
  static constexpr int kPieceK = 64;
  static constexpr int kXRowBytes = 144;  // 128 B of x + 16 B pad per token
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
  int k_split;   // columns per CTA (multiple of the piece width)
  int pmax;      // pieces per CTA (k_split / piece)
  int ppc;       // pieces per x staging chunk
  int bias_dtype;
  int off_x, off_xsum, off_sz, off_red, off_bar, off_abort;
};

// Stage x[:, kc0 : kc0 + np*PK) into shared memory (zero-padded past M and K).
// AWQ: each 8-column chunk is stored permuted [0,4,1,5,2,6,3,7] so that the
// packed pair t of the chunk holds (x_t, x_{t+4}); per-token piece sums of x
// go to xsum. FP8: stored in order.
template <int FMT, bool BF16, int MPAD>
__device__ __forceinline__ void stage_x(const DecodeParams& p, uint32_t xbuf, float* xsum, int kc0,
                                        int np, int tid) {
  using F = DecFmt<FMT>;
  const int total = np * MPAD * F::kChunksPerPiece;
  const uint16_t* x = static_cast<const uint16_t*>(p.x);
  for (int base = 0; base < total; base += kWarps * 32) {
    const int item = base + tid;
    const bool valid = item < total;
    const int q = item % F::kChunksPerPiece;
    const int pt = item / F::kChunksPerPiece;  // jl * MPAD + t
    const int t = pt % MPAD;
    const int jl = pt / MPAD;
    const int k = kc0 + jl * F::kPieceK + q * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (valid && t < p.M && k < p.K) {
      v = __ldg(reinterpret_cast<const uint4*>(x + (int64_t)t * p.K + k));
    }
    if constexpr (FMT == 0) {
      // piece sum of x for this token (16 chunks = one half-warp)
      const uint32_t r[4] = {v.x, v.y, v.z, v.w};
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        s += elem_to_float<BF16>(static_cast<uint16_t>(r[i] & 0xFFFFu));
        s += elem_to_float<BF16>(static_cast<uint16_t>(r[i] >> 16));
      }
      s += __shfl_xor_sync(0xffffffffu, s, 8);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      if (valid) {
        if (q == 0) xsum[pt] = s;
        const uint32_t p0 = prmt(v.x, v.z, 0x5410), p1 = prmt(v.x, v.z, 0x7632);
        const uint32_t p2 = prmt(v.y, v.w, 0x5410), p3 = prmt(v.y, v.w, 0x7632);
        const int cq = q >> 2, iq = q & 3;
        sts128(xbuf + pt * F::kXRowBytes + iq * 64 + cq * 16, p0, p1, p2, p3);
      }
    } else {
      if (valid) sts128(xbuf + pt * F::kXRowBytes + q * 16, v.x, v.y, v.z, v.w);
    }
  }
}

template <bool BF16, int MT>
__device__ __forceinline__ void awq_piece(float (&acc)[MT][4], const uint4& wa, const uint4& wb,
                                          uint32_t xpiece, const float* xs, float s0, float z0,
                                          float s1, float z1, int g, int c) {
  float part[MT][4];
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) part[jt][0] = part[jt][1] = part[jt][2] = part[jt][3] = 0.f;
  const uint32_t wg[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t wh[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t eg[4], eh[4];
    unpack_nibble_pairs<BF16>(wg[i], eg);
    unpack_nibble_pairs<BF16>(wh[i], eh);
    uint4 xv[MT];
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) {
      xv[jt] = lds128(xpiece + (8 * jt + g) * DecFmt<0>::kXRowBytes + i * 64 + c * 16);
    }
    const uint32_t a0[4] = {eg[0], eh[0], eg[1], eh[1]};
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) mma_16816<BF16>(part[jt], a0, xv[jt].x, xv[jt].y);
    const uint32_t a1[4] = {eg[2], eh[2], eg[3], eh[3]};
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) mma_16816<BF16>(part[jt], a1, xv[jt].z, xv[jt].w);
  }
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) {
    const float xa = xs[8 * jt + 2 * c], xb = xs[8 * jt + 2 * c + 1];
    acc[jt][0] = fmaf(s0, fmaf(-z0, xa, part[jt][0]), acc[jt][0]);
    acc[jt][1] = fmaf(s0, fmaf(-z0, xb, part[jt][1]), acc[jt][1]);
    acc[jt][2] = fmaf(s1, fmaf(-z1, xa, part[jt][2]), acc[jt][2]);
    acc[jt][3] = fmaf(s1, fmaf(-z1, xb, part[jt][3]), acc[jt][3]);
  }
}

template <bool BF16, int MT>
__device__ __forceinline__ void fp8_piece(float (&acc)[MT][4], const uint4& wa, const uint4& wb,
                                          uint32_t xpiece, int g, int c) {
  const uint32_t wg[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t wh[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int i = 0; i < 4; i += 2) {
    uint4 xv[MT];
#pragma unroll
    for (int jt = 0; jt < MT; ++jt) {
      xv[jt] = lds128(xpiece + (8 * jt + g) * DecFmt<1>::kXRowBytes + (16 * c + 4 * i) * 2);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int s = i + h;
      const uint32_t a[4] = {e4m3x2_to_pair<BF16>(static_cast<uint16_t>(wg[s] & 0xFFFFu)),
                             e4m3x2_to_pair<BF16>(static_cast<uint16_t>(wh[s] & 0xFFFFu)),
                             e4m3x2_to_pair<BF16>(static_cast<uint16_t>(wg[s] >> 16)),
                             e4m3x2_to_pair<BF16>(static_cast<uint16_t>(wh[s] >> 16))};
#pragma unroll
      for (int jt = 0; jt < MT; ++jt) {
        mma_16816<BF16>(acc[jt], a, h ? xv[jt].z : xv[jt].x, h ? xv[jt].w : xv[jt].y);
      }
    }
  }
}

template <int FMT, bool BF16, int MT>
__global__ void __launch_bounds__(kWarps * 32) decode_linear_kernel(
    const __grid_constant__ CUtensorMap wmap, const DecodeParams p) {
  using F = DecFmt<FMT>;
  constexpr int MPAD = MT * 8;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rank = blockIdx.x;  // split-K rank == rank in the cluster
  const int S = gridDim.x;
  const int n0 = blockIdx.y * kRows;
  const int k_begin = rank * p.k_split;
  const int k_end = min(p.K, k_begin + p.k_split);
  const int P = (k_end - k_begin + F::kPieceK - 1) / F::kPieceK;

  const uint32_t wring = smem_u32(smem);
  const uint32_t xbuf = smem_u32(smem + p.off_x);
  float* xsum = reinterpret_cast<float*>(smem + p.off_xsum);
  float* sz = reinterpret_cast<float*>(smem + p.off_sz);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  uint64_t* wbar = reinterpret_cast<uint64_t*>(smem + p.off_bar) + warp * kNst;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.off_abort);

  if (tid == 0) *abort_flag = 0;
  if (lane == 0) {
    for (int s = 0; s < kNst; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  auto issue = [&](int j) {
    const int buf = j % kNst;
    mbar_arrive_expect_tx(&wbar[buf], kStageBytes);
    const int kk = k_begin + j * F::kPieceK;
    tma_load_2d(smem + (warp * kNst + buf) * kStageBytes, &wmap, &wbar[buf],
                FMT == 0 ? kk / 8 : kk, n0 + 16 * warp);
  };
  int issued = 0;
  if (lane == 0) {
    tma_prefetch_desc(&wmap);
    const int first = P < kNst ? P : kNst;
    for (int j = 0; j < first; ++j) issue(j);
    issued = first;
  }

  if constexpr (FMT == 0) {
    // per-piece scale and biased zero point of this CTA's 64 rows (fp32)
    for (int idx = tid; idx < P * kRows; idx += kWarps * 32) {
      const int j = idx / kRows, r = idx % kRows;
      const int n = n0 + r;
      const int grp = (k_begin + j * F::kPieceK) / p.group_size;
      float s = 0.f, zb = 0.f;
      if (n < p.N) {
        s = __half2float(p.scales[(int64_t)n * p.G + grp]);
        zb = Magic<BF16>::kValue + __half2float(p.zeros[(int64_t)n * p.G + grp]);
      }
      sz[j * kRows + r] = s;
      sz[(p.pmax + j) * kRows + r] = zb;
    }
  }

  // x and bias may be produced by the previous kernel on the stream
  pdl_wait_prior_grids();

  float acc[MT][4];
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) acc[jt][0] = acc[jt][1] = acc[jt][2] = acc[jt][3] = 0.f;

  bool ok = true;
  int consumed = 0;
  const int nchunks = (P + p.ppc - 1) / p.ppc;
  for (int ch = 0; ch < nchunks; ++ch) {
    const int j0 = ch * p.ppc;
    const int j1 = min(P, j0 + p.ppc);
    __syncthreads();  // previous chunk fully consumed (and sz/abort init visible)
    stage_x<FMT, BF16, MPAD>(p, xbuf, xsum, k_begin + j0 * F::kPieceK, j1 - j0, tid);
    __syncthreads();
    for (int j = j0; j < j1; ++j) {
      const int buf = j % kNst;
      if (ok) ok = mbar_wait(&wbar[buf], (j / kNst) & 1, p.status, 1, abort_flag);
      if (ok) {
        const uint32_t wt = wring + (warp * kNst + buf) * kStageBytes;
        const uint4 wa = lds128(wt + g * 64 + c * 16);
        const uint4 wb = lds128(wt + (g + 8) * 64 + c * 16);
        const int jl = j - j0;
        const uint32_t xpiece = xbuf + jl * MPAD * F::kXRowBytes;
        if constexpr (FMT == 0) {
          const int r0 = 16 * warp + g;
          awq_piece<BF16, MT>(acc, wa, wb, xpiece, xsum + jl * MPAD, sz[j * kRows + r0],
                              sz[(p.pmax + j) * kRows + r0], sz[j * kRows + r0 + 8],
                              sz[(p.pmax + j) * kRows + r0 + 8], g, c);
        } else {
          fp8_piece<BF16, MT>(acc, wa, wb, xpiece, g, c);
        }
        consumed = j + 1;
      }
      __syncwarp();
      if (lane == 0 && ok && j + kNst < P) {
        issue(j + kNst);
        issued = j + kNst + 1;
      }
    }
  }
  pdl_launch_dependents();

  // partial tile -> shared memory, [token][row]
#pragma unroll
  for (int jt = 0; jt < MT; ++jt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = 8 * jt + 2 * c + (e & 1);
      const int row = 16 * warp + g + 8 * (e >> 1);
      red[tok * kRedStride + row] = acc[jt][e];
    }
  }
  if (S > 1) {
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  const int E = p.M * kRows;
  const int per = (E + S - 1) / S;
  const int e0 = rank * per;
  const int e1 = min(E, e0 + per);
  const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
  uint16_t* y = static_cast<uint16_t*>(p.y);
  for (int e = e0 + tid; e < e1; e += kWarps * 32) {
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
  if (S > 1) cluster_sync_all();

  // after an abort, let this warp's outstanding copies land before exiting
  if (lane == 0 && !ok) {
    for (int j = consumed; j < issued; ++j) {
      mbar_wait(&wbar[j % kNst], (j / kNst) & 1, nullptr, 0, nullptr);
    }
  }
}

struct Plan {
  int S, k_split, pmax, ppc;
  size_t smem;
  int off_x, off_xsum, off_sz, off_red, off_bar, off_abort;
};

template <int FMT>
Plan make_plan(int M, int K, int N) {
  using F = DecFmt<FMT>;
  Plan pl{};
  const int mpad = ((M + 7) / 8) * 8;
  const int pieces = (K + F::kPieceK - 1) / F::kPieceK;
  const int rt = (N + kRows - 1) / kRows;
  const int sms = num_sms();
  int S = (2 * sms + rt - 1) / rt;
  S = S < 1 ? 1 : S;
  S = S > 8 ? 8 : S;
  S = S > pieces ? pieces : S;
  int per = (pieces + S - 1) / S;
  if (FMT == 0 && per > 64) per = 64;  // bounded scale/zero staging
  S = (pieces + per - 1) / per;
  pl.S = S;
  pl.pmax = per;
  pl.k_split = per * F::kPieceK;
  int ppc = 40960 / (mpad * F::kXRowBytes);
  ppc = ppc < 1 ? 1 : ppc;
  pl.ppc = ppc > per ? per : ppc;
  size_t off = (size_t)kWarps * kNst * kStageBytes;
  pl.off_x = (int)off;
  off += (size_t)mpad * pl.ppc * F::kXRowBytes;
  pl.off_xsum = (int)off;
  off += (FMT == 0) ? (size_t)mpad * pl.ppc * 4 : 0;
  pl.off_sz = (int)off;
  off += (FMT == 0) ? (size_t)2 * per * kRows * 4 : 0;
  off = (off + 15) & ~(size_t)15;
  pl.off_red = (int)off;
  off += (size_t)mpad * kRedStride * 4;
  off = (off + 7) & ~(size_t)7;
  pl.off_bar = (int)off;
  off += (size_t)kWarps * kNst * 8;
  pl.off_abort = (int)off;
  off += 16;
  pl.smem = off;
  return pl;
}

template <int FMT, bool BF16, int MT>
cudaError_t launch_t(const CUtensorMap& map, const DecodeParams& p, const Plan& pl,
                     cudaStream_t stream) {
  auto kern = decode_linear_kernel<FMT, BF16, MT>;
  static std::atomic<size_t> configured{0};
  if (configured.load() < pl.smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)pl.smem);
    if (e != cudaSuccess) return e;
    configured.store(pl.smem);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.S, (p.N + kRows - 1) / kRows, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
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
    case 1: return launch_t<FMT, BF16, 1>(map, p, pl, s);
    case 2: return launch_t<FMT, BF16, 2>(map, p, pl, s);
    case 3: return launch_t<FMT, BF16, 3>(map, p, pl, s);
    case 4: return launch_t<FMT, BF16, 4>(map, p, pl, s);
    case 5: return launch_t<FMT, BF16, 5>(map, p, pl, s);
    case 6: return launch_t<FMT, BF16, 6>(map, p, pl, s);
    case 7: return launch_t<FMT, BF16, 7>(map, p, pl, s);
    default: return launch_t<FMT, BF16, 8>(map, p, pl, s);
  }
}

}  // namespace

int run_decode_linear(const LinearArgs& a, cudaStream_t stream) {
  const int mt = (a.M + 7) / 8;
  Plan pl = a.fmt == 0 ? make_plan<0>(a.M, a.K, a.N) : make_plan<1>(a.M, a.K, a.N);
  CUtensorMap map;
  CUresult cr;
  if (a.fmt == 0) {
    // qweight [N, K/8] int32: box = 16 words (128 columns) x 16 rows
    cr = encode_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_INT32, const_cast<void*>(a.wq),
                              (uint64_t)a.K / 8, (uint64_t)a.N, (uint64_t)a.K / 2, 16, 16,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    // weight_fp8 [N, K] uint8: box = 64 columns x 16 rows
    cr = encode_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<void*>(a.wq),
                              (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, 64, 16,
                              CU_TENSOR_MAP_SWIZZLE_NONE);
  }
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
  p.ppc = pl.ppc;
  p.bias_dtype = a.bias ? a.bias_dtype : NSQ_DTYPE_NONE;
  p.off_x = pl.off_x;
  p.off_xsum = pl.off_xsum;
  p.off_sz = pl.off_sz;
  p.off_red = pl.off_red;
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
