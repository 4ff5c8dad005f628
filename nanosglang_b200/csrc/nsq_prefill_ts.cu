// Prefill-regime quantized linear with the dequantised weight tile held in
// tensor memory: the transposed product y^T = W_deq . x^T on tcgen05, A
// operand (128 weight rows) read from TMEM, B operand (the token tile of x)
// from shared memory.
//
// Replaces AWQLinear.forward / FP8Linear.forward (nano_sglang/decode/
// quantization.py:150-152, :49-52) for prefill-sized batches whose tiles the
// shared-memory-operand kernels cannot spread over the GPU (few tokens, or few
// output features), and wherever it is measured faster.
//
// Why TMEM for the weight: with both operands in shared memory, a 64-column
// K step of a 128 x 256 tile moves ~128 KB through shared memory (TMA writes
// of x and the packed weight, the converters' read of the packed weight and
// write of the converted one, the tensor core's operand reads) -- about twice
// the MMA time of that step. The converted weight here goes from registers
// straight into tensor memory (tcgen05.st); shared memory carries only x and
// the packed weight.
//
// Warp roles, 448 threads:
//   warp 0        TMA producer: x tile [BT tokens x 64] (128-byte swizzle) and
//                 the packed weight tile [128 rows x 64 columns] of the
//                 reference layout, NS-stage ring.
//   warp 1        TMEM allocation; lane 0 issues 128 x BT x 16 UMMAs with A
//                 from TMEM and commits the barriers that free the stages.
//   warps 2..9    converters: warp w serves TMEM sub-partition w % 4 (32 weight
//                 rows, one per lane) and half (w - 2) / 4 of the 64 columns;
//                 int4 with zero point and group scale (AWQ) or e4m3 (FP8) ->
//                 MMA element type -> tcgen05.st into an NS-stage TMEM ring.
//   warps 10..13  epilogue: tcgen05.ld of the accumulator (lane = output
//                 feature, column = token), per-tensor scale (FP8), bias,
//                 rounding, stores of feature pairs exchanged between lanes.
// Accumulators are double-buffered (the epilogue of tile i overlaps the main
// loop of tile i + 1). Every wait is bounded.
#include <atomic>

#include "nsq_common.cuh"
#include "nsq_internal.h"
#include "nsq_tmem_operand.cuh"

namespace nsq {

namespace {

constexpr int BW = 128;  // weight rows per tile (UMMA M, TMEM lanes)
constexpr int BK = 64;   // columns per k-block
constexpr int NS = 4;    // stages: x tile + packed weight tile in shared memory, operand in TMEM
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpConv0 = 2;
constexpr int kConvWarps = 8;
constexpr int kWarpEpi0 = kWarpConv0 + kConvWarps;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;
constexpr int kMinSmem = 120 * 1024;  // keeps one CTA (and one TMEM owner) per SM

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
  static constexpr uint32_t kAcc = 0;           // 2 accumulators of BT columns
  static constexpr uint32_t kA = 2 * BT;        // NS operand stages of 32 columns (64 K values)
  static constexpr uint32_t kUsed = kA + NS * 32;
  static constexpr uint32_t kCols = kUsed <= 256 ? 256 : 512;
  static_assert(kUsed <= 512, "tensor memory budget");
};

template <int FMT, int BT>
struct TsSmem {
  static constexpr int kXBytes = BT * BK * 2;
  static constexpr int kX = 0;
  static constexpr int kWc = kX + NS * kXBytes;
  static constexpr int kBar = kWc + NS * TsFmt<FMT>::kWcBytes;
  // full_l[NS], read_w[NS], full_a[NS], mma_done[NS], full_acc[2], empty_acc[2]
  static constexpr int kNumBars = 4 * NS + 4;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kTotal = kAbort + 4;
  static constexpr int kNeed = kTotal + 1024;  // room to align the base to 1 KB
  static constexpr int kAlloc = kNeed > kMinSmem ? kNeed : kMinSmem;
  static_assert(kXBytes % 1024 == 0, "x stages stay 1 KB aligned");
  static_assert(kAlloc <= 227 * 1024, "shared memory per CTA");
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
};

template <int FMT, bool BF16, int BT>
__global__ void __launch_bounds__(kThreads, 1) prefill_ts_kernel(
    const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
    const TsParams p) {
  using L = TsSmem<FMT, BT>;
  using TM = TsTmem<BT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  // Per stage s: full_l (TMA bytes of x and the packed weight landed), read_w
  // (the converters read the packed weight), full_a (the converters wrote the
  // TMEM operand; implies full_l), mma_done (the UMMAs of the stage finished:
  // frees both the x tile and the TMEM operand). The MMA issuer waits on one
  // barrier and commits one per k-block: every barrier operation in its loop
  // delays the next UMMA.
  uint64_t* full_l = bars;
  uint64_t* read_w = bars + NS;
  uint64_t* full_a = bars + 2 * NS;
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
      mbar_init(&full_a[i], kConvWarps);
      mbar_init(&mma_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full_acc[i], 1);
      mbar_init(&empty_acc[i], kEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, TM::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // everything below may read what the previous kernel on the stream wrote
  pdl_wait_prior_grids();

  const int num_units = p.num_w_tiles * p.num_t_tiles;  // token tile fastest
  bool ok = true;

  if (warp == kWarpTma) {
    if (lane == 0) {
      tma_prefetch_desc(&xmap);
      tma_prefetch_desc(&wmap);
      int it = 0;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int wt = u / p.num_t_tiles;
        const int tt = u - wt * p.num_t_tiles;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const int s = it % NS;
          const uint32_t ph = ((it / NS) & 1) ^ 1;  // previous use of the stage
          if (!(ok = mbar_wait(&read_w[s], ph, p.status, 50, abort_flag))) break;
          if (!(ok = mbar_wait(&mma_done[s], ph, p.status, 57, abort_flag))) break;
          mbar_arrive_expect_tx(&full_l[s], L::kXBytes + TsFmt<FMT>::kWcBytes);
          tma_load_2d(smem + L::kX + s * L::kXBytes, &xmap, &full_l[s], kb * BK, tt * BT);
          tma_load_2d(smem + L::kWc + s * TsFmt<FMT>::kWcBytes, &wmap, &full_l[s],
                      FMT == 0 ? kb * (BK / 8) : kb * BK, wt * BW);
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
      int it = 0, tcount = 0;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++tcount) {
        const int tt = u % p.num_t_tiles;
        // UMMA N: the tile's tokens rounded up to 16 (the x rows past M are
        // zero-filled by TMA; their accumulator columns are never stored)
        int n_eff = p.M - tt * BT;
        n_eff = n_eff > BT ? BT : ((n_eff + 15) & ~15);
        const uint32_t idesc = umma_idesc_f16(BF16, BW, n_eff);
        const int acc = tcount & 1;
        if (!(ok = mbar_wait(&empty_acc[acc], ((tcount >> 1) & 1) ^ 1, p.status, 51, abort_flag))) break;
        tc_fence_after();
        const uint32_t d = tmem_base + TM::kAcc + acc * BT;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const int s = it % NS;
          if (!(ok = mbar_wait(&full_a[s], (it / NS) & 1, p.status, 53, abort_flag))) break;
          tc_fence_after();
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(smem + L::kX + s * L::kXBytes));
          const uint32_t a = tmem_base + TM::kA + s * 32;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // A: +8 TMEM columns per 16 K; B: +32 bytes inside the swizzled row
            umma_f16_ts(d, a + 8 * kk, bdesc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&mma_done[s]);
        }
        if (!ok) break;
        tc_commit(&full_acc[acc]);
      }
    }
  } else if (warp < kWarpEpi0) {
    // ---------------- converters: packed weight -> TMEM operand ----------------
    const int sub = warp & 3;                   // TMEM sub-partition = 32 weight rows
    const int half = (warp - kWarpConv0) >> 2;  // 32-column half of the k-block
    const int row = sub * 32 + lane;            // weight row within the tile
    const uint32_t a_lane = tmem_base + ((uint32_t)(sub * 32) << 16) + TM::kA + half * 16;
    // AWQ: the (scale, zero) pairs this thread needs, in the order it needs
    // them -- (unit, group) for its row -- loaded three groups ahead into a
    // register ring so their latency hides behind whole groups of k-blocks
    const unsigned short* sc16 = reinterpret_cast<const unsigned short*>(p.scales);
    const unsigned short* zr16 = reinterpret_cast<const unsigned short*>(p.zeros);
    int pu = blockIdx.x, pg = 0;
    auto load_sz = [&]() -> uint32_t {
      uint32_t v = 0;
      if (pu < num_units) {
        const int n = (pu / p.num_t_tiles) * BW + row;
        if (n < p.N) {
          const int64_t off = (int64_t)n * p.G + pg;
          v = (uint32_t)__ldg(sc16 + off) | ((uint32_t)__ldg(zr16 + off) << 16);
        }
        if (++pg == p.G) {
          pg = 0;
          pu += gridDim.x;
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
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
        const int s = it % NS;
        const uint32_t ph = (it / NS) & 1;
        if constexpr (FMT == 0) {
          if ((kb * BK) % p.group_size == 0) {  // a new group (kb = 0 included)
            rp = ts_row_dq_packed<BF16>(sz0);
            sz0 = sz1;
            sz1 = sz2;
            sz2 = load_sz();
          }
        }
        if (!(ok = mbar_wait(&full_l[s], ph, p.status, 54, abort_flag))) break;
        uint32_t o[16];
        ts_convert_k32<FMT, BF16>(smem_u32(smem + L::kWc + s * TsFmt<FMT>::kWcBytes), row, half, rp, o);
        // the packed tile is consumed (the x tile of the stage is freed by
        // the UMMAs' commit)
        __syncwarp();
        if (lane == 0) mbar_arrive(&read_w[s]);
        // the TMEM operand stage is free once the UMMAs of its previous use finished
        if (!(ok = mbar_wait(&mma_done[s], ph ^ 1, p.status, 55, abort_flag))) break;
        tc_fence_after();
        tmem_st_32x32b_x16(a_lane + s * 32, o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> y ----------------
    const int sub = warp & 3;
    const float wscale = (FMT == 1) ? __ldg(p.wscale) : 1.0f;
    int tcount = 0;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++tcount) {
      const int wt = u / p.num_t_tiles;
      const int tt = u - wt * p.num_t_tiles;
      const int acc = tcount & 1;
      if (!(ok = mbar_wait(&full_acc[acc], (tcount >> 1) & 1, p.status, 56, abort_flag))) break;
      tc_fence_after();
      const int n = wt * BW + sub * 32 + lane;  // this thread's output feature
      const float bn =
          (p.bias_dtype != NSQ_DTYPE_NONE && n < p.N) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
      const bool has_bias = p.bias_dtype != NSQ_DTYPE_NONE;
      const uint32_t taddr = tmem_base + ((uint32_t)(sub * 32) << 16) + TM::kAcc + acc * BT;
      uint16_t* y = static_cast<uint16_t*>(p.y);
      const int m0 = tt * BT;
#pragma unroll 1
      for (int c = 0; c < BT / 32 && m0 + c * 32 < p.M; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_ld_wait();
        ts_store_tokens<BF16>(y, p.M, p.N, n, m0 + c * 32, r, wscale, has_bias, bn, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_acc[acc]);
    }
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
  cudaLaunchAttribute attrs[1];
  int na = 0;
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
int run_ts(const LinearArgs& a, cudaStream_t stream) {
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
  const int units = p.num_w_tiles * p.num_t_tiles;
  const int sms = num_sms();
  const int grid = units < sms ? units : sms;
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

int prefill_ts_tokens_per_tile(int64_t M, int64_t K, int64_t N) {
  (void)K;
  // Problems with at most 2^20 outputs (the shared-memory-operand kernels'
  // 128 x 256 / 256 x 256 tiles leave most SMs idle there): the narrowest
  // token tile whose units still fit in one wave. Measured on B200 against
  // those kernels on the Qwen2.5-0.5B shapes (FP8 / AWQ): 1.7-1.9x faster at
  // M = 128, 1.3x at M = 1024 (q/k/v/o), 1.3x for k/v at M = 8192; slower
  // for the larger outputs.
  if (M <= kDecodeMaxM || M * N > ((int64_t)1 << 20)) return 0;
  const int64_t wt = (N + BW - 1) / BW;
  const int sms = num_sms();
  for (int bt : {64, 128}) {
    if (wt * ((M + bt - 1) / bt) <= sms) return bt;
  }
  return 192;
}

int run_prefill_ts_linear(const LinearArgs& a, int tokens_per_tile, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0) return NSQ_OK;
  switch (tokens_per_tile) {
    case 64: return run_ts<64>(a, stream);
    case 128: return run_ts<128>(a, stream);
    case 192: return run_ts<192>(a, stream);
    default: return NSQ_ENOTSUP;
  }
}

}  // namespace nsq
