// Bandwidth-bound elementwise kernels of libnsq:
//   * AWQ unpack+dequantise, bit-exact with AWQLinear._dequantize
//     (nano_sglang/decode/quantization.py:126-148)
//   * FP8 dequantise, bit-exact with `weight_fp8.to(dtype) * weight_scale`
//     (quantization.py:51)
//   * AWQ / FP8 quantisers, bit-exact with AWQLinear.from_linear
//     (quantization.py:154-194) and FP8Linear.from_linear (quantization.py:54-75)
//   * repack of an AutoAWQ (GEMM-format) layer into the reference layout, the
//     loader the reference's docstring names (quantization.py:7) but lacks
//
// All are grid-stride kernels sized to a multiple of the SM count; each thread
// moves 16-byte vectors where the layout allows.
#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

// One thread per packed word: 8 nibbles -> 8 fp16 outputs (one 16-byte store).
// Per element: q -> fp16 (exact), then fp16(q - z), then fp16(. * s): the same
// two correctly-rounded fp16 operations the reference performs per group.
__global__ void __launch_bounds__(256) awq_dequant_kernel(const uint32_t* __restrict__ qweight,
                                                          const __half* __restrict__ scales,
                                                          const __half* __restrict__ zeros,
                                                          __half* __restrict__ out, int64_t N,
                                                          int64_t K, int64_t gs, int64_t G) {
  const int64_t k8 = K / 8;
  const int64_t total = N * k8;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = idx / k8;
    const int64_t j = idx - n * k8;
    const uint32_t w = __ldg(qweight + idx);
    const int64_t kbase = j * 8;
    __align__(16) __half r[8];
    int64_t g_prev = -1;
    __half s = __float2half(0.f), z = __float2half(0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t g = (kbase + i) / gs;
      if (g != g_prev) {
        s = scales[n * G + g];
        z = zeros[n * G + g];
        g_prev = g;
      }
      const __half q = __uint2half_rn((w >> (4 * i)) & 0xFu);
      r[i] = __hmul(__hsub(q, z), s);
    }
    *reinterpret_cast<uint4*>(out + n * K + kbase) = *reinterpret_cast<const uint4*>(r);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(256) fp8_dequant_kernel(const uint8_t* __restrict__ w,
                                                          const float* __restrict__ scale_ptr,
                                                          uint16_t* __restrict__ out,
                                                          int64_t total) {
  const float scale = __ldg(scale_ptr);
  const int64_t nvec = total / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const uint2 codes = __ldg(reinterpret_cast<const uint2*>(w) + v);
    __align__(16) uint16_t r[8];
    const uint32_t c[2] = {codes.x, codes.y};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const __nv_fp8_e4m3 e = *reinterpret_cast<const __nv_fp8_e4m3*>(
            reinterpret_cast<const uint8_t*>(&c[h]) + b);
        r[h * 4 + b] = float_to_elem<BF16>(static_cast<float>(e) * scale);
      }
    }
    *reinterpret_cast<uint4*>(out + v * 8) = *reinterpret_cast<const uint4*>(r);
  }
  // tail (total % 8 elements)
  const int64_t tail0 = nvec * 8;
  for (int64_t i = tail0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const __nv_fp8_e4m3 e = *reinterpret_cast<const __nv_fp8_e4m3*>(w + i);
    out[i] = float_to_elem<BF16>(static_cast<float>(e) * scale);
  }
}

__device__ __forceinline__ float load_as_float(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case NSQ_DTYPE_F16:
      return __half2float(reinterpret_cast<const __half*>(p)[i]);
    case NSQ_DTYPE_BF16:
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    default:
      return reinterpret_cast<const float*>(p)[i];
  }
}

// One warp per (row, group). Lanes stride the group's columns, reduce min/max
// with shuffles, then every lane quantises its columns. Words that lie inside
// the group are OR-ed together in registers and stored once; when the group
// size is not a multiple of 8 a word can straddle two groups, so those words
// are combined with atomicOr into a zero-filled qweight.
__global__ void __launch_bounds__(256) awq_quantize_kernel(const void* __restrict__ w, int dtype,
                                                           int64_t N, int64_t K, int64_t gs,
                                                           int64_t G, uint32_t* __restrict__ qweight,
                                                           __half* __restrict__ scales,
                                                           __half* __restrict__ zeros,
                                                           int use_atomic) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t k8 = K / 8;
  for (int64_t item = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32; item < N * G;
       item += warps_total) {
    const int64_t n = item / G;
    const int64_t g = item - n * G;
    const int64_t c0 = g * gs;
    const int64_t c1 = min(c0 + gs, K);
    float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
    for (int64_t c = c0 + lane; c < c1; c += 32) {
      const float v = load_as_float(w, dtype, n * K + c);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    float scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    scale = (scale < 1e-8f) ? 1e-8f : scale;  // clamp(min=1e-8), NaN passes through
    const float zero = rintf(__fdiv_rn(-mn, scale));
    if (lane == 0) {
      scales[n * G + g] = __float2half_rn(scale);
      zeros[n * G + g] = __float2half_rn(zero);
    }
    // quantise + pack: lane handles words; each word covers columns 8j..8j+7
    const int64_t j0 = c0 / 8, j1 = (c1 + 7) / 8;
    for (int64_t j = j0 + lane; j < j1 && j < k8; j += 32) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t c = j * 8 + i;
        if (c < c0 || c >= c1) continue;
        const float v = load_as_float(w, dtype, n * K + c);
        float q = rintf(__fdiv_rn(__fsub_rn(v, mn), scale));
        q = fminf(fmaxf(q, 0.0f), 15.0f);
        word |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xFu) << (4 * i);
      }
      if (use_atomic) {
        atomicOr(qweight + n * k8 + j, word);
      } else {
        qweight[n * k8 + j] = word;
      }
    }
  }
}

// absmax over the whole weight into a zero-initialised uint (float bits; all
// values are >= 0 so unsigned order == float order, NaN sorts highest).
__global__ void __launch_bounds__(256) absmax_kernel(const void* __restrict__ w, int dtype,
                                                     int64_t total, unsigned int* __restrict__ out) {
  float m = 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = fabsf(load_as_float(w, dtype, i));
    m = (v > m || v != v) ? v : m;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, m, o);
    m = (t > m || t != t) ? t : m;
  }
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = red[0];
    for (int i = 1; i < (int)(blockDim.x / 32); ++i) b = (red[i] > b || red[i] != red[i]) ? red[i] : b;
    atomicMax(out, __float_as_uint(b));
  }
}

// float -> e4m3 code with torch's cast semantics: RNE, finite values whose
// magnitude rounds above 448 (i.e. > 464) and +-inf become NaN with the input's
// sign, NaN becomes 0x7F.
__device__ __forceinline__ uint8_t e4m3_encode_torch(float v) {
  if (v != v) return 0x7F;
  const uint8_t sign = (__float_as_uint(v) >> 24) & 0x80u;
  if (fabsf(v) > 464.0f) return sign | 0x7F;
  const __nv_fp8_storage_t c = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint8_t>(c);
}

__global__ void __launch_bounds__(256) fp8_quantize_kernel(const void* __restrict__ w, int dtype,
                                                           int64_t total,
                                                           const unsigned int* __restrict__ absmax_bits,
                                                           uint8_t* __restrict__ codes,
                                                           float* __restrict__ scale_out) {
  const float absmax = __uint_as_float(*absmax_bits);
  float scale = __fdiv_rn(absmax, 448.0f);
  if (scale == 0.0f) scale = 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    codes[i] = e4m3_encode_torch(__fdiv_rn(load_as_float(w, dtype, i), scale));
  }
}

// ---------------------------------------------------------------------------
// AutoAWQ GEMM format -> reference layout. AutoAWQ packs eight output columns
// per int32 word along N with nibble i holding column 8c + order[i], order =
// {0, 2, 4, 6, 1, 3, 5, 7}; the reference packs eight input columns per word
// along K, nibble i = column 8j + i. Column n sits in nibble kAutoAwqNibble[n % 8].
__constant__ int kAutoAwqNibble[8] = {0, 4, 1, 5, 2, 6, 3, 7};

// One thread per output word (n, j), j fastest so the stores are coalesced;
// it gathers nibble kAutoAwqNibble[n % 8] of input rows 8j .. 8j+7.
__global__ void __launch_bounds__(256) awq_from_autoawq_qweight_kernel(const uint32_t* __restrict__ qw_kn,
                                                                       uint32_t* __restrict__ out, int64_t N,
                                                                       int64_t K) {
  const int64_t k8 = K / 8, n8 = N / 8;
  const int64_t total = N * k8;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = idx / k8;
    const int64_t j = idx - n * k8;
    const int sh = 4 * kAutoAwqNibble[n & 7];
    const uint32_t* src = qw_kn + (j * 8) * n8 + (n >> 3);
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w |= ((__ldg(src + i * n8) >> sh) & 0xFu) << (4 * i);
    out[idx] = w;
  }
}

// One thread per (n, g), g fastest: zero point (int4 -> fp16, exact) and scale
// transposed from [G, N] to [N, G].
__global__ void __launch_bounds__(256) awq_from_autoawq_sz_kernel(const uint32_t* __restrict__ qz_gn,
                                                                  const __half* __restrict__ s_gn,
                                                                  __half* __restrict__ s_out,
                                                                  __half* __restrict__ z_out, int64_t N,
                                                                  int64_t G) {
  const int64_t total = N * G;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = idx / G;
    const int64_t g = idx - n * G;
    const uint32_t w = __ldg(qz_gn + g * (N / 8) + (n >> 3));
    z_out[idx] = __uint2half_rn((w >> (4 * kAutoAwqNibble[n & 7])) & 0xFu);
    s_out[idx] = s_gn[g * N + n];
  }
}

// Host launchers (validated by nsq_api.cu before they are called)
// ---------------------------------------------------------------------------
static int grid_for(int64_t items, int threads) {
  const int64_t want = (items + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 8;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

cudaError_t launch_awq_dequant(const int32_t* qweight, const uint16_t* scales,
                               const uint16_t* zeros, uint16_t* out, int64_t N, int64_t K,
                               int64_t gs, cudaStream_t stream) {
  const int64_t G = (K + gs - 1) / gs;
  const int64_t items = N * (K / 8);
  if (items == 0) return cudaSuccess;
  awq_dequant_kernel<<<grid_for(items, 256), 256, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(qweight), reinterpret_cast<const __half*>(scales),
      reinterpret_cast<const __half*>(zeros), reinterpret_cast<__half*>(out), N, K, gs, G);
  return cudaGetLastError();
}

cudaError_t launch_fp8_dequant(const uint8_t* w, const float* scale, void* out, int out_dtype,
                               int64_t total, cudaStream_t stream) {
  if (total == 0) return cudaSuccess;
  const int grid = grid_for(total / 8 + 1, 256);
  if (out_dtype == NSQ_DTYPE_BF16) {
    fp8_dequant_kernel<true><<<grid, 256, 0, stream>>>(w, scale, static_cast<uint16_t*>(out), total);
  } else {
    fp8_dequant_kernel<false><<<grid, 256, 0, stream>>>(w, scale, static_cast<uint16_t*>(out), total);
  }
  return cudaGetLastError();
}

cudaError_t launch_awq_quantize(const void* w, int dtype, int64_t N, int64_t K, int64_t gs,
                                int32_t* qweight, uint16_t* scales, uint16_t* zeros,
                                cudaStream_t stream) {
  const int64_t G = (K + gs - 1) / gs;
  const int use_atomic = (gs % 8) != 0;
  if (use_atomic) {
    cudaError_t e = cudaMemsetAsync(qweight, 0, sizeof(int32_t) * N * (K / 8), stream);
    if (e != cudaSuccess) return e;
  }
  if (N * G == 0) return cudaSuccess;
  awq_quantize_kernel<<<grid_for(N * G * 32, 256), 256, 0, stream>>>(
      w, dtype, N, K, gs, G, reinterpret_cast<uint32_t*>(qweight),
      reinterpret_cast<__half*>(scales), reinterpret_cast<__half*>(zeros), use_atomic);
  return cudaGetLastError();
}

cudaError_t launch_awq_from_autoawq(const int32_t* qweight_kn8, const int32_t* qzeros_gn8,
                                    const uint16_t* scales_gn, int64_t K, int64_t N, int64_t gs,
                                    int32_t* qweight, uint16_t* scales, uint16_t* zeros, cudaStream_t stream) {
  const int64_t G = K / gs;
  if (N * (K / 8) > 0) {
    awq_from_autoawq_qweight_kernel<<<grid_for(N * (K / 8), 256), 256, 0, stream>>>(
        reinterpret_cast<const uint32_t*>(qweight_kn8), reinterpret_cast<uint32_t*>(qweight), N, K);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (N * G > 0) {
    awq_from_autoawq_sz_kernel<<<grid_for(N * G, 256), 256, 0, stream>>>(
        reinterpret_cast<const uint32_t*>(qzeros_gn8), reinterpret_cast<const __half*>(scales_gn),
        reinterpret_cast<__half*>(scales), reinterpret_cast<__half*>(zeros), N, G);
  }
  return cudaGetLastError();
}

cudaError_t launch_fp8_quantize(const void* w, int dtype, int64_t total, uint8_t* codes,
                                float* scale, void* workspace, cudaStream_t stream) {
  unsigned int* absmax = static_cast<unsigned int*>(workspace);
  cudaError_t e = cudaMemsetAsync(absmax, 0, sizeof(unsigned int), stream);
  if (e != cudaSuccess) return e;
  if (total > 0) {
    absmax_kernel<<<grid_for(total, 256), 256, 0, stream>>>(w, dtype, total, absmax);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  fp8_quantize_kernel<<<grid_for(total > 0 ? total : 1, 256), 256, 0, stream>>>(w, dtype, total,
                                                                                absmax, codes, scale);
  return cudaGetLastError();
}

}  // namespace nsq
