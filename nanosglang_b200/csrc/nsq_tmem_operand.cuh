// Pieces shared by the prefill kernels that keep the dequantised weight tile
// in tensor memory (the A operand of tcgen05.mma) and the token tile of x in
// shared memory: per-row AWQ dequant constants, the conversion of 32 packed
// columns of one weight row into 16 MMA-element pairs, and the store of a
// transposed accumulator chunk (lane = output feature, column = token).
#pragma once

#include <type_traits>

#include "nsq_common.cuh"

namespace nsq {

template <bool BF16>
struct TsRowDq {  // per-row AWQ dequant constants in the MMA element type
  uint32_t s2, zb2, magic2, c2;
  bool exact;
};

template <bool BF16>
__device__ __forceinline__ uint32_t ts_pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <bool BF16>
__device__ __forceinline__ TsRowDq<BF16> ts_row_dq(float s, float z) {
  TsRowDq<BF16> r;
  constexpr float kMagic = Magic<BF16>::kValue;
  constexpr float kZMax = BF16 ? 127.0f : 1023.0f;
  r.exact = (z == rintf(z)) && fabsf(z) <= kZMax;
  r.s2 = ts_pack2<BF16>(s, s);
  r.zb2 = ts_pack2<BF16>(kMagic + z, kMagic + z);
  r.magic2 = ts_pack2<BF16>(kMagic, kMagic);
  r.c2 = ts_pack2<BF16>(-z * s, -z * s);
  return r;
}

// (scale, zero) packed as fp16 bits {scale | zero << 16} -> dequant constants
template <bool BF16>
__device__ __forceinline__ TsRowDq<BF16> ts_row_dq_packed(uint32_t sz) {
  return ts_row_dq<BF16>(__half2float(__ushort_as_half((unsigned short)(sz & 0xFFFFu))),
                         __half2float(__ushort_as_half((unsigned short)(sz >> 16))));
}

// {magic + q_a, magic + q_b} -> {(q_a - z) s, (q_b - z) s}; exact in the
// packed domain when z is a small integer, else fma with -z s
template <bool BF16>
__device__ __forceinline__ uint32_t ts_dq2(uint32_t e, const TsRowDq<BF16>& rp) {
  using T2 = typename std::conditional<BF16, __nv_bfloat162, __half2>::type;
  const T2 ev = *reinterpret_cast<const T2*>(&e);
  const T2 s = *reinterpret_cast<const T2*>(&rp.s2);
  T2 o;
  if (rp.exact) {
    o = __hmul2(__hsub2(ev, *reinterpret_cast<const T2*>(&rp.zb2)), s);
  } else {
    o = __hfma2(__hsub2(ev, *reinterpret_cast<const T2*>(&rp.magic2)), s,
                *reinterpret_cast<const T2*>(&rp.c2));
  }
  return *reinterpret_cast<uint32_t*>(&o);
}

// Bytes of one packed weight row per 64-column k-block, as TMA lands it:
// AWQ 8 words (32-byte swizzle), FP8 64 bytes (64-byte swizzle).
template <int FMT>
struct TsRow {
  static constexpr int kBytes = FMT == 0 ? 32 : 64;
};

// Columns [32 half, 32 half + 32) of row `row` of a packed k-block tile at
// shared address `tile` -> 16 pairs in the MMA element type, K order.
template <int FMT, bool BF16>
__device__ __forceinline__ void ts_convert_k32(uint32_t tile, int row, int half, const TsRowDq<BF16>& rp,
                                               uint32_t (&o)[16]) {
  if constexpr (FMT == 0) {
    // 32-byte swizzle: 16-byte chunk c of row r sits at c ^ ((r >> 2) & 1)
    const uint32_t wc = tile + row * 32;
    const uint4 v = lds128(wc + ((half ^ ((row >> 2) & 1)) << 4));
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t e[4];
      unpack_nibble_pairs<BF16>(words[w], e);
      // e[t] = {q_t, q_{t+4}} -> in-order pairs {q0,q1},{q2,q3},{q4,q5},{q6,q7}
      o[4 * w + 0] = ts_dq2<BF16>(prmt(e[0], e[1], 0x5410), rp);
      o[4 * w + 1] = ts_dq2<BF16>(prmt(e[2], e[3], 0x5410), rp);
      o[4 * w + 2] = ts_dq2<BF16>(prmt(e[0], e[1], 0x7632), rp);
      o[4 * w + 3] = ts_dq2<BF16>(prmt(e[2], e[3], 0x7632), rp);
    }
  } else {
    // 64-byte swizzle: 16-byte chunk c of row r sits at c ^ ((r >> 1) & 3)
    const uint32_t wc = tile + row * 64;
    const uint32_t sw = (row >> 1) & 3;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 v = lds128(wc + (((2 * half + c) ^ sw) << 4));
      e4m3x4_to_pairs<BF16>(v.x, o[8 * c + 0], o[8 * c + 1]);
      e4m3x4_to_pairs<BF16>(v.y, o[8 * c + 2], o[8 * c + 3]);
      e4m3x4_to_pairs<BF16>(v.z, o[8 * c + 4], o[8 * c + 5]);
      e4m3x4_to_pairs<BF16>(v.w, o[8 * c + 6], o[8 * c + 7]);
    }
  }
}

// Scale, bias, round and store T tokens m0 .. m0+T-1 of output feature n held
// by this lane (accumulator chunk r, fp32 bits). With N even, lanes 2i and
// 2i+1 (features n, n+1) exchange values so the even lane stores the pair of
// token 2j and the odd lane the pair of token 2j+1 (one 32-bit store each).
template <bool BF16, int T>
__device__ __forceinline__ void ts_store_tokens(uint16_t* y, int M, int N, int n, int m0, const uint32_t (&r)[T],
                                                float wscale, bool has_bias, float bn, int lane) {
  if ((N & 1) == 0) {
    const bool odd = lane & 1;
#pragma unroll
    for (int j = 0; j < T / 2; ++j) {
      const float a0 = __uint_as_float(r[2 * j]), a1 = __uint_as_float(r[2 * j + 1]);
      const float v0 = has_bias ? fmaf(a0, wscale, bn) : a0 * wscale;
      const float v1 = has_bias ? fmaf(a1, wscale, bn) : a1 * wscale;
      const float recv = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
      const int m = m0 + 2 * j + (odd ? 1 : 0);
      const int nn = odd ? n - 1 : n;
      if (m < M && nn < N) {
        const uint32_t w = odd ? ts_pack2<BF16>(recv, v1) : ts_pack2<BF16>(v0, recv);
        *reinterpret_cast<uint32_t*>(y + (int64_t)m * N + nn) = w;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < T; ++j) {
      const float a = __uint_as_float(r[j]);
      const float v = has_bias ? fmaf(a, wscale, bn) : a * wscale;
      const int m = m0 + j;
      if (m < M && n < N) y[(int64_t)m * N + n] = static_cast<uint16_t>(ts_pack2<BF16>(v, 0.f) & 0xFFFFu);
    }
  }
}

}  // namespace nsq
