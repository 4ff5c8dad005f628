// Host-side declarations shared by libnsq's translation units.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nsq {

struct DevStatus;

int num_sms();                  // SM count of the current device (cached per device)
int device_ready();             // NSQ_OK if the current device is sm_100, else an NSQ_E* code
DevStatus* device_status_ptr(); // device address of this device's status word (lazily set up)
bool pdl_enabled();
bool test_withhold();  // failure-path test hook: the multi-wave decode kernel skips one weight load

// cuTensorMapEncodeTiled through the runtime's driver entry point (libnsq does
// not link libcuda directly, so it also loads on machines without a driver).
CUresult encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, void* base,
                              uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);
// Rank 3: dims d0 (contiguous), d1, d2 with byte strides of d1 and d2; box b0 x b1 x b2
// (shared memory gets the box with d0 fastest, then d1, then d2).
CUresult encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, void* base, uint64_t d0, uint64_t d1,
                              uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                              uint32_t b2, CUtensorMapSwizzle swizzle);

// elementwise
cudaError_t launch_awq_dequant(const int32_t* qweight, const uint16_t* scales,
                               const uint16_t* zeros, uint16_t* out, int64_t N, int64_t K,
                               int64_t gs, cudaStream_t stream);
cudaError_t launch_fp8_dequant(const uint8_t* w, const float* scale, void* out, int out_dtype,
                               int64_t total, cudaStream_t stream);
cudaError_t launch_awq_quantize(const void* w, int dtype, int64_t N, int64_t K, int64_t gs,
                                int32_t* qweight, uint16_t* scales, uint16_t* zeros,
                                cudaStream_t stream);
cudaError_t launch_awq_from_autoawq(const int32_t* qweight_kn8, const int32_t* qzeros_gn8,
                                    const uint16_t* scales_gn, int64_t K, int64_t N, int64_t gs,
                                    int32_t* qweight, uint16_t* scales, uint16_t* zeros, cudaStream_t stream);
cudaError_t launch_fp8_quantize(const void* w, int dtype, int64_t total, uint8_t* codes,
                                float* scale, void* workspace, cudaStream_t stream);

// linears. fmt: 0 = AWQ int4, 1 = FP8 e4m3. Return an NSQ_* code.
struct LinearArgs {
  int fmt;
  const void* x;
  int x_bf16;
  int M, K, N;
  const void* wq;          // qweight (AWQ) or weight_fp8 (FP8)
  const uint16_t* scales;  // AWQ
  const uint16_t* zeros;   // AWQ
  int group_size;          // AWQ
  const float* wscale;     // FP8
  const void* bias;
  int bias_dtype;
  void* y;
  void* ws;  // caller workspace (may be null)
  size_t ws_bytes;
};
int run_decode_wave_linear(const LinearArgs& a, cudaStream_t stream);  // M <= 64, one wave of CTAs
int run_decode_stream_linear(const LinearArgs& a, cudaStream_t stream);  // M <= 64, persistent weight ring
int run_decode_linear(const LinearArgs& a, cudaStream_t stream);   // M <= 64, one or more waves
int decode_linear_ctas(const LinearArgs& a);  // CTAs run_decode_linear launches, -1 if it cannot
// Row-streaming decode kernel over 1..3 weights sharing x (M <= 32). mode 0:
// weight i writes y columns [ycol, ycol + n); mode 1: w[0] = gate, w[1] =
// up (same n), y[:, :n] = SiLU(x gate^T) * (x up^T).
struct RowsWeight {
  const void* w;           // qweight [n, K/8] (AWQ) or weight_fp8 [n, K] (FP8)
  const uint16_t* scales;  // AWQ
  const uint16_t* zeros;   // AWQ
  const float* wscale;     // FP8
  const void* bias;        // [n] or null (dtype: RowsLaunch::bias_dtype)
  int n;
  int ycol;
};
struct RowsLaunch {
  int fmt;
  const void* x;
  int x_bf16;
  int M, K;
  void* y;
  int ldy;  // row stride of y (elements)
  int group_size;
  int bias_dtype;
  int mode;
  int nw;
  RowsWeight w[3];
};
int run_decode_rows(const RowsLaunch& L, cudaStream_t stream);
int run_decode_rows_linear(const LinearArgs& a, cudaStream_t stream);
// Tensor-core decode kernel (M <= 64, K % 128 == 0, AWQ groups of 128 k, 64 to
// 128 weight rows per CTA; one CTA per SM, fewer on layers of fewer than 64
// rows per SM): rows of the tallest CTA, or 0 if it does not apply.
int decode_tc_rows(const LinearArgs& a);
// Workspace with which the kernel takes precomputed x terms (one small kernel
// ahead of it instead of every CTA computing them); without it, the CTAs do.
size_t decode_tc_workspace_bytes(const LinearArgs& a);
int run_decode_tc_linear(const LinearArgs& a, cudaStream_t stream);
// prefill: the weight tile dequantised into tensor memory (A operand), tokens
// as UMMA N. One CTA per 128 weight rows x 64/128 tokens, K optionally split
// over a cluster (small outputs, few-tile long-K layers), or CTA pairs with
// 256 weight rows x 256 tokens (the rest).
struct TsPlan {
  int tokens_per_tile;  // 64 or 128; 0: use the paired kernel
  int ksplit;           // CTAs per tile along K (cluster size)
};
TsPlan prefill_ts_plan(int fmt, int64_t M, int64_t K, int64_t N);  // fmt: 0 AWQ, 1 FP8
int run_prefill_ts_linear(const LinearArgs& a, TsPlan plan, cudaStream_t stream);
int run_prefill_ts2_linear(const LinearArgs& a, cudaStream_t stream);

constexpr int kDecodeMaxM = 64;

}  // namespace nsq
