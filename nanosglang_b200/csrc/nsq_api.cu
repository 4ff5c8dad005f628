// C ABI of libnsq (declared in include/nsq.h): host-side validation, device
// capability checks, tensor-map encoding and dispatch to the kernels.
//
// Validation happens before any launch and mirrors the reference's own
// failure modes where it has them (e.g. in_features % 8 != 0 raises in
// AWQLinear._dequantize, quantization.py:134-137); everything else the
// kernels need (alignment, K multiples for TMA) is reported as an error code.
#include <atomic>
#include <cstddef>
#include <mutex>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

__device__ DevStatus g_device_status;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
// per-device caches, written once under g_mu and read without it
std::atomic<int> g_sms[kMaxDevices];
std::atomic<int> g_arch_ok[kMaxDevices];  // 0 unknown, 1 ok, -1 not sm_100
std::atomic<DevStatus*> g_status_ptr[kMaxDevices];
std::atomic<int> g_pdl{0};
std::atomic<int> g_withhold{0};  // failure-path test hook (nsq_test_withhold_weight_load)
std::atomic<int> g_sm_reserve{0};  // SMs the linear kernels leave free (nsq_set_sm_reserve)

std::atomic<PFN_cuTensorMapEncodeTiled_v12000> g_encode{nullptr};

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return (d >= 0 && d < kMaxDevices) ? d : -1;
}

// NSQ_OK if the current device is an sm_100 part, else an error code.
int check_device() {
  const int d = current_device();
  if (d < 0) return NSQ_ECUDA;
  const int known = g_arch_ok[d].load(std::memory_order_acquire);
  if (known == 1) return NSQ_OK;
  if (known == -1) return NSQ_ENOTSUP;
  std::lock_guard<std::mutex> lk(g_mu);
  int major = 0, minor = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess) {
    return NSQ_ECUDA;
  }
  g_sms[d].store(sms, std::memory_order_relaxed);
  const int arch = (major == 10 && minor == 0) ? 1 : -1;
  g_arch_ok[d].store(arch, std::memory_order_release);
  return arch == 1 ? NSQ_OK : NSQ_ENOTSUP;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline bool valid_act_dtype(int t) { return t == NSQ_DTYPE_F16 || t == NSQ_DTYPE_BF16; }
inline bool valid_bias_dtype(int t) {
  return t == NSQ_DTYPE_NONE || t == NSQ_DTYPE_F16 || t == NSQ_DTYPE_BF16 || t == NSQ_DTYPE_F32;
}

constexpr int64_t kIntMax = 0x7FFFFFFF;

}  // namespace

int num_sms() {
  const int d = current_device();
  if (d < 0) return 148;
  if (g_sms[d].load(std::memory_order_acquire) == 0) check_device();
  const int sms = g_sms[d].load(std::memory_order_acquire);
  const int all = sms > 0 ? sms : 148;
  const int use = all - g_sm_reserve.load(std::memory_order_relaxed);
  return use >= all / 2 ? use : all / 2;
}

DevStatus* device_status_ptr() {
  const int d = current_device();
  if (d < 0) return nullptr;
  DevStatus* cached = g_status_ptr[d].load(std::memory_order_acquire);
  if (cached != nullptr) return cached;
  std::lock_guard<std::mutex> lk(g_mu);
  cached = g_status_ptr[d].load(std::memory_order_relaxed);
  if (cached == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    cached = static_cast<DevStatus*>(p);
    g_status_ptr[d].store(cached, std::memory_order_release);
  }
  return cached;
}

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

bool test_withhold() { return g_withhold.load(std::memory_order_relaxed) != 0; }

int device_ready() { return check_device(); }

namespace {
// Per-thread cache of encoded tensor maps: an eager forward encodes the same
// maps (same weight, same x buffer from the caching allocator) call after
// call. The key is every input of the encoding, so a hit is exactly what the
// driver would return.
struct MapKey {
  uint64_t base, dim[3], stride[2];
  uint32_t box[3];
  int rank, dtype, swizzle;
  bool operator==(const MapKey& o) const {
    return base == o.base && dim[0] == o.dim[0] && dim[1] == o.dim[1] && dim[2] == o.dim[2] &&
           stride[0] == o.stride[0] && stride[1] == o.stride[1] && box[0] == o.box[0] && box[1] == o.box[1] &&
           box[2] == o.box[2] && rank == o.rank && dtype == o.dtype && swizzle == o.swizzle;
  }
};
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kMapCache = 64;
thread_local MapEntry t_map_cache[kMapCache];

inline uint32_t map_slot(const MapKey& k) {
  uint64_t h = k.base * 0x9E3779B97F4A7C15ull ^ (k.dim[0] * 0xC2B2AE3D27D4EB4Full) ^ (k.dim[1] << 17) ^
               (k.dim[2] << 33) ^ (k.stride[0] << 7) ^ (k.stride[1] << 21) ^ ((uint64_t)k.box[0] << 40) ^
               ((uint64_t)k.box[1] << 24) ^ ((uint64_t)k.box[2] << 48) ^ ((uint64_t)k.dtype << 56) ^
               ((uint64_t)k.swizzle << 60) ^ ((uint64_t)k.rank << 62);
  h ^= h >> 29;
  return (uint32_t)(h % kMapCache);
}
}  // namespace

static CUresult encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, void* base, int rank,
                                  const uint64_t (&dim)[3], const uint64_t (&stride)[2], const uint32_t (&boxd)[3],
                                  CUtensorMapSwizzle swizzle) {
  const MapKey key{reinterpret_cast<uint64_t>(base), {dim[0], dim[1], dim[2]}, {stride[0], stride[1]},
                   {boxd[0], boxd[1], boxd[2]}, rank, (int)dtype, (int)swizzle};
  MapEntry& slot = t_map_cache[map_slot(key)];
  if (slot.valid && slot.key == key) {
    *map = slot.map;
    return CUDA_SUCCESS;
  }
  PFN_cuTensorMapEncodeTiled_v12000 encode = g_encode.load(std::memory_order_acquire);
  if (encode == nullptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    encode = g_encode.load(std::memory_order_relaxed);
    if (encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                           &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr) {
        return CUDA_ERROR_NOT_FOUND;
      }
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      g_encode.store(encode, std::memory_order_release);
    }
  }
  const cuuint64_t dims[3] = {dim[0], dim[1], dim[2]};
  const cuuint64_t strides[2] = {stride[0], stride[1]};
  const cuuint32_t box[3] = {boxd[0], boxd[1], boxd[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, dtype, (cuuint32_t)rank, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) {
    slot.key = key;
    slot.map = *map;
    slot.valid = true;
  }
  return r;
}

CUresult encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, void* base,
                              uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  return encode_tensor_map(map, dtype, base, 2, {inner, outer, 0}, {row_stride_bytes, 0}, {box_inner, box_outer, 0},
                           swizzle);
}

CUresult encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, void* base, uint64_t d0, uint64_t d1,
                              uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                              uint32_t b2, CUtensorMapSwizzle swizzle) {
  return encode_tensor_map(map, dtype, base, 3, {d0, d1, d2}, {stride1_bytes, stride2_bytes}, {b0, b1, b2}, swizzle);
}

}  // namespace nsq

using namespace nsq;

extern "C" {

const char* nsq_strerror(int code) {
  switch (code) {
    case NSQ_OK: return "ok";
    case NSQ_EINVAL: return "invalid argument (shape, size or dtype)";
    case NSQ_EALIGN: return "pointer or row stride not 16-byte aligned";
    case NSQ_ENOTSUP: return "unsupported device (needs sm_100) or unsupported shape";
    case NSQ_ECUDA: return "CUDA error while launching";
    case NSQ_EWORKSPACE: return "workspace missing or too small";
    case NSQ_EDEVICE_TIMEOUT: return "a bounded device-side wait ran out (kernel wound down)";
    default: return "unknown nsq error";
  }
}

int nsq_version(void) { return 100; }

int nsq_set_pdl(int enable) { return g_pdl.exchange(enable ? 1 : 0); }

int nsq_device_status(int* where, int* block) {
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  DevStatus st{};
  if (cudaMemcpyFromSymbol(&st, g_device_status, sizeof(st)) != cudaSuccess) return NSQ_ECUDA;
  if (where) *where = static_cast<int>(st.where);
  if (block) *block = static_cast<int>(st.block);
  return static_cast<int>(st.code);
}

int nsq_device_status_reset(void) {
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  DevStatus st{};
  return cudaMemcpyToSymbol(g_device_status, &st, sizeof(st)) == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

int nsq_set_wait_limit_ns(uint64_t ns) {
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  const unsigned long long v = ns;
  return cudaMemcpyToSymbol(g_device_status, &v, sizeof(v), offsetof(DevStatus, wait_limit_ns)) == cudaSuccess
             ? NSQ_OK
             : NSQ_ECUDA;
}

int nsq_test_withhold_weight_load(int enable) { return g_withhold.exchange(enable ? 1 : 0); }

int nsq_set_sm_reserve(int n) { return g_sm_reserve.exchange(n < 0 ? 0 : n); }

int nsq_awq_dequant(const int32_t* qweight, const uint16_t* scales, const uint16_t* zeros,
                    uint16_t* w_out, int64_t N, int64_t K, int64_t group_size, void* stream) {
  if (N < 0 || K <= 0 || group_size <= 0 || K % 8 != 0) return NSQ_EINVAL;
  if (N == 0) return NSQ_OK;
  if (!qweight || !scales || !zeros || !w_out) return NSQ_EINVAL;
  if (!aligned16(qweight) || !aligned16(w_out) || ((K * 2) % 16) != 0) return NSQ_EALIGN;
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  cudaError_t e = launch_awq_dequant(qweight, scales, zeros, w_out, N, K, group_size,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

int nsq_fp8_dequant(const uint8_t* weight_fp8, const float* weight_scale, void* w_out,
                    int out_dtype, int64_t N, int64_t K, void* stream) {
  if (N < 0 || K <= 0 || !valid_act_dtype(out_dtype)) return NSQ_EINVAL;
  if (N > INT64_MAX / K) return NSQ_EINVAL;
  if (N == 0) return NSQ_OK;
  if (!weight_fp8 || !weight_scale || !w_out) return NSQ_EINVAL;
  if (!aligned16(weight_fp8) || !aligned16(w_out)) return NSQ_EALIGN;
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  cudaError_t e = launch_fp8_dequant(weight_fp8, weight_scale, w_out, out_dtype, N * K,
                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

// Layers of 64-128 rows per SM: the tensor-core decode kernel (x as two
// narrow terms; FP8 A read from the TMA tile, AWQ A widened into tensor
// memory). Where it wins (B200, CUDA-graph chains of distinct weights,
// PDL; us, tensor core vs the best other kernel):
//   FP8, K >= 2048, every M: 4096 -> 14336 17.8 vs 20.7 (M = 1), 18.0 vs
//   23.7 (16), 23.4 vs 30.0 (32); 8192 -> 18944 32.5 vs 38.3 (1).
//   FP8, K < 2048 (896 -> 9472, 1024 -> 10000): within 0.5 us either way;
//   it takes 9..16 and 25..32 tokens.
//   AWQ, K >= 2048: 25..32 tokens (4096 -> 14336 32.0 vs 37.9); 17..24
//   and 9..16 tokens on weights of 64 M / 56 M+ elements (3584 -> 18944
//   at M = 16 21.7 vs 23.9, 4096 -> 12288 stays on the weight ring, 21.7
//   vs 22.9); up to 8 tokens only where the weight ring does not fit
//   (8192 -> 18944: 51 us, no ring plan).
//   33..64 tokens (with a workspace), K >= 2048: AWQ 4096 -> 14336 at M = 64
//   40.9 vs 47.3 (the one-CTA prefill kernel), 8192 -> 18944 76.4 vs 92.3;
//   FP8 4096 -> 14336 24.6 vs 25.8, 8192 -> 18944 40.5 vs 47.0; FP8 below
//   32 M weight elements (2048 -> 10000) is a tie and stays.
// pre: the call has the workspace for precomputed x terms (AWQ at 9..32
// tokens then wins from K >= 2048 on: 4096 -> 12288 at M = 16 19.4 vs 21.7).
static bool tc_decode_chosen(const LinearArgs& a, bool pre) {
  if (a.M > 64 || (a.fmt == 0 && a.group_size % 128 != 0)) return false;
  const int64_t kn = (int64_t)a.K * a.N;
  // 33..64 tokens run only with precomputed x terms (a workspace)
  const bool tc_wins =
      a.M > 32     ? pre && a.K >= 2048 && (a.fmt == 0 || kn >= ((int64_t)1 << 25))
      : a.fmt == 1 ? (a.K >= 2048 || (a.M > 8 && a.M <= 16) || a.M > 24)
      : a.K < 2048 ? false
      : a.M > 8    ? (pre || a.M > 24 || kn >= (a.M > 16 ? ((int64_t)1 << 26) : ((int64_t)7 << 23)))
                   : kn >= ((int64_t)1 << 27);
  // Layers of fewer than 64 rows per SM run on fewer CTAs of 64+ rows: a win
  // for K <= 4096 at up to 32 tokens (TP shards: AWQ 4096 -> 7168 at M = 16
  // 23.4 -> 18.3 us, FP8 at M = 32 20.9 -> 17.4 us), a loss at 64 tokens or
  // K = 8192 (FP8 8192 -> 7392 at M = 64 28.1 -> 38.6 us), and below 96 CTAs.
  const bool full_grid = (int64_t)a.N >= (int64_t)64 * num_sms();
  if (!full_grid && (a.N < 6144 || a.K > 4096 || a.M > 32)) return false;
  return tc_wins && decode_tc_rows(a) > 0;
}

static int linear_common(LinearArgs& a, cudaStream_t stream) {
  if (a.M == 0) return NSQ_OK;
  if (a.M <= kDecodeMaxM) {
    // Three decode kernels, chosen by shape (measured in CUDA-graph chains of
    // distinct weights on B200):
    //   * layers whose multi-wave plan needs more than two CTAs per SM: the
    //     persistent weight-ring kernel (up to 32 tokens);
    //   * short K (one 1 KB slice per row) with few tokens or few rows: the
    //     single-wave kernel;
    //   * otherwise the multi-wave kernel; the tensor-core GEMM when no
    //     decode plan fits.
    // 33..64 tokens on a large weight: the tcgen05 kernel with the dequantised
    // weight tile in tensor memory beats the mma.sync kernels, whose tensor
    // work grows with the token count (B200, CUDA-graph chains, AWQ at
    // M = 64: Llama-3-8B gate 140 -> 47 us, down 146 -> 47 us, q 52 -> 18 us,
    // 896 -> 9728 19.5 -> 12.6 us; 4096 -> 1024 stays faster on mma.sync)
    if (tc_decode_chosen(a, a.ws_bytes >= decode_tc_workspace_bytes(a) && ((uintptr_t)a.ws & 15) == 0)) {
      const int rc = run_decode_tc_linear(a, stream);
      if (rc != NSQ_ENOTSUP) return rc;
    }
    if (a.M > 32 && (int64_t)a.K * a.N >= ((int64_t)1 << 23)) {
      const TsPlan tp = prefill_ts_plan(a.fmt, a.M, a.K, a.N);
      if (tp.tokens_per_tile > 0) return run_prefill_ts_linear(a, tp, stream);
    }
    // Large weights at up to 32 tokens (FP8) or 17..32 tokens (AWQ): the
    // row-streaming kernel (B200, CUDA-graph chains: FP8 4096 -> 14336 at
    // M = 16 27.7 -> 20.7 us; AWQ at M = 32: 4096 -> 14336 45 -> 37 us,
    // 14336 -> 4096 90 -> 49 us, 4096 -> 4096 26 -> 17 us; AWQ at M <= 16
    // and the Qwen2.5-0.5B shapes stay on the kernels below). AWQ group sizes
    // 32 and 64 run here for every M <= 32.
    const bool small_group = a.fmt == 0 && a.group_size % 128 != 0;
    if (a.M <= 32 && (small_group ||((int64_t)a.K * a.N >= ((int64_t)1 << 24) && (a.fmt == 1 || a.M > 16)))) {
      const int rc = run_decode_rows_linear(a, stream);
      if (rc != NSQ_ENOTSUP || small_group) return rc;
    }
    if (small_group) {  // 33..64 tokens: the one-CTA tcgen05 kernel handles groups of 32 and 64
      const TsPlan tp = prefill_ts_plan(a.fmt, a.M, a.K, a.N);
      return run_prefill_ts_linear(a, tp.tokens_per_tile > 0 ? tp : TsPlan{64, 1}, stream);
    }
    const int ctas = decode_linear_ctas(a);
    if (ctas < 0 || ctas > 2 * num_sms()) {
      int rc = run_decode_stream_linear(a, stream);
      if (rc != NSQ_ENOTSUP) return rc;
      // no weight-ring plan (AWQ 8192 -> 29568 at M <= 16): the row-streaming
      // kernel, not the multi-wave one (74 vs 122 us, B200)
      if (a.M <= 32) {
        rc = run_decode_rows_linear(a, stream);
        if (rc != NSQ_ENOTSUP) return rc;
      }
    }
    if (a.K <= 1024 && (a.M <= 8 || a.N <= 1024)) {
      const int rc = run_decode_wave_linear(a, stream);
      if (rc != NSQ_ENOTSUP) return rc;
    }
    int rc = run_decode_linear(a, stream);
    if (rc != NSQ_ENOTSUP) return rc;
    rc = run_decode_wave_linear(a, stream);
    if (rc != NSQ_ENOTSUP) return rc;
  }
  // Prefill: the weight tile dequantised into tensor memory -- one CTA per
  // 128 rows (K split over a cluster when the tiles are few) for problems
  // that 256 x 256 pair tiles would leave mostly idle, CTA pairs otherwise.
  // Groups of 32 columns (two per 64-column k-block) take the one-CTA kernel.
  const TsPlan tp = prefill_ts_plan(a.fmt, a.M, a.K, a.N);
  if (tp.tokens_per_tile > 0) return run_prefill_ts_linear(a, tp, stream);
  if (a.fmt == 0 && a.group_size < 64) return run_prefill_ts_linear(a, TsPlan{128, 1}, stream);
  return run_prefill_ts2_linear(a, stream);
}

size_t nsq_linear_workspace_size(int quant, int64_t M, int64_t K, int64_t N, int64_t group_size) {
  if (M <= 0 || K <= 0 || N <= 0 || M > kIntMax || K > kIntMax || N > kIntMax || (quant != 0 && quant != 1)) return 0;
  LinearArgs a{};
  a.fmt = quant;
  a.M = (int)M;
  a.K = (int)K;
  a.N = (int)N;
  a.group_size = quant == 0 ? (int)group_size : 0;
  if (quant == 0 && (group_size <= 0 || group_size > kIntMax)) return 0;
  return tc_decode_chosen(a, true) ? decode_tc_workspace_bytes(a) : 0;
}

int nsq_awq_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N,
                   const int32_t* qweight, const uint16_t* scales, const uint16_t* zeros,
                   int64_t group_size, const void* bias, int bias_dtype, void* y,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || M > kIntMax || K > kIntMax || N > kIntMax) return NSQ_EINVAL;
  if (!valid_act_dtype(x_dtype) || !valid_bias_dtype(bias_dtype)) return NSQ_EINVAL;
  if ((bias_dtype == NSQ_DTYPE_NONE) != (bias == nullptr)) return NSQ_EINVAL;
  // groups of 32, 64 or any multiple of 128 columns (the reference accepts any size)
  if (!(group_size == 32 || group_size == 64 || (group_size > 0 && group_size % 128 == 0))) return NSQ_ENOTSUP;
  if (K % 32 != 0) return NSQ_ENOTSUP;  // qweight rows must be a 16-byte multiple for TMA
  if (M == 0) return NSQ_OK;
  if (!x || !qweight || !scales || !zeros || !y) return NSQ_EINVAL;
  if (!aligned16(x) || !aligned16(y) || !aligned16(qweight)) return NSQ_EALIGN;
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  LinearArgs a{};
  a.fmt = 0;
  a.x = x;
  a.x_bf16 = x_dtype == NSQ_DTYPE_BF16;
  a.M = (int)M;
  a.K = (int)K;
  a.N = (int)N;
  a.wq = qweight;
  a.scales = scales;
  a.zeros = zeros;
  a.group_size = (int)group_size;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.y = y;
  a.ws = workspace;
  a.ws_bytes = workspace ? workspace_bytes : 0;
  return linear_common(a, static_cast<cudaStream_t>(stream));
}

int nsq_fp8_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N,
                   const uint8_t* weight_fp8, const float* weight_scale, const void* bias,
                   int bias_dtype, void* y, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (M < 0 || K <= 0 || N <= 0 || M > kIntMax || K > kIntMax || N > kIntMax) return NSQ_EINVAL;
  if (!valid_act_dtype(x_dtype) || !valid_bias_dtype(bias_dtype)) return NSQ_EINVAL;
  if ((bias_dtype == NSQ_DTYPE_NONE) != (bias == nullptr)) return NSQ_EINVAL;
  if (K % 16 != 0) return NSQ_ENOTSUP;  // weight rows must be a 16-byte multiple for TMA
  if (M == 0) return NSQ_OK;
  if (!x || !weight_fp8 || !weight_scale || !y) return NSQ_EINVAL;
  if (!aligned16(x) || !aligned16(y) || !aligned16(weight_fp8)) return NSQ_EALIGN;
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  LinearArgs a{};
  a.fmt = 1;
  a.x = x;
  a.x_bf16 = x_dtype == NSQ_DTYPE_BF16;
  a.M = (int)M;
  a.K = (int)K;
  a.N = (int)N;
  a.wq = weight_fp8;
  a.wscale = weight_scale;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.y = y;
  a.ws = workspace;
  a.ws_bytes = workspace ? workspace_bytes : 0;
  return linear_common(a, static_cast<cudaStream_t>(stream));
}

// Fused projections over weights that share x (M <= 32, the decode batches):
// mode 0 writes weight i's outputs to y columns [sum n_<i, + n_i); mode 1
// takes (gate, up) and writes SiLU(x gate^T) * (x up^T).
static int fused_common(int fmt, int mode, const void* x, int x_dtype, int64_t M, int64_t K, int nw,
                        const void* const* w, const uint16_t* const* scales, const uint16_t* const* zeros,
                        const float* const* wscales, const int64_t* ns, int64_t group_size,
                        const void* const* biases, int bias_dtype, void* y, int64_t ldy, void* stream) {
  if (nw < 1 || nw > 3 || (mode == 1 && nw != 2)) return NSQ_EINVAL;
  if (M < 0 || K <= 0 || M > kIntMax || K > kIntMax || ldy <= 0 || ldy > kIntMax) return NSQ_EINVAL;
  if (!valid_act_dtype(x_dtype) || !valid_bias_dtype(bias_dtype)) return NSQ_EINVAL;
  if (!w || !ns || (fmt == 0 && (!scales || !zeros)) || (fmt == 1 && !wscales)) return NSQ_EINVAL;
  if ((bias_dtype == NSQ_DTYPE_NONE) != (biases == nullptr)) return NSQ_EINVAL;
  if (fmt == 0 && !(group_size == 32 || group_size == 64 || (group_size > 0 && group_size % 128 == 0))) {
    return NSQ_ENOTSUP;
  }
  if (K % (fmt == 0 ? 32 : 16) != 0) return NSQ_ENOTSUP;  // 16-byte row pitch of the weights for TMA
  if (M > 32) return NSQ_ENOTSUP;                         // decode batches only: call the single linears
  int64_t cols = 0;
  for (int i = 0; i < nw; ++i) {
    if (ns[i] <= 0 || ns[i] > kIntMax || !w[i]) return NSQ_EINVAL;
    if (!aligned16(w[i])) return NSQ_EALIGN;
    if (fmt == 0 && (!scales[i] || !zeros[i])) return NSQ_EINVAL;
    if (fmt == 1 && !wscales[i]) return NSQ_EINVAL;
    if (mode == 1 && ns[i] != ns[0]) return NSQ_EINVAL;
    cols += mode == 0 ? ns[i] : 0;
  }
  if (mode == 1) cols = ns[0];
  if (cols > ldy) return NSQ_EINVAL;
  if (M == 0) return NSQ_OK;
  if (!x || !y) return NSQ_EINVAL;
  if (!aligned16(x) || !aligned16(y)) return NSQ_EALIGN;
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  RowsLaunch L{};
  L.fmt = fmt;
  L.x = x;
  L.x_bf16 = x_dtype == NSQ_DTYPE_BF16;
  L.M = (int)M;
  L.K = (int)K;
  L.y = y;
  L.ldy = (int)ldy;
  L.group_size = fmt == 0 ? (int)group_size : 0;
  L.bias_dtype = bias_dtype;
  L.mode = mode;
  L.nw = nw;
  int64_t col = 0;
  for (int i = 0; i < nw; ++i) {
    L.w[i] = RowsWeight{w[i], fmt == 0 ? scales[i] : nullptr, fmt == 0 ? zeros[i] : nullptr,
                        fmt == 1 ? wscales[i] : nullptr, biases ? biases[i] : nullptr, (int)ns[i],
                        mode == 0 ? (int)col : 0};
    col += ns[i];
  }
  return run_decode_rows(L, static_cast<cudaStream_t>(stream));
}

int nsq_awq_linear_multi(const void* x, int x_dtype, int64_t M, int64_t K, int nw, const int32_t* const* qweights,
                         const uint16_t* const* scales, const uint16_t* const* zeros, const int64_t* ns,
                         int64_t group_size, const void* const* biases, int bias_dtype, void* y, int64_t ldy,
                         void* stream) {
  return fused_common(0, 0, x, x_dtype, M, K, nw, reinterpret_cast<const void* const*>(qweights), scales, zeros,
                      nullptr, ns, group_size, biases, bias_dtype, y, ldy, stream);
}

int nsq_fp8_linear_multi(const void* x, int x_dtype, int64_t M, int64_t K, int nw, const uint8_t* const* weights,
                         const float* const* weight_scales, const int64_t* ns, const void* const* biases,
                         int bias_dtype, void* y, int64_t ldy, void* stream) {
  return fused_common(1, 0, x, x_dtype, M, K, nw, reinterpret_cast<const void* const*>(weights), nullptr, nullptr,
                      weight_scales, ns, 0, biases, bias_dtype, y, ldy, stream);
}

int nsq_awq_gate_up_silu(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N, const int32_t* qweight_gate,
                         const uint16_t* scales_gate, const uint16_t* zeros_gate, const int32_t* qweight_up,
                         const uint16_t* scales_up, const uint16_t* zeros_up, int64_t group_size, void* y,
                         void* stream) {
  const int32_t* qw[2] = {qweight_gate, qweight_up};
  const uint16_t* sc[2] = {scales_gate, scales_up};
  const uint16_t* zr[2] = {zeros_gate, zeros_up};
  const int64_t ns[2] = {N, N};
  return fused_common(0, 1, x, x_dtype, M, K, 2, reinterpret_cast<const void* const*>(qw), sc, zr, nullptr, ns,
                      group_size, nullptr, NSQ_DTYPE_NONE, y, N, stream);
}

int nsq_fp8_gate_up_silu(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N, const uint8_t* weight_gate,
                         const float* scale_gate, const uint8_t* weight_up, const float* scale_up, void* y,
                         void* stream) {
  const uint8_t* wt[2] = {weight_gate, weight_up};
  const float* ws[2] = {scale_gate, scale_up};
  const int64_t ns[2] = {N, N};
  return fused_common(1, 1, x, x_dtype, M, K, 2, reinterpret_cast<const void* const*>(wt), nullptr, nullptr, ws, ns,
                      0, nullptr, NSQ_DTYPE_NONE, y, N, stream);
}

int nsq_awq_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int64_t group_size,
                     int32_t* qweight, uint16_t* scales, uint16_t* zeros, void* stream) {
  if (N < 0 || K < 8 || group_size <= 0) return NSQ_EINVAL;
  if (!(w_dtype == NSQ_DTYPE_F16 || w_dtype == NSQ_DTYPE_BF16 || w_dtype == NSQ_DTYPE_F32)) {
    return NSQ_EINVAL;
  }
  if (N == 0) return NSQ_OK;
  if (!w || !qweight || !scales || !zeros) return NSQ_EINVAL;
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  cudaError_t e = launch_awq_quantize(w, w_dtype, N, K, group_size, qweight, scales, zeros,
                                      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

int nsq_awq_from_autoawq(const int32_t* qweight_kn8, const int32_t* qzeros_gn8, const uint16_t* scales_gn,
                         int64_t K, int64_t N, int64_t group_size, int32_t* qweight, uint16_t* scales,
                         uint16_t* zeros, void* stream) {
  if (K <= 0 || N <= 0 || group_size <= 0 || K % 8 != 0 || N % 8 != 0 || K % group_size != 0) return NSQ_EINVAL;
  if (K > kIntMax || N > kIntMax) return NSQ_EINVAL;
  if (!qweight_kn8 || !qzeros_gn8 || !scales_gn || !qweight || !scales || !zeros) return NSQ_EINVAL;
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  cudaError_t e = launch_awq_from_autoawq(qweight_kn8, qzeros_gn8, scales_gn, K, N, group_size, qweight, scales,
                                          zeros, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

size_t nsq_fp8_quantize_workspace_size(int64_t N, int64_t K) {
  (void)N;
  (void)K;
  return 256;
}

int nsq_fp8_quantize(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* weight_fp8,
                     float* weight_scale, void* workspace, size_t workspace_bytes, void* stream) {
  if (N < 0 || K < 0) return NSQ_EINVAL;
  if (K > 0 && N > INT64_MAX / K) return NSQ_EINVAL;  // N * K must not overflow
  if (!(w_dtype == NSQ_DTYPE_F16 || w_dtype == NSQ_DTYPE_BF16 || w_dtype == NSQ_DTYPE_F32)) {
    return NSQ_EINVAL;
  }
  if (!weight_scale || (N * K > 0 && (!w || !weight_fp8))) return NSQ_EINVAL;
  if (!workspace || workspace_bytes < nsq_fp8_quantize_workspace_size(N, K)) return NSQ_EWORKSPACE;
  int rc = check_device();
  if (rc != NSQ_OK) return rc;
  cudaError_t e = launch_fp8_quantize(w, w_dtype, N * K, weight_fp8, weight_scale, workspace,
                                      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // extern "C"
