// Allocation-free variant of nsq_fp8_quantize.
//
// Some callers cannot allocate device memory at the moment they quantise a
// weight to FP8: code that runs while a CUDA stream capture is active in
// global mode (cudaMalloc is not allowed then and would invalidate the
// capture), serving engines that hand nearly all HBM to a pre-reserved pool
// (the KV cache) at start-up and keep no allocator for later requests, and
// programs that call the C ABI directly without a device allocator of their
// own. nsq_fp8_quantize needs a small workspace for its absmax reduction;
// this entry point takes that workspace from a file-scope device array
// instead, so it allocates nothing.
//
// Scratch: kNoAllocScratchBytes (256 bytes), a static __device__ array that
// every GPU which loads the library keeps until the process exits. All calls
// share it and it keeps whatever the previous call left there, so each call
// clears the absmax word first (cudaMemsetAsync: stream-ordered, no
// allocation). Calls that overlap on the GPU (for example on two streams at
// once) race on the shared scratch and must be serialised by the caller.
//
// The device address of the array is looked up once per device with that
// device current (cudaGetSymbolAddress); the first call on a device does this
// set-up, so make that first call before any stream capture begins.
#include <atomic>
#include <mutex>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr size_t kNoAllocScratchBytes = 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDev = 64;
std::mutex g_noalloc_mu;
std::atomic<void*> g_noalloc_addr[kMaxDev];  // zero-initialised (static storage)

// Device address of g_noalloc_scratch on the current device (set up once per
// device), or nullptr if the runtime refuses.
void* noalloc_scratch_on_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  void* cached = g_noalloc_addr[dev].load(std::memory_order_acquire);
  if (cached != nullptr) return cached;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  cached = g_noalloc_addr[dev].load(std::memory_order_relaxed);
  if (cached == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return nullptr;
    g_noalloc_addr[dev].store(p, std::memory_order_release);
    cached = p;
  }
  return cached;
}

}  // namespace

}  // namespace nsq

using namespace nsq;

extern "C" int nsq_fp8_quantize_noalloc(const void* w, int w_dtype, int64_t N, int64_t K,
                                        uint8_t* weight_fp8, float* weight_scale, void* stream) {
  if (N < 0 || K < 0) return NSQ_EINVAL;
  if (K > 0 && N > INT64_MAX / K) return NSQ_EINVAL;  // N * K must not overflow
  if (!(w_dtype == NSQ_DTYPE_F16 || w_dtype == NSQ_DTYPE_BF16 || w_dtype == NSQ_DTYPE_F32)) {
    return NSQ_EINVAL;
  }
  if (!weight_scale || (N * K > 0 && (!w || !weight_fp8))) return NSQ_EINVAL;
  // the static scratch must hold what the workspace-taking variant would need
  if (nsq_fp8_quantize_workspace_size(N, K) > kNoAllocScratchBytes) return NSQ_EWORKSPACE;
  const int rc = device_ready();
  if (rc != NSQ_OK) return rc;
  void* scratch = noalloc_scratch_on_current_device();
  if (scratch == nullptr) return NSQ_ECUDA;
  cudaError_t e = launch_fp8_quantize(w, w_dtype, N * K, weight_fp8, weight_scale, scratch,
                                      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}
