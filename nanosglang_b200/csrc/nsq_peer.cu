// One-shot all-reduce (sum) over NVLink peer memory, for the small row-
// parallel outputs of tensor-parallel decode (nano_sglang/distributed/
// tensor_parallel.py:134-140 reduces them with all_reduce(SUM) after o_proj
// and down_proj; 64 of them per Llama-3-8B decode step, ~0.5 MB each).
//
// Every rank owns one workspace (cudaMalloc by the caller) whose CUDA IPC
// handle the other ranks open, so every rank addresses every workspace. A
// workspace holds, for each of two parities, one slot per rank and a flag
// per (source rank, CTA). A call with epoch e (parity e & 1):
//   1. each CTA stores its chunk of this rank's partial into slot `rank` of
//      every rank's workspace (plain 16-byte stores; NVLink for the peers);
//   2. its thread 0 fences at system scope and writes e into flag
//      (rank, cta) of every rank's workspace (release stores);
//   3. it waits (bounded) until flags (q, cta) of its own workspace reach e
//      for every rank q (acquire loads), then
//   4. the CTA sums the slots of its chunk in rank order 0..world-1 in fp32
//      and writes the result: every rank computes the same sum in the same
//      order, so all ranks hold bit-identical outputs.
// Parities alternate between calls: a rank writes epoch e + 2 into a peer's
// slot only after it saw that peer's flag of epoch e + 1, which the peer
// writes after its epoch-e kernel (which read the slot) completed. The epoch
// lives in device memory and advances by one per call (the last CTA to
// finish bumps it), so calls can be captured in CUDA graphs. No multimem, no
// TMA: plain loads and stores to peer memory.
#include <atomic>
#include <cstring>

#include "nsq_common.cuh"
#include "nsq_internal.h"

namespace nsq {

namespace {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerThreads = 512;
constexpr int kPeerMaxCtas = 64;

// Workspace layout (bytes from the base), identical on every rank:
//   [0, 64)                      control: epoch (u64), finished-CTA count (u32)
//   [64, 64 + 2*R*C*8)           flags[parity][src rank][cta] (u64)
//   [kDataOff, + 2*R*max_bytes)  slots[parity][src rank] (max_bytes each)
constexpr size_t kFlagsOff = 64;
__host__ __device__ constexpr size_t peer_data_off() {
  return kFlagsOff + (size_t)2 * kPeerMaxRanks * kPeerMaxCtas * 8;
}

struct PeerParams {
  uint8_t* bases[kPeerMaxRanks];  // every rank's workspace, as mapped in this process
  int rank, world;
  const void* in;
  void* out;
  int64_t n;         // elements
  int dtype;         // NSQ_DTYPE_BF16 / F16 / F32
  int64_t max_bytes; // slot size
  DevStatus* status;
};

__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void add8(float (&a)[8], const uint4& v, int dtype) {
  const uint32_t r[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (dtype == NSQ_DTYPE_BF16) {
      a[2 * i] += __uint_as_float(r[i] << 16);
      a[2 * i + 1] += __uint_as_float(r[i] & 0xFFFF0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r[i]));
      a[2 * i] += f.x;
      a[2 * i + 1] += f.y;
    }
  }
}
__device__ __forceinline__ uint4 pack8(const float (&a)[8], int dtype) {
  uint32_t r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (dtype == NSQ_DTYPE_BF16) {
      __nv_bfloat162 b = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
      r[i] = *reinterpret_cast<uint32_t*>(&b);
    } else {
      __half2 h = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
      r[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_kernel(const PeerParams p) {
  __shared__ uint64_t s_epoch;
  __shared__ int s_ok;
  uint8_t* own = p.bases[p.rank];
  uint64_t* ctl = reinterpret_cast<uint64_t*>(own);
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint64_t*>(ctl) + 1;
    s_ok = 1;
  }
  __syncthreads();
  const uint64_t epoch = s_epoch;
  const int par = (int)(epoch & 1);
  const int esize = p.dtype == NSQ_DTYPE_F32 ? 4 : 2;
  const int64_t bytes = p.n * esize;
  // this CTA's byte range, in 16-byte units
  const int64_t units = bytes / 16;
  const int64_t per = (units + gridDim.x - 1) / gridDim.x;
  const int64_t u0 = blockIdx.x * per;
  const int64_t u1 = u0 + per < units ? u0 + per : units;
  const size_t slot_off = peer_data_off() + ((size_t)par * p.world + p.rank) * (size_t)p.max_bytes;

  // 1. this rank's partial into slot `rank` of every workspace
  const uint4* src = reinterpret_cast<const uint4*>(p.in);
  for (int64_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
    const uint4 v = src[u];
#pragma unroll 1
    for (int q = 0; q < p.world; ++q) {
      reinterpret_cast<uint4*>(p.bases[q] + slot_off)[u] = v;
    }
  }
  __syncthreads();
  // 2. publish: every peer's flag (rank, cta) of this parity = epoch
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < p.world; ++q) {
      uint64_t* f = reinterpret_cast<uint64_t*>(p.bases[q] + kFlagsOff) +
                    ((size_t)par * kPeerMaxRanks + p.rank) * kPeerMaxCtas + blockIdx.x;
      st_release_sys_u64(f, epoch);
    }
    // 3. wait for every rank's chunk (bounded)
    const unsigned long long t0 = globaltimer_ns();
    unsigned long long limit = kWaitTimeoutNs;
    if (p.status != nullptr) {
      const unsigned long long l = *reinterpret_cast<volatile unsigned long long*>(&p.status->wait_limit_ns);
      if (l != 0ull) limit = l;
    }
    for (int q = 0; q < p.world && s_ok; ++q) {
      const uint64_t* f = reinterpret_cast<const uint64_t*>(own + kFlagsOff) +
                          ((size_t)par * kPeerMaxRanks + q) * kPeerMaxCtas + blockIdx.x;
      while (ld_acquire_sys_u64(f) < epoch) {
        if (globaltimer_ns() - t0 > limit) {
          if (p.status != nullptr && atomicCAS(&p.status->code, 0u, (unsigned)NSQ_EDEVICE_TIMEOUT) == 0u) {
            p.status->where = 90;
            p.status->block = blockIdx.x;
          }
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. sum the slots in rank order (the same order on every rank)
  if (s_ok) {
    const size_t base_off = peer_data_off() + (size_t)par * p.world * (size_t)p.max_bytes;
    uint4* dst = reinterpret_cast<uint4*>(p.out);
    if (p.dtype == NSQ_DTYPE_F32) {
      for (int64_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < p.world; ++q) {
          const float4 v = reinterpret_cast<const float4*>(own + base_off + (size_t)q * p.max_bytes)[u];
          a.x += v.x;
          a.y += v.y;
          a.z += v.z;
          a.w += v.w;
        }
        reinterpret_cast<float4*>(p.out)[u] = a;
      }
    } else {
      for (int64_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < p.world; ++q) {
          add8(a, reinterpret_cast<const uint4*>(own + base_off + (size_t)q * p.max_bytes)[u], p.dtype);
        }
        dst[u] = pack8(a, p.dtype);
      }
    }
  }
  // the last CTA to finish advances the epoch (every CTA read it at its start)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int* done = reinterpret_cast<unsigned int*>(own + 8);
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      *reinterpret_cast<volatile uint64_t*>(ctl) = epoch;
      __threadfence();
    }
  }
}

}  // namespace

}  // namespace nsq

using namespace nsq;

extern "C" {

size_t nsq_peer_workspace_size(int world, int64_t max_bytes) {
  if (world < 1 || world > kPeerMaxRanks || max_bytes <= 0) return 0;
  const int64_t mb = (max_bytes + 15) / 16 * 16;
  return peer_data_off() + (size_t)2 * world * (size_t)mb;
}

int nsq_peer_workspace_alloc(size_t bytes, void** ptr_out) {
  if (bytes == 0 || !ptr_out) return NSQ_EINVAL;
  const int rc = device_ready();
  if (rc != NSQ_OK) return rc;
  void* p = nullptr;
  // a dedicated allocation, so its IPC handle maps exactly this buffer
  if (cudaMalloc(&p, bytes) != cudaSuccess) return NSQ_ECUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return NSQ_ECUDA;
  }
  *ptr_out = p;
  return NSQ_OK;
}

int nsq_peer_workspace_free(void* ptr) {
  if (!ptr) return NSQ_EINVAL;
  return cudaFree(ptr) == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

int nsq_ipc_handle(const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return NSQ_EINVAL;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return NSQ_ECUDA;
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle_out, &h, sizeof(h));
  return NSQ_OK;
}

int nsq_ipc_open(const void* handle, void** dev_ptr_out) {
  if (!handle || !dev_ptr_out) return NSQ_EINVAL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return NSQ_ECUDA;
  *dev_ptr_out = p;
  return NSQ_OK;
}

int nsq_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return NSQ_EINVAL;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

int nsq_peer_allreduce(void* const* workspaces, int rank, int world, int64_t max_bytes, const void* in, void* out,
                       int64_t n, int dtype, void* stream) {
  if (!workspaces || world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world) return NSQ_EINVAL;
  if (!(dtype == NSQ_DTYPE_BF16 || dtype == NSQ_DTYPE_F16 || dtype == NSQ_DTYPE_F32)) return NSQ_EINVAL;
  if (n < 0 || max_bytes <= 0 || max_bytes % 16 != 0) return NSQ_EINVAL;
  const int64_t esize = dtype == NSQ_DTYPE_F32 ? 4 : 2;
  if (n * esize > max_bytes) return NSQ_EWORKSPACE;
  if ((n * esize) % 16 != 0) return NSQ_EALIGN;  // whole 16-byte units
  if (n == 0) return NSQ_OK;
  if (!in || !out) return NSQ_EINVAL;
  if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) return NSQ_EALIGN;
  PeerParams p{};
  for (int q = 0; q < world; ++q) {
    if (!workspaces[q] || (reinterpret_cast<uintptr_t>(workspaces[q]) & 15u)) return NSQ_EALIGN;
    p.bases[q] = static_cast<uint8_t*>(workspaces[q]);
  }
  const int rc = device_ready();
  if (rc != NSQ_OK) return rc;
  p.rank = rank;
  p.world = world;
  p.in = in;
  p.out = out;
  p.n = n;
  p.dtype = dtype;
  p.max_bytes = max_bytes;
  p.status = device_status_ptr();
  const int64_t units = n * esize / 16;
  int grid = (int)((units + kPeerThreads * 2 - 1) / (kPeerThreads * 2));  // ~2 units per thread
  if (grid < 1) grid = 1;
  if (grid > kPeerMaxCtas) grid = kPeerMaxCtas;
  peer_allreduce_kernel<<<grid, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? NSQ_OK : NSQ_ECUDA;
}

}  // extern "C"
