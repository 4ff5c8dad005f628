/*
 * nsq.h -- C ABI of libnsq, the B200 (sm_100a) quantized-linear library.
 *
 * Each entry point replaces one operation of nanoSGLang's quantized-linear
 * path (xiehuanyi/nanoSGLang, nano_sglang/decode/quantization.py) and takes
 * the reference's own buffer layouts, unchanged:
 *   AWQ: qweight int32 [N, K/8] (nibble i of word j = column 8j+i),
 *        scales fp16 [N, G], zeros fp16 [N, G], G = ceil(K / group_size).
 *   FP8: weight_fp8 e4m3 [N, K] row-major, weight_scale one fp32 (device).
 * x is row-major [M, K], y is row-major [M, N], both in the activation dtype.
 *
 * Conventions
 *   - All pointers are device pointers; `stream` is a cudaStream_t (may be 0).
 *   - Every call is stream-ordered and asynchronous; nothing allocates or
 *     frees device memory, nothing synchronises the host, so every call can
 *     be captured in a CUDA graph. Workspaces belong to the caller.
 *   - Shapes, dtypes and alignment are validated on the host before any
 *     launch; a violation returns an error code and launches nothing.
 *   - Kernels never trap: a bounded on-device wait that runs out records
 *     NSQ_EDEVICE_TIMEOUT in the library's device status word, readable with
 *     nsq_device_status().
 */
#ifndef NSQ_H_
#define NSQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types of activations / bias */
#define NSQ_DTYPE_NONE (-1)
#define NSQ_DTYPE_F16 0
#define NSQ_DTYPE_BF16 1
#define NSQ_DTYPE_F32 2

/* return codes */
#define NSQ_OK 0
#define NSQ_EINVAL 1          /* bad shape, size or argument */
#define NSQ_EALIGN 2          /* pointer or stride not aligned as required */
#define NSQ_ENOTSUP 3         /* device is not sm_100 / shape not supported */
#define NSQ_ECUDA 4           /* CUDA runtime/driver error at launch */
#define NSQ_EWORKSPACE 5      /* workspace missing or too small */
#define NSQ_EDEVICE_TIMEOUT 6 /* a bounded device-side wait ran out */

/* Human-readable text for a return code (static storage). */
const char* nsq_strerror(int code);

/* Library version: major * 10000 + minor * 100 + patch. */
int nsq_version(void);

/* Device status word: 0 when no kernel has reported a problem since the last
 * reset, else an NSQ_E* code. `where`/`block` (may be NULL) receive the tag
 * of the wait that gave up and the block index. Synchronises the device. */
int nsq_device_status(int* where, int* block);
int nsq_device_status_reset(void);

/*
 * AWQ unpack + dequantise, bit-exact:
 *   w_out[n, k] = fp16( fp16(q[n,k] - zeros[n, k/gs]) * scales[n, k/gs] )
 * Replaces AWQLinear._dequantize (quantization.py:126-148).
 * Requires K % 8 == 0 (the reference raises otherwise), group_size >= 1,
 * qweight/w_out 16-byte aligned.
 */
int nsq_awq_dequant(const int32_t* qweight, const uint16_t* scales, const uint16_t* zeros,
                    uint16_t* w_out, int64_t N, int64_t K, int64_t group_size, void* stream);

/*
 * Workspace bytes with which nsq_awq_linear (quant 0) / nsq_fp8_linear
 * (quant 1) of this shape runs its faster form: 0 when the call needs none.
 * The workspace holds x converted for the tensor-core decode kernel (two
 * narrow terms and a scale per token and 128-column block), written by a
 * small kernel the call launches ahead of the linear. No counterpart in the
 * reference.
 */
size_t nsq_linear_workspace_size(int quant, int64_t M, int64_t K, int64_t N, int64_t group_size);

/*
 * AWQ W4A16 linear:  y = x @ dequant(qweight, scales, zeros)^T + bias.
 * Replaces AWQLinear.forward (quantization.py:150-152). x_dtype is F16 or
 * BF16 (y has the same dtype; the reference accepts fp16 only and raises on
 * bf16). bias_dtype is NONE/F16/BF16/F32. Requires K % 32 == 0,
 * group_size % 128 == 0, x/y/qweight 16-byte aligned.
 * M <= 64 runs a decode kernel, larger M the tcgen05 GEMM. Workspace may be
 * NULL; with nsq_linear_workspace_size() bytes (16-byte aligned, stream-
 * ordered like y) the tensor-core decode kernel takes x in a precomputed form
 * instead of every CTA converting it.
 */
int nsq_awq_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N,
                   const int32_t* qweight, const uint16_t* scales, const uint16_t* zeros,
                   int64_t group_size, const void* bias, int bias_dtype, void* y,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * FP8 W8A16 linear:  y = x @ (float(weight_fp8) * weight_scale)^T + bias.
 * Replaces FP8Linear.forward (quantization.py:49-52). weight_scale points to
 * ONE fp32 on the device (the reference's 0-dim / [1] buffer) and is read on
 * the device, never on the host. Requires K % 16 == 0, x/y/weight 16-byte
 * aligned. Workspace: as for nsq_awq_linear.
 */
int nsq_fp8_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N,
                   const uint8_t* weight_fp8, const float* weight_scale, const void* bias,
                   int bias_dtype, void* y, void* workspace, size_t workspace_bytes,
                   void* stream);

/*
 * FP8 dequantise, bit-exact with the reference's weight materialisation
 * `weight_fp8.to(dtype) * weight_scale` (quantization.py:51):
 *   w_out[n, k] = round_to_out_dtype(float(e4m3) * weight_scale).
 * out_dtype is F16 or BF16.
 */
int nsq_fp8_dequant(const uint8_t* weight_fp8, const float* weight_scale, void* w_out,
                    int out_dtype, int64_t N, int64_t K, void* stream);

/*
 * Fused projections for decode batches (M <= 32): one launch over nw = 1..3
 * weights of one format that read the same x, e.g. q/k/v, whose reference
 * call sites are three separate linears (nano_sglang/model/causal_lm.py:
 * 295-297). Weight i (its own buffers in the reference layout, ns[i] output
 * rows, optional bias biases[i]) writes y columns [n_0 + .. + n_{i-1}, + n_i)
 * of y [M, ldy]; the result equals the separate AWQLinear / FP8Linear
 * forwards. Streams every weight row once (row-streaming kernel).
 * M > 32 returns NSQ_ENOTSUP: call the single linears.
 */
int nsq_awq_linear_multi(const void* x, int x_dtype, int64_t M, int64_t K, int nw, const int32_t* const* qweights,
                         const uint16_t* const* scales, const uint16_t* const* zeros, const int64_t* ns,
                         int64_t group_size, const void* const* biases, int bias_dtype, void* y, int64_t ldy,
                         void* stream);
int nsq_fp8_linear_multi(const void* x, int x_dtype, int64_t M, int64_t K, int nw, const uint8_t* const* weights,
                         const float* const* weight_scales, const int64_t* ns, const void* const* biases,
                         int bias_dtype, void* y, int64_t ldy, void* stream);

/*
 * Fused gate/up projection with the SwiGLU activation for decode batches
 * (M <= 32): y [M, N] = SiLU(x gate^T) * (x up^T) in one launch, the inner
 * expression of MLP.forward (nano_sglang/model/causal_lm.py:482) computed in
 * fp32 and rounded once. gate and up are two separate weights [N, K] in the
 * reference layout (no concatenated copy). M > 32 returns NSQ_ENOTSUP.
 */
int nsq_awq_gate_up_silu(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N, const int32_t* qweight_gate,
                         const uint16_t* scales_gate, const uint16_t* zeros_gate, const int32_t* qweight_up,
                         const uint16_t* scales_up, const uint16_t* zeros_up, int64_t group_size, void* y,
                         void* stream);
int nsq_fp8_gate_up_silu(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N, const uint8_t* weight_gate,
                         const float* scale_gate, const uint8_t* weight_up, const float* scale_up, void* y,
                         void* stream);

/*
 * AWQ quantiser, bit-exact with AWQLinear.from_linear/*
 * AWQ quantiser, bit-exact with AWQLinear.from_linear
 * (quantization.py:154-194): per (row, group) asymmetric min/max int4,
 * sequential nibble packing, columns past 8*(K/8) dropped. w is row-major
 * [N, K] in w_dtype (F16/BF16/F32). Writes qweight [N, K/8], scales/zeros
 * [N, G] fp16. Requires K >= 8.
 */
int nsq_awq_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int64_t group_size,
                     int32_t* qweight, uint16_t* scales, uint16_t* zeros, void* stream);

/*
 * AutoAWQ checkpoint layer -> the reference layout, bit-exact repack (no
 * arithmetic on the values). The reference's module docstring names AutoAWQ
 * checkpoints (quantization.py:7) but ships no loader; this is that loader's
 * device step. Input, AutoAWQ's GEMM format for in_features K, out_features N,
 * G = K / group_size: qweight_kn8 int32 [K, N/8] and qzeros_gn8 int32
 * [G, N/8], eight int4 values per word along N with nibble i holding column
 * 8c + {0,2,4,6,1,3,5,7}[i]; scales_gn fp16 [G, N]. Output, the AWQLinear
 * buffers (quantization.py:107-119): qweight int32 [N, K/8], scales and
 * zeros fp16 [N, G]. Requires K % 8 == 0, N % 8 == 0, K % group_size == 0.
 */
int nsq_awq_from_autoawq(const int32_t* qweight_kn8, const int32_t* qzeros_gn8, const uint16_t* scales_gn,
                         int64_t K, int64_t N, int64_t group_size, int32_t* qweight, uint16_t* scales,
                         uint16_t* zeros, void* stream);

/* Bytes of device workspace nsq_fp8_quantize needs (absmax reduction). */
size_t nsq_fp8_quantize_workspace_size(int64_t N, int64_t K);

/*
 * FP8 quantiser, bit-exact with FP8Linear.from_linear (quantization.py:54-75):
 * scale = absmax / 448 (1 if absmax == 0), codes = RNE e4m3 of w / scale,
 * non-saturating like torch's cast. Writes weight_fp8 [N, K] and the scale
 * (one fp32, device). workspace >= nsq_fp8_quantize_workspace_size().
 */
int nsq_fp8_quantize(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* weight_fp8,
                     float* weight_scale, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Allocation-free FP8 quantiser: the same result as nsq_fp8_quantize, but the
 * absmax scratch comes from a 256-byte array inside the library instead of a
 * caller workspace. No counterpart in the reference. For callers that cannot
 * allocate device memory when they quantise (inside a global-mode stream
 * capture, engines whose HBM is pre-reserved for the KV cache, C callers with
 * no device allocator). Returns NSQ_EWORKSPACE if a shape would need more
 * scratch than the array holds. Calls share the array: calls that overlap on
 * the GPU race, so serialise them. The first call on a device looks up the
 * array's device address; make it before any stream capture begins.
 */
int nsq_fp8_quantize_noalloc(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* weight_fp8,
                             float* weight_scale, void* stream);

/* Limit, in nanoseconds, of every bounded device-side wait that reports to the
 * status word (0 restores the default of 2 s; nsq_device_status_reset also
 * restores it). The wind-down waits that let in-flight copies land after a
 * failure always use the default. No counterpart in the reference (its path
 * has no device-side waits); used by the failure-path tests. */
int nsq_set_wait_limit_ns(uint64_t ns);

/* Failure-path test hook, off by default; returns the previous setting. While
 * on, the multi-wave decode kernel (the AWQ/FP8 linear with M <= 64 when it is
 * chosen, e.g. M = 16, K = 896, N = 9728) never requests the first weight box
 * of its first row group, so that group's bounded wait runs out: the kernel
 * records NSQ_EDEVICE_TIMEOUT (tag 1) in the status word, lets every copy it
 * did request land, and returns. Its output is then undefined. No counterpart
 * in the reference. Not for production use. */
int nsq_test_withhold_weight_load(int enable);

/*
 * One-shot all-reduce (sum) over NVLink peer memory for tensor parallelism:
 * the row-parallel all_reduce(SUM) of nano_sglang/distributed/
 * tensor_parallel.py:134-140 for outputs of at most `max_bytes`. Set-up (not
 * in the launch path): every rank allocates one workspace of
 * nsq_peer_workspace_size(world, max_bytes) bytes with
 * nsq_peer_workspace_alloc (zeroed), exports it with nsq_ipc_handle (64
 * bytes), and opens every other rank's handle with nsq_ipc_open.
 * nsq_peer_allreduce(workspaces[world] as mapped in this process, ...) then
 * sums `in` over the ranks into `out` (may alias `in`): every rank stores its
 * partial into every workspace, signals, waits (bounded) for the others and
 * sums the slots in rank order, so every rank gets bit-identical results.
 * Every rank must make the same sequence of calls. Stream-ordered, no host
 * synchronisation, graph-capturable. n * sizeof(dtype) must be a multiple of
 * 16 and at most max_bytes (else NSQ_EALIGN / NSQ_EWORKSPACE). A rank whose
 * wait runs out records NSQ_EDEVICE_TIMEOUT (tag 90) and returns.
 */
size_t nsq_peer_workspace_size(int world, int64_t max_bytes);
int nsq_peer_workspace_alloc(size_t bytes, void** ptr_out);
int nsq_peer_workspace_free(void* ptr);
int nsq_ipc_handle(const void* dev_ptr, void* handle_out);
int nsq_ipc_open(const void* handle, void** dev_ptr_out);
int nsq_ipc_close(void* dev_ptr);
int nsq_peer_allreduce(void* const* workspaces, int rank, int world, int64_t max_bytes, const void* in, void* out,
                       int64_t n, int dtype, void* stream);

/* Number of SMs the linear kernels leave free when they size their grids
 * (default 0; at most half the SMs), so that a collective launched on
 * another stream can run beside them. Returns the previous setting. No
 * counterpart in the reference (its all-reduce is serial). */
int nsq_set_sm_reserve(int n);

/* Opt in (1) or out (0, default) of programmatic dependent launch for the
 * linear kernels: with it on, a linear starts streaming its weights while the
 * previous kernel on the stream drains. Only valid when no kernel earlier on
 * the stream writes the weights being read. Returns the previous setting. */
int nsq_set_pdl(int enable);

#ifdef __cplusplus
}
#endif

#endif /* NSQ_H_ */
