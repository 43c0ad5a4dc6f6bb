/*
 * axq8.h — C ABI of the B200 (sm_100a) Q8_0 linear hot path.
 *
 * Plain C: pointers, sizes and status codes only; no C++ or torch types, no
 * exceptions cross this boundary.  Device pointers are caller-owned unless a
 * function says it allocates.  `stream` is a cudaStream_t passed as void*
 * (NULL = the legacy default stream).  Every function returns AXQ8_OK (0) or a
 * negative AXQ8_ERR_* code; axq8_last_error() gives the message of the most
 * recent failure on the calling host thread.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   gguf_tensor_byte_size            inference/cpp/gguf/gguf.hpp:34-37, gguf.cpp:36-67
 *   GGUFLoader::load_tensor (Q8_0)   inference/cpp/gguf/gguf.hpp:92-94, gguf.cpp:784-882
 *   linear_from_gguf                 inference/cpp/runtime/linear.hpp:22-25, linear.cpp:27-71
 *   quantize_weight / quantized_matmul (Q8_0)
 *                                    inference/cpp/runtime/quantized_matmul.hpp:38-48
 */
#ifndef AXION_B200_AXQ8_H
#define AXION_B200_AXQ8_H

#include <stdint.h>

#include "axq8_status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Activation handling of axq8_linear. */
enum {
    /* A8: activations quantized on the fly to Q8 blocks of 32 (amax/127
     * scale kept in fp32, round half away from zero), exact int32 block dot
     * products, fp32 accumulation of d_w*d_x*dot.  The decode default. */
    AXQ8_ACT_Q8 = 0,
    /* A32: fp32 activations against the dequantized weight, i.e. the
     * arithmetic of linear_from_gguf(x, load_tensor(W)). */
    AXQ8_ACT_F32 = 1
};

/* A Q8_0 weight [N, K] resident in device memory in the repacked row layout:
 * row n occupies `row_stride` bytes at rows + n*row_stride: K int8 quants,
 * K/32 fp16 scales, zero padding to a 16-byte multiple. */
typedef struct axq8_weight {
    void* rows;          /* device pointer, 256-byte aligned when allocated here */
    int64_t N;           /* output features (GGUF outer dim) */
    int64_t K;           /* input features, multiple of 32 */
    int64_t row_stride;  /* bytes, = axq8_row_stride(K) */
    int32_t owns;        /* 1: allocated by axq8_weight_upload, freed by axq8_weight_free */
    int32_t device;      /* CUDA device ordinal holding `rows` */
} axq8_weight_t;

/* Bytes of a GGUF Q8_0 tensor of n elements: (n/32)*34.
 * Replaces gguf_tensor_byte_size(GGUFType::Q8_0, n) (gguf.cpp:51). */
uint64_t axq8_q8_0_byte_size(uint64_t n);

/* Bytes of one repacked device row for K inputs. */
int64_t axq8_row_stride(int64_t K);

/* Upload GGUF Q8_0 blocks (host memory, N*K/32 blocks of 34 bytes, rows in
 * GGUF order) once and repack them on the device.  ALLOCATES device memory
 * (cudaMalloc); the copy and repack run on `stream` and are complete when the
 * call returns.  Replaces the per-token GGUFLoader::load_tensor + dequant of
 * the reference (gguf.cpp:784-882): the raw blocks stay resident instead. */
int axq8_weight_upload(const void* host_blocks, int64_t N, int64_t K, void* stream,
                       axq8_weight_t* out);

/* Repack GGUF Q8_0 blocks already in device memory into caller-owned
 * `dev_rows` (N*axq8_row_stride(K) bytes, 16-byte aligned).  No allocation. */
int axq8_weight_repack(const void* dev_blocks, int64_t N, int64_t K, void* dev_rows,
                       void* stream);

/* Describe caller-owned repacked rows as a weight (no allocation). */
int axq8_weight_wrap(void* dev_rows, int64_t N, int64_t K, axq8_weight_t* out);

/* Free a weight made by axq8_weight_upload (no-op for wrapped weights). */
int axq8_weight_free(axq8_weight_t* w);

/* Device dequantization to fp32 [N, K], the values GGUFLoader::load_tensor
 * produces for a Q8_0 tensor: out[n,k] = (float)q * fp16_to_fp32(d)
 * (gguf.cpp:870-882). */
int axq8_dequantize(const axq8_weight_t* w, float* out, void* stream);

/* Quantize fp32 activations x[M, K] to int8 xq[M, K] and fp32 per-block
 * scales dx[M, K/32] under the A8 convention.  Bit-exact with the oracle. */
int axq8_quantize_act(const float* x, int64_t M, int64_t K, int8_t* xq, float* dx,
                      void* stream);

/* y[M, N] = x[M, K] . W^T — linear_from_gguf(input[M,K], weight[N,K])
 * (linear.hpp:22-25) with the weight kept in Q8_0.  x and y are device fp32,
 * row-major, contiguous.  act_mode: AXQ8_ACT_Q8 or AXQ8_ACT_F32.  In A8 mode
 * the quantized activations live in a per-device workspace that this
 * library allocates on first use and grows when a larger M*K arrives (the
 * only allocation on this path); calls on different streams of one device
 * must not overlap.  A8 with 8 < M <= 64 runs the skinny tensor-core product
 * (axq8_linear_q8act_s), A8 with M > 64, N >= 128 and K % 128 == 0 the tcgen05
 * product (axq8_linear_q8act_t); everything else the streaming GEMV kernel
 * (axq8_linear_path tells which). */
int axq8_linear(const axq8_weight_t* w, const float* x, int64_t M, float* y, int act_mode,
                void* stream);

/* Which kernel axq8_linear runs for w at M rows in act_mode (see above). */
enum {
    AXQ8_PATH_GEMV = 0,
    AXQ8_PATH_TENSOR_CORE = 1,
    AXQ8_PATH_SKINNY = 2
};
int axq8_linear_path(const axq8_weight_t* w, int64_t M, int act_mode);

/* The same product for decode widths (1 <= M <= 64, any N, K % 32 == 0) with
 * mma.sync m16n8k32 int8 and register accumulators (linear_from_gguf,
 * linear.cpp:27-71, for batched decode); inputs from axq8_quantize_act_t.
 * Exact int32 block dots; fp32 combination acc += (D_b*dw)*dx per block.
 * Uses no device workspace (the K splits of a row tile are combined in shared
 * memory within one thread-block cluster) and is deterministic run to run. */
int axq8_linear_q8act_s(const axq8_weight_t* w, const int8_t* xq, const float* dxT, int64_t M,
                        const float* residual, float* y, void* stream);

/* A8 quantization for the tensor-core product: xq[M, K] int8 as
 * axq8_quantize_act, the scales transposed: dxT[K/32, Mp] fp32 with
 * Mp = M rounded up to a multiple of 4. */
int axq8_quantize_act_t(const float* x, int64_t M, int64_t K, int8_t* xq, float* dxT,
                        void* stream);

/* y[M, N] = residual + xq.W^T on the tensor cores (prefill / batched decode:
 * linear_from_gguf, linear.cpp:27-71, at M >= 32), from axq8_quantize_act_t
 * output.  Needs M >= 32, N >= 128, K % 128 == 0 (else AXQ8_ERR_UNSUPPORTED).
 * Exact int32 block dots; fp32 combination acc += (D_b*dw)*dx per block.
 * Few output tiles split K across CTAs through a per-device scratch this
 * library allocates on first use. */
int axq8_linear_q8act_t(const axq8_weight_t* w, const int8_t* xq, const float* dxT, int64_t M,
                        const float* residual, float* y, void* stream);

/* Same with pre-quantized activations (xq[M,K] int8, dx[M,K/32] fp32), as
 * written by axq8_quantize_act or a fused producer.  `residual` (nullable,
 * [M, N] fp32) is added to the product: y = residual + x.W^T. */
int axq8_linear_q8act(const axq8_weight_t* w, const int8_t* xq, const float* dx, int64_t M,
                      const float* residual, float* y, void* stream);

/* axq8_linear in A8 mode for callers that cannot allocate device memory:
 * code running under a fixed, pre-planned memory budget (an allocator that
 * owns all of HBM) or code that must not risk the device synchronization
 * cudaMalloc/cudaFree can cause.  No counterpart in the reference (its
 * linear runs on the host).  Allocates nothing: the quantized activation
 * goes to a fixed 1.1875 MiB static device array that every GPU loading this
 * library reserves until exit.  Limit: M*K <= 1,048,576, else
 * AXQ8_ERR_INVALID.  Kernels: the GEMV for M <= 8 and M > 64, the skinny
 * product for 8 < M <= 64 (both as axq8_linear picks them); above 64 rows
 * axq8_linear's tcgen05 product needs split-K scratch, so this entry point
 * stays on the GEMV there (slower; same values up to fp32 combination
 * order).  The array is shared by all calls on a device: calls that overlap
 * on the GPU race and must be serialized by the caller.  The first call on a
 * device looks up the array's address and keeps it; make it before any
 * stream capture, and do not use the library across a cudaDeviceReset. */
int axq8_linear_noalloc(const axq8_weight_t* w, const float* x, int64_t M, float* y,
                        void* stream);

/* Exact int32 block dot products dots[M, N, K/32] = sum_i qw*qx over each
 * 32-block; a debug/parity entry point (slow). */
int axq8_block_dots(const axq8_weight_t* w, const int8_t* xq, int64_t M, int32_t* dots,
                    void* stream);

/* The same block dots read back from the tensor cores' TMEM accumulators
 * (axq8_linear_q8act_t's kernel in a debug mode that also stores every
 * int32 block result; y receives the product).  Same shape limits. */
int axq8_block_dots_tc(const axq8_weight_t* w, const int8_t* xq, const float* dxT, int64_t M,
                       int32_t* dots, float* y, void* stream);

/* Per-tensor Q8_0 runtime format of quantize_weight / quantized_matmul
 * (quantized_matmul.cpp:35-204, QuantType::Q8_0): W[K, N] fp32 ->
 * q[K, N] int8 = clamp(lround(w/scale), +-127), scale = max(max|w|, 1e-8)/127.
 * The scale is written to *scale_dev (device fp32). */
int axq8_quantize_weight_tensor(const float* w, int64_t K, int64_t N, int8_t* q,
                                float* scale_dev, void* stream);

/* quantized_matmul for that format: y[M, N] = (sum_k x[m,k]*q[k,n]) * scale. */
int axq8_quantized_matmul(const float* x, int64_t M, int64_t K, const int8_t* q,
                          const float* scale_dev, int64_t N, float* y, void* stream);

/* Random-init Q8_0 weight [N, K] generated on the device (benchmark
 * workloads): element n*K+k of stream `seed` is approximately
 * N(mean, std^2) (Irwin-Hall sum of twelve splitmix64 uniforms), then each
 * 32-block is quantized as a GGUF writer does (d = amax/127 stored as fp16,
 * q = round-half-away(w/d)).  layout 0 writes GGUF blocks (N*K/32*34 bytes),
 * layout 1 writes repacked rows (N*axq8_row_stride(K) bytes).  No
 * counterpart in the reference, which reads weights from a GGUF file. */
int axq8_synth_q8_0(uint64_t seed, int64_t N, int64_t K, float mean, float std, int layout,
                    void* out, void* stream);

/* Device status word shared by all kernels of this library on the current
 * device: 0, or the AXQ8_ERR_* code of the first bounded wait that gave up.
 * axq8_status_read synchronizes the device; axq8_status_clear resets it. */
int axq8_status_read(int* code);
int axq8_status_clear(void);

/* Message of the last failure on this host thread ("" if none). */
const char* axq8_last_error(void);

/* Library build identification (for logs). */
const char* axq8_version(void);

#ifdef __cplusplus
}
#endif
#endif /* AXION_B200_AXQ8_H */
