// Q8_0 linear hot path for sm_100a: weight repack/dequantize, activation
// quantization, the decode GEMV, debug block dots and the per-tensor Q8_0
// runtime format.  C ABI in include/axq8.h.
//
// Reference semantics (paths inside the reference project):
//   Q8_0 block decode       inference/cpp/gguf/gguf.cpp:870-882
//   linear_from_gguf        inference/cpp/runtime/linear.cpp:27-71
//   quantize_weight (Q8_0)  inference/cpp/runtime/quantized_matmul.cpp:35-66
//   quantized_matmul (Q8_0) inference/cpp/runtime/quantized_matmul.cpp:110-204
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "axq8.h"
#include "common.cuh"
#include "q8_gemv.cuh"
#include "q8_mma.h"
#include "runtime.h"

using namespace axq8;

namespace {

// ---- repack GGUF blocks -> Q8R rows ------------------------------------------
// One thread per (row, block).  The 34-byte source block is read as 17
// half-words (block offsets are even), the quants are written as two 16-byte
// stores and the scale as one half-word.  Thread (n, 0) also zero-fills the
// row's padding so the rows are fully defined.
__global__ void repack_kernel(const uint16_t* __restrict__ src, int64_t N, int64_t K,
                              uint8_t* __restrict__ dst) {
    const int64_t nb = K / QK;
    const int64_t rs = q8r_row_stride(K);
    const int64_t total = N * nb;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = t / nb, b = t - n * nb;
        const uint16_t* s = src + t * (Q8_0_BYTES / 2);
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = (uint32_t)s[1 + 2 * i] | ((uint32_t)s[2 + 2 * i] << 16);
        uint8_t* row = dst + n * rs;
        reinterpret_cast<uint4*>(row + b * QK)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4*>(row + b * QK)[1] = make_uint4(w[4], w[5], w[6], w[7]);
        reinterpret_cast<uint16_t*>(row + K)[b] = s[0];
        if (b == 0) {
            for (int64_t p = K + 2 * nb; p < rs; p++) row[p] = 0;
        }
    }
}

// ---- dequantize (load_tensor values) -----------------------------------------
__global__ void dequant_kernel(const uint8_t* __restrict__ rows, int64_t N, int64_t K,
                               float* __restrict__ out) {
    const int64_t rs = q8r_row_stride(K);
    const int64_t total = N * K;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = t / K, k = t - n * K;
        const uint8_t* row = rows + n * rs;
        const float d = __half2float(reinterpret_cast<const __half*>(row + K)[k / QK]);
        out[t] = __fmul_rn((float)(int8_t)row[k], d);
    }
}

// ---- activation quantization ---------------------------------------------------
// One warp per 32-block.  amax by a warp max-reduction of |x| bit patterns
// (order-free), then the convention shared with the oracle:
// d = amax/127, id = 127/amax (IEEE divisions), q = round-half-away(x*id).
__global__ void quantize_act_kernel(const float* __restrict__ x, int64_t nblocks,
                                    int8_t* __restrict__ xq, float* __restrict__ dx) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t blk = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
         blk < nblocks; blk += warps) {
        const float v = ld_cg(x + blk * QK + lane);
        const uint32_t abits = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
        const float amax = __uint_as_float(abits);
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
        xq[blk * QK + lane] = (int8_t)q8_round(__fmul_rn(v, id));
        if (lane == 0) dx[blk] = d;
    }
}

// ---- debug: exact int32 block dots ---------------------------------------------
__global__ void block_dots_kernel(const uint8_t* __restrict__ rows, int64_t N, int64_t K,
                                  const int8_t* __restrict__ xq, int64_t M,
                                  int32_t* __restrict__ dots) {
    const int64_t nb = K / QK;
    const int64_t rs = q8r_row_stride(K);
    const int64_t total = M * N * nb;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = t % nb;
        const int64_t n = (t / nb) % N;
        const int64_t m = t / (nb * N);
        const int* w = reinterpret_cast<const int*>(rows + n * rs + b * QK);
        const int* a = reinterpret_cast<const int*>(xq + m * K + b * QK);
        int s = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) s = __dp4a(w[i], a[i], s);
        dots[t] = s;
    }
}

// ---- per-tensor Q8_0 runtime format (quantize_weight / quantized_matmul) ------
__global__ void absmax_kernel(const float* __restrict__ w, int64_t n, unsigned* amax_bits) {
    unsigned m = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        m = max(m, __float_as_uint(fabsf(w[i])));
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, m);
}

__global__ void quantize_tensor_kernel(const float* __restrict__ w, int64_t n,
                                       const unsigned* amax_bits, int8_t* __restrict__ q,
                                       float* scale_out) {
    float m = __uint_as_float(*amax_bits);
    m = m < 1e-8f ? 1e-8f : m;                          // max_abs_2d floor
    const float scale = __fdiv_rn(m, 127.0f);
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        long v = lroundf(__fdiv_rn(w[i], scale));       // std::lround(w/scale)
        v = v > 127 ? 127 : (v < -127 ? -127 : v);
        q[i] = (int8_t)v;
    }
}

// One thread per output; the k loop runs in order with separately rounded
// products and sums, as the reference's scalar loop does, so the result is
// bit-identical to quantized_matmul on the same inputs.
__global__ void quantized_matmul_kernel(const float* __restrict__ x, int64_t M, int64_t K,
                                        const int8_t* __restrict__ q, const float* scale,
                                        int64_t N, float* __restrict__ y) {
    const int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t m = blockIdx.y;
    if (n >= N || m >= M) return;
    const float* xr = x + m * K;
    float acc = 0.0f;
    for (int64_t k = 0; k < K; k++) acc = __fadd_rn(acc, __fmul_rn(xr[k], (float)q[k * N + n]));
    y[m * N + n] = __fmul_rn(acc, *scale);
}

// ---- synthetic Q8_0 weights --------------------------------------------------
// The benchmark workloads use random-init weights.  Element i (row-major
// index n*K + k) of stream `seed` is the Irwin-Hall sum of twelve 16-bit
// uniforms from splitmix64 at counters 3i..3i+2, scaled by std and shifted
// by mean with separately rounded fp32 operations; each 32-block is then
// quantized like a GGUF Q8_0 writer: d = amax/127, q = round-half-away(w/d),
// stored d = fp16(d).  Host code computing the same recipe gets identical
// bytes, which the tests check.
__device__ inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ inline float synth_value(uint64_t seed, uint64_t i, float mean, float stdv) {
    int acc = 0;
#pragma unroll
    for (int t = 0; t < 3; t++) {
        const uint64_t r = splitmix64(seed ^ ((3 * i + (uint64_t)t) * 0xD1B54A32D192ED03ull));
        acc += (int)(r & 0xffff) + (int)((r >> 16) & 0xffff) + (int)((r >> 32) & 0xffff) +
               (int)(r >> 48);
    }
    const float z = __fmul_rn((float)(acc - 393210), 1.0f / 65536.0f);
    return __fadd_rn(__fmul_rn(z, stdv), mean);
}

// layout 0: GGUF blocks (34 bytes each, row-major); layout 1: Q8R rows.
// Rows [row0, row0 + N) and columns [col0, col0 + K) of a synthetic
// [*, Kfull] tensor: element (r, k) is value number r * Kfull + k of the
// generator, so a slice holds exactly the blocks of the whole tensor.
__global__ void synth_q8_0_kernel(uint64_t seed, int64_t N, int64_t K, int64_t row0, int64_t col0,
                                  int64_t Kfull, float mean, float stdv, int layout,
                                  uint8_t* __restrict__ out) {
    const int64_t nb = K / QK;
    const int64_t rs = q8r_row_stride(K);
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < N * nb;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = t / nb, b = t - n * nb;
        float v[QK];
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < QK; i++) {
            v[i] = synth_value(seed, (uint64_t)((row0 + n) * Kfull + col0 + b * QK + i), mean, stdv);
            amax = fmaxf(amax, fabsf(v[i]));
        }
        const float d = __fdiv_rn(amax, 127.0f);
        const __half dh = __float2half_rn(d);
        uint8_t* qdst;
        if (layout == 0) {
            uint8_t* blk = out + t * Q8_0_BYTES;   // even offset: 2-byte aligned
            *reinterpret_cast<uint16_t*>(blk) = __half_as_ushort(dh);
            qdst = blk + 2;
        } else {
            uint8_t* row = out + n * rs;
            reinterpret_cast<__half*>(row + K)[b] = dh;
            if (b == 0)
                for (int64_t p = K + 2 * nb; p < rs; p++) row[p] = 0;
            qdst = row + b * QK;
        }
#pragma unroll
        for (int i = 0; i < QK; i++) {
            int q = 0;
            if (d != 0.0f) {
                float r = roundf(__fdiv_rn(v[i], d));
                q = (int)fminf(fmaxf(r, -127.0f), 127.0f);
            }
            qdst[i] = (uint8_t)(int8_t)q;
        }
    }
}

inline int grid_for(DeviceState* ds, int64_t work, int threads) {
    int64_t g = (work + threads - 1) / threads;
    int64_t cap = (int64_t)ds->sm_count * 16;
    if (g > cap) g = cap;
    return g < 1 ? 1 : (int)g;
}

int check_weight(const axq8_weight_t* w, const char* who) {
    if (!w || !w->rows) return fail(AXQ8_ERR_INVALID, "%s: null weight", who);
    if (w->N <= 0 || w->K <= 0 || (w->K % QK) != 0)
        return fail(AXQ8_ERR_INVALID, "%s: bad weight shape [%lld, %lld] (K %% 32 != 0)", who,
                    (long long)w->N, (long long)w->K);
    if (w->row_stride != q8r_row_stride(w->K))
        return fail(AXQ8_ERR_INVALID, "%s: row_stride %lld != %lld", who,
                    (long long)w->row_stride, (long long)q8r_row_stride(w->K));
    if ((reinterpret_cast<uintptr_t>(w->rows) & 15) != 0)
        return fail(AXQ8_ERR_INVALID, "%s: rows not 16-byte aligned", who);
    return AXQ8_OK;
}

}  // namespace

extern "C" {

uint64_t axq8_q8_0_byte_size(uint64_t n) { return (n / QK) * Q8_0_BYTES; }

int64_t axq8_row_stride(int64_t K) { return q8r_row_stride(K); }

int axq8_weight_repack(const void* dev_blocks, int64_t N, int64_t K, void* dev_rows,
                       void* stream) {
    if (!dev_blocks || !dev_rows) return fail(AXQ8_ERR_INVALID, "axq8_weight_repack: null pointer");
    if (N <= 0 || K <= 0 || K % QK)
        return fail(AXQ8_ERR_INVALID, "axq8_weight_repack: bad shape [%lld, %lld]", (long long)N,
                    (long long)K);
    if ((reinterpret_cast<uintptr_t>(dev_blocks) & 1) || (reinterpret_cast<uintptr_t>(dev_rows) & 15))
        return fail(AXQ8_ERR_INVALID, "axq8_weight_repack: misaligned pointer");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    repack_kernel<<<grid_for(ds, N * (K / QK), 256), 256, 0, s>>>(
        static_cast<const uint16_t*>(dev_blocks), N, K, static_cast<uint8_t*>(dev_rows));
    AXQ8_CUDA_TRY(cudaGetLastError(), "repack_kernel launch");
    return AXQ8_OK;
}

int axq8_weight_wrap(void* dev_rows, int64_t N, int64_t K, axq8_weight_t* out) {
    if (!out) return fail(AXQ8_ERR_INVALID, "axq8_weight_wrap: null out");
    out->rows = dev_rows;
    out->N = N;
    out->K = K;
    out->row_stride = q8r_row_stride(K);
    out->owns = 0;
    out->device = -1;
    int rc = check_weight(out, "axq8_weight_wrap");
    if (rc) return rc;
    int dev = 0;
    AXQ8_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    out->device = dev;
    return AXQ8_OK;
}

int axq8_weight_upload(const void* host_blocks, int64_t N, int64_t K, void* stream,
                       axq8_weight_t* out) {
    if (!host_blocks || !out) return fail(AXQ8_ERR_INVALID, "axq8_weight_upload: null pointer");
    if (N <= 0 || K <= 0 || K % QK)
        return fail(AXQ8_ERR_INVALID, "axq8_weight_upload: bad shape [%lld, %lld]", (long long)N,
                    (long long)K);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t src_bytes = (size_t)N * (K / QK) * Q8_0_BYTES;
    const size_t dst_bytes = (size_t)N * q8r_row_stride(K);
    void* staging = nullptr;
    void* rows = nullptr;
    cudaError_t e = cudaMalloc(&staging, src_bytes);
    if (e != cudaSuccess) return cuda_fail(e, "axq8_weight_upload: cudaMalloc(staging)");
    e = cudaMalloc(&rows, dst_bytes);
    if (e != cudaSuccess) {
        cudaFree(staging);
        return cuda_fail(e, "axq8_weight_upload: cudaMalloc(rows)");
    }
    int rc = AXQ8_OK;
    e = cudaMemcpyAsync(staging, host_blocks, src_bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) rc = cuda_fail(e, "axq8_weight_upload: H2D copy");
    if (rc == AXQ8_OK) rc = axq8_weight_repack(staging, N, K, rows, stream);
    if (rc == AXQ8_OK) {
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = cuda_fail(e, "axq8_weight_upload: synchronize");
    }
    cudaFree(staging);
    if (rc != AXQ8_OK) {
        cudaFree(rows);
        return rc;
    }
    rc = axq8_weight_wrap(rows, N, K, out);
    out->owns = 1;
    return rc;
}

int axq8_weight_free(axq8_weight_t* w) {
    if (!w) return AXQ8_OK;
    if (w->owns && w->rows) AXQ8_CUDA_TRY(cudaFree(w->rows), "axq8_weight_free");
    w->rows = nullptr;
    w->owns = 0;
    return AXQ8_OK;
}

int axq8_dequantize(const axq8_weight_t* w, float* out, void* stream) {
    int rc = check_weight(w, "axq8_dequantize");
    if (rc) return rc;
    if (!out) return fail(AXQ8_ERR_INVALID, "axq8_dequantize: null out");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    dequant_kernel<<<grid_for(ds, w->N * w->K, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(w->rows), w->N, w->K, out);
    AXQ8_CUDA_TRY(cudaGetLastError(), "dequant_kernel launch");
    return AXQ8_OK;
}

int axq8_quantize_act(const float* x, int64_t M, int64_t K, int8_t* xq, float* dx,
                      void* stream) {
    if (M < 0 || K <= 0 || K % QK)
        return fail(AXQ8_ERR_INVALID, "axq8_quantize_act: bad shape [%lld, %lld]", (long long)M,
                    (long long)K);
    if (M == 0) return AXQ8_OK;
    if (!x || !xq || !dx) return fail(AXQ8_ERR_INVALID, "axq8_quantize_act: null pointer");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    const int64_t nblocks = M * (K / QK);
    int grid = grid_for(ds, nblocks * 32, 256);
    AXQ8_CUDA_TRY(launch_k(quantize_act_kernel, dim3(grid), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), true, x, nblocks, xq, dx),
                  "quantize_act_kernel launch");
    return AXQ8_OK;
}

int axq8_linear_q8act(const axq8_weight_t* w, const int8_t* xq, const float* dx, int64_t M,
                      const float* residual, float* y, void* stream) {
    int rc = check_weight(w, "axq8_linear_q8act");
    if (rc) return rc;
    if (M < 0) return fail(AXQ8_ERR_INVALID, "axq8_linear_q8act: M < 0");
    if (M == 0) return AXQ8_OK;
    if (!xq || !dx || !y) return fail(AXQ8_ERR_INVALID, "axq8_linear_q8act: null pointer");
    if (reinterpret_cast<uintptr_t>(xq) & 15)
        return fail(AXQ8_ERR_INVALID, "axq8_linear_q8act: xq not 16-byte aligned");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    GemvArgs a = {};
    a.rows = static_cast<const uint8_t*>(w->rows);
    a.N = w->N;
    a.K = w->K;
    a.row_stride = w->row_stride;
    a.M = (int)M;
    a.xq = xq;
    a.dx = dx;
    a.residual = residual;
    a.y = y;
    a.ldy = w->N;
    a.status = ds->status;
    return gemv_launch(ds, a, /*a32=*/false, static_cast<cudaStream_t>(stream));
}

int axq8_linear(const axq8_weight_t* w, const float* x, int64_t M, float* y, int act_mode,
                void* stream) {
    int rc = check_weight(w, "axq8_linear");
    if (rc) return rc;
    if (M < 0) return fail(AXQ8_ERR_INVALID, "axq8_linear: M < 0");
    if (M == 0) return AXQ8_OK;
    if (!x || !y) return fail(AXQ8_ERR_INVALID, "axq8_linear: null pointer");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (act_mode == AXQ8_ACT_F32) {
        if (reinterpret_cast<uintptr_t>(x) & 15)
            return fail(AXQ8_ERR_INVALID, "axq8_linear: x not 16-byte aligned");
        GemvArgs a = {};
        a.rows = static_cast<const uint8_t*>(w->rows);
        a.N = w->N;
        a.K = w->K;
        a.row_stride = w->row_stride;
        a.M = (int)M;
        a.x = x;
        a.y = y;
        a.ldy = w->N;
        a.status = ds->status;
        return gemv_launch(ds, a, /*a32=*/true, s);
    }
    if (act_mode != AXQ8_ACT_Q8) return fail(AXQ8_ERR_INVALID, "axq8_linear: bad act_mode %d", act_mode);
    const int64_t nb = w->K / QK;
    if (skinny_eligible(w, M) || mma_eligible(w, M)) {
        // tensor-core paths: xq [M][K] + transposed scales dxT [K/32][Mp]
        const size_t q_bytes = ((size_t)M * w->K + 255) / 256 * 256;
        const size_t d_bytes = sizeof(float) * (size_t)nb * mma_scale_pitch(M);
        uint8_t* ws = static_cast<uint8_t*>(workspace(ds, q_bytes + d_bytes, s));
        if (!ws) return capture_active(s) ? AXQ8_ERR_STATE : AXQ8_ERR_ALLOC;
        int8_t* xq = reinterpret_cast<int8_t*>(ws);
        float* dxT = reinterpret_cast<float*>(ws + q_bytes);
        if ((rc = mma_quantize(ds, x, M, w->K, xq, dxT, s))) return rc;
        if (skinny_eligible(w, M)) return mmq_linear(ds, w, xq, dxT, M, nullptr, y, w->N, s);
        return mma_linear(ds, w, xq, dxT, M, nullptr, y, w->N, nullptr, s);
    }
    const size_t q_bytes = ((size_t)M * w->K + 255) / 256 * 256;
    uint8_t* ws = static_cast<uint8_t*>(workspace(ds, q_bytes + (size_t)M * nb * sizeof(float), s));
    if (!ws) return capture_active(s) ? AXQ8_ERR_STATE : AXQ8_ERR_ALLOC;
    int8_t* xq = reinterpret_cast<int8_t*>(ws);
    float* dx = reinterpret_cast<float*>(ws + q_bytes);
    rc = axq8_quantize_act(x, M, w->K, xq, dx, stream);
    if (rc) return rc;
    return axq8_linear_q8act(w, xq, dx, M, nullptr, y, stream);
}

int axq8_block_dots(const axq8_weight_t* w, const int8_t* xq, int64_t M, int32_t* dots,
                    void* stream) {
    int rc = check_weight(w, "axq8_block_dots");
    if (rc) return rc;
    if (M == 0) return AXQ8_OK;
    if (M < 0 || !xq || !dots) return fail(AXQ8_ERR_INVALID, "axq8_block_dots: bad argument");
    if (reinterpret_cast<uintptr_t>(xq) & 15)
        return fail(AXQ8_ERR_INVALID, "axq8_block_dots: xq not 16-byte aligned");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    block_dots_kernel<<<grid_for(ds, M * w->N * (w->K / QK), 256), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(w->rows), w->N, w->K, xq, M, dots);
    AXQ8_CUDA_TRY(cudaGetLastError(), "block_dots_kernel launch");
    return AXQ8_OK;
}

int axq8_quantize_weight_tensor(const float* w, int64_t K, int64_t N, int8_t* q,
                                float* scale_dev, void* stream) {
    if (!w || !q || !scale_dev || K <= 0 || N <= 0)
        return fail(AXQ8_ERR_INVALID, "axq8_quantize_weight_tensor: bad argument");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned* amax = static_cast<unsigned*>(workspace(ds, 256, s));
    if (!amax) return capture_active(s) ? AXQ8_ERR_STATE : AXQ8_ERR_ALLOC;
    AXQ8_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(unsigned), s), "memset amax");
    const int64_t n = K * N;
    absmax_kernel<<<grid_for(ds, n, 256), 256, 0, s>>>(w, n, amax);
    AXQ8_CUDA_TRY(cudaGetLastError(), "absmax_kernel launch");
    quantize_tensor_kernel<<<grid_for(ds, n, 256), 256, 0, s>>>(w, n, amax, q, scale_dev);
    AXQ8_CUDA_TRY(cudaGetLastError(), "quantize_tensor_kernel launch");
    return AXQ8_OK;
}

int axq8_quantized_matmul(const float* x, int64_t M, int64_t K, const int8_t* q,
                          const float* scale_dev, int64_t N, float* y, void* stream) {
    if (M == 0 || N == 0) return AXQ8_OK;
    if (!x || !q || !scale_dev || !y || M < 0 || K <= 0 || N < 0 || M > 65535)
        return fail(AXQ8_ERR_INVALID, "axq8_quantized_matmul: bad argument");
    dim3 grid((unsigned)((N + 255) / 256), (unsigned)M);
    quantized_matmul_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, M, K, q,
                                                                                  scale_dev, N, y);
    AXQ8_CUDA_TRY(cudaGetLastError(), "quantized_matmul_kernel launch");
    return AXQ8_OK;
}

int axq8_synth_q8_0(uint64_t seed, int64_t N, int64_t K, float mean, float stdv, int layout,
                    void* out, void* stream) {
    if (!out || N <= 0 || K <= 0 || K % QK || (layout != 0 && layout != 1))
        return fail(AXQ8_ERR_INVALID, "axq8_synth_q8_0: bad argument");
    if (layout == 1 && (reinterpret_cast<uintptr_t>(out) & 15))
        return fail(AXQ8_ERR_INVALID, "axq8_synth_q8_0: rows not 16-byte aligned");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    synth_q8_0_kernel<<<grid_for(ds, N * (K / QK), 128), 128, 0,
                        static_cast<cudaStream_t>(stream)>>>(seed, N, K, 0, 0, K, mean, stdv,
                                                             layout, static_cast<uint8_t*>(out));
    AXQ8_CUDA_TRY(cudaGetLastError(), "synth_q8_0_kernel launch");
    return AXQ8_OK;
}

}  // extern "C"

namespace axq8 {

int synth_q8_0_slice(uint64_t seed, int64_t N, int64_t K, int64_t row0, int64_t col0,
                     int64_t Kfull, float mean, float stdv, void* rows, cudaStream_t stream) {
    if (!rows || N <= 0 || K <= 0 || K % QK || col0 % QK || col0 + K > Kfull || row0 < 0)
        return fail(AXQ8_ERR_INVALID, "synth slice: bad argument");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    synth_q8_0_kernel<<<grid_for(ds, N * (K / QK), 128), 128, 0, stream>>>(
        seed, N, K, row0, col0, Kfull, mean, stdv, 1, static_cast<uint8_t*>(rows));
    AXQ8_CUDA_TRY(cudaGetLastError(), "synth_q8_0_kernel launch");
    return AXQ8_OK;
}

}  // namespace axq8
