// Decode GEMV / skinny GEMM over repacked Q8_0 rows (sm_100a).
//
// y[m, n] = residual[m, n] + sum_b d_w[n,b] * d_x[m,b] * sum_{k in b} qw[n,k]*qx[m,k]
//   (A8: exact int32 block dots via dp4a, fp32 accumulation), or
// y[m, n] = residual[m, n] + sum_b d_w[n,b] * sum_{k in b} x[m,k]*qw[n,k]
//   (A32: the arithmetic of linear_from_gguf on the dequantized weight,
//    inference/cpp/runtime/linear.cpp:57-68, up to fp32 summation order).
//
// Structure.  Each CTA owns a contiguous range of output rows, so its share
// of the weight is one contiguous span of HBM.  A producer warp streams that
// span row by row into a ring of shared-memory slots with 1-D bulk async
// copies (TMA engine), one mbarrier per slot; eight consumer warps take rows
// round-robin, each row reduced by one warp.  Weights do not depend on the
// previous kernel in the stream, so the producer starts before
// griddepcontrol.wait: under programmatic dependent launch the weight stream
// of this GEMV overlaps the tail of the kernel that produces its activations.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "axq8.h"
#include "common.cuh"
#include "runtime.h"

namespace axq8 {

struct GemvArgs {
    const uint8_t* rows;      // Q8R rows
    int64_t N, K, row_stride;
    int M;
    const int8_t* xq;         // A8: [M, K] int8, 16-byte aligned
    const float* dx;          // A8: [M, K/32]
    const float* x;           // A32: [M, K] fp32, 16-byte aligned
    const float* residual;    // nullable, [M, ldy]
    float* y;                 // [M, ldy]
    int64_t ldy;
    int* status;
    int nslot;                // ring slots (rows in flight per CTA)
};

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kGemvRingBytes = 64 * 1024;

__device__ inline int dot16_i8(const int4 w, const int4 a) {
    int s = __dp4a(w.x, a.x, 0);
    s = __dp4a(w.y, a.y, s);
    s = __dp4a(w.z, a.z, s);
    return __dp4a(w.w, a.w, s);
}

// 16 int8 weights against 16 fp32 activations.
__device__ inline float dot16_f32(const int4 w, const float* __restrict__ xa) {
    const float4* x4 = reinterpret_cast<const float4*>(xa);
    const int ws[4] = {w.x, w.y, w.z, w.w};
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 v = __ldg(x4 + i);
        const int q = ws[i];
        s = fmaf(v.x, (float)(int8_t)(q & 0xff), s);
        s = fmaf(v.y, (float)(int8_t)((q >> 8) & 0xff), s);
        s = fmaf(v.z, (float)(int8_t)((q >> 16) & 0xff), s);
        s = fmaf(v.w, (float)(int8_t)((q >> 24) & 0xff), s);
    }
    return s;
}

// One warp reduces one staged row against MT activation rows starting at m0.
// Lane l owns 16-byte chunks l, l+32, ...; the two lanes holding the halves
// of a 32-block combine their int32 partials with one shuffle so every block
// dot is exact before it is scaled.
template <int MT, bool A32>
__device__ inline void gemv_row(const uint8_t* __restrict__ row, const GemvArgs& a, int m0,
                                int lane, float (&acc)[MT]) {
    const int64_t K = a.K;
    const int64_t nb = K / QK;
    const int nchunks = (int)(K / 16);
    const __half* dw = reinterpret_cast<const __half*>(row + K);
#pragma unroll
    for (int j = 0; j < MT; j++) acc[j] = 0.0f;
    for (int base = 0; base < nchunks; base += 32) {
        const int c = base + lane;
        const bool valid = c < nchunks;
        const int b = c >> 1;
        const bool lead = valid && ((lane & 1) == 0);
        const int4 w = valid ? *reinterpret_cast<const int4*>(row + (int64_t)c * 16)
                             : make_int4(0, 0, 0, 0);
        const float d = lead ? __half2float(dw[b]) : 0.0f;
#pragma unroll
        for (int j = 0; j < MT; j++) {
            const int m = m0 + j;
            if (m >= a.M) break;   // uniform across the warp
            if (A32) {
                float p = valid ? dot16_f32(w, a.x + (int64_t)m * K + (int64_t)c * 16) : 0.0f;
                p += __shfl_xor_sync(0xffffffffu, p, 1);
                if (lead) acc[j] = fmaf(d, p, acc[j]);
            } else {
                const int4 xa = valid ? __ldg(reinterpret_cast<const int4*>(
                                            a.xq + (int64_t)m * K + (int64_t)c * 16))
                                      : make_int4(0, 0, 0, 0);
                int s = dot16_i8(w, xa);
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                if (lead) acc[j] = fmaf(d * __ldg(a.dx + (int64_t)m * nb + b), (float)s, acc[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < MT; j++) acc[j] = warp_sum(acc[j]);
}

template <int MT, bool A32>
__global__ void __launch_bounds__(kGemvThreads) q8_gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int nslot = a.nslot;
    const int64_t rs = a.row_stride;
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (int64_t)nslot * rs);
    uint64_t* empty = full + nslot;

    const int64_t r0 = a.N * blockIdx.x / gridDim.x;
    const int64_t r1 = a.N * (blockIdx.x + 1) / gridDim.x;
    const int nrows = (int)(r1 - r0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < nslot; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kGemvConsumerWarps) {
        // Producer: weights are independent of the previous grid, so no
        // griddepcontrol.wait here.
        if (lane == 0) {
            const uint8_t* src = a.rows + r0 * rs;
            for (int i = 0; i < nrows; i++) {
                const int s = i % nslot;
                if (i >= nslot &&
                    !mbar_wait_bounded(&empty[s], ((i / nslot) - 1) & 1, a.status,
                                       AXQ8_ERR_WAIT_TIMEOUT))
                    break;
                mbar_arrive_expect_tx(&full[s], (uint32_t)rs);
                bulk_g2s(ring + (int64_t)s * rs, src + (int64_t)i * rs, (uint32_t)rs, &full[s]);
            }
        }
        return;
    }

    pdl_wait();   // activations and residual come from the previous grid
    for (int i = warp; i < nrows; i += kGemvConsumerWarps) {
        const int s = i % nslot;
        if (!mbar_wait_bounded(&full[s], (i / nslot) & 1, a.status, AXQ8_ERR_WAIT_TIMEOUT)) break;
        const uint8_t* row = ring + (int64_t)s * rs;
        const int64_t n = r0 + i;
        for (int m0 = 0; m0 < a.M; m0 += MT) {
            float acc[MT];
            gemv_row<MT, A32>(row, a, m0, lane, acc);
            if (lane == 0) {
#pragma unroll
                for (int j = 0; j < MT; j++) {
                    const int m = m0 + j;
                    if (m < a.M) {
                        float v = acc[j];
                        if (a.residual) v += a.residual[(int64_t)m * a.ldy + n];
                        a.y[(int64_t)m * a.ldy + n] = v;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

template <int MT, bool A32>
inline int gemv_launch_t(DeviceState* ds, GemvArgs a, cudaStream_t stream) {
    const int64_t rs = a.row_stride;
    int nslot = (int)(kGemvRingBytes / rs);
    if (nslot < 1) nslot = 1;
    if (nslot > 64) nslot = 64;
    const size_t smem = (size_t)nslot * rs + 2 * nslot * sizeof(uint64_t);
    if (smem > (size_t)ds->max_smem_optin)
        return fail(AXQ8_ERR_UNSUPPORTED, "q8 gemv: K=%lld needs %zu B shared memory",
                    (long long)a.K, smem);
    a.nslot = nslot;
    auto kern = q8_gemv_kernel<MT, A32>;
    static int configured_for[64] = {0};   // per device: opted-in smem bytes
    int dev = ds->device < 64 ? ds->device : 63;
    if (configured_for[dev] < (int)smem) {
        AXQ8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)ds->max_smem_optin),
                      "cudaFuncSetAttribute(q8_gemv)");
        configured_for[dev] = ds->max_smem_optin;
    }
    int64_t grid = ds->sm_count;
    if (grid > a.N) grid = a.N;
    AXQ8_CUDA_TRY(launch_k(kern, dim3((unsigned)grid), dim3(kGemvThreads), smem, stream, true, a),
                  "q8_gemv launch");
    return AXQ8_OK;
}

inline int gemv_launch(DeviceState* ds, const GemvArgs& a, bool a32, cudaStream_t stream) {
    if (a.M <= 1) return a32 ? gemv_launch_t<1, true>(ds, a, stream) : gemv_launch_t<1, false>(ds, a, stream);
    if (a.M <= 2) return a32 ? gemv_launch_t<2, true>(ds, a, stream) : gemv_launch_t<2, false>(ds, a, stream);
    if (a.M <= 4) return a32 ? gemv_launch_t<4, true>(ds, a, stream) : gemv_launch_t<4, false>(ds, a, stream);
    return a32 ? gemv_launch_t<8, true>(ds, a, stream) : gemv_launch_t<8, false>(ds, a, stream);
}

}  // namespace axq8
