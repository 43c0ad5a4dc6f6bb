// Host interface of the tensor-core (tcgen05 kind::i8) Q8_0 x A8 product,
// used by the C ABI in q8_linear.cu and by the decoder.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "axq8.h"
#include "runtime.h"

namespace axq8 {

// Smallest M routed to the tensor-core path by default (AXQ8_MMA_MIN_M
// overrides it; a large value keeps every M on the GEMV).
constexpr int kMmaMinM = 32;

// Whether the tensor-core path handles w at M rows: M >= the threshold,
// N >= 128, K a multiple of 128.
bool mma_eligible(const axq8_weight_t* w, int64_t M);

// The skinny product is preferred up to kMmqMaxM rows for every shape: with
// its weight tiles streamed through a shared-memory ring it matches or beats
// the tcgen05 product there (measured on B200, M = 32..64, Llama-3-8B shapes
// and their tensor-parallel slices: e.g. [128256x4096] 307 vs 336 us and
// [28672x4096] 98 vs 158 us at M = 48, [768x4096] 16 vs 37 us at M = 64).
constexpr int kMmqMaxM = 64;
inline bool skinny_preferred(int64_t N, int64_t M) {
    (void)N;
    return M <= kMmqMaxM;
}

// Whether axq8_linear takes the skinny product for w at M rows: 8 < M <= 64.
bool skinny_eligible(const axq8_weight_t* w, int64_t M);

// Caller-owned split-K scratch (partials and per-tile counters, the counters
// zero before first use); without it the library's per-device scratch is used
// (allocated, and grown, on demand: not usable inside a graph capture).
struct MmaScratch {
    float* part = nullptr;
    size_t part_bytes = 0;
    int* counters = nullptr;
    int64_t counter_slots = 0;
};

// y[M][ldy] = residual + xq . W^T with xq [M][K] int8 (16-byte aligned rows)
// and the activation scales transposed, dxT [K/32][Mp] fp32 (Mp = M rounded
// up to 4).  dots, when not null, receives every raw int32 block dot
// [M][N][K/32].  Requires the shape part of mma_eligible (any M >= 32).
int mma_linear(DeviceState* ds, const axq8_weight_t* w, const int8_t* xq, const float* dxT,
               int64_t M, const float* residual, float* y, int64_t ldy, int32_t* dots,
               cudaStream_t stream, const MmaScratch* scratch = nullptr);

// Split-K scratch a call with these sizes needs: partial bytes and counters.
void mma_split_needs(DeviceState* ds, int64_t N, int64_t K, int64_t M, size_t* part_bytes,
                     int64_t* counters);

// Whether the tensor-core path takes this shape at all (M >= 32, N >= 128,
// K % 128 == 0), ignoring the AXQ8_MMA_MIN_M threshold.
inline bool mma_shape_ok(int64_t N, int64_t K, int64_t M) {
    return M >= 32 && M <= (1 << 24) && N >= 128 && N <= (1 << 24) && K >= 128 && K % 128 == 0 &&
           K <= (1 << 20);
}

// Skinny product for decode widths (1 <= M <= 64, any N, K % 32 == 0):
// mma.sync m16n8k32 with register accumulators (q8_mmq.cuh), same inputs and
// result as mma_linear.  Its K splits combine on chip: no scratch.
int mmq_linear(DeviceState* ds, const axq8_weight_t* w, const int8_t* xq, const float* dxT,
               int64_t M, const float* residual, float* y, int64_t ldy, cudaStream_t stream);

// The skinny product of the stacked gate|up weight stored interleaved (rows
// gate_j, up_j; N % 64 == 0) fused with SiLU*up and its A8 quantization:
// sq [M][N/2] int8 and its block scales sdx ([b * sdxt + m] for sdxt > 0, else
// [m * N/64 + b]); bit-identical to mmq_linear into fp32 followed by
// silu_mul_kernel<true>.  sq / sdx must not alias xq / dxT.
int mmq_linear_silu(DeviceState* ds, const axq8_weight_t* w, const int8_t* xq, const float* dxT,
                    int64_t M, int8_t* sq, float* sdx, int sdxt, cudaStream_t stream);

// Mp for a given M (row pitch of dxT).
inline int64_t mma_scale_pitch(int64_t M) { return (M + 3) / 4 * 4; }

// Quantize x [M][K] into xq [M][K] and dxT [K/32][Mp] (A8 convention).
int mma_quantize(DeviceState* ds, const float* x, int64_t M, int64_t K, int8_t* xq, float* dxT,
                 cudaStream_t stream);

// dx [M][K/32] -> dxT [K/32][Mp].
int mma_transpose_scales(DeviceState* ds, const float* dx, int64_t M, int64_t K, float* dxT,
                         cudaStream_t stream);

}  // namespace axq8
