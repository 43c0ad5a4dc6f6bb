// Decode GEMV / skinny GEMM over repacked Q8_0 rows (sm_100a).
//
// y[m, n] = residual[m, n] + sum_b d_w[n,b] * d_x[m,b] * sum_{k in b} qw[n,k]*qx[m,k]
//   (A8: exact int32 block dots via dp4a, fp32 accumulation), or
// y[m, n] = residual[m, n] + sum_b d_w[n,b] * sum_{k in b} x[m,k]*qw[n,k]
//   (A32: the arithmetic of linear_from_gguf on the dequantized weight,
//    inference/cpp/runtime/linear.cpp:57-68, up to fp32 summation order).
//
// Structure.  The kernel is a pure weight stream, and HBM bandwidth is reached
// only with enough bytes in flight per SM (measured on B200: a read stream
// needs >= 8 outstanding 16-byte loads per thread at >= 1024 threads per SM
// for ~7 TB/s; 1-D bulk copies need >= 16 KB per copy, 4 KB copies cap at
// ~2.6 TB/s).  So:
//  * two CTAs of 16 warps per SM, each CTA owning a contiguous range of rows;
//  * each warp reduces TWO rows at a time with kChunks 16-byte loads per row
//    per lane in flight (non-allocating, read-once);
//  * the warp's first loads are issued before griddepcontrol.wait: weights do
//    not depend on the previous kernel, so under programmatic dependent launch
//    their HBM latency overlaps the tail of the kernel producing the input;
//  * when a CTA has fewer row pairs than warps (short N, long K), the K range
//    of each pair is split over several warps and the partial sums are
//    reduced through shared memory in a fixed order (SPLIT instantiation);
//  * in A8 mode the quantized activation and its scales are staged once per
//    CTA in shared memory.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>

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
    int act_smem;             // bytes of staged activation (0: read from global)
};

constexpr int kGemvWarps = 16;                 // warps per CTA
constexpr int kGemvCtasPerSm = 2;
constexpr int kChunks = 4;                     // 16-byte loads per row per lane in flight
constexpr int kGemvActSmemMax = 32 * 1024;     // largest staged activation
constexpr int kGemvMaxMT = 4;
constexpr int kPartBytes = kGemvWarps * 2 * kGemvMaxMT * 4;   // split-K partials

__device__ inline int4 ldg_stream(const void* p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ inline int dot16_i8(const int4 w, const int4 a) {
    int s = __dp4a(w.x, a.x, 0);
    s = __dp4a(w.y, a.y, s);
    s = __dp4a(w.z, a.z, s);
    return __dp4a(w.w, a.w, s);
}

// 16 int8 weights against 16 fp32 activations (global memory).
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

// The 2 x kChunks weight chunks (and their block scales) a lane holds for one
// step of a row pair: rows ra, rb, chunk columns base + 32u + lane, u < kChunks,
// limited to chunks below `cend`.
struct PairLoad {
    int4 w[2][kChunks];
    __half2 d[kChunks];   // .x: row a, .y: row b
};

__device__ __forceinline__ void pair_load(PairLoad& L, const uint8_t* ra, const uint8_t* rb,
                                          bool has_b, int K, int base, int cend, int lane) {
    const __half* da = reinterpret_cast<const __half*>(ra + K);
    const __half* db = reinterpret_cast<const __half*>(rb + K);
#pragma unroll
    for (int u = 0; u < kChunks; u++) {
        const int c = base + 32 * u + lane;
        const bool v = c < cend;
        L.w[0][u] = v ? ldg_stream(ra + c * 16) : make_int4(0, 0, 0, 0);
        L.w[1][u] = (v && has_b) ? ldg_stream(rb + c * 16) : make_int4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kChunks; u++) {
        const int c = base + 32 * u + lane;
        const bool v = c < cend;
        const __half z = __ushort_as_half(0);
        L.d[u] = __halves2half2(v ? __ldg(da + (c >> 1)) : z,
                                (v && has_b) ? __ldg(db + (c >> 1)) : z);
    }
}

// Accumulate one loaded step into acc[row][j] for MT activation rows from m0.
// The two lanes holding the halves of a 32-block combine their int32
// partials with one shuffle, so each block dot is exact before it is scaled.
template <int MT, bool A32>
__device__ __forceinline__ void pair_compute(const PairLoad& L, const GemvArgs& a,
                                             const int8_t* __restrict__ xq,
                                             const float* __restrict__ dx, int base, int cend,
                                             int m0, int lane, float (&acc)[2][MT]) {
    const int K = (int)a.K;
    const int nb = K / QK;
#pragma unroll
    for (int u = 0; u < kChunks; u++) {
        if (base + 32 * u >= cend) break;   // uniform across the warp
        const int c = base + 32 * u + lane;
        const bool valid = c < cend;
        const bool lead = valid && ((lane & 1) == 0);
        const int b = c >> 1;
#pragma unroll
        for (int j = 0; j < MT; j++) {
            const int m = m0 + j;
            if (m >= a.M) break;   // uniform across the warp
            if (A32) {
                const float* xr = a.x + (int64_t)m * K + c * 16;
                float p0 = valid ? dot16_f32(L.w[0][u], xr) : 0.0f;
                float p1 = valid ? dot16_f32(L.w[1][u], xr) : 0.0f;
                p0 += __shfl_xor_sync(0xffffffffu, p0, 1);
                p1 += __shfl_xor_sync(0xffffffffu, p1, 1);
                if (lead) {
                    const float2 d = __half22float2(L.d[u]);
                    acc[0][j] = fmaf(d.x, p0, acc[0][j]);
                    acc[1][j] = fmaf(d.y, p1, acc[1][j]);
                }
            } else {
                const int4 xa = valid ? *reinterpret_cast<const int4*>(xq + m * K + c * 16)
                                      : make_int4(0, 0, 0, 0);
                int s0 = dot16_i8(L.w[0][u], xa);
                int s1 = dot16_i8(L.w[1][u], xa);
                s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
                s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
                if (lead) {
                    const float dxv = dx[m * nb + b];
                    const float2 d = __half22float2(L.d[u]);
                    acc[0][j] = fmaf(d.x * dxv, (float)s0, acc[0][j]);
                    acc[1][j] = fmaf(d.y * dxv, (float)s1, acc[1][j]);
                }
            }
        }
    }
}

template <int MT>
__device__ __forceinline__ void pair_store(const GemvArgs& a, int64_t n, bool has_b, int m0,
                                           int lane, float (&acc)[2][MT]) {
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int j = 0; j < MT; j++) acc[r][j] = warp_sum(acc[r][j]);
    if (lane < 2 && (lane == 0 || has_b)) {
        const int r = lane;
#pragma unroll
        for (int j = 0; j < MT; j++) {
            const int m = m0 + j;
            if (m < a.M) {
                float v = acc[r][j];
                if (a.residual) v += a.residual[(int64_t)m * a.ldy + n + r];
                a.y[(int64_t)m * a.ldy + n + r] = v;
            }
        }
    }
}

template <int MT>
__device__ __forceinline__ void acc_zero(float (&acc)[2][MT]) {
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int j = 0; j < MT; j++) acc[r][j] = 0.0f;
}

template <int MT, bool A32, bool SPLIT>
__global__ void __launch_bounds__(kGemvWarps * 32, kGemvCtasPerSm) q8_gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    float* part = reinterpret_cast<float*>(smem);   // [kGemvWarps][2][MT] split-K partials
    uint8_t* act = smem + kPartBytes;               // staged activation
    const int64_t rs = a.row_stride;
    const int K = (int)a.K;
    const int nchunks = K / 16;
    const int64_t r0 = a.N * blockIdx.x / gridDim.x;
    const int64_t r1 = a.N * (blockIdx.x + 1) / gridDim.x;
    const int nrows = (int)(r1 - r0);
    const int npairs = (nrows + 1) / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Warps per row pair (SPLIT only): a power of two with wpp * npairs <=
    // warps, so each warp has at most one (pair, K slice); slices are whole
    // 32-chunk warp steps, so the two halves of a block never straddle them.
    const int nsteps = (nchunks + 31) / 32;
    int wpp = 1;
    if (SPLIT)
        while (2 * wpp <= kGemvWarps && 2 * wpp * npairs <= kGemvWarps && 2 * wpp <= nsteps)
            wpp *= 2;
    const int slice = warp % wpp;
    const int sps = (nsteps + wpp - 1) / wpp;
    const int c_begin = min(nchunks, slice * sps * 32);
    const int c_end = min(nchunks, (slice + 1) * sps * 32);
    int p = warp / wpp;
    const int conc = kGemvWarps / wpp;

    // First weight loads of this warp before the dependency wait.
    PairLoad L;
    if (p < npairs && c_begin < c_end) {
        const uint8_t* ra = a.rows + (r0 + 2 * p) * rs;
        const bool has_b = 2 * p + 1 < nrows;
        pair_load(L, ra, has_b ? ra + rs : ra, has_b, K, c_begin, c_end, lane);
    }
    pdl_launch_dependents();
    pdl_wait();   // activations and residual come from the previous grid

    const int8_t* xq = a.xq;
    const float* dx = a.dx;
    if (!A32 && a.act_smem > 0) {
        int8_t* act_q = reinterpret_cast<int8_t*>(act);
        float* act_d = reinterpret_cast<float*>(act + ((int64_t)a.M * K + 15) / 16 * 16);
        const int qbytes = a.M * K;
        for (int o = threadIdx.x * 16; o < qbytes; o += kGemvWarps * 32 * 16)
            *reinterpret_cast<int4*>(act_q + o) = __ldg(reinterpret_cast<const int4*>(a.xq + o));
        const int nd = a.M * (K / QK);
        for (int o = threadIdx.x; o < nd; o += kGemvWarps * 32) act_d[o] = __ldg(a.dx + o);
        __syncthreads();
        xq = act_q;
        dx = act_d;
    }

    if (!SPLIT || wpp == 1) {
        for (; p < npairs; p += conc) {
            const uint8_t* ra = a.rows + (r0 + 2 * p) * rs;
            const bool has_b = 2 * p + 1 < nrows;
            const uint8_t* rb = has_b ? ra + rs : ra;
            if (a.M <= MT) {
                float acc[2][MT];
                acc_zero(acc);
                for (int base = 0; base < nchunks; base += 32 * kChunks) {
                    if (base > 0 || p != warp) pair_load(L, ra, rb, has_b, K, base, nchunks, lane);
                    pair_compute<MT, A32>(L, a, xq, dx, base, nchunks, 0, lane, acc);
                }
                pair_store<MT>(a, r0 + 2 * p, has_b, 0, lane, acc);
                continue;
            }
            // more activation rows than one pass holds: re-read the (L2-hot)
            // row pair for each group of MT rows
            for (int m0 = 0; m0 < a.M; m0 += MT) {
                float acc[2][MT];
                acc_zero(acc);
                for (int base = 0; base < nchunks; base += 32 * kChunks) {
                    if (base > 0 || p != warp || m0 > 0)
                        pair_load(L, ra, rb, has_b, K, base, nchunks, lane);
                    pair_compute<MT, A32>(L, a, xq, dx, base, nchunks, m0, lane, acc);
                }
                pair_store<MT>(a, r0 + 2 * p, has_b, m0, lane, acc);
            }
        }
        return;
    }
    if (!SPLIT) return;

    // split-K: every warp reaches the barriers, including warps without work
    const bool active = p < npairs && c_begin < c_end;
    const uint8_t* ra = a.rows + (r0 + 2 * (p < npairs ? p : 0)) * rs;
    const bool has_b = 2 * p + 1 < nrows;
    const uint8_t* rb = has_b ? ra + rs : ra;
    for (int m0 = 0; m0 < a.M; m0 += MT) {
        float acc[2][MT];
        acc_zero(acc);
        if (active) {
            for (int base = c_begin; base < c_end; base += 32 * kChunks) {
                if (base > c_begin || m0 > 0) pair_load(L, ra, rb, has_b, K, base, c_end, lane);
                pair_compute<MT, A32>(L, a, xq, dx, base, c_end, m0, lane, acc);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
            for (int j = 0; j < MT; j++) acc[r][j] = warp_sum(acc[r][j]);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < 2; r++)
#pragma unroll
                for (int j = 0; j < MT; j++) part[(warp * 2 + r) * MT + j] = acc[r][j];
        }
        __syncthreads();
        if (slice == 0 && p < npairs && lane < 2 && (lane == 0 || has_b)) {
            const int r = lane;
            const int64_t n = r0 + 2 * p + r;
#pragma unroll
            for (int j = 0; j < MT; j++) {
                const int m = m0 + j;
                if (m < a.M) {
                    float v = 0.0f;
                    for (int s = 0; s < wpp; s++) v += part[((warp + s) * 2 + r) * MT + j];
                    if (a.residual) v += a.residual[(int64_t)m * a.ldy + n];
                    a.y[(int64_t)m * a.ldy + n] = v;
                }
            }
        }
        __syncthreads();
    }
}

template <int MT, bool A32>
inline int gemv_launch_t(DeviceState* ds, GemvArgs a, cudaStream_t stream) {
    if (a.K > (1 << 24) || (int64_t)a.M * a.K > (1ll << 31))
        return fail(AXQ8_ERR_UNSUPPORTED, "q8 gemv: K or M*K too large");
    int64_t act = 0;
    if (!A32) {
        act = ((int64_t)a.M * a.K + 15) / 16 * 16 + (int64_t)a.M * (a.K / QK) * 4;
        act = (act + 127) / 128 * 128;
        if (act > kGemvActSmemMax) act = 0;
    }
    a.act_smem = (int)act;
    const size_t smem = (size_t)kPartBytes + (size_t)act;
    // CTAs per SM: 2 fills the SM (best for an isolated GEMV); 1 leaves room
    // for the next kernel's CTAs to co-reside and start their weight loads
    // under programmatic dependent launch.  AXQ8_GEMV_CTAS_PER_SM overrides
    // the default for tuning.
    static const int ctas_per_sm = [] {
        const char* e = getenv("AXQ8_GEMV_CTAS_PER_SM");
        const int v = e ? atoi(e) : kGemvCtasPerSm;
        return v >= 1 && v <= 4 ? v : kGemvCtasPerSm;
    }();
    int64_t grid = (int64_t)ds->sm_count * ctas_per_sm;
    const int64_t max_grid = (a.N + 1) / 2;       // at least one row pair per CTA
    if (grid > max_grid) grid = max_grid;
    // split-K inside the CTA when its row pairs cannot occupy every warp
    const int64_t rows_per_cta = (a.N + grid - 1) / grid;
    const bool split = 2 * ((rows_per_cta + 1) / 2) <= kGemvWarps && a.K >= 1024;
    auto kern = split ? q8_gemv_kernel<MT, A32, true> : q8_gemv_kernel<MT, A32, false>;
    if (smem > 48 * 1024) {
        static int configured_for[2][64] = {{0}};
        const int dev = ds->device < 64 ? ds->device : 63;
        if (!configured_for[split][dev]) {
            AXQ8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kPartBytes + kGemvActSmemMax),
                          "cudaFuncSetAttribute(q8_gemv)");
            configured_for[split][dev] = 1;
        }
    }
    AXQ8_CUDA_TRY(launch_k(kern, dim3((unsigned)grid), dim3(kGemvWarps * 32), smem, stream, true, a),
                  "q8_gemv launch");
    return AXQ8_OK;
}

inline int gemv_launch(DeviceState* ds, const GemvArgs& a, bool a32, cudaStream_t stream) {
    if (a.M <= 1) return a32 ? gemv_launch_t<1, true>(ds, a, stream) : gemv_launch_t<1, false>(ds, a, stream);
    if (a.M <= 2) return a32 ? gemv_launch_t<2, true>(ds, a, stream) : gemv_launch_t<2, false>(ds, a, stream);
    return a32 ? gemv_launch_t<4, true>(ds, a, stream) : gemv_launch_t<4, false>(ds, a, stream);
}

}  // namespace axq8
