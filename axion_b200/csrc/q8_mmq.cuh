// Skinny Q8_0 x A8 product for decode widths (M <= 64) on the tensor cores
// with register accumulators: mma.sync m16n8k32 s8 x s8 -> s32, one MMA per
// (16 weight rows, 8 activation rows, 32-block), rescaled in registers.
//
// Reference semantics: linear_from_gguf (inference/cpp/kernels/linear.cpp:27-71)
// on the dequantized weight (gguf.cpp:870-882); with A8 activations
// y[m,n] = sum_b dw[n,b] * dx[m,b] * sum_{i<32} qw[n,32b+i] * qx[m,32b+i].
//
// The tcgen05 product reads every block's int32 result back from TMEM; at
// decode widths that round trip (and its barrier hand-off) per block is the
// whole cost.  Here the block result stays in registers:
//   D_b = C + A.B with C preset to the bits of 1.5*2^23, so the float view of
//   D_b is 1.5*2^23 + dot exactly (|dot| < 2^22), and
//   acc = fma(fma(1.5*2^23 + dot, dw, -1.5*2^23*dw), dx, acc)  (first product exact).
// Within a block the k order of the dot is free (an exact integer sum), so
// lane (g, t) takes the 8 contiguous bytes 8t..8t+7 of its rows' block for
// the fragment slots of k 4t..4t+3 and 16+4t..16+4t+3, in the weight (rows g,
// g+8) and the activation (row g of each 8-row tile) alike: every fragment is
// one 8-byte load (global memory for the weights, shared for the activation).
//
// CTA: 8 warps x 16 weight rows = 128 rows over one range of K (blockIdx.y
// splits K when the row tiles are few).  The activation rows and scales of
// each 4-block chunk are staged once per CTA in shared memory with cp.async
// (double buffered; 16-byte chunks XOR-swizzled by row so the 8-byte fragment
// reads are conflict-free; rows past M and bytes past K zero-filled) and shared
// by the 8 warps; each warp's weight fragments come straight from global
// memory one chunk ahead.  A split launch writes partial tiles and its last
// CTA (atomic counter, back to zero) adds them in split order: deterministic.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace axq8 {

constexpr int kMmqWarps = 8;
constexpr int kMmqRows = 16 * kMmqWarps;   // weight rows per CTA
constexpr int kMmqChunkKb = 4;             // 32-blocks per staged chunk (128 bytes of K)

struct MmqArgs {
    const uint8_t* rows;     // repacked Q8R rows
    int64_t row_stride;
    int N, K, M;
    const int8_t* xq;        // [M][K]
    const float* dxT;        // [K/32][Mp]
    int Mp;
    int chunks_per_split;    // 4-block chunks of K per blockIdx.y
    const float* residual;   // optional [M][ldy]
    float* y;                // [M][ldy]
    int ldy;
    float* part;             // [splits][M][N] when gridDim.y > 1
    int* counters;           // [gridDim.x]
};

__device__ __forceinline__ void mma_s8_16832(int* d, const uint32_t* a, uint32_t b0, uint32_t b1,
                                             int c) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c));
}

__device__ __forceinline__ uint2 ldg_nc8(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
}

// One chunk's weight fragments of a lane: rows g and g+8 of its warp's 16,
// bytes 8t..8t+7 of each of the 4 blocks, and the 4 block scales of both rows.
struct MmqWeights {
    uint2 a[kMmqChunkKb][2];
    uint2 s[2];
};

template <int MT8>   // 8-row activation tiles (M <= 8 * MT8)
__global__ void __launch_bounds__(kMmqWarps * 32, 2) q8_mmq_kernel(const MmqArgs a) {
    constexpr uint32_t kMagicBitsI = 0x4B400000u;   // 1.5 * 2^23 as fp32
    constexpr float kMagicF = 12582912.0f;
    constexpr int MR = 8 * MT8;                     // staged activation rows
    __shared__ __align__(16) uint8_t xs[2][MR][kMmqChunkKb * 32];
    __shared__ __align__(16) float dxs[2][kMmqChunkKb][MR];
    __shared__ int last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * kMmqRows + warp * 16;
    const int nkb = a.K / 32;
    const int nch = (nkb + kMmqChunkKb - 1) / kMmqChunkKb;
    const int ch0 = blockIdx.y * a.chunks_per_split, ch1 = min(nch, ch0 + a.chunks_per_split);
    const int ra = min(n0 + g, a.N - 1), rb = min(n0 + g + 8, a.N - 1);
    const uint8_t* wa = a.rows + (int64_t)ra * a.row_stride;
    const uint8_t* wb = a.rows + (int64_t)rb * a.row_stride;
    auto load_w = [&](int ch, MmqWeights& W) {
#pragma unroll
        for (int k4 = 0; k4 < kMmqChunkKb; k4++) {
            const int kb = ch * kMmqChunkKb + k4;
            if (kb < nkb) {
                W.a[k4][0] = ldg_nc8(wa + kb * 32 + 8 * t);
                W.a[k4][1] = ldg_nc8(wb + kb * 32 + 8 * t);
            } else {
                W.a[k4][0] = W.a[k4][1] = make_uint2(0, 0);
            }
        }
        // 4 fp16 scales per row; the row's scale area is padded to 16 bytes
        W.s[0] = ldg_nc8(wa + a.K + ch * kMmqChunkKb * 2);
        W.s[1] = ldg_nc8(wb + a.K + ch * kMmqChunkKb * 2);
    };
    auto stage_x = [&](int ch, int buf) {
        // activation quants: MR rows x 8 chunks of 16 bytes, swizzled by row
        for (int i = threadIdx.x; i < MR * 8; i += blockDim.x) {
            const int r = i >> 3, c = i & 7;
            const int64_t k = (int64_t)ch * kMmqChunkKb * 32 + c * 16;
            const bool ok = r < a.M && k < a.K;
            cp_async16_zfill(&xs[buf][r][(c ^ (r & 7)) * 16], a.xq + (ok ? (int64_t)r * a.K + k : 0), ok);
        }
        // scales: 4 blocks x MR rows, 16 bytes = 4 rows per copy
        for (int i = threadIdx.x; i < kMmqChunkKb * MR / 4; i += blockDim.x) {
            const int k4 = i / (MR / 4), r4 = (i % (MR / 4)) * 4;
            const int kb = ch * kMmqChunkKb + k4;
            const bool ok = kb < nkb && r4 < a.Mp;
            cp_async16_zfill(&dxs[buf][k4][r4], a.dxT + (ok ? (int64_t)kb * a.Mp + r4 : 0), ok);
        }
    };
    float acc[MT8][4];
#pragma unroll
    for (int j = 0; j < MT8; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
    MmqWeights Wc, Wn;
    if (ch0 < ch1) load_w(ch0, Wc);          // weights are static: before the wait
    pdl_launch_dependents();
    pdl_wait();
    if (ch0 < ch1) stage_x(ch0, 0);
    cp_async_commit();
    for (int ch = ch0; ch < ch1; ch++) {
        const int buf = (ch - ch0) & 1;
        if (ch + 1 < ch1) {
            load_w(ch + 1, Wn);
            stage_x(ch + 1, buf ^ 1);
            cp_async_commit();
            cp_async_wait_group<1>();
        } else {
            cp_async_wait_group<0>();
        }
        __syncthreads();
#pragma unroll
        for (int k4 = 0; k4 < kMmqChunkKb; k4++) {
            const uint32_t af[4] = {Wc.a[k4][0].x, Wc.a[k4][1].x, Wc.a[k4][0].y, Wc.a[k4][1].y};
            const uint32_t swa = (k4 < 2 ? Wc.s[0].x : Wc.s[0].y) >> ((k4 & 1) * 16);
            const uint32_t swb = (k4 < 2 ? Wc.s[1].x : Wc.s[1].y) >> ((k4 & 1) * 16);
            const float dwa = __half2float(__ushort_as_half((unsigned short)(swa & 0xFFFFu)));
            const float dwb = __half2float(__ushort_as_half((unsigned short)(swb & 0xFFFFu)));
            const float nca = -kMagicF * dwa, ncb = -kMagicF * dwb;
            // the chunk's 16-byte piece holding bytes 8t..8t+7 of block k4
            const int c16 = (k4 * 32 + 8 * t) >> 4, c8 = (8 * t) & 15;
#pragma unroll
            for (int j = 0; j < MT8; j++) {
                const int r = 8 * j + g;
                const uint2 B = *reinterpret_cast<const uint2*>(&xs[buf][r][((c16 ^ (r & 7)) << 4) + c8]);
                const float2 dxv = *reinterpret_cast<const float2*>(&dxs[buf][k4][8 * j + 2 * t]);
                int d[4];
                mma_s8_16832(d, af, B.x, B.y, (int)kMagicBitsI);
                acc[j][0] = fmaf(fmaf(__int_as_float(d[0]), dwa, nca), dxv.x, acc[j][0]);
                acc[j][1] = fmaf(fmaf(__int_as_float(d[1]), dwa, nca), dxv.y, acc[j][1]);
                acc[j][2] = fmaf(fmaf(__int_as_float(d[2]), dwb, ncb), dxv.x, acc[j][2]);
                acc[j][3] = fmaf(fmaf(__int_as_float(d[3]), dwb, ncb), dxv.y, acc[j][3]);
            }
        }
        Wc = Wn;
        __syncthreads();   // buffer `buf` is free for chunk ch + 2
    }
    if (ch0 >= ch1) cp_async_wait_all();
    // outputs: rows n0 + g (+8), columns 8j + 2t (+1)
    const int splits = gridDim.y;
    float* dst = splits == 1 ? a.y : a.part + (int64_t)blockIdx.y * a.M * a.N;
    const int ld = splits == 1 ? a.ldy : a.N;
#pragma unroll
    for (int j = 0; j < MT8; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int n = n0 + g + ((e & 2) ? 8 : 0);
            const int m = 8 * j + 2 * t + (e & 1);
            if (n >= a.N || m >= a.M) continue;
            const int64_t o = (int64_t)m * ld + n;
            float v = acc[j][e];
            if (splits == 1 && a.residual) v = __fadd_rn(a.residual[o], v);
            dst[o] = v;
        }
    if (splits == 1) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int* c = a.counters + blockIdx.x;
        last = atomicAdd(c, 1) == splits - 1;
        if (last) *c = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int nb0 = blockIdx.x * kMmqRows;
    for (int idx = threadIdx.x; idx < kMmqRows * a.M; idx += blockDim.x) {
        const int r = idx % kMmqRows, m = idx / kMmqRows;
        const int n = nb0 + r;
        if (n >= a.N) continue;
        float v = 0.0f;
        for (int z = 0; z < splits; z++) v = __fadd_rn(v, __ldcg(a.part + ((int64_t)z * a.M + m) * a.N + n));
        const int64_t o = (int64_t)m * a.ldy + n;
        a.y[o] = a.residual ? __fadd_rn(a.residual[o], v) : v;
    }
}

}  // namespace axq8
