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
// memory one chunk ahead.  The K splits of a row tile (blockIdx.y, at most 8)
// run as one thread-block cluster: each CTA leaves its fp32 partial tile in
// shared memory and, after a cluster barrier, every CTA adds one slice of the
// tile over the cluster's partials in split order (distributed shared memory),
// so the combine needs no global workspace and stays deterministic.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cooperative_groups.h>

#include "common.cuh"

namespace axq8 {

constexpr int kMmqWarps = 8;
constexpr int kMmqRows = 16 * kMmqWarps;   // weight rows per CTA
constexpr int kMmqChunkKb = 4;             // 32-blocks per staged chunk (128 bytes of K)
constexpr int kMmqMaxSplits = 8;           // cluster size limit (portable)

// Shared memory of one CTA: the double-buffered activation chunk and scales
// during the main loop, then (split launches) the fp32 partial tile [MR][kMmqTilePitch].
constexpr int kMmqTilePitch = kMmqRows + 4;   // conflict-free fragment stores
template <int MT8>
struct MmqSmem {
    static constexpr int MR = 8 * MT8;
    static constexpr int XS = 2 * MR * kMmqChunkKb * 32;
    static constexpr int DXS = 2 * kMmqChunkKb * MR * 4;
    static constexpr int TILE = MR * kMmqTilePitch * 4;
    static constexpr int BYTES = XS + DXS > TILE ? XS + DXS : TILE;
};

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

// Launched with cluster dimensions (1, gridDim.y, 1) when gridDim.y > 1.
template <int MT8>   // 8-row activation tiles (M <= 8 * MT8)
__global__ void __launch_bounds__(kMmqWarps * 32, 2) q8_mmq_kernel(const MmqArgs a) {
    constexpr uint32_t kMagicBitsI = 0x4B400000u;   // 1.5 * 2^23 as fp32
    constexpr float kMagicF = 12582912.0f;
    using SM = MmqSmem<MT8>;
    constexpr int MR = SM::MR;                      // staged activation rows
    __shared__ __align__(16) uint8_t smem[SM::BYTES];
    auto xs = reinterpret_cast<uint8_t(*)[MR][kMmqChunkKb * 32]>(smem);
    auto dxs = reinterpret_cast<float(*)[kMmqChunkKb][MR]>(smem + SM::XS);
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
    float2 acc[MT8][2];   // [j][0]: row g, columns 8j + 2t (+1); [j][1]: row g + 8
#pragma unroll
    for (int j = 0; j < MT8; j++) acc[j][0] = acc[j][1] = make_float2(0.0f, 0.0f);
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
                const float2 ta = ffma2(make_float2(__int_as_float(d[0]), __int_as_float(d[1])),
                                        make_float2(dwa, dwa), make_float2(nca, nca));
                const float2 tb = ffma2(make_float2(__int_as_float(d[2]), __int_as_float(d[3])),
                                        make_float2(dwb, dwb), make_float2(ncb, ncb));
                acc[j][0] = ffma2(ta, dxv, acc[j][0]);
                acc[j][1] = ffma2(tb, dxv, acc[j][1]);
            }
        }
        Wc = Wn;
        __syncthreads();   // buffer `buf` is free for chunk ch + 2
    }
    if (ch0 >= ch1) cp_async_wait_all();
    // outputs: rows n0 + g (+8), columns 8j + 2t (+1)
    const int splits = gridDim.y;
    if (splits == 1) {
#pragma unroll
        for (int j = 0; j < MT8; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int n = n0 + g + ((e & 2) ? 8 : 0);
                const int m = 8 * j + 2 * t + (e & 1);
                if (n >= a.N || m >= a.M) continue;
                const int64_t o = (int64_t)m * a.ldy + n;
                const float v = (e & 1) ? acc[j][e >> 1].y : acc[j][e >> 1].x;
                a.y[o] = a.residual ? __fadd_rn(a.residual[o], v) : v;
            }
        return;
    }
    // split launch: partial tile -> shared memory, then the cluster's combine
    float* tile = reinterpret_cast<float*>(smem);   // [MR][kMmqTilePitch], over the stage buffers
    __syncthreads();
#pragma unroll
    for (int j = 0; j < MT8; j++)
#pragma unroll
        for (int e = 0; e < 4; e++)
            tile[(8 * j + 2 * t + (e & 1)) * kMmqTilePitch + warp * 16 + g + ((e & 2) ? 8 : 0)] =
                (e & 1) ? acc[j][e >> 1].y : acc[j][e >> 1].x;
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const float* peer[kMmqMaxSplits];
#pragma unroll
    for (int z = 0; z < kMmqMaxSplits; z++)
        peer[z] = z < splits ? cluster.map_shared_rank(tile, z) : tile;
    // this CTA's slice of the M x 128 outputs, in row-major (m, r) order
    const int total = a.M * kMmqRows;
    const int rank = (int)cluster.block_rank();
    const int lo = (int)((int64_t)total * rank / splits), hi = (int)((int64_t)total * (rank + 1) / splits);
    const int nb0 = blockIdx.x * kMmqRows;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int m = i / kMmqRows, r = i % kMmqRows;
        const int off = m * kMmqTilePitch + r;
        float p[kMmqMaxSplits];
#pragma unroll
        for (int z = 0; z < kMmqMaxSplits; z++) p[z] = z < splits ? peer[z][off] : 0.0f;
        float v = 0.0f;
#pragma unroll
        for (int z = 0; z < kMmqMaxSplits; z++)
            if (z < splits) v = __fadd_rn(v, p[z]);
        const int n = nb0 + r;
        if (n < a.N) {
            const int64_t o = (int64_t)m * a.ldy + n;
            a.y[o] = a.residual ? __fadd_rn(a.residual[o], v) : v;
        }
    }
    cluster.sync();   // peers' tiles stay alive until every slice is read
}

}  // namespace axq8
