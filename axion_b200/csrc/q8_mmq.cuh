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
// one 8-byte load from shared memory.
//
// CTA: 8 warps x 16 weight rows = 128 rows over one range of K (blockIdx.y
// splits K when the row tiles are few).  Each 4-block chunk of K — the CTA's
// 128 weight rows (16 KB, 16-byte pieces XOR-swizzled by row, kSwz, so the
// 8-byte fragment reads are conflict-free), their block scales, the activation rows
// (swizzled alike, zero-filled past M and K) and their scales — goes through a
// ring of shared-memory stages (MmqSmem) with cp.async, several chunks in
// flight: a weight stream needs about 44 KB in flight per SM to cover the HBM
// latency, and one chunk ahead in registers left the warps waiting on it.
// The first stages' weights are requested before the dependency wait
// (programmatic dependent launch), the activations after it.  The K splits of
// a row tile (blockIdx.y, at most 8) run as one thread-block cluster: each CTA
// leaves its fp32 partial tile in shared memory (over the stages) and, after a
// cluster barrier, every CTA adds one slice of the tile over the cluster's
// partials in split order (distributed shared memory), so the combine needs
// no global workspace and stays deterministic.
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

constexpr int kMmqTilePitch = kMmqRows + 4;   // fp32 partial tile row: conflict-free stores

// Shared memory of one CTA: MmqSmem<MT8>::STAGES stages (2..6, about 104 KB) of
//   W  [128 rows][128 B]  weight pieces (swizzled)      16 KB
//   WS [128 rows][8 B]    their 4 fp16 block scales      1 KB
//   X  [MR rows][128 B]   activation pieces (swizzled)
//   DX [4 blocks][MR]     activation scales
// then, for split launches, the fp32 partial tile [MR][kMmqTilePitch] over them.
template <int MT8>
struct MmqSmem {
    static constexpr int MR = 8 * MT8;
    static constexpr int W = 0;
    static constexpr int WS = kMmqRows * kMmqChunkKb * 32;
    static constexpr int X = WS + kMmqRows * 8;
    static constexpr int DX = X + MR * kMmqChunkKb * 32;
    static constexpr int STAGE = DX + kMmqChunkKb * MR * 4;
    static constexpr int STAGES = 106496 / STAGE > 6 ? 6 : (106496 / STAGE < 2 ? 2 : 106496 / STAGE);
    static constexpr int TILE = MR * kMmqTilePitch * 4;
    static constexpr int BYTES = STAGES * STAGE > TILE ? STAGES * STAGE : TILE;
};

// Swizzle of a staged 128-byte row: its 16-byte piece p is stored at piece
// p ^ kSwz(row).  A fragment read by a half-warp (4 rows g, 4 lanes t, each
// lane 8 bytes at 32*k4 + 8t of its row) then touches 16 distinct 8-byte slots
// of the 128-byte bank window: 32*(k4 ^ (g & 3)) + 8t.
__device__ __forceinline__ int kSwz(int row) { return (row & 3) << 1; }

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
    // SILU launches: the rows are (gate_j, up_j) pairs; out = A8(silu(gate) * up)
    int8_t* sq;              // [M][N/2]
    float* sdx;              // its block scales: [b * sdxt + m] (sdxt > 0), else [m * N/64 + b]
    int sdxt;
};

__device__ __forceinline__ void mma_s8_16832(int* d, const uint32_t* a, uint32_t b0, uint32_t b1,
                                             int c) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c));
}

// Launched with cluster dimensions (1, gridDim.y, 1) when gridDim.y > 1, and
// MmqSmem<MT8>::BYTES of dynamic shared memory.
// SILU: the weight rows are the stacked gate|up weight stored interleaved
// (gate row j, up row j), N % 64 == 0; instead of y the combine writes
// a = silu(gate) * up, rounded per op as silu_mul_kernel does, quantized to A8
// (quant_block_quad) into sq / sdx: the SiLU*up kernel and the fp32 gate|up
// round trip are folded into the product.
template <int MT8, bool SILU = false>   // 8-row activation tiles (M <= 8 * MT8)
__global__ void __launch_bounds__(kMmqWarps * 32, 2) q8_mmq_kernel(const MmqArgs a) {
    constexpr uint32_t kMagicBitsI = 0x4B400000u;   // 1.5 * 2^23 as fp32
    constexpr float kMagicF = 12582912.0f;
    using SM = MmqSmem<MT8>;
    constexpr int MR = SM::MR;                      // staged activation rows
    constexpr int NST = SM::STAGES;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nbase = blockIdx.x * kMmqRows;
    const int n0 = nbase + warp * 16;
    const int nkb = a.K / 32;
    const int nch = (nkb + kMmqChunkKb - 1) / kMmqChunkKb;
    const int ch0 = blockIdx.y * a.chunks_per_split, ch1 = min(nch, ch0 + a.chunks_per_split);
    // Copy assignment, fixed over the chunks: thread -> 16-byte piece cpc of
    // rows cr + 32q.  kSwz(cr + 32q) == kSwz(cr), so the swizzled piece offset
    // is one per thread, and the rows' global addresses are computed once and
    // advance by 128 bytes per chunk.
    const int cr = threadIdx.x >> 3, cpc = threadIdx.x & 7;
    const int cpiece = (cpc ^ kSwz(cr)) << 4;
    const uint8_t* wsrc[kMmqRows / 32];
#pragma unroll
    for (int q = 0; q < kMmqRows / 32; q++)
        wsrc[q] = a.rows + (int64_t)min(nbase + cr + 32 * q, a.N - 1) * a.row_stride + cpc * 16;
    // 4 fp16 scales per row (the row's scale area is padded to 16 bytes): thread r < 128
    const uint8_t* wssrc = a.rows + (int64_t)min(nbase + (int)threadIdx.x, a.N - 1) * a.row_stride + a.K;
    // weights (and their scales) of chunk ch into stage st
    auto issue_w = [&](int ch, int st) {
        uint8_t* W = smem + st * SM::STAGE + SM::W + cr * 128 + cpiece;
        const bool ok = ch * kMmqChunkKb * 32 + cpc * 16 < a.K;   // a partial last chunk
        const int koff = ok ? ch * kMmqChunkKb * 32 : -cpc * 16;  // zero fill: the row's start
#pragma unroll
        for (int q = 0; q < kMmqRows / 32; q++) cp_async16_zfill(W + q * 32 * 128, wsrc[q] + koff, ok);
        if (threadIdx.x < kMmqRows)
            cp_async8(smem + st * SM::STAGE + SM::WS + threadIdx.x * 8, wssrc + ch * kMmqChunkKb * 2);
    };
    // activation rows and scales of chunk ch into stage st
    auto issue_x = [&](int ch, int st) {
        uint8_t* X = smem + st * SM::STAGE + SM::X + cr * 128 + cpiece;
        const int64_t k = (int64_t)ch * kMmqChunkKb * 32 + cpc * 16;
#pragma unroll
        for (int q = 0; q < (MR + 31) / 32; q++) {
            const int r = cr + 32 * q;
            if (r < MR) {
                const bool ok = r < a.M && k < a.K;
                cp_async16_zfill(X + q * 32 * 128, a.xq + (ok ? (int64_t)r * a.K + k : 0), ok);
            }
        }
        // scales: 4 blocks x MR rows, 16 bytes = 4 rows per copy
        float* DX = reinterpret_cast<float*>(smem + st * SM::STAGE + SM::DX);
        for (int i = threadIdx.x; i < kMmqChunkKb * MR / 4; i += blockDim.x) {
            const int k4 = i / (MR / 4), r4 = (i % (MR / 4)) * 4;
            const int kb = ch * kMmqChunkKb + k4;
            const bool ok = kb < nkb && r4 < a.Mp;
            cp_async16_zfill(DX + k4 * MR + r4, a.dxT + (ok ? (int64_t)kb * a.Mp + r4 : 0), ok);
        }
    };
    float2 acc[MT8][2];   // [j][0]: row g, columns 8j + 2t (+1); [j][1]: row g + 8
#pragma unroll
    for (int j = 0; j < MT8; j++) acc[j][0] = acc[j][1] = make_float2(0.0f, 0.0f);
    // weights are static: the first NST - 1 chunks' weights before the wait
    for (int s = 0; s < NST - 1; s++)
        if (ch0 + s < ch1) issue_w(ch0 + s, s);
    pdl_launch_dependents();
    pdl_wait();
    for (int s = 0; s < NST - 1; s++) {
        if (ch0 + s < ch1) issue_x(ch0 + s, s);
        cp_async_commit();   // group s (group 0 also holds the early weights)
    }
    const int ra = warp * 16 + g, rb = ra + 8;   // this lane's rows in the tile; both & 3 == g & 3
    const int lane_off = (t >> 1) * 16 + (t & 1) * 8;   // byte 8t of a block, within its piece pair
    for (int ch = ch0; ch < ch1; ch++) {
        const int i = ch - ch0;
        cp_async_wait_group<NST - 2>();   // chunk ch has landed
        __syncthreads();                  // ... for every thread; stage (i - 1) % NST is free
        if (ch + NST - 1 < ch1) {
            issue_w(ch + NST - 1, (i + NST - 1) % NST);
            issue_x(ch + NST - 1, (i + NST - 1) % NST);
        }
        cp_async_commit();
        const uint8_t* st = smem + (i % NST) * SM::STAGE;
        const uint8_t* Wl = st + SM::W + ra * 128 + lane_off;   // + the block's piece offset
        const uint8_t* Xl = st + SM::X + g * 128 + lane_off;    // + the block's piece offset + 1024 j
        const float* DXl = reinterpret_cast<const float*>(st + SM::DX) + 2 * t;
        const uint2 sa = *reinterpret_cast<const uint2*>(st + SM::WS + ra * 8);
        const uint2 sb = *reinterpret_cast<const uint2*>(st + SM::WS + rb * 8);
#pragma unroll
        for (int k4 = 0; k4 < kMmqChunkKb; k4++) {
            // bytes 8t..8t+7 of block k4 sit in 16-byte piece 2 k4 + t/2 of the row,
            // stored at piece (2 k4 + t/2) ^ kSwz(g) = (2 k4 ^ kSwz(g)) + t/2
            const int poff = ((2 * k4) ^ kSwz(g)) << 4;
            const uint2 A0 = *reinterpret_cast<const uint2*>(Wl + poff);
            const uint2 A1 = *reinterpret_cast<const uint2*>(Wl + poff + 8 * 128);
            const uint32_t af[4] = {A0.x, A1.x, A0.y, A1.y};
            const uint32_t swa = (k4 < 2 ? sa.x : sa.y) >> ((k4 & 1) * 16);
            const uint32_t swb = (k4 < 2 ? sb.x : sb.y) >> ((k4 & 1) * 16);
            const float dwa = __half2float(__ushort_as_half((unsigned short)(swa & 0xFFFFu)));
            const float dwb = __half2float(__ushort_as_half((unsigned short)(swb & 0xFFFFu)));
            const float nca = -kMagicF * dwa, ncb = -kMagicF * dwb;
#pragma unroll
            for (int j = 0; j < MT8; j++) {
                // activation row 8j + g: kSwz(8j + g) == kSwz(g)
                const uint2 B = *reinterpret_cast<const uint2*>(Xl + poff + j * 8 * 128);
                const float2 dxv = *reinterpret_cast<const float2*>(DXl + k4 * MR + 8 * j);
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
    }
    cp_async_wait_all();   // nothing of this CTA still lands in the stages
    // outputs: rows n0 + g (+8), columns 8j + 2t (+1)
    const int splits = gridDim.y;
    if (!SILU && splits == 1) {
#pragma unroll
        for (int j = 0; j < MT8; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int n = n0 + g + ((e & 2) ? 8 : 0);
                const int m = 8 * j + 2 * t + (e & 1);
                if (n >= a.N || m >= a.M) continue;
                const int64_t o = (int64_t)m * a.ldy + n;
                const float v = (e & 1) ? acc[j][e >> 1].y : acc[j][e >> 1].x;
                a.y[o] = a.residual ? __fadd_rn(ld_cg(a.residual + o), v) : v;
            }
        return;
    }
    // split launch (and every SILU launch): partial tile -> shared memory, then
    // the cluster's combine (a single CTA combines its own tile)
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
    if (splits > 1) cluster.sync();
    else __syncthreads();
    const float* peer[kMmqMaxSplits];
#pragma unroll
    for (int z = 0; z < kMmqMaxSplits; z++)
        peer[z] = z < splits && splits > 1 ? cluster.map_shared_rank(tile, z) : tile;
    const int rank = splits > 1 ? (int)cluster.block_rank() : 0;
    const int nb0 = blockIdx.x * kMmqRows;
    if (SILU) {
        // 32-output blocks of the tile (two per activation row: pairs 0-31,
        // 32-63), whole blocks per CTA; 4 consecutive threads take a block, 8
        // outputs (16 rows) each, the trip count uniform over the CTA for the
        // quantizer's shuffles.  Sums in split order, as the plain combine.
        const int F = a.N / 2, nbf = F / 32;
        const int nblk = a.M * 2;
        const int lo = nblk * rank / splits, hi = nblk * (rank + 1) / splits;
        const int lane = threadIdx.x & 31;
        for (int base = 4 * lo; base < 4 * hi; base += blockDim.x) {
            const int u = base + threadIdx.x;
            const int bk = u >> 2, gq = u & 3;
            const int m = bk >> 1, hb = bk & 1;
            const int r0 = 64 * hb + 16 * gq;
            const bool valid = u < 4 * hi && nb0 + r0 < a.N;
            float act[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                float gs = 0.0f, us = 0.0f;
                if (valid) {
                    const int off = m * kMmqTilePitch + r0 + 2 * e;
                    float pg[kMmqMaxSplits], pu[kMmqMaxSplits];
#pragma unroll
                    for (int z = 0; z < kMmqMaxSplits; z++) {
                        pg[z] = z < splits ? peer[z][off] : 0.0f;
                        pu[z] = z < splits ? peer[z][off + 1] : 0.0f;
                    }
#pragma unroll
                    for (int z = 0; z < kMmqMaxSplits; z++)
                        if (z < splits) {
                            gs = __fadd_rn(gs, pg[z]);
                            us = __fadd_rn(us, pu[z]);
                        }
                }
                act[e] = __fmul_rn(__fdiv_rn(gs, __fadd_rn(1.0f, expf(-gs))), us);
            }
            const int jg = nb0 / 2 + 32 * hb + 8 * gq;   // output index in [0, F)
            const int b = jg / 32;
            quant_block_quad(act, lane, valid, a.sq + (int64_t)(valid ? m : 0) * F + (valid ? jg : 0),
                             a.sdx + (a.sdxt ? (int64_t)b * a.sdxt + m : (int64_t)m * nbf + b));
        }
        if (splits > 1) cluster.sync();   // peers' tiles stay alive until every block is read
        return;
    }
    // this CTA's slice of the M x 128 outputs, in row-major (m, r) order
    const int total = a.M * kMmqRows;
    const int lo = (int)((int64_t)total * rank / splits), hi = (int)((int64_t)total * (rank + 1) / splits);
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
            a.y[o] = a.residual ? __fadd_rn(ld_cg(a.residual + o), v) : v;
        }
    }
    cluster.sync();   // peers' tiles stay alive until every slice is read
}

}  // namespace axq8
