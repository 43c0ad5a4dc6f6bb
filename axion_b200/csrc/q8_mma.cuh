// Q8_0 x A8 matrix product on the 5th-generation tensor cores (sm_100a):
// tcgen05.mma kind::i8, operands staged by TMA in 128-byte-swizzled shared
// memory tiles, int32 block dots accumulated in TMEM, per-block rescale in
// the epilogue.
//
// Reference semantics: linear_from_gguf (inference/cpp/kernels/linear.cpp:27-71)
// on the dequantized weight (gguf.cpp:870-882); with A8 activations
// y[m,n] = sum_b dw[n,b] * dx[m,b] * sum_{i<32} qw[n,32b+i] * qx[m,32b+i].
//
// One CTA computes a tile of 128 weight rows (TMEM lanes) x BN activation
// rows (TMEM columns).  Q8_0 scales change every 32 values of K and one
// kind::i8 MMA consumes exactly K = 32, so every MMA is one block: its
// int32 result D_b (exact, |D_b| <= 32*128*128 < 2^22) is read back by the
// epilogue warps, scaled and added to fp32 accumulators held in registers:
//     t   = D_b * dw   (exact product, one rounding: the integer add of the
//                       bits of 1.5*2^23 turns D_b into the float 1.5*2^23 + D_b,
//                       then fma(1.5*2^23 + D_b, dw, -1.5*2^23*dw))
//     acc = fma(t, dx, acc)
// TMEM holds four D buffers, one per block of a 4-block stage; each MMA
// overwrites its buffer, and the epilogue hands a buffer back to the MMA
// issuer as soon as its 32 columns are in registers, so the MMAs of the next
// blocks run while block b is rescaled.
//
// Warp roles: warp 0 lane 0 issues TMA loads (weight quants [128 x 128 B],
// activation quants [BN x 128 B], transposed activation scales [4 x BN] fp32
// per 4-block stage), warp 1 lane 0 issues the MMAs, warps 2-3 idle; warps
// 4.. are the epilogue, BN/8 of them (warp w reads TMEM lanes 32*(w%4).. and
// the 32 columns of group (w-4)/4).  For BN >= 64 warpgroup 0 hands registers
// to the epilogue warpgroups (setmaxnreg), which hold 32 accumulators and 32
// TMEM values per thread.  Every wait is bounded (WAIT_BUDGET_CYCLES); a
// wait that gives up records AXQ8_ERR_WAIT_TIMEOUT and its role stops, the
// CTA then waits (bounded) for its MMAs to retire and frees TMEM.
//
// Split-K: with few output tiles, blockIdx.z takes a contiguous range of
// stages; partial tiles go to a workspace and the last CTA of a tile (atomic
// counter, returned to zero) adds them in split order (deterministic) and
// writes y (+ residual).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace axq8 {

constexpr int kMmaBM = 128;          // weight rows per tile (TMEM lanes)
constexpr int kMmaKC = 128;          // K bytes per stage: one 128-byte swizzle row = 4 blocks
constexpr uint32_t kMagicBits = 0x4B400000u;   // 1.5 * 2^23 as fp32
constexpr float kMagic = 12582912.0f;

template <int BN>
struct MmaCfg {
    static_assert(BN == 32 || BN == 64 || BN == 128, "BN");
    static constexpr int W_BYTES = kMmaBM * kMmaKC;          // 16 KB
    static constexpr int X_BYTES = BN * kMmaKC;
    static constexpr int D_BYTES = 4 * BN * 4;                // [4 blocks][BN] fp32
    static constexpr int STAGE = (W_BYTES + X_BYTES + D_BYTES + 1023) / 1024 * 1024;
    // BN = 64 runs two CTAs per SM: two independent pipelines overlap one
    // CTA's TMEM traffic with the other's rescale arithmetic
    static constexpr int CTAS_PER_SM = BN == 64 ? 2 : 1;
    static constexpr int SMEM_BUDGET = CTAS_PER_SM == 2 ? 100 * 1024 : 200 * 1024;
    static constexpr int STAGES = SMEM_BUDGET / STAGE > 8 ? 8 : SMEM_BUDGET / STAGE;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = 1024 /* alignment slack */ + STAGES * STAGE + BAR_BYTES;
    static constexpr int NBUF = 4;                            // D buffers: one per block of a stage
    static constexpr int TMEM_COLS = NBUF * BN;
    static constexpr int CW = 32;                             // columns per epilogue thread
    static constexpr int EPI_WARPS = 4 * (BN / CW);           // 4 lane quarters x column groups
    static constexpr int EPI_WARP0 = 4;                       // warpgroup 0: TMA, MMA, two idle warps
    static constexpr int THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
    // Register split (setmaxnreg) where the launch cap would make the
    // epilogue spill: warpgroup 0 gives registers back, the epilogue
    // warpgroups take them.  The CTA's pool is THREADS x the launch register
    // count, which the launcher checks against LAUNCH_REGS_MIN before launching
    // (setmaxnreg.inc waits until the pool can serve it).
    static constexpr bool REG_SPLIT = BN >= 64;
    static constexpr int REGS_WG0 = 32;
    static constexpr int REGS_EPI = BN == 128 ? 112 : 104;
    static constexpr int LAUNCH_REGS_MIN =
        (128 * REGS_WG0 + EPI_WARPS * 32 * REGS_EPI + THREADS - 1) / THREADS;
};

struct MmaArgs {
    const uint8_t* rows;    // repacked Q8R weight rows (scales follow the K quants)
    int64_t row_stride;
    int N, K, M;
    int stages_per_split;   // stages of K per blockIdx.z
    const float* residual;  // optional [M][ldy]
    float* y;               // [M][ldy]
    int ldy;
    float* part;            // split-K partials [splits][M][N]
    int* counters;          // one per (m tile, n tile), zero between launches
    int32_t* dots;          // optional [M][N][K/32] raw block dots (debug)
    int* status;
};

// ---- tcgen05 / TMA wrappers ---------------------------------------------------

__device__ inline void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ inline void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ inline void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ inline void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// D[tmem] (=|+=) A[smem desc] . B[smem desc]^T, int8 x int8 -> int32.
__device__ inline void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes, and the wait
// for them: the registers of the load are tied to the wait so no use of
// them is scheduled before it.
__device__ inline void tmem_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
        "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
        "%30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
          "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
          "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ inline void tmem_wait_ld32(uint32_t* r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}
template <int N>
__device__ inline void setmaxnreg_dec() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ inline void setmaxnreg_inc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// 2-D tiled TMA load (no multicast) into shared memory, completion as
// transaction bytes on `bar`.  x (innermost) must be a multiple of 16 bytes.
__device__ inline void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], "
        "[%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile written by TMA
// with 128-byte swizzling: rows of 128 bytes, 8-row groups 1024 bytes apart
// (SBO), leading offset field 1 (unused for swizzled K-major), descriptor
// version 1 (bits 46-47), swizzle mode 2 = 128 B (bits 61-63).  The tile
// must start on a 1024-byte boundary; advancing K inside the 128-byte row
// adds bytes/16 to the start address field.
__device__ inline uint64_t sw128_kmajor_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A and B signed
// int8 (bits 7-9, 10-12 = 1), both K-major, N>>3 at bit 17, M>>4 at bit 24.
__host__ __device__ constexpr uint32_t mma_i8_idesc(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ inline bool wait_or_flag(uint64_t* bar, uint32_t parity, int* status, volatile int* abort) {
    if (*abort) return false;
    if (mbar_wait_bounded(bar, parity, status, AXQ8_ERR_WAIT_TIMEOUT)) return true;
    *abort = 1;
    return false;
}

template <int BN, bool DOTS>
__global__ void __launch_bounds__(MmaCfg<BN>::THREADS, MmaCfg<BN>::CTAS_PER_SM)
    q8_mma_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                  const __grid_constant__ CUtensorMap tm_d, const MmaArgs a) {
    using C = MmaCfg<BN>;
    constexpr int S = C::STAGES;
    constexpr int CW = C::CW;
    constexpr int EW = C::EPI_WARPS;
    constexpr int NB = C::NBUF;
    extern __shared__ uint8_t mma_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(mma_smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * C::STAGE);
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;     // [NB] D buffer written
    uint64_t* tempty = tfull + NB;   // [NB] D buffer read back
    uint64_t* done = tempty + NB;    // every MMA retired
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* last_flag = reinterpret_cast<int*>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // m tiles vary fastest: CTAs in flight together share weight tiles in L2
    const int m0 = blockIdx.x * BN, n0 = blockIdx.y * kMmaBM;
    const int nst_total = a.K / kMmaKC;
    const int st0 = blockIdx.z * a.stages_per_split;
    const int st1 = min(nst_total, st0 + a.stages_per_split);
    const int nst = max(0, st1 - st0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + EW);
        }
        for (int b = 0; b < NB; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], EW);
        }
        mbar_init(done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch_dependents();
    pdl_wait();

    auto stage_w = [&](int s) { return smem + s * C::STAGE; };
    auto stage_x = [&](int s) { return smem + s * C::STAGE + C::W_BYTES; };
    auto stage_d = [&](int s) {
        return reinterpret_cast<float*>(smem + s * C::STAGE + C::W_BYTES + C::X_BYTES);
    };

    if (warp < C::EPI_WARP0) {
        if (C::REG_SPLIT) setmaxnreg_dec<C::REGS_WG0>();
        if (warp == 0) {
            if (lane == 0) {
                int issued = 0;
                for (int i = 0; i < nst; i++) {
                    const int s = i % S, u = i / S;
                    if (!wait_or_flag(&empty[s], (u & 1) ^ 1, a.status, abort)) break;
                    mbar_arrive_expect_tx(&full[s], C::W_BYTES + C::X_BYTES + C::D_BYTES);
                    const int st = st0 + i;
                    tma_load_2d(stage_w(s), &tm_w, st * kMmaKC, n0, &full[s]);
                    tma_load_2d(stage_x(s), &tm_x, st * kMmaKC, m0, &full[s]);
                    tma_load_2d(stage_d(s), &tm_d, m0, st * 4, &full[s]);
                    issued++;
                }
                // no copy may still be landing when the CTA exits
                for (int i = max(0, issued - S); i < issued; i++)
                    mbar_wait_bounded(&full[i % S], (i / S) & 1, a.status, AXQ8_ERR_WAIT_TIMEOUT);
            }
        } else if (warp == 1) {
            if (lane == 0) {
                const uint32_t idesc = mma_i8_idesc(kMmaBM, BN);
                for (int i = 0; i < nst; i++) {
                    const int s = i % S, u = i / S;
                    if (!wait_or_flag(&full[s], u & 1, a.status, abort)) break;
                    tc_fence_after();
                    const uint64_t ad = sw128_kmajor_desc(smem_u32(stage_w(s)));
                    const uint64_t bd = sw128_kmajor_desc(smem_u32(stage_x(s)));
                    bool ok = true;
                    for (int k4 = 0; k4 < 4; k4++) {       // D buffer k4 holds block 4i+k4
                        if (!wait_or_flag(&tempty[k4], (i & 1) ^ 1, a.status, abort)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        mma_i8(tmem + k4 * BN, ad + 2 * k4, bd + 2 * k4, idesc, 0);   // D_b overwrites
                        tc_commit(&tfull[k4]);
                    }
                    if (!ok) break;
                    tc_commit(&empty[s]);
                }
                tc_commit(done);
            }
        }
    } else {
        if (C::REG_SPLIT) setmaxnreg_inc<C::REGS_EPI>();
        // epilogue
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int half = (warp - C::EPI_WARP0) >> 2;   // column group
        const int nl = q * 32 + lane;           // row of the tile
        const int n = n0 + nl;
        const int nc = min(n, a.N - 1);
        const uint8_t* srow = a.rows + (int64_t)nc * a.row_stride + a.K;   // fp16 scales
        const int kb0 = st0 * 4;
        float2 acc[CW / 2];
#pragma unroll
        for (int j = 0; j < CW / 2; j++) acc[j] = make_float2(0.0f, 0.0f);
        // weight scales of this row, 8 blocks (16 bytes) per load, one group ahead
        const int nbt = a.K / QK;
        uint4 sc_cur = __ldg(reinterpret_cast<const uint4*>(srow + (kb0 & ~7) * 2));
        uint4 sc_nxt = make_uint4(0, 0, 0, 0);
        if ((kb0 & ~7) + 8 < nbt)
            sc_nxt = __ldg(reinterpret_cast<const uint4*>(srow + ((kb0 & ~7) + 8) * 2));
        const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + half * CW;
        // One TMEM load (32 columns) and one wait per block; the buffer goes
        // back to the MMA issuer as soon as it is in registers, before the
        // rescale.  D_b arrives as a plain int32: the integer add of the bits
        // of 1.5*2^23 (ALU pipe) gives the float 1.5*2^23 + D_b, exact for
        // |D_b| < 2^22.  Waits are warp-uniform: the TMEM accesses are .sync.aligned.
        uint32_t r[CW];
        bool ok = nst > 0 && __all_sync(0xffffffffu, wait_or_flag(&full[0], 0, a.status, abort));
        for (int i = 0; ok && i < nst; i++) {
            const int s = i % S;
            const int kbase = kb0 + 4 * i;                 // multiple of 4
            if (i > 0) {
                if (!__all_sync(0xffffffffu, wait_or_flag(&full[s], (i / S) & 1, a.status, abort))) break;
                if ((kbase & 7) == 0) {
                    sc_cur = sc_nxt;
                    if (kbase + 8 < nbt)
                        sc_nxt = __ldg(reinterpret_cast<const uint4*>(srow + (kbase + 8) * 2));
                }
            }
            const uint32_t w01 = (kbase & 4) ? sc_cur.z : sc_cur.x;
            const uint32_t w23 = (kbase & 4) ? sc_cur.w : sc_cur.y;
            const float* dxs = stage_d(s) + half * CW;
#pragma unroll 1
            for (int k4 = 0; k4 < 4; k4++) {              // block kbase + k4 is in D buffer k4
                if (!__all_sync(0xffffffffu, wait_or_flag(&tfull[k4], i & 1, a.status, abort))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                tmem_ld32(tq + k4 * BN, r);
                const uint32_t wsel = ((k4 & 2) ? w23 : w01) >> ((k4 & 1) * 16);
                const float dw = __half2float(__ushort_as_half((unsigned short)(wsel & 0xFFFFu)));
                const float ncw = -kMagic * dw;
                const float2 dw2 = make_float2(dw, dw), ncw2 = make_float2(ncw, ncw);
                const float* dxb = dxs + k4 * BN;
                tmem_wait_ld32(r);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[k4]);   // buffer k4 free for block kbase + k4 + 4
                if (DOTS && n < a.N) {
                    const int nb = a.K / QK;
#pragma unroll
                    for (int j = 0; j < CW; j++) {
                        const int m = m0 + half * CW + j;
                        if (m < a.M) a.dots[((int64_t)m * a.N + n) * nb + kbase + k4] = (int32_t)r[j];
                    }
                }
#pragma unroll
                for (int j = 0; j < CW; j += 4) {
                    const float4 d4 = *reinterpret_cast<const float4*>(dxb + j);
                    const float2 t0 = ffma2(make_float2(__uint_as_float(r[j] + kMagicBits),
                                                        __uint_as_float(r[j + 1] + kMagicBits)),
                                            dw2, ncw2);
                    const float2 t1 = ffma2(make_float2(__uint_as_float(r[j + 2] + kMagicBits),
                                                        __uint_as_float(r[j + 3] + kMagicBits)),
                                            dw2, ncw2);
                    acc[j / 2] = ffma2(t0, make_float2(d4.x, d4.y), acc[j / 2]);
                    acc[j / 2 + 1] = ffma2(t1, make_float2(d4.z, d4.w), acc[j / 2 + 1]);
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);   // the stage's activation scales are read
        }
        // ---- output ----
        const int splits = gridDim.z;
        if (splits == 1) {
            if (n < a.N) {
#pragma unroll
                for (int j = 0; j < CW; j++) {
                    const int m = m0 + half * CW + j;
                    if (m < a.M) {
                        const float v = (j & 1) ? acc[j / 2].y : acc[j / 2].x;
                        const int64_t o = (int64_t)m * a.ldy + n;
                        a.y[o] = a.residual ? __fadd_rn(ld_cg(a.residual + o), v) : v;
                    }
                }
            }
        } else {
            float* pz = a.part + (int64_t)blockIdx.z * a.M * a.N;
            if (n < a.N) {
#pragma unroll
                for (int j = 0; j < CW; j++) {
                    const int m = m0 + half * CW + j;
                    if (m < a.M) pz[(int64_t)m * a.N + n] = (j & 1) ? acc[j / 2].y : acc[j / 2].x;
                }
            }
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"n"(EW * 32) : "memory");
            if (warp == C::EPI_WARP0 && lane == 0) {
                int* c = a.counters + blockIdx.y * gridDim.x + blockIdx.x;
                const int last = atomicAdd(c, 1) == splits - 1;
                if (last) *c = 0;
                *last_flag = last;
            }
            asm volatile("bar.sync 1, %0;" ::"n"(EW * 32) : "memory");
            if (*last_flag && n < a.N) {
                __threadfence();
                // the thread's CW outputs in batches of 16: each split's 16
                // loads are in flight together, the adds stay in split order
#pragma unroll
                for (int j0 = 0; j0 < CW; j0 += 16) {
                    const int mb = m0 + half * CW + j0;
                    if (mb >= a.M) break;
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] = 0.0f;
                    for (int z = 0; z < splits; z++) {
                        const float* pz2 = a.part + ((int64_t)z * a.M + mb) * a.N + n;
                        float p[16];
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            p[j] = mb + j < a.M ? __ldcg(pz2 + (int64_t)j * a.N) : 0.0f;
#pragma unroll
                        for (int j = 0; j < 16; j++) v[j] = __fadd_rn(v[j], p[j]);
                    }
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        if (mb + j >= a.M) break;
                        const int64_t o = (int64_t)(mb + j) * a.ldy + n;
                        a.y[o] = a.residual ? __fadd_rn(ld_cg(a.residual + o), v[j]) : v[j];
                    }
                }
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        // every MMA this CTA issued has retired before TMEM is released
        mbar_wait_bounded(done, 0, a.status, AXQ8_ERR_WAIT_TIMEOUT);
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// Activation quantization for the tensor-core path: xq [M][K] int8 (same
// convention as quantize_act_kernel) and the scales transposed, dxT [K/32][Mp].
__global__ void quantize_act_t_kernel(const float* __restrict__ x, int M, int K, int Mp,
                                      int8_t* __restrict__ xq, float* __restrict__ dxT) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int nb = K / QK;
    const int64_t nblocks = (int64_t)M * nb;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t blk = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); blk < nblocks;
         blk += warps) {
        const float v = ld_cg(x + blk * QK + lane);
        const uint32_t abits = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
        const float amax = __uint_as_float(abits);
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
        xq[blk * QK + lane] = (int8_t)q8_round(__fmul_rn(v, id));
        if (lane == 0) {
            const int m = (int)(blk / nb), b = (int)(blk % nb);
            dxT[(int64_t)b * Mp + m] = d;
        }
    }
}

// dx [M][K/32] -> dxT [K/32][Mp].
__global__ void transpose_scales_kernel(const float* __restrict__ dx, int M, int nb, int Mp,
                                        float* __restrict__ dxT) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t total = (int64_t)M * nb;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / nb), b = (int)(i % nb);
        dxT[(int64_t)b * Mp + m] = ld_cg(dx + i);
    }
}

}  // namespace axq8
