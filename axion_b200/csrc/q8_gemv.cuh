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
//  * two CTAs of 16 warps per SM, each CTA owning a contiguous range of row
//    PAIRS (rows 2p, 2p+1);
//  * each warp reduces one row pair at a time with kChunks 16-byte loads per
//    row per lane in flight (non-allocating, read-once);
//  * the warp's first loads are issued before griddepcontrol.wait: weights do
//    not depend on the previous kernel, so under programmatic dependent launch
//    their HBM latency overlaps the tail of the kernel producing the input;
//  * when a CTA has fewer row pairs than warps (short N, long K), the K range
//    of each pair is split over several warps and the partial sums are
//    reduced through shared memory in a fixed order (SPLIT instantiation).
//
// Prologues (PRO) produce the activation after the dependency wait:
//   PRO_Q8    pre-quantized xq/dx (staged in shared memory when it fits);
//   PRO_F32   fp32 x read from global memory (A32);
//   PRO_RMS   RMSNorm of src[M,K] by norm_w, quantized to Q8 in shared memory
//             (every CTA computes the same bytes; replaces a producer kernel);
//   PRO_QNT   fp32 src[M, K] quantized to Q8 in shared memory (the SiLU*up
//             rows an EPI_SILU launch wrote).
// Epilogues (EPI) consume the two sums of a row pair:
//   EPI_STORE   y = residual + sum;
//   EPI_ROPE_KV the rows of Q and K are stored permuted so that a pair is
//               (dim j, dim j + hd/2) of one head: rotate (NEOX RoPE) and
//               write q back in natural order / k into the KV pages; v rows
//               go to the V pages (replaces rope_apply_row_at + append_row);
//   EPI_SILU    the rows are (gate_j, up_j) pairs (the stacked gate|up weight
//               stored interleaved): y[m, j] = silu(gate_j) * up_j, rounded per op
//               as silu.cpp:53-61 and elementwise.cpp:55-63 do (ldy = N / 2);
//   EPI_ARGMAX  store the logits and reduce the greedy argmax over the grid
//               (packed atomicMax); the last CTA to finish advances the
//               decode state (next input token, position, generated token).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>
#include <stdlib.h>

#include "axq8.h"
#include "common.cuh"
#include "runtime.h"

namespace axq8 {

enum { PRO_Q8 = 0, PRO_F32 = 1, PRO_RMS = 2, PRO_QNT = 3 };
enum { EPI_STORE = 0, EPI_ROPE_KV = 1, EPI_ARGMAX = 2, EPI_SILU = 3 };

struct GemvArgs {
    const uint8_t* rows;      // Q8R rows
    int64_t N, K, row_stride;
    int M;
    const int8_t* xq;         // PRO_Q8: [M, K] int8, 16-byte aligned
    const float* dx;          // PRO_Q8: [M, K/32]
    const float* x;           // PRO_F32: [M, K] fp32, 16-byte aligned
    const float* residual;    // nullable, [M, ldy]
    float* y;                 // [M, ldy]
    int64_t ldy;
    int* status;
    int act_smem;             // bytes of staged activation (0: read from global)
    // PRO_RMS / PRO_QNT
    const float* src;         // RMS, QNT: [M, K]
    const float* norm_w;      // RMS weight [K]
    float eps;
    // EPI_ROPE_KV
    int* pos;                 // [M] (advanced by the EPI_ARGMAX tail)
    const float2* rope;       // [max_ctx][hd/2] (cos, sin)
    int max_ctx, n_heads, n_kv, hd;
    void* kc;                 // [pages][n_kv][B][hd]
    void* vc;
    const int* block_table;   // [M][max_blocks]
    int max_blocks, kv_block;
    // EPI_ARGMAX
    unsigned long long* amax_key;  // [M], zero between uses
    int* done;                     // grid completion counter, zero between uses
    int* tokens;                   // [M] next input token
    const int* feed;               // [M][feed_len]
    const int* ctl;                // {n_prompt, feed_len, max_out}
    int* out_tokens;               // [M][max_out]
    int* argmax_out;               // [M]
    int idx_offset;                // vocabulary index of row 0 (tensor-parallel LM head slice)
    int no_advance;                // 1: leave the keys for a cross-rank reduction, no advance
};

constexpr int kGemvWarps = 16;                 // warps per CTA
constexpr int kGemvCtasPerSm = 2;
constexpr int kChunks = 4;                     // 16-byte loads per row per lane in flight
constexpr int kGemvActSmemMax = 32 * 1024;     // largest staged activation
constexpr int kGemvMaxMT = 4;
constexpr int kPartBytes = kGemvWarps * 2 * kGemvMaxMT * 4;   // split-K partials / scratch

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
        const float4 v = __ldcg(x4 + i);
        const int q = ws[i];
        s = fmaf(v.x, (float)(int8_t)(q & 0xff), s);
        s = fmaf(v.y, (float)(int8_t)((q >> 8) & 0xff), s);
        s = fmaf(v.z, (float)(int8_t)((q >> 16) & 0xff), s);
        s = fmaf(v.w, (float)(int8_t)((q >> 24) & 0xff), s);
    }
    return s;
}

__device__ inline float kv_to_float(__half v) { return __half2float(v); }
__device__ inline float kv_to_float(float v) { return v; }
__device__ inline void kv_store(__half* p, float v) { *p = __float2half_rn(v); }
__device__ inline void kv_store(float* p, float v) { *p = v; }

// Quantize one 32-block held one element per lane (all 32 lanes active),
// the convention of axq8_quantize_act.
__device__ __forceinline__ void quant_block_warp(float v, int lane, int8_t* q, float* d) {
    const uint32_t abits = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
    const float amax = __uint_as_float(abits);
    const float id = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
    q[lane] = (int8_t)q8_round(__fmul_rn(v, id));
    if (lane == 0) *d = __fdiv_rn(amax, 127.0f);
}

// Orderable 64-bit key of (logit, index): larger logit wins, then the smaller
// index (the first maximum, as the reference's greedy argmax keeps).
__device__ inline unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}
__device__ inline int argmax_key_index(unsigned long long k) {
    return (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
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
                                             const int8_t* xq, const float* dx, int base, int cend,
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
__device__ __forceinline__ void acc_zero(float (&acc)[2][MT]) {
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int j = 0; j < MT; j++) acc[r][j] = 0.0f;
}

constexpr int kArgmaxMaxM = 64;   // sequences an EPI_ARGMAX launch reduces

// Epilogue of one row pair (rows n, n+1) for activation row m, run by one
// lane holding both sums.  EPI_ARGMAX folds each stored logit into the CTA's
// shared key of row m.
template <int EPI, typename KV>
__device__ __forceinline__ void epi_pair(const GemvArgs& a, int m, int64_t n, bool has_b,
                                         float v0, float v1, unsigned long long* keys) {
    if (EPI == EPI_ROPE_KV) {
        const int hd = a.hd, half = hd / 2, B = a.kv_block;
        const int64_t Nq = (int64_t)a.n_heads * hd, Nkv = (int64_t)a.n_kv * hd;
        const int p = ld_cg(a.pos + m);
        if (p < 0 || p >= a.max_ctx) {
            record_status(a.status, AXQ8_ERR_INVALID);
            return;
        }
        const int page = a.block_table[m * a.max_blocks + p / B];
        const int slot = p % B;
        if (n < Nq + Nkv) {
            const bool isk = n >= Nq;
            const int local = (int)(n - (isk ? Nq : 0));
            const int head = local / hd, j = (local % hd) >> 1;
            const float2 cs = a.rope[(int64_t)p * half + j];
            const float r0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
            const float r1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
            if (!isk) {
                float* q = a.y + (int64_t)m * a.ldy + (int64_t)head * hd;
                q[j] = r0;
                q[j + half] = r1;
            } else {
                KV* dst = static_cast<KV*>(a.kc) + (((int64_t)page * a.n_kv + head) * B + slot) * hd;
                kv_store(dst + j, r0);
                kv_store(dst + j + half, r1);
            }
        } else {
            const int d0 = (int)(n - Nq - Nkv);
            const int head = d0 / hd, d = d0 % hd;
            KV* dst = static_cast<KV*>(a.vc) + (((int64_t)page * a.n_kv + head) * B + slot) * hd + d;
            kv_store(dst, v0);
            if (has_b) kv_store(dst + 1, v1);
        }
        return;
    }
    if (EPI == EPI_SILU) {   // rows n, n + 1 = gate_j, up_j with j = n / 2
        const float act = __fmul_rn(__fdiv_rn(v0, __fadd_rn(1.0f, expf(-v0))), v1);
        a.y[(int64_t)m * a.ldy + n / 2] = act;
        return;
    }
#pragma unroll
    for (int r = 0; r < 2; r++) {
        if (r == 1 && !has_b) break;
        float v = r ? v1 : v0;
        if (a.residual) v += ld_cg(a.residual + (int64_t)m * a.ldy + n + r);
        a.y[(int64_t)m * a.ldy + n + r] = v;
        if (EPI == EPI_ARGMAX) atomicMax(keys + m, argmax_key(v, (int)(n + r) + a.idx_offset));
    }
}

// Fused prologues.  Their inputs are first copied to a shared-memory staging
// area with cp.async (every 16-byte copy in flight at once, no registers
// held), then thread t handles 4 consecutive elements at a time; the 8 lanes
// holding one 32-block quantize it together.
constexpr int kProMaxK = 8192;                      // largest K of a fused prologue
constexpr int kProStageMax = 64 * 1024;             // largest staging area

// Quantize the 4 values a lane holds; the block is 8 consecutive lanes.
__device__ __forceinline__ void quant_quad(const float (&v)[4], int lane, int8_t* q4, float* d) {
    float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float id = a == 0.0f ? 0.0f : __fdiv_rn(127.0f, a);
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; i++)
        packed |= (uint32_t)(uint8_t)(int8_t)q8_round(__fmul_rn(v[i], id)) << (8 * i);
    *reinterpret_cast<uint32_t*>(q4) = packed;
    if ((lane & 7) == 0) *d = __fdiv_rn(a, 127.0f);
}

// PRO_RMS: act <- Q8(rmsnorm(src[m,:]) * w): out = (x * (1/sqrt(mean(x^2) +
// eps))) * w with the reference's separately rounded operations
// (rmsnorm.cpp:47-96); the sum of squares is a fixed tree.
// stage: x [M][K] then w [K] (fp32).
template <int NW>
__device__ __forceinline__ void prologue_rms(const GemvArgs& a, int8_t* act_q, float* act_d,
                                             float* red, float* stage) {
    const int K = (int)a.K, nb = K / QK, M = a.M;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int T = NW * 32;
    float* xs = stage;
    float* ws = stage + (int64_t)M * K;
    for (int i = threadIdx.x; i < M * K / 4; i += T) cp_async16(xs + 4 * i, a.src + 4 * i);
    for (int i = threadIdx.x; i < K / 4; i += T) cp_async16(ws + 4 * i, a.norm_w + 4 * i);
    cp_async_wait_all();
    __syncthreads();
    for (int m = 0; m < M; m++) {
        const float4* x4 = reinterpret_cast<const float4*>(xs + (int64_t)m * K);
        float s = 0.0f;
        for (int q = threadIdx.x; q < K / 4; q += T) {
            const float4 v = x4[q];
            s = fmaf(v.x, v.x, s);
            s = fmaf(v.y, v.y, s);
            s = fmaf(v.z, v.z, s);
            s = fmaf(v.w, v.w, s);
        }
        s = warp_sum(s);
        if (lane == 0) red[warp] = s;
        __syncthreads();
        float t = lane < NW ? red[lane] : 0.0f;
        t = warp_sum(t);
        const float ms = __fdiv_rn(t, (float)K);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
        const float4* w4 = reinterpret_cast<const float4*>(ws);
        for (int q0 = 0; q0 < K / 4; q0 += T) {      // uniform trip count: the 8-lane groups
            const int q = q0 + threadIdx.x;          // of a block are whole (K % 32 == 0)
            if (q < K / 4) {
                const float4 xv = x4[q], wv = w4[q];
                const float v[4] = {__fmul_rn(__fmul_rn(xv.x, inv), wv.x),
                                    __fmul_rn(__fmul_rn(xv.y, inv), wv.y),
                                    __fmul_rn(__fmul_rn(xv.z, inv), wv.z),
                                    __fmul_rn(__fmul_rn(xv.w, inv), wv.w)};
                quant_quad(v, lane, act_q + m * K + 4 * q, act_d + m * nb + q / 8);
            }
        }
        __syncthreads();   // red reused by the next row; act complete
    }
}

// PRO_QNT: act <- Q8(src[m, :]).  stage: src [M][K].
template <int NW>
__device__ __forceinline__ void prologue_qnt(const GemvArgs& a, int8_t* act_q, float* act_d,
                                             float* stage) {
    const int K = (int)a.K, nb = K / QK, M = a.M;
    const int lane = threadIdx.x & 31;
    constexpr int T = NW * 32;
    for (int i = threadIdx.x; i < M * K / 4; i += T) cp_async16(stage + 4 * i, a.src + 4 * i);
    cp_async_wait_all();
    __syncthreads();
    for (int m = 0; m < M; m++) {
        const float4* x4 = reinterpret_cast<const float4*>(stage + (int64_t)m * K);
        for (int q0 = 0; q0 < K / 4; q0 += T) {      // uniform trip count: whole 8-lane groups
            const int q = q0 + threadIdx.x;
            if (q < K / 4) {
                const float4 xv = x4[q];
                const float v[4] = {xv.x, xv.y, xv.z, xv.w};
                quant_quad(v, lane, act_q + m * K + 4 * q, act_d + m * nb + q / 8);
            }
        }
    }
    __syncthreads();
}

// EPI_ARGMAX tail: grid reduction of the CTA keys by packed atomicMax, and
// the decode-state advance by the last CTA (the completion counter pattern:
// fence, count, fence).
__device__ __forceinline__ void argmax_tail(const GemvArgs& a, const unsigned long long* keys) {
    __syncthreads();
    for (int m = threadIdx.x; m < a.M; m += blockDim.x)
        if (keys[m]) atomicMax(a.amax_key + m, keys[m]);
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) last = atomicAdd(a.done, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (a.no_advance) {     // the keys go to a cross-rank max first (argmax_advance_kernel)
        if (threadIdx.x == 0) *a.done = 0;
        return;
    }
    {   // one thread per sequence
        const int n_prompt = ld_cg(a.ctl), feed_len = ld_cg(a.ctl + 1), max_out = ld_cg(a.ctl + 2);
        for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
            const unsigned long long k = atomicExch(a.amax_key + m, 0ull);
            const int idx = k == 0ull ? 0 : argmax_key_index(k);
            const int p = ld_cg(a.pos + m);
            const int np = p + 1;
            a.argmax_out[m] = idx;
            if (np >= n_prompt && np - n_prompt < max_out)
                a.out_tokens[m * max_out + (np - n_prompt)] = idx;
            a.tokens[m] = np < feed_len ? ld_cg(a.feed + m * feed_len + np) : idx;
            a.pos[m] = np;
        }
        if (threadIdx.x == 0) *a.done = 0;
    }
}

template <int MT, int PRO, int EPI, bool SPLIT, typename KV>
__global__ void __launch_bounds__(kGemvWarps * 32, kGemvCtasPerSm) q8_gemv_kernel(const GemvArgs a) {
    constexpr bool A32 = PRO == PRO_F32;
    extern __shared__ __align__(128) uint8_t smem[];
    float* part = reinterpret_cast<float*>(smem);   // [kGemvWarps][2][MT] split-K partials
    uint8_t* act = smem + kPartBytes;               // staged activation
    float* stage = reinterpret_cast<float*>(act + a.act_smem);   // fused-prologue inputs
    const int64_t rs = a.row_stride;
    const int K = (int)a.K;
    const int nchunks = K / 16;
    const int64_t npt = (a.N + 1) / 2;               // row pairs in the matrix
    const int64_t p0 = npt * blockIdx.x / gridDim.x;
    const int64_t p1 = npt * (blockIdx.x + 1) / gridDim.x;
    const int64_t r0 = 2 * p0;
    const int nrows = (int)(min(a.N, 2 * p1) - r0);
    const int npairs = (int)(p1 - p0);
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
    {
        int8_t* act_q = reinterpret_cast<int8_t*>(act);
        float* act_d = reinterpret_cast<float*>(act + ((int64_t)a.M * K + 15) / 16 * 16);
        if (PRO == PRO_Q8 && a.act_smem > 0) {
            const int qbytes = a.M * K;
            for (int o = threadIdx.x * 16; o < qbytes; o += kGemvWarps * 32 * 16)
                *reinterpret_cast<int4*>(act_q + o) = __ldcg(reinterpret_cast<const int4*>(a.xq + o));
            const int nd = a.M * (K / QK);
            for (int o = threadIdx.x; o < nd; o += kGemvWarps * 32) act_d[o] = __ldcg(a.dx + o);
            __syncthreads();
            xq = act_q;
            dx = act_d;
        } else if (PRO == PRO_RMS) {
            prologue_rms<kGemvWarps>(a, act_q, act_d, part, stage);
            xq = act_q;
            dx = act_d;
        } else if (PRO == PRO_QNT) {
            prologue_qnt<kGemvWarps>(a, act_q, act_d, stage);
            xq = act_q;
            dx = act_d;
        }
    }

    __shared__ unsigned long long keys[EPI == EPI_ARGMAX ? kArgmaxMaxM : 1];
    if (EPI == EPI_ARGMAX) {
        for (int m = threadIdx.x; m < a.M; m += blockDim.x) keys[m] = 0ull;
        __syncthreads();
    }

    if (!SPLIT || wpp == 1) {
        for (; p < npairs; p += conc) {
            const uint8_t* ra = a.rows + (r0 + 2 * p) * rs;
            const bool has_b = 2 * p + 1 < nrows;
            const uint8_t* rb = has_b ? ra + rs : ra;
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
#pragma unroll
                for (int r = 0; r < 2; r++)
#pragma unroll
                    for (int j = 0; j < MT; j++) acc[r][j] = warp_sum(acc[r][j]);
                if (lane == 0) {
#pragma unroll
                    for (int j = 0; j < MT; j++)
                        if (m0 + j < a.M)
                            epi_pair<EPI, KV>(a, m0 + j, r0 + 2 * p, has_b, acc[0][j], acc[1][j],
                                              keys);
                }
            }
        }
    } else {
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
            if (slice == 0 && p < npairs && lane == 0) {
#pragma unroll
                for (int j = 0; j < MT; j++) {
                    if (m0 + j >= a.M) break;
                    float v0 = 0.0f, v1 = 0.0f;
                    for (int s = 0; s < wpp; s++) {
                        v0 += part[((warp + s) * 2 + 0) * MT + j];
                        v1 += part[((warp + s) * 2 + 1) * MT + j];
                    }
                    epi_pair<EPI, KV>(a, m0 + j, r0 + 2 * p, has_b, v0, v1, keys);
                }
            }
            __syncthreads();
        }
    }
    if (EPI == EPI_ARGMAX) argmax_tail(a, keys);
}

// Host side ---------------------------------------------------------------------

inline int64_t gemv_act_bytes(int M, int64_t K) {
    int64_t act = ((int64_t)M * K + 15) / 16 * 16 + (int64_t)M * (K / QK) * 4;
    return (act + 127) / 128 * 128;
}

// Bytes of the fused prologue's input staging area.
inline int64_t gemv_stage_bytes(int pro, int M, int64_t K) {
    if (pro == PRO_RMS) return ((int64_t)M * K + K) * 4;
    if (pro == PRO_QNT) return (int64_t)M * K * 4;
    return 0;
}

// Whether a fused prologue (PRO_RMS / PRO_QNT) fits for M rows of K.
inline bool gemv_fused_prologue_fits(int pro, int M, int64_t K) {
    return M <= kGemvMaxMT && K <= kProMaxK && gemv_act_bytes(M, K) <= kGemvActSmemMax &&
           gemv_stage_bytes(pro, M, K) <= kProStageMax;
}

template <int MT, int PRO, int EPI, typename KV>
inline int gemv_launch_t(DeviceState* ds, GemvArgs a, cudaStream_t stream) {
    if (a.K > (1 << 24) || (int64_t)a.M * a.K > (1ll << 31))
        return fail(AXQ8_ERR_UNSUPPORTED, "q8 gemv: K or M*K too large");
    if ((PRO == PRO_RMS || PRO == PRO_QNT) && (a.M > MT || a.K > kProMaxK))
        return fail(AXQ8_ERR_UNSUPPORTED, "q8 gemv: fused prologue with M=%d, K=%lld", a.M,
                    (long long)a.K);
    if (EPI == EPI_ARGMAX && a.M > kArgmaxMaxM)
        return fail(AXQ8_ERR_UNSUPPORTED, "q8 gemv: argmax epilogue with M=%d > %d", a.M,
                    kArgmaxMaxM);
    int64_t act = 0;
    if (PRO != PRO_F32) {
        act = gemv_act_bytes(a.M, a.K);
        if (act > kGemvActSmemMax) {
            if (PRO != PRO_Q8)
                return fail(AXQ8_ERR_UNSUPPORTED, "q8 gemv: fused prologue needs %lld B",
                            (long long)act);
            act = 0;
        }
    }
    a.act_smem = (int)act;
    const int64_t stage = gemv_stage_bytes(PRO, a.M, a.K);
    if (stage > kProStageMax)
        return fail(AXQ8_ERR_UNSUPPORTED, "q8 gemv: fused prologue staging needs %lld B",
                    (long long)stage);
    const size_t smem = (size_t)kPartBytes + (size_t)act + (size_t)stage;
    // CTAs per SM: 2 fills the SM (best for an isolated GEMV); 1 leaves room
    // for the next kernel's CTAs to co-reside and start their weight loads
    // under programmatic dependent launch.  AXQ8_GEMV_CTAS_PER_SM overrides
    // the default for tuning.
    static const int ctas_per_sm = [] {
        const char* e = getenv("AXQ8_GEMV_CTAS_PER_SM");
        const int v = e ? atoi(e) : kGemvCtasPerSm;
        return v >= 1 && v <= 4 ? v : kGemvCtasPerSm;
    }();
    const int64_t npt = (a.N + 1) / 2;
    int64_t grid = (int64_t)ds->sm_count * ctas_per_sm;
    if (grid > npt) grid = npt;                    // at least one row pair per CTA
    // split-K inside the CTA when its row pairs cannot occupy every warp
    const int64_t pairs_per_cta = (npt + grid - 1) / grid;
    const bool split = 2 * pairs_per_cta <= kGemvWarps && a.K >= 1024;
    auto kern = split ? q8_gemv_kernel<MT, PRO, EPI, true, KV> : q8_gemv_kernel<MT, PRO, EPI, false, KV>;
    if (smem > 48 * 1024) {
        static int configured_for[2][64] = {{0}};
        const int dev = ds->device < 64 ? ds->device : 63;
        if (!configured_for[split][dev]) {
            AXQ8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kPartBytes + kGemvActSmemMax + kProStageMax),
                          "cudaFuncSetAttribute(q8_gemv)");
            configured_for[split][dev] = 1;
        }
    }
    AXQ8_CUDA_TRY(launch_k(kern, dim3((unsigned)grid), dim3(kGemvWarps * 32), smem, stream, true, a),
                  "q8_gemv launch");
    return AXQ8_OK;
}

template <int PRO, int EPI, typename KV>
inline int gemv_launch_mt(DeviceState* ds, const GemvArgs& a, cudaStream_t stream) {
    if (a.M <= 1) return gemv_launch_t<1, PRO, EPI, KV>(ds, a, stream);
    if (a.M <= 2) return gemv_launch_t<2, PRO, EPI, KV>(ds, a, stream);
    return gemv_launch_t<4, PRO, EPI, KV>(ds, a, stream);
}

// The plain linear of the axq8 API: pre-quantized (A8) or fp32 (A32) input,
// y = residual + x.W^T.
inline int gemv_launch(DeviceState* ds, const GemvArgs& a, bool a32, cudaStream_t stream) {
    return a32 ? gemv_launch_mt<PRO_F32, EPI_STORE, float>(ds, a, stream)
               : gemv_launch_mt<PRO_Q8, EPI_STORE, float>(ds, a, stream);
}

}  // namespace axq8
