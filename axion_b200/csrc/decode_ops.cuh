// Decode-step kernels around the Q8_0 GEMV (sm_100a).
//
// Reference semantics (paths inside the reference project):
//   token_embedding           inference/cpp/runtime/token_embedding.cpp (row of the
//                             dequantized token_embd, gguf.cpp:870-882)
//   rmsnorm                   inference/cpp/kernels/rmsnorm.cpp:12-100
//   mha_attention_incremental inference/cpp/runtime/mha.cpp:227-285
//   silu * up                 inference/cpp/kernels/silu.cpp:13-65, elementwise.cpp:13-67
//
// Every kernel calls griddepcontrol.wait before its first global write or
// its first read of data another kernel produced, and every kernel of the
// step (these and the GEMVs of q8_gemv.cuh, whose RoPE/KV-append and argmax
// epilogues also live there) does so unconditionally: completion of kernel i then implies
// completion of all earlier kernels, which is what makes programmatic
// dependent launch safe for the reuse of activation buffers across phases.
// A8 producers (Q8 = true) quantize their output in 32-blocks with the
// convention of axq8_quantize_act (bit-identical on identical inputs).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include "axq8.h"
#include "common.cuh"
#include "q8_gemv.cuh"

namespace axq8 {

// ---- embedding ----------------------------------------------------------------
// h[m, :] = dequantized row tokens[m] of token_embd (repacked Q8_0 rows).
static __global__ void embed_kernel(const uint8_t* __restrict__ rows, int64_t rs, int H, int V,
                             const int* __restrict__ tokens, float* __restrict__ h, int* status) {
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x;
    int tok = ld_cg(tokens + m);
    if (tok < 0 || tok >= V) {
        if (threadIdx.x == 0) record_status(status, AXQ8_ERR_INVALID);
        tok = 0;
    }
    const uint8_t* row = rows + (int64_t)tok * rs;
    const __half* sc = reinterpret_cast<const __half*>(row + H);
    for (int k = threadIdx.x; k < H; k += blockDim.x)
        h[(int64_t)m * H + k] = __fmul_rn((float)(int8_t)row[k], __half2float(sc[k >> 5]));
}

// ---- RMSNorm (+ A8 quantization) ------------------------------------------------
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
// load8 of data another kernel produced (coherent, through L2)
__device__ __forceinline__ void load8_cg(const float* p, float (&v)[8]) {
    const float4 a = ld_cg4(p);
    const float4 b = ld_cg4(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// One CTA per row, 8 consecutive elements per thread and up to kNormUnits such
// units per thread, all held in registers (one read of x, loads in flight
// together; the norm weight is read before the wait on the producer).
// out = (x * (1/sqrt(mean(x^2) + eps))) * w with the reference's separately
// rounded operations; the sum of squares is a fixed tree (per thread, warp
// sums, then warps in order), not the reference's sequential sum.  H % 32 == 0,
// H <= 8 * kNormUnits * blockDim.x, blockDim.x a multiple of 32.
// dxt > 0: the block scales go transposed, dx[b * dxt + m] (the tensor-core
// product's layout), else row-major dx[m * H/32 + b].  Same below.
constexpr int kNormUnits = 4;
template <bool Q8>
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ w, int H,
                                                       float eps, float* __restrict__ out,
                                                       int8_t* __restrict__ xq,
                                                       float* __restrict__ dx, int dxt) {
    __shared__ float red[32];
    const int m = blockIdx.x, nu = H / 8;
    float wv[kNormUnits][8], v[kNormUnits][8];
#pragma unroll
    for (int u = 0; u < kNormUnits; u++) {
        const int j = threadIdx.x + u * blockDim.x;
        if (j < nu) load8(w + 8 * j, wv[u]);
    }
    pdl_launch_dependents();
    pdl_wait();
    const float* xr = x + (int64_t)m * H;
    float s = 0.0f;
#pragma unroll
    for (int u = 0; u < kNormUnits; u++) {
        const int j = threadIdx.x + u * blockDim.x;
        if (j < nu) {
            load8_cg(xr + 8 * j, v[u]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[u][e] = wv[u][e] = 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 8; e++) s = fmaf(v[u][e], v[u][e], s);
    }
    s = warp_sum(s);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    const float ms = __fdiv_rn(red[0], (float)H);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    const int nb = H / QK;
#pragma unroll
    for (int u = 0; u < kNormUnits; u++) {
        const int j = threadIdx.x + u * blockDim.x;
        if (u * blockDim.x >= (unsigned)nu) break;   // uniform over the CTA
#pragma unroll
        for (int e = 0; e < 8; e++) v[u][e] = __fmul_rn(__fmul_rn(v[u][e], inv), wv[u][e]);
        if (!Q8) {
            if (j < nu) store8(out + (int64_t)m * H + 8 * j, v[u]);
        } else {
            const int b = j >> 2;
            quant_block_quad(v[u], lane, j < nu, xq + (int64_t)m * H + 8 * j,
                             dx + (dxt ? (int64_t)b * dxt + m : (int64_t)m * nb + b));
        }
    }
}

// Threads of an rmsnorm_kernel CTA for rows of H: two 8-element units per
// thread where that fits in 1024 threads; 0 when H is beyond the kernel.
inline int rmsnorm_threads(int H) {
    if (H <= 0 || H % QK) return 0;
    const int nu = H / 8;
    const int t = ((nu + 1) / 2 + 31) / 32 * 32;
    if (t <= 1024) return t;
    return nu <= 1024 * kNormUnits ? 1024 : 0;
}

// The split merge of one query head (one warp): out = sum_s acc_s e^(m_s - M)
// / sum_s l_s e^(m_s - M) over the nsplit partials of (sequence m, head h),
// then (Q8) the head's A8 quantization.  One lane per split (nsplit <= 32):
// every partial is loaded at once.
template <int HD, bool Q8>
__device__ __forceinline__ void attn_merge_head(const float* __restrict__ part, int m, int n_heads,
                                                int h, int nsplit, float* __restrict__ out,
                                                int8_t* __restrict__ xq, float* __restrict__ dx,
                                                int dxt, int lane) {
    constexpr int DL = HD / 32;
    const float* ph = part + ((int64_t)m * n_heads + h) * nsplit * (HD + 2);
    const float ms = lane < nsplit ? __ldcg(ph + lane * (HD + 2) + HD) : -CUDART_INF_F;
    const float ls = lane < nsplit ? __ldcg(ph + lane * (HD + 2) + HD + 1) : 0.0f;
    float mx = ms;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float f = ms == -CUDART_INF_F ? 0.0f : expf(ms - mx);   // empty splits weigh 0
    const float l = warp_sum(ls * f);
    float sum[DL];
#pragma unroll
    for (int i = 0; i < DL; i++) sum[i] = 0.0f;
#pragma unroll 4
    for (int t2 = 0; t2 < nsplit; t2++) {
        const float ft = __shfl_sync(0xffffffffu, f, t2);
#pragma unroll
        for (int i = 0; i < DL; i++) sum[i] = fmaf(__ldcg(ph + t2 * (HD + 2) + lane * DL + i), ft, sum[i]);
    }
    const int64_t base = (int64_t)m * n_heads * HD + (int64_t)h * HD + lane * DL;
    float v[DL];
#pragma unroll
    for (int i = 0; i < DL; i++) v[i] = __fdiv_rn(sum[i], l);
    if (!Q8) {
#pragma unroll
        for (int i = 0; i < DL; i++) out[base + i] = v[i];
        return;
    }
    // 32-dim quantization block = 32/DL consecutive lanes
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < DL; i++) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
    for (int off = 1; off < 32 / DL; off <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    const float id = am == 0.0f ? 0.0f : __fdiv_rn(127.0f, am);
#pragma unroll
    for (int i = 0; i < DL; i++) xq[base + i] = (int8_t)q8_round(__fmul_rn(v[i], id));
    if ((lane % (32 / DL)) == 0) {
        const int64_t col = (int64_t)h * HD + lane * DL;   // position in the row of n_heads*HD
        dx[dxt ? (col / QK) * dxt + m : base / QK] = __fdiv_rn(am, 127.0f);
    }
}


// ---- attention: split-K flash decode ----------------------------------------------
// Grid (n_kv, M, nsplit); G warps per CTA, warp g serving query head
// kvh*G + g (GQA: query head h reads kv head h / G, mha.cpp:253-254).  Split
// s covers KV pages [s*bps, (s+1)*bps) of the sequence's pages in use
// (ctx = pos + 1 tokens).  Up to `cp` pages (B = 16 tokens each) of K and V
// are copied to shared memory at once with cp.async, in the cache's own
// type, and shared by the G warps.  Lane l scores token l & 15 over half the
// head dims (l >> 4), walking the dims from a lane-dependent start so that
// the 32 lanes hit 32 different banks; scores are scaled by 1/sqrt(hd) after
// the dot, as the reference does.  Online softmax; the partial (acc[hd],
// running max, running sum) of each (sequence, query head, split) goes to
// `part`, and the last split CTA to finish merges them (and, with Q8,
// quantizes the head's output for the O projection).
__device__ __forceinline__ float2 kv_pair(const __half* p) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
}
__device__ __forceinline__ float2 kv_pair(const float* p) {
    return *reinterpret_cast<const float2*>(p);
}

// Shared memory of attn_decode_kernel: K and V stages, the G query rows and
// the split's page ids.
template <typename KV, int HD>
inline size_t attn_smem_bytes(int G, int cp, int bps) {
    return (size_t)4 * cp * 16 * HD * sizeof(KV) + (size_t)G * HD * sizeof(float) +
           ((size_t)bps * sizeof(int) + 15) / 16 * 16;
}

template <typename KV, int HD, bool Q8>
__global__ void attn_decode_kernel(const float* __restrict__ qkv, int ldq,
                                   const int* __restrict__ pos, const KV* __restrict__ kc,
                                   const KV* __restrict__ vc, const int* __restrict__ block_table,
                                   int max_blocks, int n_heads, int n_kv, int bps, int cp,
                                   float scale, float* __restrict__ part, int* __restrict__ counters,
                                   float* __restrict__ out, int8_t* __restrict__ xq,
                                   float* __restrict__ dx, int dxt) {
    constexpr int B = 16;
    constexpr int DL = HD / 32;            // dims per lane in the value accumulation
    constexpr int V16 = 16 / sizeof(KV);    // cache elements per 16-byte copy
    static_assert(HD % 32 == 0 && (DL == 1 || DL % 2 == 0), "head dim");
    extern __shared__ __align__(16) uint8_t attn_sm[];
    const int G = blockDim.x >> 5;
    KV* ks = reinterpret_cast<KV*>(attn_sm);              // [2][cp][B][HD] (double buffer)
    KV* vs = ks + (size_t)2 * cp * B * HD;                 // [2][cp][B][HD]
    float* qs = reinterpret_cast<float*>(vs + (size_t)2 * cp * B * HD);   // [G][HD]
    int* pg = reinterpret_cast<int*>(qs + G * HD);         // [bps] page ids
    const int kvh = blockIdx.x, m = blockIdx.y, s = blockIdx.z, nsplit = gridDim.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * G + warp;
    const int b0 = s * bps;
    // the page table is written by the host before the step: read it while
    // the previous kernel drains
    for (int i = threadIdx.x; i < bps; i += blockDim.x)
        pg[i] = b0 + i < max_blocks ? block_table[m * max_blocks + b0 + i] : 0;
    pdl_launch_dependents();
    pdl_wait();
    // a position past the page table was already reported by the KV append;
    // never read beyond the table
    const int ctx = min(ld_cg(pos + m) + 1, max_blocks * B);
    const int nblk = (ctx + B - 1) / B;
    const int b1 = min(nblk, b0 + bps);
    for (int i = threadIdx.x; i < G * HD / 4; i += blockDim.x)
        cp_async16(qs + 4 * i, qkv + (int64_t)m * ldq + (int64_t)(kvh * G) * HD + 4 * i);
    float mrun = -CUDART_INF_F, lrun = 0.0f;
    float acc[DL];
#pragma unroll
    for (int i = 0; i < DL; i++) acc[i] = 0.0f;
    const int t = lane & (B - 1), hf = lane >> 4;
    constexpr int per_page = B * HD / V16;
    // chunks of cp pages, double buffered: the copy of chunk ci + 1 is in
    // flight while chunk ci is scored
    const int nch = b1 > b0 ? (b1 - b0 + cp - 1) / cp : 0;
    auto issue = [&](int ci) {
        const int c0 = b0 + ci * cp, np = min(cp, b1 - c0);
        KV* kb = ks + (size_t)(ci & 1) * cp * B * HD;
        KV* vb = vs + (size_t)(ci & 1) * cp * B * HD;
        for (int i = threadIdx.x; i < np * per_page; i += blockDim.x) {
            const int p = i / per_page, j = i - p * per_page;
            const int64_t off = ((int64_t)pg[c0 - b0 + p] * n_kv + kvh) * B * HD + j * V16;
            cp_async16(kb + p * B * HD + j * V16, kc + off);
            cp_async16(vb + p * B * HD + j * V16, vc + off);
        }
    };
    __syncthreads();   // pg visible
    if (nch > 0) issue(0);
    cp_async_commit();   // group 0 also holds the query copies
    for (int ci = 0; ci < nch; ci++) {
        if (ci + 1 < nch) {
            issue(ci + 1);
            cp_async_commit();
            cp_async_wait_group<1>();
        } else {
            cp_async_wait_group<0>();
        }
        __syncthreads();
        const int c0 = b0 + ci * cp, np = min(cp, b1 - c0);
        const KV* kbuf = ks + (size_t)(ci & 1) * cp * B * HD;
        const KV* vbuf = vs + (size_t)(ci & 1) * cp * B * HD;
        for (int p = 0; p < np; p++) {
            const int blk = c0 + p;
            // score of token t, half hf of the dims, then combine the halves
            const float* q = qs + warp * HD + hf * (HD / 2);
            const KV* k = kbuf + ((size_t)p * B + t) * HD + hf * (HD / 2);
            float dot = 0.0f;
#pragma unroll 8
            for (int d2 = 0; d2 < HD / 4; d2++) {
                const int dd = 2 * ((d2 + lane) & (HD / 4 - 1));
                const float2 kf = kv_pair(k + dd);
                const float2 qf = *reinterpret_cast<const float2*>(q + dd);
                dot = fmaf(qf.x, kf.x, dot);
                dot = fmaf(qf.y, kf.y, dot);
            }
            dot += __shfl_xor_sync(0xffffffffu, dot, 16);
            const bool valid = blk * B + t < ctx;
            const float sc = valid ? __fmul_rn(dot, scale) : -CUDART_INF_F;
            float mt = sc;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            const float mnew = fmaxf(mrun, mt);
            const float corr = expf(mrun - mnew);   // 0 when mrun is -inf
            const float pt = valid ? expf(sc - mnew) : 0.0f;
            float ps = pt;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            lrun = fmaf(lrun, corr, ps);
#pragma unroll
            for (int i = 0; i < DL; i++) acc[i] *= corr;
            const KV* v = vbuf + (size_t)p * B * HD + lane * DL;
#pragma unroll 4
            for (int tt = 0; tt < B; tt++) {
                const float pv = __shfl_sync(0xffffffffu, pt, tt);
                if (DL == 1) {
                    acc[0] = fmaf(pv, kv_to_float(v[tt * HD]), acc[0]);
                } else {
#pragma unroll
                    for (int i = 0; i < DL; i += 2) {
                        const float2 vf = kv_pair(v + tt * HD + i);
                        acc[i] = fmaf(pv, vf.x, acc[i]);
                        acc[i + 1] = fmaf(pv, vf.y, acc[i + 1]);
                    }
                }
            }
            mrun = mnew;
        }
        __syncthreads();   // buffer ci & 1 is free for chunk ci + 2
    }
    if (nch == 0) cp_async_wait_all();   // empty split: the query copies
    float* o = part + (((int64_t)m * n_heads + h) * nsplit + s) * (HD + 2);
#pragma unroll
    for (int i = 0; i < DL; i++) o[lane * DL + i] = acc[i];
    if (lane == 0) {
        o[HD] = mrun;
        o[HD + 1] = lrun;
    }
    // The last CTA of this (sequence, kv head) merges the splits of its G
    // query heads (fence, count, fence; counters return to zero):
    // out = sum_s acc_s e^(m_s - M) / sum_s l_s e^(m_s - M).
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) {
        int* c = counters + m * n_kv + kvh;
        last = atomicAdd(c, 1) == nsplit - 1;
        if (last) *c = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    attn_merge_head<HD, Q8>(part, m, n_heads, h, nsplit, out, xq, dx, dxt, lane);
}

// ---- attention on the tensor cores (fp16 KV pages, head dim 64 / 128) ---------------
// Grid (n_kv, M, nsplit) as above; kAttnTcWarps warps per CTA, each taking
// whole pages of the split in turn (page b0 + w, b0 + w + W, ...) for all G
// query heads of the KV head.  Per page (16 tokens) and warp:
//   S [16 heads (G used) x 16 tokens] = Q K^T    mma.sync m16n8k16, fp32 accumulate
//   online softmax over the page's tokens per head (scale after the dot, as
//   the reference does; expf)
//   O [16 x hd] += P V                            mma.sync m16n8k16
// Q and P are fp32 values split into an fp16 high part and an fp16 residual,
// each multiplied separately (products with the fp16 K / V are exact in fp32),
// so the scores and the output keep fp32 accuracy.  K and V pages are copied
// per warp with cp.async, double buffered, into rows XOR-swizzled by 16-byte
// chunk so that ldmatrix reads are conflict-free.  The warps' states merge in
// shared memory into the split partial of the scalar kernel above, and the
// last split CTA merges the splits with attn_merge_head.
constexpr int kAttnTcWarps = 4;

// Shared memory: the warps' double-buffered K/V pages, reused afterwards for
// the warps' merge ([W][16 x HD + 32] fp32), then the split's page ids.
template <int HD>
struct AttnTcSmem {
    static constexpr size_t STAGE = (size_t)kAttnTcWarps * 2 /*buffers*/ * 2 /*K,V*/ * 16 * HD * 2;
    static constexpr size_t MERGE = (size_t)kAttnTcWarps * (16 * HD + 32) * 4;
    static constexpr size_t PG = STAGE > MERGE ? STAGE : MERGE;   // offset of the page ids
};
template <int HD>
inline size_t attn_tc_smem_bytes(int bps) {
    return AttnTcSmem<HD>::PG + ((size_t)bps * sizeof(int) + 15) / 16 * 16;
}

__device__ __forceinline__ void mma_f16_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// fp16 pair (lo element first) of x and y, and of their fp16 residuals.
__device__ __forceinline__ void split_pair(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __half xh = __float2half_rn(x), yh = __float2half_rn(y);
    const __half xl = __float2half_rn(x - __half2float(xh)), yl = __float2half_rn(y - __half2float(yh));
    hi = (uint32_t)__half_as_ushort(xh) | ((uint32_t)__half_as_ushort(yh) << 16);
    lo = (uint32_t)__half_as_ushort(xl) | ((uint32_t)__half_as_ushort(yl) << 16);
}

// The CTA's merge of its warps' states and, in the last split CTA of a
// (sequence, KV head), of the splits.  Warp w left in shared memory (at
// w * (16 HD + 32) floats) its unnormalised O rows [16][HD] (row = head of
// the group), then 16 running maxima and 16 sums; rows >= G are unused.
template <int HD, bool Q8>
__device__ __forceinline__ void attn_tc_merge(const uint8_t* tc_sm, int G, int n_heads, int n_kv,
                                              int kvh, int m, int s, int nsplit, float* __restrict__ part,
                                              int* __restrict__ counters, float* __restrict__ out,
                                              int8_t* __restrict__ xq, float* __restrict__ dx, int dxt,
                                              int warp, int lane) {
    constexpr int W = kAttnTcWarps;
    __syncthreads();
    const float* m0p = reinterpret_cast<const float*>(tc_sm);
    for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
        const int row = idx / HD, d = idx % HD;
        float mx = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < W; w++) mx = fmaxf(mx, m0p[(size_t)w * (16 * HD + 32) + 16 * HD + row]);
        float acc = 0.0f, l = 0.0f;
#pragma unroll
        for (int w = 0; w < W; w++) {
            const float* base = m0p + (size_t)w * (16 * HD + 32);
            const float mwv = base[16 * HD + row];
            const float f = mwv == -CUDART_INF_F ? 0.0f : expf(mwv - mx);
            acc = fmaf(base[row * HD + d], f, acc);
            l = fmaf(base[16 * HD + 16 + row], f, l);
        }
        const int h = kvh * G + row;
        float* op = part + (((int64_t)m * n_heads + h) * nsplit + s) * (HD + 2);
        op[d] = acc;
        if (d == 0) {
            op[HD] = mx;
            op[HD + 1] = l;
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) {
        int* c = counters + m * n_kv + kvh;
        last = atomicAdd(c, 1) == nsplit - 1;
        if (last) *c = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int hh = warp; hh < G; hh += W)
        attn_merge_head<HD, Q8>(part, m, n_heads, kvh * G + hh, nsplit, out, xq, dx, dxt, lane);
}

template <int HD, bool Q8>
__global__ void __launch_bounds__(kAttnTcWarps * 32)
    attn_tc_kernel(const float* __restrict__ qkv, int ldq, const int* __restrict__ pos,
                   const __half* __restrict__ kc, const __half* __restrict__ vc,
                   const int* __restrict__ block_table, int max_blocks, int n_heads, int n_kv,
                   int G, int bps, float scale, float* __restrict__ part, int* __restrict__ counters,
                   float* __restrict__ out, int8_t* __restrict__ xq, float* __restrict__ dx, int dxt) {
    constexpr int B = 16;
    constexpr int W = kAttnTcWarps;
    constexpr int KS = HD / 16;              // k-steps of the score product
    constexpr int NT = HD / 8;               // n-tiles (8 dims) of the output
    constexpr int CH = HD / 8;               // 16-byte chunks per row
    constexpr int PAGE = B * HD;             // halves per K (or V) page
    extern __shared__ __align__(16) uint8_t tc_sm[];
    __half* stage = reinterpret_cast<__half*>(tc_sm);   // [W][2 buf][K,V][B][HD]
    int* pg = reinterpret_cast<int*>(tc_sm + AttnTcSmem<HD>::PG);
    const int kvh = blockIdx.x, m = blockIdx.y, s = blockIdx.z, nsplit = gridDim.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int b0 = s * bps;
    for (int i = threadIdx.x; i < bps; i += blockDim.x)
        pg[i] = b0 + i < max_blocks ? block_table[m * max_blocks + b0 + i] : 0;
    pdl_launch_dependents();
    pdl_wait();
    const int ctx = min(ld_cg(pos + m) + 1, max_blocks * B);
    const int nblk = (ctx + B - 1) / B;
    const int b1 = min(nblk, b0 + bps);
    __syncthreads();   // pg visible
    // Q fragments (rows = heads kvh*G + row, rows >= G zero), fp16 high and residual
    uint32_t qh[KS][4], ql[KS][4];
    {
        const float* q0 = qkv + (int64_t)m * ldq + (int64_t)(kvh * G) * HD;
#pragma unroll
        for (int k = 0; k < KS; k++) {
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int row = g + ((r & 1) ? 8 : 0);
                const int col = k * 16 + 2 * t + ((r & 2) ? 8 : 0);
                float x = 0.0f, y = 0.0f;
                if (row < G) {
                    const float2 v = ld_cg2(q0 + (int64_t)row * HD + col);
                    x = v.x;
                    y = v.y;
                }
                split_pair(x, y, qh[k][r], ql[k][r]);
            }
        }
    }
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float mrun[2] = {-CUDART_INF_F, -CUDART_INF_F}, lrun[2] = {0.0f, 0.0f};
    __half* wst = stage + (size_t)warp * 2 * 2 * PAGE;
    const uint32_t wst_s = smem_u32(wst);
    // this warp's pages: b0 + warp, b0 + warp + W, ...
    const int npw = b1 > b0 + warp ? (b1 - b0 - warp + W - 1) / W : 0;
    auto issue = [&](int i) {            // page number i of this warp -> buffer i & 1
        const int blk = b0 + warp + i * W;
        const int64_t off = ((int64_t)pg[blk - b0] * n_kv + kvh) * PAGE;
        __half* kb = wst + (size_t)(i & 1) * 2 * PAGE;
        __half* vb = kb + PAGE;
#pragma unroll
        for (int c = lane; c < B * CH; c += 32) {
            const int r = c / CH, ch = c % CH;
            const int sw = r * HD + ((ch ^ (r & 7)) * 8);
            cp_async16(kb + sw, kc + off + r * HD + ch * 8);
            cp_async16(vb + sw, vc + off + r * HD + ch * 8);
        }
    };
    if (npw > 0) issue(0);
    cp_async_commit();
    for (int i = 0; i < npw; i++) {
        if (i + 1 < npw) {
            issue(i + 1);
            cp_async_commit();
            cp_async_wait_group<1>();
        } else {
            cp_async_wait_group<0>();
        }
        __syncwarp();
        const int blk = b0 + warp + i * W;
        const uint32_t kb = wst_s + (uint32_t)((i & 1) * 2 * PAGE * 2);
        const uint32_t vb = kb + PAGE * 2;
        // S = Q K^T: n-tile 0 = tokens 0-7, n-tile 1 = tokens 8-15
        float sc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
        {
            const int mi = lane >> 3, rr = lane & 7;
            const int tok = rr + ((mi >> 1) << 3);
#pragma unroll
            for (int k = 0; k < KS; k++) {
                const int ch = k * 2 + (mi & 1);
                uint32_t kf[4];
                ldsm_x4(kf, kb + (uint32_t)((tok * HD + ((ch ^ (tok & 7)) * 8)) * 2));
                mma_f16_16816(sc[0], qh[k], kf[0], kf[1]);
                mma_f16_16816(sc[0], ql[k], kf[0], kf[1]);
                mma_f16_16816(sc[1], qh[k], kf[2], kf[3]);
                mma_f16_16816(sc[1], ql[k], kf[2], kf[3]);
            }
        }
        // online softmax per head row (g: c0, c1; g + 8: c2, c3)
        float p[2][4];
#pragma unroll
        for (int hr = 0; hr < 2; hr++) {
            float mt = -CUDART_INF_F;
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int tok = blk * B + n * 8 + 2 * t + j;
                    float& v = sc[n][2 * hr + j];
                    v = tok < ctx ? __fmul_rn(v, scale) : -CUDART_INF_F;
                    mt = fmaxf(mt, v);
                }
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
            const float mnew = fmaxf(mrun[hr], mt);
            const float corr = expf(mrun[hr] - mnew);   // 0 when mrun is -inf
            float ps = 0.0f;
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const float v = sc[n][2 * hr + j];
                    const float e = v == -CUDART_INF_F ? 0.0f : expf(v - mnew);
                    p[n][2 * hr + j] = e;
                    ps += e;
                }
            lrun[hr] = fmaf(lrun[hr], corr, ps);
            mrun[hr] = mnew;
#pragma unroll
            for (int n = 0; n < NT; n++) {
                o[n][2 * hr] *= corr;
                o[n][2 * hr + 1] *= corr;
            }
        }
        // P fragments (A operand, rows = heads, k = tokens) from the S layout
        uint32_t ph[4], pl[4];
        split_pair(p[0][0], p[0][1], ph[0], pl[0]);
        split_pair(p[0][2], p[0][3], ph[1], pl[1]);
        split_pair(p[1][0], p[1][1], ph[2], pl[2]);
        split_pair(p[1][2], p[1][3], ph[3], pl[3]);
        // O += P V: pairs of 8-dim n-tiles per ldmatrix.trans
        {
            const int mi = lane >> 3, rr = lane & 7;
            const int tok = rr + ((mi & 1) << 3);
#pragma unroll
            for (int dn = 0; dn < HD / 16; dn++) {
                const int ch = dn * 2 + (mi >> 1);
                uint32_t vf[4];
                ldsm_x4_t(vf, vb + (uint32_t)((tok * HD + ((ch ^ (tok & 7)) * 8)) * 2));
                mma_f16_16816(o[2 * dn], ph, vf[0], vf[1]);
                mma_f16_16816(o[2 * dn], pl, vf[0], vf[1]);
                mma_f16_16816(o[2 * dn + 1], ph, vf[2], vf[3]);
                mma_f16_16816(o[2 * dn + 1], pl, vf[2], vf[3]);
            }
        }
        __syncwarp();   // buffer i & 1 free for page i + 2
    }
    if (npw == 0) cp_async_wait_all();
    // row sums over the quad
#pragma unroll
    for (int hr = 0; hr < 2; hr++) {
        lrun[hr] += __shfl_xor_sync(0xffffffffu, lrun[hr], 1);
        lrun[hr] += __shfl_xor_sync(0xffffffffu, lrun[hr], 2);
    }
    // merge the warps: per warp [16 rows][HD] of O, then 16 m, 16 l
    __syncthreads();   // every warp is done with the staging buffers
    float* mw = reinterpret_cast<float*>(tc_sm) + (size_t)warp * (16 * HD + 32);
#pragma unroll
    for (int n = 0; n < NT; n++) {
        mw[g * HD + n * 8 + 2 * t] = o[n][0];
        mw[g * HD + n * 8 + 2 * t + 1] = o[n][1];
        mw[(g + 8) * HD + n * 8 + 2 * t] = o[n][2];
        mw[(g + 8) * HD + n * 8 + 2 * t + 1] = o[n][3];
    }
    if (t == 0) {
        mw[16 * HD + g] = mrun[0];
        mw[16 * HD + g + 8] = mrun[1];
        mw[16 * HD + 16 + g] = lrun[0];
        mw[16 * HD + 16 + g + 8] = lrun[1];
    }
    attn_tc_merge<HD, Q8>(tc_sm, G, n_heads, n_kv, kvh, m, s, nsplit, part, counters, out, xq, dx,
                          dxt, warp, lane);
}

// Transposed tensor-core attention for query groups of at most 8 heads (the
// Llama-3 and TinyLlama groups: 4 and 8).  The 16 tokens of a page are the
// MMA rows and the heads the 8 columns, so no MMA row is padding:
//   S^T [16 tokens x 8 heads] = K Q^T   (A = K page rows by ldmatrix, B = Q^T in registers)
//   O^T [HD x 8 heads] += V^T P^T        (A = V^T by ldmatrix.trans, B = P^T)
// P^T's B fragments come from the S^T accumulators by one register transpose
// (movmatrix) per 8x8 block.  Q and P keep the fp16 high + residual split of
// the kernel above (fp32 accuracy); half the MMAs of the 16-head layout and
// half the output registers.  Grid, shared memory, splits and merge as above.
constexpr int kAttnTctBufs = 3;   // page buffers per warp: two pages in flight ahead
template <int HD>
struct AttnTctSmem {
    static constexpr size_t STAGE = (size_t)kAttnTcWarps * kAttnTctBufs * 2 /*K,V*/ * 16 * HD * 2;
    static constexpr size_t MERGE = AttnTcSmem<HD>::MERGE;
    static constexpr size_t PG = STAGE > MERGE ? STAGE : MERGE;   // offset of the page ids
};
template <int HD>
inline size_t attn_tct_smem_bytes(int bps) {
    return AttnTctSmem<HD>::PG + ((size_t)bps * sizeof(int) + 15) / 16 * 16;
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

template <int HD, bool Q8>
__global__ void __launch_bounds__(kAttnTcWarps * 32)
    attn_tct_kernel(const float* __restrict__ qkv, int ldq, const int* __restrict__ pos,
                    const __half* __restrict__ kc, const __half* __restrict__ vc,
                    const int* __restrict__ block_table, int max_blocks, int n_heads, int n_kv,
                    int G, int bps, float scale, float* __restrict__ part, int* __restrict__ counters,
                    float* __restrict__ out, int8_t* __restrict__ xq, float* __restrict__ dx, int dxt) {
    constexpr int B = 16;
    constexpr int W = kAttnTcWarps;
    constexpr int KS = HD / 16;              // k-steps of the score product
    constexpr int MT = HD / 16;              // 16-dim row tiles of O^T
    constexpr int CH = HD / 8;               // 16-byte chunks per row
    constexpr int PAGE = B * HD;             // halves per K (or V) page
    extern __shared__ __align__(16) uint8_t tc_sm[];
    constexpr int NBUF = kAttnTctBufs;
    __half* stage = reinterpret_cast<__half*>(tc_sm);   // [W][NBUF][K,V][B][HD]
    int* pg = reinterpret_cast<int*>(tc_sm + AttnTctSmem<HD>::PG);
    const int kvh = blockIdx.x, m = blockIdx.y, s = blockIdx.z, nsplit = gridDim.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int b0 = s * bps;
    for (int i = threadIdx.x; i < bps; i += blockDim.x)
        pg[i] = b0 + i < max_blocks ? block_table[m * max_blocks + b0 + i] : 0;
    pdl_launch_dependents();
    pdl_wait();
    const int ctx = min(ld_cg(pos + m) + 1, max_blocks * B);
    const int nblk = (ctx + B - 1) / B;
    const int b1 = min(nblk, b0 + bps);
    __syncthreads();   // pg visible
    // Q^T fragments (B operand, column = head g of the group, zero for g >= G):
    // [k][0] dims 16k + 2t (+1), [k][1] dims 16k + 8 + 2t (+1); fp16 high and residual
    uint32_t qh[KS][2], ql[KS][2];
    {
        const float* q0 = qkv + (int64_t)m * ldq + (int64_t)(kvh * G) * HD;
#pragma unroll
        for (int k = 0; k < KS; k++) {
#pragma unroll
            for (int r = 0; r < 2; r++) {
                float x = 0.0f, y = 0.0f;
                if (g < G) {
                    const float2 v = ld_cg2(q0 + (int64_t)g * HD + k * 16 + 8 * r + 2 * t);
                    x = v.x;
                    y = v.y;
                }
                split_pair(x, y, qh[k][r], ql[k][r]);
            }
        }
    }
    // O^T tile mt: [0] dim 16 mt + g, head 2t; [1] head 2t + 1; [2], [3] dim + 8
    float o[MT][4];
#pragma unroll
    for (int n = 0; n < MT; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float mrun[2] = {-CUDART_INF_F, -CUDART_INF_F}, lrun[2] = {0.0f, 0.0f};   // heads 2t, 2t + 1
    __half* wst = stage + (size_t)warp * NBUF * 2 * PAGE;
    const uint32_t wst_s = smem_u32(wst);
    const int npw = b1 > b0 + warp ? (b1 - b0 - warp + W - 1) / W : 0;
    auto issue = [&](int i) {            // page number i of this warp -> buffer i % NBUF
        const int blk = b0 + warp + i * W;
        const int64_t off = ((int64_t)pg[blk - b0] * n_kv + kvh) * PAGE;
        __half* kb = wst + (size_t)(i % NBUF) * 2 * PAGE;
        __half* vb = kb + PAGE;
#pragma unroll
        for (int c = lane; c < B * CH; c += 32) {
            const int r = c / CH, ch = c % CH;
            const int sw = r * HD + ((ch ^ (r & 7)) * 8);
            cp_async16(kb + sw, kc + off + r * HD + ch * 8);
            cp_async16(vb + sw, vc + off + r * HD + ch * 8);
        }
    };
    // NBUF - 1 pages ahead: page i + NBUF - 1 is requested while page i is used
    static_assert(NBUF == 3, "wait counts below");
    for (int i = 0; i < NBUF - 1; i++) {
        if (i < npw) issue(i);
        cp_async_commit();
    }
    const int mi = lane >> 3, rr = lane & 7;
    for (int i = 0; i < npw; i++) {
        if (i + NBUF - 1 < npw) issue(i + NBUF - 1);
        cp_async_commit();                 // (possibly empty) group of page i + NBUF - 1
        cp_async_wait_group<NBUF - 1>();   // page i has landed
        __syncwarp();
        const int blk = b0 + warp + i * W;
        const uint32_t kb = wst_s + (uint32_t)((i % NBUF) * 2 * PAGE * 2);
        const uint32_t vb = kb + PAGE * 2;
        // S^T = K Q^T.  A fragment of K for k-step k: matrices (tokens 0-7 | 8-15) x
        // (dims 16k..+7 | 16k+8..+15), lane l addressing row l % 8 of matrix l / 8
        float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // tok g: heads 2t, 2t+1; tok g + 8: same
        {
            const int tok = rr + ((mi & 1) << 3);
#pragma unroll
            for (int k = 0; k < KS; k++) {
                const int ch = k * 2 + (mi >> 1);
                uint32_t kf[4];
                ldsm_x4(kf, kb + (uint32_t)((tok * HD + ((ch ^ (tok & 7)) * 8)) * 2));
                mma_f16_16816(sc, kf, qh[k][0], qh[k][1]);
                mma_f16_16816(sc, kf, ql[k][0], ql[k][1]);
            }
        }
        // online softmax per head column (2t + hh): tokens g, g + 8 of this lane,
        // the other tokens across the 8 lanes of the same t
        float p[4];
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            float mt = -CUDART_INF_F;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int tok = blk * B + g + 8 * j;
                float& v = sc[2 * j + hh];
                v = tok < ctx ? __fmul_rn(v, scale) : -CUDART_INF_F;
                mt = fmaxf(mt, v);
            }
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
            const float mnew = fmaxf(mrun[hh], mt);
            const float corr = expf(mrun[hh] - mnew);   // 0 when mrun is -inf
            float ps = 0.0f;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const float v = sc[2 * j + hh];
                const float e = v == -CUDART_INF_F ? 0.0f : expf(v - mnew);
                p[2 * j + hh] = e;
                ps += e;
            }
            lrun[hh] = fmaf(lrun[hh], corr, ps);
            mrun[hh] = mnew;
#pragma unroll
            for (int n = 0; n < MT; n++) {
                o[n][hh] *= corr;
                o[n][2 + hh] *= corr;
            }
        }
        // P^T fragments (B operand: k = tokens, n = head g) by transposing the
        // 8x8 blocks (tokens 0-7, 8-15) x heads held in the S^T layout
        uint32_t h01, l01, h23, l23;
        split_pair(p[0], p[1], h01, l01);   // token g, heads 2t, 2t+1
        split_pair(p[2], p[3], h23, l23);   // token g + 8
        const uint32_t pbh0 = movmatrix_t(h01), pbh1 = movmatrix_t(h23);
        const uint32_t pbl0 = movmatrix_t(l01), pbl1 = movmatrix_t(l23);
        // O^T += V^T P^T.  A fragment of V^T for row tile mt: matrices (dims 16mt..+7 |
        // +8..+15) x (tokens 0-7 | 8-15), each the transpose of a stored 8x8 block
        {
            const int tok = rr + ((mi >> 1) << 3);
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                const int ch = mt * 2 + (mi & 1);
                uint32_t vf[4];
                ldsm_x4_t(vf, vb + (uint32_t)((tok * HD + ((ch ^ (tok & 7)) * 8)) * 2));
                mma_f16_16816(o[mt], vf, pbh0, pbh1);
                mma_f16_16816(o[mt], vf, pbl0, pbl1);
            }
        }
        __syncwarp();   // buffer i % NBUF free for page i + NBUF
    }
    cp_async_wait_all();
    // column sums over the 8 lanes of the same t
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
        lrun[hh] += __shfl_xor_sync(0xffffffffu, lrun[hh], 4);
        lrun[hh] += __shfl_xor_sync(0xffffffffu, lrun[hh], 8);
        lrun[hh] += __shfl_xor_sync(0xffffffffu, lrun[hh], 16);
    }
    // the warp's state in the merge layout: rows = heads, [16][HD], then m, l
    __syncthreads();   // every warp is done with the staging buffers
    float* mw = reinterpret_cast<float*>(tc_sm) + (size_t)warp * (16 * HD + 32);
#pragma unroll
    for (int n = 0; n < MT; n++) {
        const int d = n * 16 + g;
        mw[(2 * t) * HD + d] = o[n][0];
        mw[(2 * t + 1) * HD + d] = o[n][1];
        mw[(2 * t) * HD + d + 8] = o[n][2];
        mw[(2 * t + 1) * HD + d + 8] = o[n][3];
    }
    if (g == 0) {
        mw[16 * HD + 2 * t] = mrun[0];
        mw[16 * HD + 2 * t + 1] = mrun[1];
        mw[16 * HD + 16 + 2 * t] = lrun[0];
        mw[16 * HD + 16 + 2 * t + 1] = lrun[1];
    }
    attn_tc_merge<HD, Q8>(tc_sm, G, n_heads, n_kv, kvh, m, s, nsplit, part, counters, out, xq, dx,
                          dxt, warp, lane);
}

// ---- RoPE + KV append over product rows (wide batches, prefill chunks) ----------
// The tensor-core product writes qkv [M][Nq + 2 Nkv] with the Q and K rows of
// each head in the (j, j + hd/2) pair order of the permuted weight.  One warp
// per (row, head): it reads the whole head, then rotates Q back into natural
// order in place and writes K (rotated) and V into the KV page of the row's
// position, as the GEMV's RoPE/KV epilogue does.  Decode steps (T == 0): row
// m is sequence m at position pos[m].  Prefill chunks (T > 0): row m is
// sequence m / T at position p0 + m % T.
template <typename KV>
__global__ void rope_kv_rows_kernel(float* __restrict__ qkv, int M, int n_heads, int n_kv, int hd,
                                   const int* __restrict__ pos, int T, int p0,
                                   const float2* __restrict__ rope,
                                   int max_ctx, const int* __restrict__ block_table, int max_blocks,
                                   int B, KV* __restrict__ kc, KV* __restrict__ vc,
                                   int* __restrict__ status) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int heads = n_heads + 2 * n_kv;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (gw >= M * heads) return;
    const int m = gw / heads, hh = gw % heads;
    const int half = hd / 2;
    const int seq = T > 0 ? m / T : m;
    const int p = T > 0 ? p0 + m % T : ld_cg(pos + m);
    if (p < 0 || p >= max_ctx) {
        if (lane == 0) record_status(status, AXQ8_ERR_INVALID);
        return;
    }
    const int page = block_table[seq * max_blocks + p / B], slot = p % B;
    const int ldq = (n_heads + 2 * n_kv) * hd;
    float* row = qkv + (int64_t)m * ldq + (int64_t)hh * hd;
    if (hh >= n_heads + n_kv) {                       // V: natural order, copy
        KV* dst = vc + (((int64_t)page * n_kv + (hh - n_heads - n_kv)) * B + slot) * hd;
        for (int d = lane; d < hd; d += 32) kv_store(dst + d, ld_cg(row + d));
        return;
    }
    // pairs j = lane, lane + 32 (hd <= 128)
    float v0[2], v1[2];
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int j = lane + 32 * t;
        if (j < half) {
            const float2 pr = ld_cg2(row + 2 * j);
            v0[t] = pr.x;
            v1[t] = pr.y;
        }
    }
    __syncwarp();
    const bool isk = hh >= n_heads;
    KV* kdst = isk ? kc + (((int64_t)page * n_kv + (hh - n_heads)) * B + slot) * hd : nullptr;
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int j = lane + 32 * t;
        if (j >= half) continue;
        const float2 cs = rope[(int64_t)p * half + j];
        const float r0 = __fsub_rn(__fmul_rn(v0[t], cs.x), __fmul_rn(v1[t], cs.y));
        const float r1 = __fadd_rn(__fmul_rn(v0[t], cs.y), __fmul_rn(v1[t], cs.x));
        if (!isk) {
            row[j] = r0;
            row[j + half] = r1;
        } else {
            kv_store(kdst + j, r0);
            kv_store(kdst + j + half, r1);
        }
    }
}

// ---- batched prefill: prompt tokens of a chunk ------------------------------------
// ptok[s * T + t] = feed[s * feed_len + p0 + t]: the chunk's rows, sequence-major.
static __global__ void gather_chunk_tokens_kernel(const int* __restrict__ feed, int feed_len, int n_seq,
                                           int T, int p0, int* __restrict__ ptok) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_seq * T) return;
    ptok[i] = ld_cg(feed + (int64_t)(i / T) * feed_len + p0 + i % T);
}

// ---- causal attention over a prompt chunk (batched prefill) ----------------------
// Reference: mha_attention / sdpa_causal (inference/cpp/runtime/mha.cpp:126-198):
// query position i of a head attends to keys 0..i of its GQA kv head
// (kv = h / (n_head / n_kv)), scores scaled by 1/sqrt(hd) after the dot,
// max-subtracted softmax, out = sum p*v / sum p.
//
// The chunk's rows r = s * T + t hold sequence s at position p0 + t; its K and
// V (and those of every earlier position) are already in the fp16 pages.
// Grid (tiles * HG, n_kv, n_seq) with HG = G / Gc head groups of Gc = min(G, 8)
// heads; 8 warps per CTA, warp w serving query head (w % Gc) of the group for
// the 16 positions tile*TQ + 16*(w / Gc) .. +15 (TQ = 16 * 8 / Gc positions per
// CTA), so the G heads of a kv head share every staged page.  The CTA walks
// the pages 0 .. of its last position in stages of kPrefPages pages (K and V
// by cp.async, double buffered, rows XOR-swizzled by 16-byte chunk for
// conflict-free ldmatrix), each warp skipping pages past its own positions.
// Per page and warp, as the decode kernel above: S [16 positions x 16 keys] =
// Q K^T and O += P V with mma.sync m16n8k16, Q and P split into an fp16 high
// part and an fp16 residual (fp32 accuracy against the exact fp16 K, V), the
// causal mask key > position applied to the scaled scores, online softmax
// with expf.  The output row (position, head) is divided by its sum and, with
// Q8, quantized to A8 in 32-dim blocks (transposed scales, pitch dxt) for the
// O projection, else stored as fp32 rows of `out`.
constexpr int kPrefWarps = 8;
constexpr int kPrefPages = 4;
template <int HD>
constexpr size_t attn_prefill_smem_bytes() {
    return (size_t)2 /*buffers*/ * kPrefPages * 2 /*K,V*/ * 16 * HD * 2;
}

template <int HD, bool Q8>
__global__ void __launch_bounds__(kPrefWarps * 32)
    attn_prefill_kernel(const float* __restrict__ qkv, int ldq, int T, int p0,
                        const __half* __restrict__ kc, const __half* __restrict__ vc,
                        const int* __restrict__ block_table, int max_blocks, int n_kv, int G,
                        float scale, int8_t* __restrict__ xq, int ldo, float* __restrict__ dxT,
                        int dxt, float* __restrict__ out) {
    constexpr int B = 16;
    constexpr int KS = HD / 16;          // k-steps of the score product
    constexpr int NT = HD / 8;           // n-tiles (8 dims) of the output
    constexpr int CH = HD / 8;           // 16-byte chunks per K/V row
    constexpr int PAGE = B * HD;         // halves per K (or V) page
    constexpr int SP = kPrefPages;
    extern __shared__ __align__(16) uint8_t pf_sm[];
    __half* stage = reinterpret_cast<__half*>(pf_sm);   // [2][SP][K,V][B][HD]
    const uint32_t stage_s = smem_u32(stage);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int Gc = G < 8 ? G : 8, HG = G / Gc;
    const int TQ = 16 * (kPrefWarps / Gc);
    const int tile = blockIdx.x / HG, hgrp = blockIdx.x % HG;
    const int kvh = blockIdx.y, s = blockIdx.z;
    const int head = kvh * G + hgrp * Gc + warp % Gc;
    const int t0 = tile * TQ + (warp / Gc) * 16;          // this warp's first chunk position
    const int cta_end = min(T, tile * TQ + TQ);           // the CTA's positions end here
    const int npages = (p0 + cta_end + B - 1) / B;         // keys 0 .. p0 + cta_end - 1
    const int nst = (npages + SP - 1) / SP;
    const bool active = t0 < T && warp / Gc < kPrefWarps / Gc;
    const int my_last = p0 + min(t0 + 15, T - 1);          // last position of this warp
    const int qp0 = p0 + t0 + g, qp1 = qp0 + 8;            // positions of rows g, g + 8
    pdl_launch_dependents();
    pdl_wait();
    const int* bt = block_table + (int64_t)s * max_blocks;
    auto issue = [&](int st) {
        __half* buf = stage + (size_t)(st & 1) * SP * 2 * PAGE;
        for (int c = threadIdx.x; c < SP * B * CH; c += blockDim.x) {
            const int j = c / (B * CH), r = (c / CH) % B, ch = c % CH;
            const int pg = st * SP + j;
            if (pg >= npages) continue;
            const int64_t off = (((int64_t)bt[pg] * n_kv + kvh) * B + r) * HD + ch * 8;
            const int sw = r * HD + ((ch ^ (r & 7)) * 8);
            __half* kb = buf + (size_t)j * 2 * PAGE;
            cp_async16(kb + sw, kc + off);
            cp_async16(kb + PAGE + sw, vc + off);
        }
    };
    // Q fragments: rows = positions t0 + g (+8) of `head`, fp16 high and residual
    uint32_t qh[KS][4], ql[KS][4];
    {
#pragma unroll
        for (int k = 0; k < KS; k++) {
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int tr = t0 + g + ((r & 1) ? 8 : 0);
                const int col = k * 16 + 2 * t + ((r & 2) ? 8 : 0);
                float x = 0.0f, y = 0.0f;
                if (active && tr < T) {
                    const float2 v =
                        ld_cg2(qkv + ((int64_t)s * T + tr) * ldq + (int64_t)head * HD + col);
                    x = v.x;
                    y = v.y;
                }
                split_pair(x, y, qh[k][r], ql[k][r]);
            }
        }
    }
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float mrun[2] = {-CUDART_INF_F, -CUDART_INF_F}, lrun[2] = {0.0f, 0.0f};
    issue(0);
    cp_async_commit();
    for (int st = 0; st < nst; st++) {
        if (st + 1 < nst) {
            issue(st + 1);
            cp_async_commit();
            cp_async_wait_group<1>();
        } else {
            cp_async_wait_group<0>();
        }
        __syncthreads();   // stage st visible to every warp
#pragma unroll 1
        for (int j = 0; j < SP; j++) {
            const int pg = st * SP + j;
            if (!active || pg >= npages || pg * B > my_last) break;   // warp-uniform
            const uint32_t kb = stage_s + (uint32_t)((((st & 1) * SP + j) * 2 * PAGE) * 2);
            const uint32_t vb = kb + PAGE * 2;
            float sc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
            {
                const int mi = lane >> 3, rr = lane & 7;
                const int tok = rr + ((mi >> 1) << 3);
#pragma unroll
                for (int k = 0; k < KS; k++) {
                    const int ch = k * 2 + (mi & 1);
                    uint32_t kf[4];
                    ldsm_x4(kf, kb + (uint32_t)((tok * HD + ((ch ^ (tok & 7)) * 8)) * 2));
                    mma_f16_16816(sc[0], qh[k], kf[0], kf[1]);
                    mma_f16_16816(sc[0], ql[k], kf[0], kf[1]);
                    mma_f16_16816(sc[1], qh[k], kf[2], kf[3]);
                    mma_f16_16816(sc[1], ql[k], kf[2], kf[3]);
                }
            }
            float p[2][4];
#pragma unroll
            for (int hr = 0; hr < 2; hr++) {
                const int qp = hr ? qp1 : qp0;
                float mt = -CUDART_INF_F;
#pragma unroll
                for (int n = 0; n < 2; n++)
#pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
                        const int key = pg * B + n * 8 + 2 * t + jj;
                        float& v = sc[n][2 * hr + jj];
                        v = key <= qp ? __fmul_rn(v, scale) : -CUDART_INF_F;
                        mt = fmaxf(mt, v);
                    }
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
                // page 0 holds key 0 <= every position, so mrun is finite after it
                const float mnew = fmaxf(mrun[hr], mt);
                const float corr = mrun[hr] == -CUDART_INF_F ? 0.0f : expf(mrun[hr] - mnew);
                float ps = 0.0f;
#pragma unroll
                for (int n = 0; n < 2; n++)
#pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
                        const float v = sc[n][2 * hr + jj];
                        const float e = v == -CUDART_INF_F ? 0.0f : expf(v - mnew);
                        p[n][2 * hr + jj] = e;
                        ps += e;
                    }
                lrun[hr] = fmaf(lrun[hr], corr, ps);
                mrun[hr] = mnew;
#pragma unroll
                for (int n = 0; n < NT; n++) {
                    o[n][2 * hr] *= corr;
                    o[n][2 * hr + 1] *= corr;
                }
            }
            uint32_t ph[4], pl[4];
            split_pair(p[0][0], p[0][1], ph[0], pl[0]);
            split_pair(p[0][2], p[0][3], ph[1], pl[1]);
            split_pair(p[1][0], p[1][1], ph[2], pl[2]);
            split_pair(p[1][2], p[1][3], ph[3], pl[3]);
            {
                const int mi = lane >> 3, rr = lane & 7;
                const int tok = rr + ((mi & 1) << 3);
#pragma unroll
                for (int dn = 0; dn < HD / 16; dn++) {
                    const int ch = dn * 2 + (mi >> 1);
                    uint32_t vf[4];
                    ldsm_x4_t(vf, vb + (uint32_t)((tok * HD + ((ch ^ (tok & 7)) * 8)) * 2));
                    mma_f16_16816(o[2 * dn], ph, vf[0], vf[1]);
                    mma_f16_16816(o[2 * dn], pl, vf[0], vf[1]);
                    mma_f16_16816(o[2 * dn + 1], ph, vf[2], vf[3]);
                    mma_f16_16816(o[2 * dn + 1], pl, vf[2], vf[3]);
                }
            }
        }
        __syncthreads();   // every warp is done with buffer st & 1 before it is refilled
    }
    if (!active) return;
#pragma unroll
    for (int hr = 0; hr < 2; hr++) {
        lrun[hr] += __shfl_xor_sync(0xffffffffu, lrun[hr], 1);
        lrun[hr] += __shfl_xor_sync(0xffffffffu, lrun[hr], 2);
    }
    // out = O / l, quantized per 32-dim block (n-tiles 4b .. 4b + 3; the quad
    // t = 0..3 holds the block's 32 values of each row)
#pragma unroll
    for (int hr = 0; hr < 2; hr++) {
        const int tr = t0 + g + 8 * hr;
        const bool ok = tr < T;
        const int64_t row = (int64_t)s * T + tr;
#pragma unroll
        for (int b = 0; b < HD / 32; b++) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                v[2 * i] = __fdiv_rn(o[4 * b + i][2 * hr], lrun[hr]);
                v[2 * i + 1] = __fdiv_rn(o[4 * b + i][2 * hr + 1], lrun[hr]);
            }
            if (!Q8) {   // fp32 rows [n_seq * T][ldo]
                if (ok) {
                    float* orow = out + row * ldo + (int64_t)head * HD + 32 * b;
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        *reinterpret_cast<float2*>(orow + 8 * i + 2 * t) = make_float2(v[2 * i], v[2 * i + 1]);
                }
                continue;
            }
            uint32_t ab = 0;
#pragma unroll
            for (int e = 0; e < 8; e++) ab = max(ab, __float_as_uint(fabsf(v[e])));
            ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, 1));
            ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, 2));
            const float amax = __uint_as_float(ab);
            const float id = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
            if (!ok) continue;
            int8_t* qrow = xq + row * ldo + (int64_t)head * HD + 32 * b;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t q0 = (uint32_t)(uint8_t)(int8_t)q8_round(__fmul_rn(v[2 * i], id));
                const uint32_t q1 = (uint32_t)(uint8_t)(int8_t)q8_round(__fmul_rn(v[2 * i + 1], id));
                *reinterpret_cast<uint16_t*>(qrow + 8 * i + 2 * t) = (uint16_t)(q0 | (q1 << 8));
            }
            if (t == 0)
                dxT[((int64_t)head * HD / QK + b) * dxt + row] = __fdiv_rn(amax, 127.0f);
        }
    }
}

// ---- greedy argmax over logit rows (wide batches) ---------------------------------
// Grid (chunks, M): each CTA folds its part of row m into amax_key[m] (zero
// before; argmax_advance_kernel consumes and clears it).
static __global__ void argmax_rows_kernel(const float* __restrict__ logits, int V, int idx_offset,
                                   unsigned long long* __restrict__ amax_key) {
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.y;
    const float* row = logits + (int64_t)m * V;
    unsigned long long best = 0ull;
    // 4 consecutive logits per load, 4 loads in flight per thread (rows of V %
    // 4 == 0 floats start 16-byte aligned; other widths take the scalar loop)
    const int stride = gridDim.x * blockDim.x;
    const int i0 = blockIdx.x * blockDim.x + threadIdx.x;
    if ((V & 3) == 0) {
        const int V4 = V / 4;
        for (int i = i0; i < V4; i += 4 * stride) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                v[u] = i + u * stride < V4 ? ld_cg4(row + 4 * (i + u * stride))
                                           : make_float4(-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F,
                                                         -CUDART_INF_F);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (i + u * stride >= V4) break;
                const int c = 4 * (i + u * stride) + idx_offset;
                const unsigned long long k0 = argmax_key(v[u].x, c), k1 = argmax_key(v[u].y, c + 1);
                const unsigned long long k2 = argmax_key(v[u].z, c + 2), k3 = argmax_key(v[u].w, c + 3);
                best = k0 > best ? k0 : best;
                best = k1 > best ? k1 : best;
                best = k2 > best ? k2 : best;
                best = k3 > best ? k3 : best;
            }
        }
    } else {
        for (int i = i0; i < V; i += stride) {
            const unsigned long long k = argmax_key(ld_cg(row + i), i + idx_offset);
            best = k > best ? k : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if ((threadIdx.x & 31) == 0 && best) atomicMax(amax_key + m, best);
}

// ---- greedy step advance after a cross-rank argmax ------------------------------
// The tensor-parallel LM head (and the wide-batch argmax) leave each
// sequence's packed (logit, global index) key in amax_key; after the max
// all-reduce over ranks one thread per sequence performs the advance of the argmax epilogue: record the token,
// feed the next input (prompt token or the argmax), move the position, and
// zero the key for the next step.
static __global__ void argmax_advance_kernel(unsigned long long* __restrict__ amax_key, int M,
                                      int* __restrict__ pos, int* __restrict__ tokens,
                                      const int* __restrict__ feed, const int* __restrict__ ctl,
                                      int* __restrict__ out_tokens, int* __restrict__ argmax_out) {
    pdl_launch_dependents();
    pdl_wait();
    const int n_prompt = ld_cg(ctl), feed_len = ld_cg(ctl + 1), max_out = ld_cg(ctl + 2);
    // one thread per sequence: the sequences' advances are independent
    for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
        const unsigned long long k = __ldcg(amax_key + m);
        amax_key[m] = 0ull;
        const int idx = k == 0ull ? 0 : argmax_key_index(k);
        const int p = ld_cg(pos + m);
        const int np = p + 1;
        argmax_out[m] = idx;
        if (np >= n_prompt && np - n_prompt < max_out) out_tokens[m * max_out + (np - n_prompt)] = idx;
        tokens[m] = np < feed_len ? ld_cg(feed + m * feed_len + np) : idx;
        pos[m] = np;
    }
}

// ---- SiLU(gate) * up (+ A8 quantization) -------------------------------------------
// gu row = (gate_0, up_0, gate_1, up_1, ...): the product of the gate|up weight
// stored with gate row j and up row j interleaved.  a = (g / (1 + e^-g)) * u,
// rounded per op as silu.cpp and elementwise.cpp do.  8 consecutive outputs
// per thread (4 threads per 32-block); F % 32 == 0.
template <bool Q8>
__global__ void silu_mul_kernel(const float* __restrict__ gu, int F, int M,
                                float* __restrict__ out, int8_t* __restrict__ xq,
                                float* __restrict__ dx, int dxt) {
    pdl_launch_dependents();
    pdl_wait();
    const int nu = F / 8, nb = F / QK;
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const bool valid = j < (int64_t)M * nu;
    const int m = valid ? (int)(j / nu) : 0, c = valid ? (int)(j % nu) : 0;
    float g[8], u[8], a[8];
    if (valid) {
        float p[16];
        load8_cg(gu + (int64_t)m * 2 * F + 16 * c, *reinterpret_cast<float(*)[8]>(p));
        load8_cg(gu + (int64_t)m * 2 * F + 16 * c + 8, *reinterpret_cast<float(*)[8]>(p + 8));
#pragma unroll
        for (int e = 0; e < 8; e++) {
            g[e] = p[2 * e];
            u[e] = p[2 * e + 1];
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) g[e] = u[e] = 0.0f;
    }
#pragma unroll
    for (int e = 0; e < 8; e++) a[e] = __fmul_rn(__fdiv_rn(g[e], __fadd_rn(1.0f, expf(-g[e]))), u[e]);
    if (!Q8) {
        if (valid) store8(out + (int64_t)m * F + 8 * c, a);
    } else {
        const int b = c >> 2;
        quant_block_quad(a, lane, valid, xq + (int64_t)m * F + 8 * c,
                         dx + (dxt ? (int64_t)b * dxt + m : (int64_t)m * nb + b));
    }
}

}  // namespace axq8
