// Decode-step kernels around the Q8_0 GEMV (sm_100a).
//
// Reference semantics (paths inside the reference project):
//   token_embedding           inference/cpp/runtime/token_embedding.cpp (row of the
//                             dequantized token_embd, gguf.cpp:870-882)
//   rmsnorm                   inference/cpp/kernels/rmsnorm.cpp:12-100
//   rope_apply_row_at (NEOX)  inference/cpp/runtime/mha.cpp:15-55, :200-225
//   append_row                inference/cpp/runtime/streaming_executor.cpp:255-266
//   mha_attention_incremental inference/cpp/runtime/mha.cpp:227-285
//   silu * up                 inference/cpp/kernels/silu.cpp:13-65, elementwise.cpp:13-67
//   greedy argmax             inference/cpp/runtime/sampler.cpp:11-24
//
// Every kernel calls griddepcontrol.wait before its first global write or
// its first read of data another kernel produced, and every kernel of the
// step does so unconditionally: completion of kernel i then implies
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

namespace axq8 {

__device__ inline float kv_to_float(__half v) { return __half2float(v); }
__device__ inline float kv_to_float(float v) { return v; }
__device__ inline void kv_store(__half* p, float v) { *p = __float2half_rn(v); }
__device__ inline void kv_store(float* p, float v) { *p = v; }

// Quantize one 32-block held one element per lane (all 32 lanes active).
__device__ __forceinline__ void quant_block_warp(float v, int lane, int8_t* q, float* d) {
    const uint32_t abits = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
    const float amax = __uint_as_float(abits);
    const float id = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
    q[lane] = (int8_t)q8_round(__fmul_rn(v, id));
    if (lane == 0) *d = __fdiv_rn(amax, 127.0f);
}

// ---- embedding ----------------------------------------------------------------
// h[m, :] = dequantized row tokens[m] of token_embd (repacked Q8_0 rows).
__global__ void embed_kernel(const uint8_t* __restrict__ rows, int64_t rs, int H, int V,
                             const int* __restrict__ tokens, float* __restrict__ h, int* status) {
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x;
    int tok = tokens[m];
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
// One CTA per row.  out = (x * (1/sqrt(mean(x^2) + eps))) * w with the
// reference's separately rounded operations; the sum of squares is a fixed
// tree (warp sums, then warps in order), not the reference's sequential sum.
template <bool Q8>
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, int H,
                               float eps, float* __restrict__ out, int8_t* __restrict__ xq,
                               float* __restrict__ dx) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x;
    const float* xr = x + (int64_t)m * H;
    float s = 0.0f;
    for (int k = threadIdx.x; k < H; k += blockDim.x) s = fmaf(xr[k], xr[k], s);
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
    if (!Q8) {
        for (int k = threadIdx.x; k < H; k += blockDim.x)
            out[(int64_t)m * H + k] = __fmul_rn(__fmul_rn(xr[k], inv), w[k]);
    } else {
        const int nb = H / QK;
        for (int b = warp; b < nb; b += nw) {
            const int k = b * QK + lane;
            const float v = __fmul_rn(__fmul_rn(xr[k], inv), w[k]);
            quant_block_warp(v, lane, xq + (int64_t)m * H + b * QK, dx + (int64_t)m * nb + b);
        }
    }
}

// ---- RoPE (NEOX) + KV page append ----------------------------------------------
// One CTA per sequence.  qkv row = [q (n_heads*hd) | k (n_kv*hd) | v (n_kv*hd)].
// The rotation uses the host-computed table tab[pos][i] = (cos, sin) of
// pos * theta^(-2i/hd), evaluated with the same expressions as the
// reference, and rounds a*c - b*s / a*s + b*c like its scalar code.  Rotated
// k and v are stored in the layer's pages: page = block_table[m][pos / B],
// layout [page][n_kv][B][hd].
template <typename KV>
__global__ void rope_kv_kernel(float* __restrict__ qkv, int ldq, const int* __restrict__ pos,
                               const float2* __restrict__ tab, int max_ctx, int n_heads, int n_kv,
                               int hd, KV* __restrict__ kc, KV* __restrict__ vc,
                               const int* __restrict__ block_table, int max_blocks, int B,
                               int* status) {
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x;
    const int p = pos[m];
    if (p < 0 || p >= max_ctx) {
        if (threadIdx.x == 0) record_status(status, AXQ8_ERR_INVALID);
        return;
    }
    const int half = hd / 2;
    float* row = qkv + (int64_t)m * ldq;
    const float2* t = tab + (int64_t)p * half;
    const int page = block_table[m * max_blocks + p / B];
    const int slot = p % B;
    const int nq_pairs = n_heads * half;
    const int nk_pairs = n_kv * half;
    for (int i = threadIdx.x; i < nq_pairs + nk_pairs; i += blockDim.x) {
        const bool is_k = i >= nq_pairs;
        const int ii = is_k ? i - nq_pairs : i;
        const int head = ii / half, j = ii % half;
        float* base = row + (is_k ? n_heads * hd : 0) + head * hd;
        const float a = base[j], b = base[j + half];
        const float2 cs = t[j];
        const float r0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        const float r1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
        if (!is_k) {
            base[j] = r0;
            base[j + half] = r1;
        } else {
            KV* dst = kc + (((int64_t)page * n_kv + head) * B + slot) * hd;
            kv_store(dst + j, r0);
            kv_store(dst + j + half, r1);
        }
    }
    const float* v = row + (n_heads + n_kv) * hd;
    for (int i = threadIdx.x; i < n_kv * hd; i += blockDim.x) {
        const int head = i / hd, d = i % hd;
        kv_store(vc + (((int64_t)page * n_kv + head) * B + slot) * hd + d, v[i]);
    }
}

// ---- attention: split-K flash decode ----------------------------------------------
// Grid (n_kv, M, nsplit); G warps per CTA, warp g serving query head
// kvh*G + g (GQA: query head h reads kv head h / G, mha.cpp:253-254).  Split
// s covers KV pages [s*bps, (s+1)*bps) of the sequence's pages in use
// (ctx = pos + 1 tokens).  Each page (B = 16 tokens) is staged in shared
// memory as fp32 and shared by the G warps.  Lane l scores token l & 15 over
// half the head dims (l >> 4); scores are scaled by 1/sqrt(hd) after the
// dot, as the reference does.  Online softmax; the partial
// (acc[hd], running max, running sum) of each (sequence, query head, split)
// goes to `part` and attn_combine_kernel merges the splits.
template <typename KV, int HD>
__global__ void attn_partial_kernel(const float* __restrict__ qkv, int ldq,
                                    const int* __restrict__ pos, const KV* __restrict__ kc,
                                    const KV* __restrict__ vc, const int* __restrict__ block_table,
                                    int max_blocks, int n_heads, int n_kv, int bps, float scale,
                                    float* __restrict__ part) {
    constexpr int B = 16;
    constexpr int DL = HD / 32;            // dims per lane in the value accumulation
    extern __shared__ __align__(16) float sm[];
    const int G = blockDim.x >> 5;
    float* ks = sm;                         // [B][HD]
    float* vs = ks + B * HD;                // [B][HD]
    float* qs = vs + B * HD;                // [G][HD]
    pdl_launch_dependents();
    pdl_wait();
    const int kvh = blockIdx.x, m = blockIdx.y, s = blockIdx.z, nsplit = gridDim.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * G + warp;
    // a position past the page table was already reported by rope_kv_kernel;
    // never read beyond the table
    const int ctx = min(pos[m] + 1, max_blocks * B);
    const int nblk = (ctx + B - 1) / B;
    const int b0 = s * bps, b1 = min(nblk, b0 + bps);
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x)
        qs[i] = qkv[(int64_t)m * ldq + (int64_t)(kvh * G) * HD + i];
    float mrun = -CUDART_INF_F, lrun = 0.0f;
    float acc[DL];
#pragma unroll
    for (int i = 0; i < DL; i++) acc[i] = 0.0f;
    const int t = lane & (B - 1), hf = lane >> 4;
    for (int blk = b0; blk < b1; blk++) {
        __syncthreads();   // previous page fully consumed (and qs written)
        const int page = block_table[m * max_blocks + blk];
        const KV* kp = kc + ((int64_t)page * n_kv + kvh) * B * HD;
        const KV* vp = vc + ((int64_t)page * n_kv + kvh) * B * HD;
        for (int i = threadIdx.x; i < B * HD; i += blockDim.x) {
            ks[i] = kv_to_float(kp[i]);
            vs[i] = kv_to_float(vp[i]);
        }
        __syncthreads();
        // score of token t, half hf of the dims, then combine the halves
        const float* q = qs + warp * HD + hf * (HD / 2);
        const float* k = ks + t * HD + hf * (HD / 2);
        float dot = 0.0f;
#pragma unroll 8
        for (int d = 0; d < HD / 2; d++) dot = fmaf(q[d], k[d], dot);
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
        for (int tt = 0; tt < B; tt++) {
            const float p = __shfl_sync(0xffffffffu, pt, tt);
#pragma unroll
            for (int i = 0; i < DL; i++) acc[i] = fmaf(p, vs[tt * HD + lane * DL + i], acc[i]);
        }
        mrun = mnew;
    }
    float* o = part + (((int64_t)m * n_heads + h) * nsplit + s) * (HD + 2);
#pragma unroll
    for (int i = 0; i < DL; i++) o[lane * DL + i] = acc[i];
    if (lane == 0) {
        o[HD] = mrun;
        o[HD + 1] = lrun;
    }
}

// Merge the nsplit partials of each (sequence, query head): one warp each.
// out = sum_s acc_s * e^(m_s - M) / sum_s l_s * e^(m_s - M).  With Q8 the
// head's output is quantized in 32-dim blocks (groups of 32/DL lanes).
template <int HD, bool Q8>
__global__ void attn_combine_kernel(const float* __restrict__ part, int M, int n_heads, int nsplit,
                                    float* __restrict__ out, int8_t* __restrict__ xq,
                                    float* __restrict__ dx) {
    constexpr int DL = HD / 32;
    pdl_launch_dependents();
    pdl_wait();
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gw >= M * n_heads) return;
    const int m = gw / n_heads, h = gw % n_heads;
    const float* p = part + ((int64_t)m * n_heads + h) * nsplit * (HD + 2);
    float mx = -CUDART_INF_F;
    for (int s = 0; s < nsplit; s++) mx = fmaxf(mx, p[s * (HD + 2) + HD]);
    float l = 0.0f;
    float acc[DL];
#pragma unroll
    for (int i = 0; i < DL; i++) acc[i] = 0.0f;
    for (int s = 0; s < nsplit; s++) {
        const float ms = p[s * (HD + 2) + HD];
        if (ms == -CUDART_INF_F) continue;      // empty split
        const float f = expf(ms - mx);
        l = fmaf(p[s * (HD + 2) + HD + 1], f, l);
#pragma unroll
        for (int i = 0; i < DL; i++) acc[i] = fmaf(p[s * (HD + 2) + lane * DL + i], f, acc[i]);
    }
    const int64_t base = (int64_t)m * n_heads * HD + (int64_t)h * HD + lane * DL;
    float v[DL];
#pragma unroll
    for (int i = 0; i < DL; i++) v[i] = __fdiv_rn(acc[i], l);
    if (!Q8) {
#pragma unroll
        for (int i = 0; i < DL; i++) out[base + i] = v[i];
        return;
    }
    // 32-dim block = 32/DL consecutive lanes
    float a = 0.0f;
#pragma unroll
    for (int i = 0; i < DL; i++) a = fmaxf(a, fabsf(v[i]));
#pragma unroll
    for (int o = 1; o < 32 / DL; o <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float id = a == 0.0f ? 0.0f : __fdiv_rn(127.0f, a);
#pragma unroll
    for (int i = 0; i < DL; i++) xq[base + i] = (int8_t)q8_round(__fmul_rn(v[i], id));
    if ((lane % (32 / DL)) == 0) dx[base / QK] = __fdiv_rn(a, 127.0f);
}

// ---- SiLU(gate) * up (+ A8 quantization) -------------------------------------------
// gu row = [gate (F) | up (F)].  a = (g / (1 + e^-g)) * u, rounded per op as
// silu.cpp and elementwise.cpp do.  One warp per 32-block.
template <bool Q8>
__global__ void silu_mul_kernel(const float* __restrict__ gu, int F, int M,
                                float* __restrict__ out, int8_t* __restrict__ xq,
                                float* __restrict__ dx) {
    pdl_launch_dependents();
    pdl_wait();
    const int nb = F / QK;
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gw >= M * nb) return;
    const int m = gw / nb, b = gw % nb;
    const int i = b * QK + lane;
    const float g = gu[(int64_t)m * 2 * F + i];
    const float u = gu[(int64_t)m * 2 * F + F + i];
    const float a = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    if (!Q8) {
        out[(int64_t)m * F + i] = a;
    } else {
        quant_block_warp(a, lane, xq + (int64_t)m * F + b * QK, dx + (int64_t)m * nb + b);
    }
}

// ---- greedy argmax + advance ----------------------------------------------------------
// One CTA per sequence.  next = first index of the maximum logit.  Then the
// next input is the fed token when one remains (prompt / teacher forcing),
// else `next`; generated tokens are recorded; pos advances by one.
// ctl = {n_prompt, feed_len, max_out}.
__global__ void argmax_advance_kernel(const float* __restrict__ logits, int V,
                                      int* __restrict__ tokens, int* __restrict__ pos,
                                      const int* __restrict__ feed, const int* __restrict__ ctl,
                                      int* __restrict__ out_tokens, int* __restrict__ argmax_out) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x;
    const float* lg = logits + (int64_t)m * V;
    float best = -CUDART_INF_F;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = lg[i];
        if (v > best) { best = v; idx = i; }   // ascending i: keeps the first maximum
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) { bv[warp] = best; bi[warp] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < nw; w++)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) { best = bv[w]; idx = bi[w]; }
        if (idx == 0x7fffffff) idx = 0;            // all logits NaN/-inf
        const int n_prompt = ctl[0], feed_len = ctl[1], max_out = ctl[2];
        const int p = pos[m];
        const int np = p + 1;
        argmax_out[m] = idx;
        if (np >= n_prompt && np - n_prompt < max_out) out_tokens[m * max_out + (np - n_prompt)] = idx;
        tokens[m] = np < feed_len ? feed[m * feed_len + np] : idx;
        pos[m] = np;
    }
}

}  // namespace axq8
