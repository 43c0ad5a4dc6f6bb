// Paged KV cache entry points (include/axkv.h): KV append over caller-owned
// pages, and the decode attention kernels of the decode step (decode_ops.cuh)
// over them with fp32 output.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <type_traits>

#include "axkv.h"
#include "common.cuh"
#include "decode_ops.cuh"
#include "runtime.h"

using namespace axq8;

namespace {

// One warp per (row, kv head): its K and V head vectors into the page slot.
template <typename KV>
__global__ void kv_append_kernel(const float* __restrict__ k_rows, const float* __restrict__ v_rows,
                                 int n_rows, const int* __restrict__ row_seq,
                                 const int* __restrict__ row_pos, KV* __restrict__ kc,
                                 KV* __restrict__ vc, const int* __restrict__ block_table,
                                 int max_blocks, int n_pages, int n_kv, int hd, int B,
                                 int* __restrict__ status) {
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gw >= n_rows * n_kv) return;
    const int r = gw / n_kv, h = gw % n_kv;
    const int p = row_pos[r], s = row_seq[r];
    const int page = p >= 0 && p < max_blocks * B && s >= 0
                         ? block_table[(int64_t)s * max_blocks + p / B] : -1;
    if (page < 0 || page >= n_pages) {
        if (lane == 0) record_status(status, AXQ8_ERR_INVALID);
        return;
    }
    const int64_t dst = (((int64_t)page * n_kv + h) * B + p % B) * hd;
    const int64_t src = (int64_t)r * n_kv * hd + (int64_t)h * hd;
    for (int d = lane; d < hd; d += 32) {
        kv_store(kc + dst + d, k_rows[src + d]);
        kv_store(vc + dst + d, v_rows[src + d]);
    }
}

bool n_kv_ok(const axkv_cache_t* c, int n_heads) {
    return n_heads > 0 && n_heads % c->n_kv_heads == 0;
}

int check_cache(const axkv_cache_t* c, const char* what) {
    if (!c || !c->k_pages || !c->v_pages || !c->block_table)
        return fail(AXQ8_ERR_INVALID, "%s: null cache pointer", what);
    if (c->page_tokens != 16)
        return fail(AXQ8_ERR_UNSUPPORTED, "%s: page_tokens must be 16", what);
    if (c->head_dim != 32 && c->head_dim != 64 && c->head_dim != 128)
        return fail(AXQ8_ERR_UNSUPPORTED, "%s: head_dim %d (32, 64, 128)", what, c->head_dim);
    if (c->n_pages <= 0 || c->max_blocks <= 0 || c->n_kv_heads <= 0)
        return fail(AXQ8_ERR_INVALID, "%s: non-positive cache dimension", what);
    return AXQ8_OK;
}

// Context splits of the decode attention: about four CTAs per SM, down to
// one page per split, at most 32 (the merge gives one lane to each split).
void plan_splits(const axkv_cache_t* c, int n_seq, int sm_count, int* nsplit, int* bps) {
    const int target = (4 * sm_count + c->n_kv_heads * n_seq - 1) / (c->n_kv_heads * n_seq);
    int ns = std::max(1, std::min(std::min(target, c->max_blocks), 32));
    *bps = (c->max_blocks + ns - 1) / ns;
    *nsplit = (c->max_blocks + *bps - 1) / *bps;
}

template <typename KV, int HD>
int launch_attn(DeviceState* ds, const axkv_cache_t* c, const float* q, int n_seq, int n_heads,
                const int* q_pos, float* out, float* part, int* counters, int nsplit, int bps,
                cudaStream_t s) {
    const int G = n_heads / c->n_kv_heads;
    const float scale = 1.0f / std::sqrt((float)HD);   // mha.cpp:250
    if constexpr (std::is_same<KV, __half>::value && HD >= 64) {
        if (n_seq >= 2) {
            const bool tr = G <= 8;   // groups of at most 8 heads: tokens as the MMA rows
            const size_t smem = tr ? attn_tct_smem_bytes<HD>(bps) : attn_tc_smem_bytes<HD>(bps);
            auto kern = tr ? attn_tct_kernel<HD, false> : attn_tc_kernel<HD, false>;
            constexpr int kMaxSmem = 200 * 1024;
            if (smem > (size_t)kMaxSmem) return fail(AXQ8_ERR_UNSUPPORTED, "attention: shared memory");
            static int configured[2][64] = {{0}};
            const int dev = ds->device < 64 ? ds->device : 63;
            if (smem > 48 * 1024 && !configured[tr][dev]) {
                AXQ8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   kMaxSmem),
                              "attention smem attribute");
                configured[tr][dev] = 1;
            }
            AXQ8_CUDA_TRY(launch_k(kern, dim3(c->n_kv_heads, n_seq, nsplit), dim3(kAttnTcWarps * 32),
                                   smem, s, false, q, n_heads * HD, q_pos, (const __half*)c->k_pages,
                                   (const __half*)c->v_pages, c->block_table, c->max_blocks, n_heads,
                                   c->n_kv_heads, G, bps, scale, part, counters, out,
                                   (int8_t*)nullptr, (float*)nullptr, 0),
                          "axkv_paged_decode_attn launch");
            return AXQ8_OK;
        }
    }
    const int cp = std::max(1, std::min(bps, (int)(32768 / (4 * 16 * HD * sizeof(KV)))));
    const size_t smem = attn_smem_bytes<KV, HD>(G, cp, bps);
    if (smem > 48 * 1024) return fail(AXQ8_ERR_UNSUPPORTED, "attention: %zu B of shared memory", smem);
    AXQ8_CUDA_TRY(launch_k(attn_decode_kernel<KV, HD, false>, dim3(c->n_kv_heads, n_seq, nsplit),
                           dim3(G * 32), smem, s, false, q, n_heads * HD, q_pos,
                           (const KV*)c->k_pages, (const KV*)c->v_pages, c->block_table,
                           c->max_blocks, n_heads, c->n_kv_heads, bps, cp, scale, part, counters,
                           out, (int8_t*)nullptr, (float*)nullptr, 0),
                  "axkv_paged_decode_attn launch");
    return AXQ8_OK;
}

template <int HD, bool Q8>
int prefill_launch(DeviceState* ds, const axkv_cache_t* c, dim3 grid, const float* q, int64_t ldq,
                   int T, int p0, int G, int n_heads, float scale, int8_t* xq, float* dxT, int dxt,
                   float* out, cudaStream_t s) {
    constexpr size_t smem = attn_prefill_smem_bytes<HD>();
    auto kern = attn_prefill_kernel<HD, Q8>;
    static int configured[64] = {0};
    const int dev = ds->device < 64 ? ds->device : 63;
    if (smem > 48 * 1024 && !configured[dev]) {
        AXQ8_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                      "prefill attention smem attribute");
        configured[dev] = 1;
    }
    AXQ8_CUDA_TRY(launch_k(kern, grid, dim3(kPrefWarps * 32), smem, s, false, q, (int)ldq, T, p0,
                           (const __half*)c->k_pages, (const __half*)c->v_pages, c->block_table,
                           c->max_blocks, c->n_kv_heads, G, scale, xq, n_heads * HD, dxT, dxt, out),
                  "axkv_paged_prefill_attn launch");
    return AXQ8_OK;
}

}  // namespace

extern "C" {

int64_t axkv_pages_bytes(const axkv_cache_t* c) {
    if (!c) return 0;
    return (int64_t)c->n_pages * c->n_kv_heads * c->page_tokens * c->head_dim *
           (c->kv_fp32 ? 4 : 2);
}

int axkv_paged_append(const axkv_cache_t* c, const float* k_rows, const float* v_rows,
                      int32_t n_rows, const int32_t* row_seq, const int32_t* row_pos,
                      void* stream) {
    int rc = check_cache(c, "axkv_paged_append");
    if (rc) return rc;
    if (n_rows < 0) return fail(AXQ8_ERR_INVALID, "axkv_paged_append: n_rows < 0");
    if (n_rows == 0) return AXQ8_OK;
    if (!k_rows || !v_rows || !row_seq || !row_pos)
        return fail(AXQ8_ERR_INVALID, "axkv_paged_append: null pointer");
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    const int64_t warps = (int64_t)n_rows * c->n_kv_heads;
    const dim3 grid((unsigned)((warps + 7) / 8));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (c->kv_fp32)
        AXQ8_CUDA_TRY(launch_k(kv_append_kernel<float>, grid, dim3(256), 0, s, false, k_rows, v_rows,
                               (int)n_rows, row_seq, row_pos, (float*)c->k_pages, (float*)c->v_pages,
                               c->block_table, c->max_blocks, c->n_pages, c->n_kv_heads, c->head_dim,
                               c->page_tokens, ds->status),
                      "axkv_paged_append launch");
    else
        AXQ8_CUDA_TRY(launch_k(kv_append_kernel<__half>, grid, dim3(256), 0, s, false, k_rows, v_rows,
                               (int)n_rows, row_seq, row_pos, (__half*)c->k_pages, (__half*)c->v_pages,
                               c->block_table, c->max_blocks, c->n_pages, c->n_kv_heads, c->head_dim,
                               c->page_tokens, ds->status),
                      "axkv_paged_append launch");
    return AXQ8_OK;
}

int64_t axkv_decode_attn_workspace(const axkv_cache_t* c, int32_t n_seq, int32_t n_heads) {
    if (check_cache(c, "axkv_decode_attn_workspace") || n_seq <= 0 || n_heads <= 0) return -1;
    DeviceState* ds = device_state();
    if (!ds) return -1;
    int nsplit, bps;
    plan_splits(c, n_seq, ds->sm_count, &nsplit, &bps);
    const int64_t part = (int64_t)n_seq * n_heads * nsplit * (c->head_dim + 2) * 4;
    return (part + 255) / 256 * 256 + (int64_t)n_seq * c->n_kv_heads * 4;
}

int axkv_paged_decode_attn(const axkv_cache_t* c, const float* q, int32_t n_seq, int32_t n_heads,
                           const int32_t* q_pos, float* out, void* workspace,
                           int64_t workspace_bytes, void* stream) {
    int rc = check_cache(c, "axkv_paged_decode_attn");
    if (rc) return rc;
    if (n_seq <= 0 || n_heads <= 0 || n_heads % c->n_kv_heads || n_heads / c->n_kv_heads > 16)
        return fail(AXQ8_ERR_INVALID,
                    "axkv_paged_decode_attn: n_heads must be a multiple of n_kv_heads (<= 16x)");
    if (!q || !q_pos || !out || !workspace)
        return fail(AXQ8_ERR_INVALID, "axkv_paged_decode_attn: null pointer");
    if (reinterpret_cast<uintptr_t>(q) & 15 || reinterpret_cast<uintptr_t>(workspace) & 15)
        return fail(AXQ8_ERR_INVALID, "axkv_paged_decode_attn: q / workspace not 16-byte aligned");
    const int64_t need = axkv_decode_attn_workspace(c, n_seq, n_heads);
    if (workspace_bytes < need)
        return fail(AXQ8_ERR_INVALID, "axkv_paged_decode_attn: workspace %lld B < %lld B",
                    (long long)workspace_bytes, (long long)need);
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    int nsplit, bps;
    plan_splits(c, n_seq, ds->sm_count, &nsplit, &bps);
    float* part = static_cast<float*>(workspace);
    const int64_t part_bytes = (int64_t)n_seq * n_heads * nsplit * (c->head_dim + 2) * 4;
    int* counters = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + (part_bytes + 255) / 256 * 256);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int hd = c->head_dim;
    if (c->kv_fp32) {
        if (hd == 32) return launch_attn<float, 32>(ds, c, q, n_seq, n_heads, q_pos, out, part, counters, nsplit, bps, s);
        if (hd == 64) return launch_attn<float, 64>(ds, c, q, n_seq, n_heads, q_pos, out, part, counters, nsplit, bps, s);
        return launch_attn<float, 128>(ds, c, q, n_seq, n_heads, q_pos, out, part, counters, nsplit, bps, s);
    }
    if (hd == 32) return launch_attn<__half, 32>(ds, c, q, n_seq, n_heads, q_pos, out, part, counters, nsplit, bps, s);
    if (hd == 64) return launch_attn<__half, 64>(ds, c, q, n_seq, n_heads, q_pos, out, part, counters, nsplit, bps, s);
    return launch_attn<__half, 128>(ds, c, q, n_seq, n_heads, q_pos, out, part, counters, nsplit, bps, s);
}

int axkv_paged_prefill_attn(const axkv_cache_t* c, const float* q, int64_t ldq, int32_t n_seq,
                            int32_t T, int32_t p0, int32_t n_heads, float* out, int8_t* xq,
                            float* dxT, void* stream) {
    int rc = check_cache(c, "axkv_paged_prefill_attn");
    if (rc) return rc;
    const int G = n_kv_ok(c, n_heads) ? n_heads / c->n_kv_heads : 0;
    if (!G || (G > 8 && G % 8))
        return fail(AXQ8_ERR_INVALID, "axkv_paged_prefill_attn: n_heads / n_kv_heads must be "
                                      "<= 8 or a multiple of 8");
    if (c->kv_fp32 || (c->head_dim != 64 && c->head_dim != 128))
        return fail(AXQ8_ERR_UNSUPPORTED, "axkv_paged_prefill_attn: fp16 pages, head dim 64 or 128");
    if (n_seq <= 0 || T <= 0 || p0 < 0 || (int64_t)p0 + T > (int64_t)c->max_blocks * c->page_tokens ||
        ldq < (int64_t)n_heads * c->head_dim)
        return fail(AXQ8_ERR_INVALID, "axkv_paged_prefill_attn: bad sizes");
    if (!q || (reinterpret_cast<uintptr_t>(q) & 7) ||
        (xq ? !dxT || (reinterpret_cast<uintptr_t>(xq) & 1)
            : !out || (reinterpret_cast<uintptr_t>(out) & 7)))
        return fail(AXQ8_ERR_INVALID, "axkv_paged_prefill_attn: null or unaligned pointer");
    const int dxt = (int)(((int64_t)n_seq * T + 3) / 4 * 4);
    DeviceState* ds = device_state();
    if (!ds) return AXQ8_ERR_CUDA;
    const int Gc = std::min(G, 8), HG = G / Gc, TQ = 16 * (kPrefWarps / Gc);
    const dim3 grid((unsigned)(((T + TQ - 1) / TQ) * HG), c->n_kv_heads, n_seq);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float scale = 1.0f / std::sqrt((float)c->head_dim);   // mha.cpp:131
    if (c->head_dim == 64)
        return xq ? prefill_launch<64, true>(ds, c, grid, q, ldq, T, p0, G, n_heads, scale, xq, dxT,
                                             dxt, out, s)
                  : prefill_launch<64, false>(ds, c, grid, q, ldq, T, p0, G, n_heads, scale, xq,
                                              dxT, dxt, out, s);
    return xq ? prefill_launch<128, true>(ds, c, grid, q, ldq, T, p0, G, n_heads, scale, xq, dxT,
                                          dxt, out, s)
              : prefill_launch<128, false>(ds, c, grid, q, ldq, T, p0, G, n_heads, scale, xq, dxT,
                                           dxt, out, s);
}

}  // extern "C"
