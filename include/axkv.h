/*
 * axkv.h — C ABI of the paged KV cache and its decode attention on B200.
 *
 * The cache lives in caller-owned device memory.  Per layer, K and V are
 * arrays of pages [n_pages][n_kv_heads][page_tokens][head_dim] (fp16, or fp32
 * with kv_fp32 = 1); token p of sequence s lives in page
 * block_table[s * max_blocks + p / page_tokens], slot p % page_tokens (the
 * block table is a caller-owned device array of int32).  Same conventions as
 * axq8.h: plain C, status codes, axq8_last_error().
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   PagedKVCache::initialize / append   inference/cpp/runtime/paged_kv.hpp:18-41,
 *                                       paged_kv.cpp:44-120 (fp32 rows of
 *                                       page_size x hidden; here fp16 pages of
 *                                       16 tokens per KV head)
 *   append_row (KV append per token)    inference/cpp/runtime/streaming_executor.cpp:255-266
 *   mha_attention_incremental           inference/cpp/runtime/mha.cpp:227-285
 *   mha_attention (causal, prefill)     inference/cpp/runtime/mha.cpp:126-198
 */
#ifndef AXION_B200_AXKV_H
#define AXION_B200_AXKV_H

#include <stdint.h>

#include "axq8_status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct axkv_cache {
    void* k_pages;               /* device, n_pages * n_kv_heads * page_tokens * head_dim elements */
    void* v_pages;               /* device, same shape */
    const int32_t* block_table;  /* device [sequences][max_blocks] page ids */
    int32_t n_pages;
    int32_t max_blocks;          /* pages per sequence (block table row length) */
    int32_t n_kv_heads;
    int32_t head_dim;            /* 32, 64 or 128 */
    int32_t page_tokens;         /* 16 */
    int32_t kv_fp32;             /* 0: fp16 pages, 1: fp32 pages */
} axkv_cache_t;

/* Bytes of one layer's K (or V) pages. */
int64_t axkv_pages_bytes(const axkv_cache_t* c);

/* Append n_rows token rows: row r of k_rows / v_rows (device fp32
 * [n_rows][n_kv_heads * head_dim], K after RoPE) is written, rounded to the
 * page type, at position row_pos[r] of sequence row_seq[r] (device int32
 * arrays).  PagedKVCache::append for one layer. */
int axkv_paged_append(const axkv_cache_t* c, const float* k_rows, const float* v_rows,
                      int32_t n_rows, const int32_t* row_seq, const int32_t* row_pos,
                      void* stream);

/* Workspace bytes axkv_paged_decode_attn needs for n_seq sequences of
 * n_heads query heads (split partials and per-(sequence, kv head) counters). */
int64_t axkv_decode_attn_workspace(const axkv_cache_t* c, int32_t n_seq, int32_t n_heads);

/* One query row per sequence against its cached tokens:
 * mha_attention_incremental (mha.cpp:227-285) — GQA kv head h / (n_heads /
 * n_kv_heads), scores scaled by 1/sqrt(head_dim) after the dot, max-subtracted
 * softmax.  q [n_seq][n_heads * head_dim] (device fp32, after RoPE); query s
 * sits at position q_pos[s] (device int32) and attends to tokens 0 ..
 * q_pos[s] of sequence s (append its own K/V first); out [n_seq][n_heads *
 * head_dim] device fp32.  The workspace (axkv_decode_attn_workspace bytes,
 * 16-byte aligned) must be zero before its first use; every call leaves it
 * zero again.  Calls sharing a workspace must not overlap on the GPU. */
int axkv_paged_decode_attn(const axkv_cache_t* c, const float* q, int32_t n_seq, int32_t n_heads,
                           const int32_t* q_pos, float* out, void* workspace,
                           int64_t workspace_bytes, void* stream);

/* Causal attention of a prompt chunk over the cache: mha_attention /
 * sdpa_causal (mha.cpp:126-198) for positions p0 .. p0 + T - 1 of n_seq
 * sequences whose K/V (those positions included) are already in the pages.
 * q rows [n_seq * T][n_heads * head_dim] (device fp32, after RoPE; row
 * s * T + t is sequence s at position p0 + t) with row pitch ldq floats;
 * out rows [n_seq * T][n_heads * head_dim] device fp32.  When xq is not null
 * the rows are instead quantized for the next Q8_0 product (the O
 * projection): xq [n_seq * T][n_heads * head_dim] int8 and transposed block
 * scales dxT [n_heads * head_dim / 32][Mp], Mp = n_seq * T rounded up to 4
 * (the layout of axq8_quantize_act_t); out is then unused.  fp16 pages, head
 * dim 64 or 128, n_heads / n_kv_heads <= 8 or a multiple of 8.  No workspace. */
int axkv_paged_prefill_attn(const axkv_cache_t* c, const float* q, int64_t ldq, int32_t n_seq,
                            int32_t T, int32_t p0, int32_t n_heads, float* out, int8_t* xq,
                            float* dxT, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AXION_B200_AXKV_H */
