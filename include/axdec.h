/*
 * axdec.h — C ABI of the B200 decode step built on the Q8_0 linear path.
 *
 * A Llama-architecture decoder (RMSNorm, GQA attention with NEOX RoPE over a
 * paged KV cache, SwiGLU FFN, LM head) whose every linear is the Q8_0 GEMV of
 * axq8.h.  It replaces, for Q8_0 GGUF models (paths inside the reference):
 *   StreamingExecutor::begin_decode / decode_step / decode_layer
 *       inference/cpp/runtime/streaming_executor.hpp:58-67, .cpp:244-420
 *   ModelRunner::generate (greedy)            inference/cpp/runtime/model_runner.cpp:245-317
 *   mha_attention_incremental + append_row    inference/cpp/runtime/mha.cpp:227-285,
 *                                             streaming_executor.cpp:255-266
 *   PagedKVCache (fp32 pages)                 inference/cpp/runtime/paged_kv.hpp:18-41
 * Weights are uploaded once and stay resident; the KV cache is paged
 * (fixed-size blocks of tokens, per-sequence block tables); one decode step
 * for a batch of sequences is a CUDA graph of fused kernels.
 *
 * Same conventions as axq8.h: plain C, status codes, axq8_last_error().
 */
#ifndef AXION_B200_AXDEC_H
#define AXION_B200_AXDEC_H

#include <stdint.h>

#include "axq8_status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct axdec_config {
    int32_t n_layers;     /* <arch>.block_count */
    int32_t hidden;       /* <arch>.embedding_length */
    int32_t ffn;          /* <arch>.feed_forward_length */
    int32_t n_heads;      /* <arch>.attention.head_count */
    int32_t n_kv_heads;   /* <arch>.attention.head_count_kv */
    int32_t head_dim;     /* <arch>.rope.dimension_count (hidden / n_heads) */
    int32_t vocab;
    float rope_theta;     /* <arch>.rope.freq_base */
    float rms_eps;        /* <arch>.attention.layer_norm_rms_epsilon */
    int32_t max_batch;    /* sequences decoded together */
    int32_t max_ctx;      /* tokens per sequence (prompt + generated) */
    int32_t kv_block;     /* tokens per KV page, power of two (16) */
    int32_t act_mode;     /* AXQ8_ACT_Q8 (decode default) or AXQ8_ACT_F32 */
    int32_t kv_fp32;      /* 0: fp16 KV pages (default), 1: fp32 pages */
    /* Tensor parallelism over tp_size GPUs (0 or 1: none), this model being
     * rank tp_rank: Q, K, V, gate and up split by output rows (whole heads),
     * O and down by input columns, the LM head by vocabulary; the embedding
     * and norms are replicated.  Needs n_kv_heads, ffn / 32 and vocab
     * divisible by tp_size. */
    int32_t tp_size;
    int32_t tp_rank;
} axdec_config_t;

typedef struct axdec_model axdec_model_t;

/* Create a model on the current device and allocate its weights, KV pages and
 * activation buffers (the only allocations; none happen per step). */
int axdec_create(const axdec_config_t* cfg, axdec_model_t** out);
int axdec_destroy(axdec_model_t* m);

/* Set one tensor by its GGUF name (token_embd.weight, blk.N.attn_q.weight,
 * ..., output_norm.weight, output.weight) from host memory: Q8_0 blocks
 * (ggml_type 8) for the linears and the embedding, F32 (ggml_type 0) for the
 * norm weights.  rows x cols is the row-major shape ([out, in]).  When
 * output.weight is never set the LM head is tied to token_embd.weight
 * (select_output_weight_name, model_runner.cpp:179-189). */
int axdec_set_tensor(axdec_model_t* m, const char* name, const void* host_data, int ggml_type,
                     int64_t rows, int64_t cols);

/* Random-init every weight on the device: each Q8_0 tensor from
 * axq8_synth_q8_0(seed + axdec_tensor_index(name), std), norm weights 1.0. */
int axdec_init_random(axdec_model_t* m, uint64_t seed, float std);

/* Canonical index of a tensor name (the per-tensor seed offset above), or -1:
 * token_embd 0, output 1, output_norm 2, then per layer i: 3 + 9*i + slot
 * with slots attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm,
 * ffn_gate, ffn_up, ffn_down. */
int axdec_tensor_index(const axdec_config_t* cfg, const char* name);

/* Greedy generation for n_seq sequences (<= max_batch) sharing one prompt
 * length: prompts[n_seq, n_prompt] (host), then n_new greedy tokens written
 * to out_tokens[n_seq, n_new] (host).  Prompt positions 0 .. n_prompt - 2 run
 * as a batched prefill where axdec_prefill_batched says so (A8, fp16 pages,
 * head dim 64 / 128), else one position at a time through the decode step, as
 * ModelRunner::generate does (model_runner.cpp:291-295); the last prompt
 * position always goes through the decode step and yields the first token.  When
 * logits_out is non-null it receives the LM-head logits of every generated
 * step [n_new, n_seq, vocab] (host; slows the loop: one copy per step).
 * The decode step runs as a CUDA graph on `stream`.  On return *decode_ms
 * (nullable) holds the device time of the n_new generation steps alone. */
int axdec_generate(axdec_model_t* m, const int32_t* prompts, int32_t n_seq, int32_t n_prompt,
                   int32_t n_new, int32_t* out_tokens, float* logits_out, float* decode_ms,
                   void* stream);

/* Teacher-forced variant: feeds tokens[n_seq, n_steps] (prompt followed by
 * forced continuations) and returns, for every position p >= n_prompt - 1,
 * the logits of the next token: logits_out[n_steps - n_prompt + 1, n_seq, vocab]. */
int axdec_forced(axdec_model_t* m, const int32_t* tokens, int32_t n_seq, int32_t n_prompt,
                 int32_t n_steps, float* logits_out, void* stream);

/* Batched prefill: prompt positions as wide products (rows = sequences x
 * positions, in chunks of up to 4096 rows: the tcgen05 product above 64 rows,
 * the skinny one up to 64) and a causal GQA attention kernel over the paged
 * cache — StreamingExecutor::execute_layer (streaming_executor.cpp:110-238)
 * with mha_attention (mha.cpp:167-198) for a whole prompt.  mode 1 (default):
 * used wherever supported; mode 0: prompts go through the decode step one
 * position at a time.  axdec_prefill_batched tells whether prompts of n_seq
 * sequences take it.  The chunk buffers are allocated on the first batched
 * prefill and kept. */
int axdec_set_prefill(axdec_model_t* m, int mode);
int axdec_prefill_batched(const axdec_model_t* m, int32_t n_seq);

/* Step-wise decoding, StreamingExecutor::begin_decode + decode_step
 * (streaming_executor.hpp:58-67, .cpp:244-253, 403-420) for a batch.
 * axdec_prefill starts a session of n_seq sequences: tokens[n_seq, n_tok]
 * (host) fill the KV cache at positions 0 .. n_tok - 1 (no logits; n_tok may
 * be 0) and the session continues at position n_tok.  axdec_decode_step then
 * takes one input token per sequence (host tokens[n_seq]), runs one decode
 * step (the step's CUDA graph) at the session position, and writes the greedy
 * next token of each sequence to next_tokens[n_seq] (host); logits_out
 * (nullable, host) receives the step's logits [n_seq, vocab] (this rank's
 * vocabulary slice under tensor parallelism).  Synchronous: each call returns
 * when its outputs are in host memory.  axdec_generate and axdec_forced end
 * the session (AXQ8_ERR_STATE from axdec_decode_step until the next
 * axdec_prefill). */
int axdec_prefill(axdec_model_t* m, const int32_t* tokens, int32_t n_seq, int32_t n_tok,
                  void* stream);
int axdec_decode_step(axdec_model_t* m, const int32_t* tokens, int32_t n_seq, int32_t* next_tokens,
                      float* logits_out, void* stream);

/* Continue the session for n_steps greedy steps on the device (each step's
 * token fed back without a host round trip): the first step's inputs are
 * first_tokens[n_seq] (host), or, when null, the greedy tokens of the
 * session's previous step.  out_tokens[n_seq, n_steps] (host) receives the
 * tokens; *decode_ms (nullable) the device time of the n_steps steps. */
int axdec_decode_continue(axdec_model_t* m, const int32_t* first_tokens, int32_t n_seq,
                          int32_t n_steps, int32_t* out_tokens, float* decode_ms, void* stream);

/* Bytes of device memory the model holds (weights + KV pages + buffers). */
int64_t axdec_device_bytes(const axdec_model_t* m);

/* Bytes of Q8_0 weight streamed by one decode step on this rank (all linears + LM head,
 * at 34 bytes per 32 weights) — the algorithmic weight traffic per token. */
int64_t axdec_weight_bytes_per_step(const axdec_model_t* m);

/* Tensor-parallel set-up.  Rank 0 draws a communicator id (128 bytes,
 * written to id_out) and every rank passes the same id to axdec_tp_connect
 * (collectively: all tp_size ranks call it).  The step then sums the partial
 * hidden states after the O and down projections with an NCCL all-reduce
 * over NVLink and takes the greedy token as a max all-reduce of packed
 * (logit, index) keys.  With tp_size > 1, logits_out of axdec_generate /
 * axdec_forced receives this rank's vocabulary slice ([steps][n_seq][vocab /
 * tp_size], vocabulary rows tp_rank * vocab / tp_size onwards).  NCCL is
 * loaded at run time; AXQ8_ERR_UNSUPPORTED when it cannot be found. */
int axdec_tp_unique_id(void* id_out, int64_t id_bytes);
int axdec_tp_connect(axdec_model_t* m, const void* id);

/* The hidden-state all-reduce of a connected model: 0 none (tp_size 1), 1 NCCL
 * (default), 2 the NVLink peer-memory kernel of axtp.h, which
 * axdec_tp_connect sets up when AXDEC_TP_AR=nvlink and every rank can map the
 * others' buffers with CUDA IPC: each rank sums its slice of the partials in
 * rank order and writes it to every rank, so all ranks hold identical sums;
 * its waits on the peers are bounded (about two seconds), after which the
 * device status word reads AXQ8_ERR_WAIT_TIMEOUT. */
int axdec_tp_allreduce_kind(const axdec_model_t* m);

/* Failure handling.  axdec_tp_health reads, without synchronizing the device,
 * the communicator's asynchronous error (ncclResult_t, 0 = none) and the
 * device status word (AXQ8_ERR_WAIT_TIMEOUT after a peer stopped answering).
 * axdec_tp_abort aborts the communicator (ncclCommAbort), which ends pending
 * NCCL work so that a rank whose peer failed can return; the model then needs
 * a new axdec_tp_connect before the next step. */
int axdec_tp_health(axdec_model_t* m, int* nccl_error, int* device_status);
int axdec_tp_abort(axdec_model_t* m);

/* Kernels launched by one decode step of n_seq sequences: the kernel nodes
 * of the step's CUDA graph, captured by the first axdec_generate/axdec_forced
 * call with that n_seq (-1 before it). */
int axdec_step_kernels(const axdec_model_t* m, int n_seq);

#ifdef __cplusplus
}
#endif
#endif /* AXION_B200_AXDEC_H */
