// extern "C" shim over the reference's own C++ implementation of the Q8_0
// linear hot path, compiled together with the reference sources (unchanged,
// read in place) into oracle/_ref/libaxion_ref.so by oracle/Makefile.
//
// TEST INFRASTRUCTURE ONLY. Nothing in the product (axion_b200/, include/)
// links or loads this library: it is the checker the parity tests, the golden
// fixture generator and the CPU-baseline arm of bench.py use to run the
// reference code path itself on the same inputs.
//
// Every entry point returns 0 on success and a negative code on a thrown
// std::exception; the message is kept in axref_last_error().

#include "gguf/gguf.hpp"
#include "core/fp16.hpp"
#include "core/tensor_factory.hpp"
#include "runtime/linear.hpp"
#include "runtime/quantized_matmul.hpp"
#include "runtime/mha.hpp"
#include "runtime/model_runner.hpp"
#include "runtime/streaming_executor.hpp"
#include "runtime/token_embedding.hpp"
#include "runtime/final_norm.hpp"
#include "runtime/logits.hpp"
#include "kernels/rmsnorm.hpp"
#include "kernels/silu.hpp"
#include "kernels/elementwise.hpp"

#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

using namespace axion;

namespace {

thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    } catch (...) {
        g_err = "unknown exception";
        return -2;
    }
}

Tensor tensor_from(const float* p, int64_t rows, int64_t cols) {
    Tensor t = create_owned_tensor({rows, cols}, DType::FLOAT32);
    std::memcpy(t.data(), p, sizeof(float) * rows * cols);
    return t;
}

void copy_out(const Tensor& t, float* out) {
    for (int64_t i = 0; i < t.numel(); i++) out[i] = t.value(i);
}

// The loader prints progress to std::cout; silence it while a call runs so
// the parity tests and the CPU-baseline JSON line stay clean.
struct QuietCout {
    std::streambuf* old;
    std::ostringstream sink;
    QuietCout() : old(std::cout.rdbuf(sink.rdbuf())) {}
    ~QuietCout() { std::cout.rdbuf(old); }
};

}  // namespace

extern "C" {

const char* axref_last_error(void) { return g_err.c_str(); }

float axref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }

uint64_t axref_q8_0_byte_size(uint64_t n) {
    return gguf_tensor_byte_size(GGUFType::Q8_0, n);
}

// ---- GGUFLoader -----------------------------------------------------------

void* axref_gguf_open(const char* path) {
    GGUFLoader* l = new GGUFLoader();
    int rc = guarded([&] { QuietCout q; l->load_file(path); });
    if (rc != 0) { delete l; return nullptr; }
    return l;
}

void axref_gguf_close(void* h) { delete static_cast<GGUFLoader*>(h); }

// Writes the row-major shape (after the loader's GGML dim reversal) of
// `name` into shape[0..3]; returns the rank, or -1 if absent.
int axref_gguf_shape(void* h, const char* name, int64_t* shape) {
    std::vector<int64_t> s = static_cast<GGUFLoader*>(h)->tensor_shape(name);
    if (s.empty()) return -1;
    for (size_t i = 0; i < s.size() && i < 4; i++) shape[i] = s[i];
    return (int)s.size();
}

// GGUFLoader::load_tensor: raw read + dequantization to fp32.
int axref_gguf_load_tensor(void* h, const char* name, float* out, int64_t cap) {
    return guarded([&] {
        QuietCout q;
        Tensor t = static_cast<GGUFLoader*>(h)->load_tensor(name);
        if (t.numel() > cap) throw std::runtime_error("output buffer too small");
        copy_out(t, out);
    });
}

// ---- operators ------------------------------------------------------------

// linear_from_gguf(input[M,K], weight[N,K]) -> [M,N]
int axref_linear_from_gguf(const float* x, int64_t M, int64_t K,
                           const float* w, int64_t N, int64_t Kw, float* y) {
    return guarded([&] {
        Tensor in = tensor_from(x, M, K);
        Tensor wt = tensor_from(w, N, Kw);
        copy_out(linear_from_gguf(in, wt), y);
    });
}

// quantize_weight(W[K,N], Q8_0) followed by quantized_matmul(x[M,K], W).
// The per-tensor int8 payload and scale are returned as well.
int axref_quantized_matmul_q8(const float* x, int64_t M, int64_t K,
                              const float* w, int64_t N, float* y,
                              int8_t* q_out, float* scale_out) {
    return guarded([&] {
        Tensor in = tensor_from(x, M, K);
        Tensor wt = tensor_from(w, K, N);
        QuantizedWeight qw = quantize_weight(wt, QuantType::Q8_0);
        copy_out(quantized_matmul(in, qw), y);
        if (q_out) std::memcpy(q_out, qw.q8.data(), qw.q8.size());
        if (scale_out) *scale_out = qw.scale;
    });
}

int axref_rmsnorm(const float* x, int64_t rows, int64_t cols,
                  const float* w, float eps, float* out) {
    return guarded([&] {
        Tensor in = tensor_from(x, rows, cols);
        Tensor wt = tensor_from(w, 1, cols);
        copy_out(rmsnorm(in, wt, eps), out);
    });
}

// silu(gate) * up, the SwiGLU product of decode_layer.
int axref_silu_mul(const float* gate, const float* up, int64_t n, float* out) {
    return guarded([&] {
        Tensor g = tensor_from(gate, 1, n);
        Tensor u = tensor_from(up, 1, n);
        copy_out(elementwise_mul(silu(g), u), out);
    });
}

// rope_apply_row_at on a [1, n_heads*head_dim] row (NEOX convention).
int axref_rope_row_at(float* x, int n_heads, int head_dim, float theta,
                      int position) {
    return guarded([&] {
        Tensor t = tensor_from(x, 1, (int64_t)n_heads * head_dim);
        rope_apply_row_at(t, n_heads, head_dim, theta, position, RopeType::NEOX);
        copy_out(t, x);
    });
}

// mha_attention_incremental(q_row, k_cache[ctx, n_kv*hd], v_cache) -> [1, n_head*hd]
int axref_mha_incremental(const float* q, const float* k, const float* v,
                          int64_t ctx, int n_head, int n_kv, int hd, float* out) {
    return guarded([&] {
        Tensor qt = tensor_from(q, 1, (int64_t)n_head * hd);
        Tensor kt = tensor_from(k, ctx, (int64_t)n_kv * hd);
        Tensor vt = tensor_from(v, ctx, (int64_t)n_kv * hd);
        MHAConfig c;
        c.n_head = n_head; c.n_kv_head = n_kv; c.head_dim = hd;
        copy_out(mha_attention_incremental(qt, kt, vt, c), out);
    });
}

// ---- timing (CPU baseline of bench.py) -------------------------------------

// `iters` times: [GGUFLoader::load_tensor(name) when with_load] +
// linear_from_gguf(x[M,K], W) — the reference's per-token cost of one
// linear (streaming_executor.cpp:299-307 then :328-372).  Writes the last
// output to y and the elapsed wall time to *seconds.
int axref_time_linear(const char* path, const char* name, const float* x, int64_t M,
                      int iters, int with_load, float* y, double* seconds) {
    return guarded([&] {
        QuietCout q;
        GGUFLoader loader;
        loader.load_file(path);
        Tensor w = loader.load_tensor(name);
        const int64_t K = w.shape[1];
        Tensor in = tensor_from(x, M, K);
        Tensor out;
        auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < iters; i++) {
            if (with_load) w = loader.load_tensor(name);
            out = linear_from_gguf(in, w);
        }
        auto t1 = std::chrono::steady_clock::now();
        *seconds = std::chrono::duration<double>(t1 - t0).count();
        copy_out(out, y);
    });
}

// ModelRunner::generate timed: prompt + max_new greedy tokens.  Returns the
// generated ids and the wall time of the generate() call.
int axref_time_generate(const char* path, const int32_t* prompt, int n_prompt, int max_new,
                        int32_t* out_tokens, int* n_out, double* seconds) {
    return guarded([&] {
        QuietCout q;
        GGUFLoader loader;
        loader.load_file(path);
        ModelRunner runner(&loader);
        ModelRunner::GenerationParams p;
        p.max_new_tokens = max_new;
        std::vector<int> pr(prompt, prompt + n_prompt);
        auto t0 = std::chrono::steady_clock::now();
        std::vector<int> seq = runner.generate(pr, p);
        auto t1 = std::chrono::steady_clock::now();
        *seconds = std::chrono::duration<double>(t1 - t0).count();
        for (size_t i = 0; i < seq.size(); i++) out_tokens[i] = seq[i];
        *n_out = (int)seq.size();
    });
}

// ---- end-to-end decode ----------------------------------------------------

// ModelRunner::generate with greedy sampling. out_tokens receives
// prompt + generated ids; *n_out their count.
int axref_generate(const char* path, const int32_t* prompt, int n_prompt,
                   int max_new, int32_t* out_tokens, int* n_out) {
    return guarded([&] {
        QuietCout q;
        GGUFLoader loader;
        loader.load_file(path);
        ModelRunner runner(&loader);
        ModelRunner::GenerationParams p;
        p.max_new_tokens = max_new;
        std::vector<int> pr(prompt, prompt + n_prompt);
        std::vector<int> seq = runner.generate(pr, p);
        for (size_t i = 0; i < seq.size(); i++) out_tokens[i] = seq[i];
        *n_out = (int)seq.size();
    });
}

// The same incremental decode as ModelRunner::generate, composed from the
// reference's public pieces so the logits of every step are visible:
// token_embedding -> StreamingExecutor::decode_step -> final_norm ->
// compute_logits -> greedy argmax. Teacher forcing: when `forced` is
// non-null, step s feeds forced[s] instead of the argmax. logits_out is
// [n_steps, vocab]; the step-s logits are those produced after the prompt
// plus s generated/forced tokens.
int axref_decode_logits(const char* path, const int32_t* prompt, int n_prompt,
                        int n_steps, const int32_t* forced, float* logits_out,
                        int32_t* argmax_out) {
    return guarded([&] {
        QuietCout q;
        GGUFLoader loader;
        loader.load_file(path);
        ModelRunner runner(&loader);
        const ModelConfig& cfg = runner.config();
        StreamingExecutor ex(&loader);
        LayerConfig lc;
        lc.num_heads = cfg.n_heads;
        lc.n_kv_heads = cfg.n_kv_heads;
        lc.head_dim = cfg.head_dim;
        lc.rope_theta = cfg.rope_theta;
        lc.eps = cfg.rms_eps;
        lc.rope_type = cfg.rope_type;
        ex.begin_decode(cfg.n_layers, lc);
        Tensor embd = loader.load_tensor("token_embd.weight");
        Tensor norm_w = loader.load_tensor("output_norm.weight");
        std::vector<std::string> names = loader.tensor_names();
        Tensor w_out = loader.load_tensor(select_output_weight_name(names));
        Tensor last;
        for (int i = 0; i < n_prompt; i++)
            last = ex.decode_step(token_embedding(embd, prompt[i]));
        for (int s = 0; s < n_steps; s++) {
            Tensor normed = final_norm(last, norm_w, cfg.rms_eps);
            Tensor lg = compute_logits(normed, w_out);
            copy_out(lg, logits_out + (int64_t)s * lg.numel());
            int next = argmax(lg);
            argmax_out[s] = next;
            int feed = forced ? forced[s] : next;
            if (s + 1 < n_steps) last = ex.decode_step(token_embedding(embd, feed));
        }
    });
}

}  // extern "C"
