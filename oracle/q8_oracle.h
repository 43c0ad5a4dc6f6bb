/* CPU restatement of the reference's Q8_0 linear path and of the decode-layer
 * operators around it.  TEST INFRASTRUCTURE ONLY: the parity tests, the golden
 * fixture generator and bench.py's CPU-baseline leg call it as the checker.
 * The product (axion_b200/, include/) never links or loads it.
 *
 * Each function names the reference file:line it restates (paths relative to
 * the reference project root).  Scalar loops, fp32 throughout, products and
 * sums rounded separately (built with -ffp-contract=off), so that the fp32
 * functions reproduce the reference bit for bit on the same inputs; the
 * pin is checked against the reference itself in tests/test_oracle.py.
 */
#ifndef AXION_Q8_ORACLE_H
#define AXION_Q8_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AXO_QK 32          /* elements per Q8_0 block */
#define AXO_Q8_0_BYTES 34  /* fp16 d + 32 x int8 */

/* inference/cpp/core/fp16.cpp:5-66 — exact IEEE binary16 -> binary32. */
float axo_fp16_to_fp32(uint16_t h);

/* binary32 -> binary16, round to nearest even (fixture writer only; the
 * reference has no float->half conversion on its Q8_0 path). */
uint16_t axo_fp32_to_fp16(float f);

/* inference/cpp/gguf/gguf.cpp:51 — (n/32)*34. */
uint64_t axo_q8_0_byte_size(uint64_t n);

/* inference/cpp/gguf/gguf.cpp:870-882 — block b: d = fp16 bytes 0..1,
 * out[b*32+i] = (float)(int8)qs[i] * d. */
void axo_q8_0_dequant(const uint8_t* blocks, uint64_t n, float* out);

/* Weight quantizer used to make the synthetic Q8_0 weights (the recipe of
 * the benchmark workloads): per 32-block, d = amax/127 (fp32),
 * q = round-half-away(w/d) clamped to [-127,127] (0 when d == 0), and the
 * block stores fp16_rne(d).  Row-major [rows, K], K % 32 == 0. */
void axo_q8_0_quantize(const float* w, int64_t rows, int64_t K, uint8_t* blocks);

/* Activation Q8 quantization (A8 mode), the convention the device kernels
 * reproduce bit for bit: per 32-block of each row, amax = max|x|,
 * d = amax/127 and id = 127/amax (IEEE fp32 divisions, id = 0 when
 * amax == 0), q = round-half-away(x*id) clamped to [-127,127]; d is kept
 * in fp32.  The reference has no activation quantization; this is the only
 * new numeric convention. */
void axo_quantize_act(const float* x, int64_t M, int64_t K, int8_t* q, float* d);

/* Integer block dots: dots[(m*N + n)*(K/32) + b] = sum_{i<32} qw[n,b,i]*qx[m,b,i]. */
void axo_block_dots(const uint8_t* wblocks, int64_t N, int64_t K,
                    const int8_t* xq, int64_t M, int32_t* dots);

/* A8W8 linear: y[m,n] = sum_b (d_w[n,b]*d_x[m,b]) * dot[m,n,b], fp32, b in order. */
void axo_linear_a8(const uint8_t* wblocks, int64_t N, int64_t K,
                   const int8_t* xq, const float* dx, int64_t M, float* y);

/* inference/cpp/runtime/linear.cpp:27-71 applied to the Q8_0 weight as
 * GGUFLoader::load_tensor dequantizes it (gguf.cpp:870-882):
 * y[m,n] = sum_k x[m,k]*w[n,k], one fp32 accumulator, k ascending. */
void axo_linear_a32(const float* x, int64_t M, int64_t K,
                    const uint8_t* wblocks, int64_t N, float* y);

/* Same loop on an already-fp32 weight [N,K] (linear.cpp:57-68). */
void axo_linear_f32(const float* x, int64_t M, int64_t K,
                    const float* w, int64_t N, float* y);

/* inference/cpp/kernels/rmsnorm.cpp:12-100. */
void axo_rmsnorm(const float* x, int64_t rows, int64_t cols,
                 const float* w, float eps, float* out);

/* inference/cpp/runtime/mha.cpp:15-55 (NEOX branch) + :200-225:
 * rotate pairs (i, i+hd/2) of every head of one row at `position`. */
void axo_rope_neox_row(float* x, int n_heads, int head_dim, float theta, int position);

/* inference/cpp/runtime/mha.cpp:227-285: one query row against a
 * contiguous fp32 cache [ctx, n_kv*hd], GQA kv = h / (n_head/n_kv). */
void axo_attention_decode(const float* q, const float* k_cache, const float* v_cache,
                          int64_t ctx, int n_head, int n_kv, int hd, float* out);

/* inference/cpp/kernels/silu.cpp:13-65 then elementwise.cpp:13-67. */
void axo_silu_mul(const float* gate, const float* up, int64_t n, float* out);

/* inference/cpp/runtime/residual.cpp:8-46. */
void axo_residual_add(const float* a, const float* b, int64_t n, float* out);

/* inference/cpp/runtime/sampler.cpp:11-24 — first index of the maximum. */
int64_t axo_argmax(const float* x, int64_t n);

/* Counter-based approximately-N(mean, std) generator used for the synthetic
 * weights of the large workloads.  The device generator computes the same
 * values bit for bit: element i of stream `seed` is the Irwin-Hall sum of
 * twelve 16-bit uniforms taken from three splitmix64 outputs at counter
 * 3*i..3*i+2, centred and scaled with one exact conversion, one fp32
 * multiply and one fp32 add (no transcendental function, so no library
 * rounding differences between host and device). */
void axo_gen_normal(uint64_t seed, uint64_t start, int64_t n, float mean,
                    float std, float* out);

#ifdef __cplusplus
}
#endif
#endif
