/* CPU restatement of the reference's Q8_0 linear path (test infrastructure;
 * see q8_oracle.h for the contract and the reference lines each function
 * restates).  Written from the reference's behaviour, not copied from it. */
#include "q8_oracle.h"

#include <math.h>
#include <string.h>

/* ---- binary16 ------------------------------------------------------------ */

float axo_fp16_to_fp32(uint16_t h) {
    /* IEEE-754 binary16: 1 sign, 5 exponent (bias 15), 10 fraction bits. */
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f;
    uint32_t f = h & 0x3ff;
    uint32_t bits;
    if (e == 0x1f) {
        bits = sign | 0x7f800000u | (f << 13);           /* inf / nan */
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (f << 13);    /* normal: rebias 15 -> 127 */
    } else if (f == 0) {
        bits = sign;                                      /* +-0 */
    } else {
        /* subnormal: value = f * 2^-24; normalise the fraction */
        int shift = 0;
        while ((f & 0x400u) == 0) { f <<= 1; shift++; }
        f &= 0x3ffu;
        bits = sign | ((uint32_t)(113 - shift) << 23) | (f << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

uint16_t axo_fp32_to_fp16(float v) {
    uint32_t x;
    memcpy(&x, &v, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {                               /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (ax < 0x33000001u) return sign;                      /* < 2^-25: rounds to 0 */
    int32_t e = (int32_t)(ax >> 23) - 127;
    uint32_t mant = (ax & 0x7fffffu) | 0x800000u;           /* 24-bit significand */
    int shift;                                              /* bits to drop */
    uint32_t base;
    if (e < -14) {                                          /* subnormal half */
        shift = 13 + (-14 - e);
        base = 0;
    } else {
        shift = 13;
        base = (uint32_t)(e + 15) << 10;
        mant &= 0x7fffffu;
    }
    uint32_t q = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    uint32_t r = base + q;                                  /* carries propagate into exponent */
    if (rem > half || (rem == half && (q & 1u))) r += 1;
    return (uint16_t)(sign | r);
}

/* ---- Q8_0 format ----------------------------------------------------------- */

uint64_t axo_q8_0_byte_size(uint64_t n) { return (n / AXO_QK) * AXO_Q8_0_BYTES; }

void axo_q8_0_dequant(const uint8_t* blocks, uint64_t n, float* out) {
    uint64_t nb = n / AXO_QK;
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* blk = blocks + b * AXO_Q8_0_BYTES;
        uint16_t dh = (uint16_t)(blk[0] | (blk[1] << 8));
        float d = axo_fp16_to_fp32(dh);
        for (int i = 0; i < AXO_QK; i++) {
            out[b * AXO_QK + i] = (float)(int8_t)blk[2 + i] * d;
        }
    }
}

static int round_half_away_clamp127(float v) {
    float r = roundf(v);                 /* C99 roundf: halves away from zero */
    if (r > 127.0f) r = 127.0f;
    if (r < -127.0f) r = -127.0f;
    return (int)r;
}

void axo_q8_0_quantize(const float* w, int64_t rows, int64_t K, uint8_t* blocks) {
    int64_t nb = K / AXO_QK;
    #pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t b = 0; b < nb; b++) {
            const float* src = w + r * K + b * AXO_QK;
            uint8_t* blk = blocks + (r * nb + b) * AXO_Q8_0_BYTES;
            float amax = 0.0f;
            for (int i = 0; i < AXO_QK; i++) {
                float a = fabsf(src[i]);
                if (a > amax) amax = a;
            }
            float d = amax / 127.0f;
            uint16_t dh = axo_fp32_to_fp16(d);
            blk[0] = (uint8_t)(dh & 0xff);
            blk[1] = (uint8_t)(dh >> 8);
            for (int i = 0; i < AXO_QK; i++) {
                int q = (d == 0.0f) ? 0 : round_half_away_clamp127(src[i] / d);
                blk[2 + i] = (uint8_t)(int8_t)q;
            }
        }
    }
}

void axo_quantize_act(const float* x, int64_t M, int64_t K, int8_t* q, float* d) {
    int64_t nb = K / AXO_QK;
    for (int64_t m = 0; m < M; m++) {
        for (int64_t b = 0; b < nb; b++) {
            const float* src = x + m * K + b * AXO_QK;
            float amax = 0.0f;
            for (int i = 0; i < AXO_QK; i++) {
                float a = fabsf(src[i]);
                if (a > amax) amax = a;
            }
            float db = amax / 127.0f;
            float id = (amax == 0.0f) ? 0.0f : 127.0f / amax;
            d[m * nb + b] = db;
            for (int i = 0; i < AXO_QK; i++) {
                q[m * K + b * AXO_QK + i] = (int8_t)round_half_away_clamp127(src[i] * id);
            }
        }
    }
}

void axo_block_dots(const uint8_t* wblocks, int64_t N, int64_t K,
                    const int8_t* xq, int64_t M, int32_t* dots) {
    int64_t nb = K / AXO_QK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            for (int64_t b = 0; b < nb; b++) {
                const uint8_t* blk = wblocks + (n * nb + b) * AXO_Q8_0_BYTES;
                const int8_t* xs = xq + m * K + b * AXO_QK;
                int32_t s = 0;
                for (int i = 0; i < AXO_QK; i++) s += (int32_t)(int8_t)blk[2 + i] * (int32_t)xs[i];
                dots[(m * N + n) * nb + b] = s;
            }
        }
    }
}

void axo_linear_a8(const uint8_t* wblocks, int64_t N, int64_t K,
                   const int8_t* xq, const float* dx, int64_t M, float* y) {
    int64_t nb = K / AXO_QK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            float acc = 0.0f;
            for (int64_t b = 0; b < nb; b++) {
                const uint8_t* blk = wblocks + (n * nb + b) * AXO_Q8_0_BYTES;
                const int8_t* xs = xq + m * K + b * AXO_QK;
                int32_t s = 0;
                for (int i = 0; i < AXO_QK; i++) s += (int32_t)(int8_t)blk[2 + i] * (int32_t)xs[i];
                float dw = axo_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8)));
                float scale = dw * dx[m * nb + b];
                acc += scale * (float)s;
            }
            y[m * N + n] = acc;
        }
    }
}

void axo_linear_f32(const float* x, int64_t M, int64_t K,
                    const float* w, int64_t N, float* y) {
    #pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            const float* a = x + m * K;
            const float* b = w + n * K;
            float acc = 0.0f;
            for (int64_t k = 0; k < K; k++) acc += a[k] * b[k];
            y[m * N + n] = acc;
        }
    }
}

void axo_linear_a32(const float* x, int64_t M, int64_t K,
                    const uint8_t* wblocks, int64_t N, float* y) {
    int64_t nb = K / AXO_QK;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            const float* a = x + m * K;
            float acc = 0.0f;
            for (int64_t b = 0; b < nb; b++) {
                const uint8_t* blk = wblocks + (n * nb + b) * AXO_Q8_0_BYTES;
                float d = axo_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8)));
                for (int i = 0; i < AXO_QK; i++) {
                    float wv = (float)(int8_t)blk[2 + i] * d;   /* load_tensor's value */
                    acc += a[b * AXO_QK + i] * wv;
                }
            }
            y[m * N + n] = acc;
        }
    }
}

/* ---- decode-layer operators ----------------------------------------------- */

void axo_rmsnorm(const float* x, int64_t rows, int64_t cols,
                 const float* w, float eps, float* out) {
    for (int64_t r = 0; r < rows; r++) {
        const float* row = x + r * cols;
        float ms = 0.0f;
        for (int64_t c = 0; c < cols; c++) ms += row[c] * row[c];
        ms /= (float)cols;
        float inv = 1.0f / sqrtf(ms + eps);
        for (int64_t c = 0; c < cols; c++) out[r * cols + c] = (row[c] * inv) * w[c];
    }
}

void axo_rope_neox_row(float* x, int n_heads, int head_dim, float theta, int position) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        float* v = x + (int64_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
            float ang = (float)position * freq;
            float c = cosf(ang), s = sinf(ang);
            float a = v[i], b = v[i + half];
            v[i] = a * c - b * s;
            v[i + half] = a * s + b * c;
        }
    }
}

void axo_attention_decode(const float* q, const float* k_cache, const float* v_cache,
                          int64_t ctx, int n_head, int n_kv, int hd, float* out) {
    int group = n_head / n_kv;
    float scale = 1.0f / sqrtf((float)hd);
    int64_t kvw = (int64_t)n_kv * hd;
    float* sc = (float*)__builtin_alloca(sizeof(float) * (ctx > 0 ? ctx : 1));
    for (int h = 0; h < n_head; h++) {
        int kv = h / group;
        const float* qh = q + (int64_t)h * hd;
        float mx = -INFINITY;
        for (int64_t j = 0; j < ctx; j++) {
            const float* kj = k_cache + j * kvw + (int64_t)kv * hd;
            float dot = 0.0f;
            for (int d = 0; d < hd; d++) dot += qh[d] * kj[d];
            dot *= scale;
            sc[j] = dot;
            if (dot > mx) mx = dot;
        }
        float sum = 0.0f;
        for (int64_t j = 0; j < ctx; j++) {
            sc[j] = expf(sc[j] - mx);
            sum += sc[j];
        }
        for (int d = 0; d < hd; d++) {
            float acc = 0.0f;
            for (int64_t j = 0; j < ctx; j++) acc += sc[j] * v_cache[j * kvw + (int64_t)kv * hd + d];
            out[(int64_t)h * hd + d] = acc / sum;
        }
    }
}

void axo_silu_mul(const float* gate, const float* up, int64_t n, float* out) {
    for (int64_t i = 0; i < n; i++) {
        float g = gate[i];
        float s = g / (1.0f + expf(-g));
        out[i] = s * up[i];
    }
}

void axo_residual_add(const float* a, const float* b, int64_t n, float* out) {
    for (int64_t i = 0; i < n; i++) out[i] = a[i] + b[i];
}

int64_t axo_argmax(const float* x, int64_t n) {
    int64_t best = 0;
    float bv = -INFINITY;
    for (int64_t i = 0; i < n; i++) {
        if (x[i] > bv) { bv = x[i]; best = i; }
    }
    return best;
}

/* ---- synthetic weights ------------------------------------------------------ */

static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void axo_gen_normal(uint64_t seed, uint64_t start, int64_t n, float mean,
                    float std, float* out) {
    #pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; j++) {
        uint64_t i = start + (uint64_t)j;
        int32_t acc = 0;
        for (int t = 0; t < 3; t++) {
            uint64_t r = splitmix64(seed ^ (3 * i + (uint64_t)t) * 0xD1B54A32D192ED03ull);
            acc += (int32_t)(r & 0xffff) + (int32_t)((r >> 16) & 0xffff) +
                   (int32_t)((r >> 32) & 0xffff) + (int32_t)(r >> 48);
        }
        /* 12 uniforms on [0, 65536): mean 6*65535, exact integers < 2^24 */
        float z = (float)(acc - 393210) * (1.0f / 65536.0f);   /* exact */
        /* Irwin-Hall(12) of unit-width uniforms has variance 1 */
        out[j] = z * std + mean;
    }
}
