/* CPU ORACLE -- test infrastructure only (see xp_oracle.h).
 *
 * Plain C restatement of the reference's Gemma-3 decode path. Arithmetic is
 * written in the same fp32 operation order as the reference kernels so that,
 * built with -ffp-contract=off like oracle/_ref, the two agree bit-for-bit on
 * the matvec, norms, RoPE and GeGLU (tests/test_oracle_pin.py).
 */
#include "xp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* generator                                                                 */
/* ------------------------------------------------------------------------ */
uint64_t xo_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return xo_splitmix64(seed ^ xo_splitmix64(stream + 0x632BE59BD9B4E019ull));
}

/* Irwin-Hall(12): sum of twelve 24-bit uniforms, centred, scaled. The sum is
 * formed in integers (exact), converted once (correctly rounded) and scaled
 * by sigma * 2^-24 in one fp32 multiply, so any IEEE implementation that
 * rounds to nearest produces the same bits. */
void xo_gen_normal(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float sigma,
                   float* out) {
    const uint64_t key = stream_key(seed, stream);
    const float mul = sigma * (1.0f / 16777216.0f);
#pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)n; ++ii) {
        const uint64_t i = (uint64_t)ii + offset;
        int64_t s = 0;
        for (uint64_t j = 0; j < 6; ++j) {
            const uint64_t h = xo_splitmix64(key + (i * 6 + j) * 0x9E3779B97F4A7C15ull);
            s += (int64_t)(h >> 40) + (int64_t)((h >> 8) & 0xFFFFFFull);
        }
        s -= 6ll * 16777216ll;
        out[ii] = (float)s * mul;
    }
}

void xo_gen_tokens(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab, uint32_t* out) {
    const uint64_t key = stream_key(seed, stream);
    for (uint64_t i = 0; i < n; ++i)
        out[i] = (uint32_t)((xo_splitmix64(key + i * 0x9E3779B97F4A7C15ull) >> 32) % vocab);
}

float xo_uniform(uint64_t seed, uint64_t stream, uint64_t index) {
    const uint64_t key = stream_key(seed, stream);
    const uint64_t h = xo_splitmix64(key + index * 0x9E3779B97F4A7C15ull);
    return (float)(h >> 40) * (1.0f / 16777216.0f);
}

/* ------------------------------------------------------------------------ */
/* fp16                                                                      */
/* ------------------------------------------------------------------------ */
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t xo_f32_to_f16(float f) {
    const uint32_t u = f2u(f);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t a = u & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (a > 0x7F800000u ? 0x200u : 0u));
    if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 -> inf */
    if (a < 0x38800000u) {                                    /* fp16 subnormal or zero */
        /* value = a_float; fp16 subnormal unit is 2^-24 */
        const float v = u2f(a) * 16777216.0f; /* exact scaling by 2^24 */
        /* round half to even on an integer */
        float r = rintf(v);
        return (uint16_t)(sign | (uint32_t)r);
    }
    /* normal: rebias exponent, round mantissa 23 -> 10 bits, ties to even */
    uint32_t m = a - 0x38000000u; /* exponent rebias (127 - 15) << 23 */
    const uint32_t lsb = (m >> 13) & 1u;
    m += 0x0FFFu + lsb;
    return (uint16_t)(sign | (m >> 13));
}

float xo_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    const uint32_t m = h & 0x3FFu;
    if (e == 0) {
        const float v = (float)m * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* ------------------------------------------------------------------------ */
/* packer: examples/llm/decode.cpp:94-229                                    */
/* ------------------------------------------------------------------------ */
/* decode.cpp:101-103 -- symmetric int4, nibble = clamp(lround(v*inv)+8, 0, 15) */
uint32_t xo_quantise(float v, float inv_scale) {
    long r = lroundf(v * inv_scale);
    long q = r + 8;
    if (q < 0) q = 0;
    if (q > 15) q = 15;
    return (uint32_t)q;
}

/* decode.cpp:109-113 */
static uint32_t bf16_bits(float f) { return f2u(f) >> 16; }

static double block_err(const float* blk, float s) {
    if (!(s > 0.0f)) return INFINITY;
    const float inv = 1.0f / s;
    double e = 0.0;
    for (int t = 0; t < 32; ++t) {
        const double d = (double)((int)xo_quantise(blk[t], inv) - 8) * (double)s - (double)blk[t];
        e += d * d;
    }
    return e;
}

/* decode.cpp:127-147 -- of the truncated bf16 of s0 and the next bf16 up,
 * keep the one with the smaller squared reconstruction error; ties -> lower. */
float xo_best_bf16_scale(const float* blk, float s0) {
    if (!(s0 > 0.0f)) return 0.0f;
    const uint32_t ulo = f2u(s0) & 0xFFFF0000u;
    const uint32_t uhi = ulo + 0x10000u;
    const float lo = u2f(ulo), hi = u2f(uhi);
    return block_err(blk, lo) <= block_err(blk, hi) ? lo : hi;
}

/* decode.cpp:177-229 (KM4 branch :212-227) and decode.cpp:157-169. */
int xo_pack_km4bf16(const float* w, uint32_t rows, uint32_t cols, uint32_t* words,
                    uint32_t* scales) {
    if (rows % 128u || cols % 64u) return -1;
    const uint32_t nblk = rows / 32u;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t gg = 0; gg < (int64_t)(cols / 64u); ++gg) {
        const uint32_t g = (uint32_t)gg;
        const float* cols64 = w + (size_t)g * 64u * rows;
        float inv[64];
        for (uint32_t b = 0; b < nblk; ++b) {
            for (uint32_t c = 0; c < 64u; ++c) {
                const float* r = cols64 + (size_t)c * rows + b * 32u;
                float amax = 0.0f;
                for (uint32_t t = 0; t < 32u; ++t) {
                    const float a = fabsf(r[t]);
                    if (amax < a) amax = a; /* std::max(amax, a) */
                }
                const float s = xo_best_bf16_scale(r, amax / 7.0f);
                const uint32_t j = g * 64u + c;
                /* decode.cpp:157-169: four bf16 block scales per uint2, blocks
                 * 4q..4q+3 in the low/high halves of .x then .y */
                const uint32_t q = b / 4u, i = b % 4u;
                uint32_t* d = scales + ((size_t)q * cols + j) * 2u + (i >> 1);
                if ((i & 1u) == 0u) *d = (*d & 0xFFFF0000u) | bf16_bits(s);
                else *d = (*d & 0x0000FFFFu) | (bf16_bits(s) << 16);
                inv[c] = s > 0.0f ? 1.0f / s : 0.0f;
            }
            const size_t base = ((size_t)g * nblk + b) * 64u;
            for (uint32_t c = 0; c < 64u; ++c) {
                uint32_t wd[4] = {0, 0, 0, 0};
                for (uint32_t t = 0; t < 32u; ++t) {
                    const uint32_t k = b * 32u + t;
                    wd[(t >> 3) & 3u] |= xo_quantise(cols64[(size_t)c * rows + k], inv[c])
                                         << ((t & 7u) * 4u);
                }
                memcpy(words + (base + c) * 4u, wd, 16);
            }
        }
    }
    return 0;
}

static float bf16lo(uint32_t w) { return u2f(w << 16); }
static float bf16hi(uint32_t w) { return u2f(w & 0xFFFF0000u); }

float xo_dequant(const uint32_t* words, const uint32_t* scales, uint32_t rows, uint32_t cols,
                 uint32_t k, uint32_t j) {
    const uint32_t nblk = rows / 32u, b = k / 32u, t = k % 32u;
    const size_t u4 = ((size_t)(j / 64u) * nblk + b) * 64u + (j % 64u);
    const uint32_t w = words[u4 * 4u + ((t >> 3) & 3u)];
    const uint32_t nib = (w >> ((t & 7u) * 4u)) & 15u;
    const uint32_t sw = scales[((size_t)(b / 4u) * cols + j) * 2u + ((b % 4u) >> 1)];
    const float s = (b % 2u) ? bf16hi(sw) : bf16lo(sw);
    return ((float)nib - 8.0f) * s;
}

/* ------------------------------------------------------------------------ */
/* matvec: kernels/llm_matvec.cl:55-72 (q4dot8/32), :407-456 (mv_km4_bs*)     */
/* ------------------------------------------------------------------------ */
static float q4dot8(uint32_t w, const float* v) {
    float s;
    s = v[0] * ((float)((w) & 15u) - 8.0f);
    s += v[1] * ((float)((w >> 4) & 15u) - 8.0f);
    s += v[2] * ((float)((w >> 8) & 15u) - 8.0f);
    s += v[3] * ((float)((w >> 12) & 15u) - 8.0f);
    s += v[4] * ((float)((w >> 16) & 15u) - 8.0f);
    s += v[5] * ((float)((w >> 20) & 15u) - 8.0f);
    s += v[6] * ((float)((w >> 24) & 15u) - 8.0f);
    s += v[7] * ((float)((w >> 28) & 15u) - 8.0f);
    return s;
}
static float q4dot32(const uint32_t* w4, const float* v) {
    return q4dot8(w4[0], v) + q4dot8(w4[1], v + 8) + q4dot8(w4[2], v + 16) +
           q4dot8(w4[3], v + 24);
}
static float km4_quad(const uint32_t* wq, size_t base, const float* in, uint32_t b,
                      const uint32_t* s) {
    float a;
    a = q4dot32(wq + (base + (size_t)(b)*64u) * 4u, in + (b)*32u) * bf16lo(s[0]);
    a += q4dot32(wq + (base + (size_t)(b + 1u) * 64u) * 4u, in + (b + 1u) * 32u) * bf16hi(s[0]);
    a += q4dot32(wq + (base + (size_t)(b + 2u) * 64u) * 4u, in + (b + 2u) * 32u) * bf16lo(s[1]);
    a += q4dot32(wq + (base + (size_t)(b + 3u) * 64u) * 4u, in + (b + 3u) * 32u) * bf16hi(s[1]);
    return a;
}
static float mv_col(const float* in, const uint32_t* wq, const uint32_t* sc, uint32_t rows,
                    uint32_t cols, uint32_t j, uint32_t q0, uint32_t q1) {
    const uint32_t nblk = rows / 32u;
    const size_t base = (size_t)(j / 64u) * nblk * 64u + (j % 64u);
    float acc = 0.0f;
    for (uint32_t q = q0; q < q1; ++q) acc += km4_quad(wq, base, in, q * 4u, sc + ((size_t)q * cols + j) * 2u);
    return acc;
}

void xo_mv_km4_bs(float* out, const float* in, const uint32_t* wq, const uint32_t* sc,
                  uint32_t rows, uint32_t cols) {
    const uint32_t nq = rows / 128u;
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < (int64_t)cols; ++j)
        out[j] = mv_col(in, wq, sc, rows, cols, (uint32_t)j, 0, nq);
}

/* llm_matvec.cl:439-456 + :128-135 (mv_reduce) */
void xo_mv_km4_bs_split(float* out, const float* in, const uint32_t* wq, const uint32_t* sc,
                        uint32_t rows, uint32_t cols, uint32_t split) {
    const uint32_t nq = rows / 128u;
    const uint32_t per = (nq + split - 1u) / split;
#pragma omp parallel for schedule(static)
    for (int64_t jj = 0; jj < (int64_t)cols; ++jj) {
        const uint32_t j = (uint32_t)jj;
        float acc = 0.0f;
        for (uint32_t p = 0; p < split; ++p) {
            uint32_t q0 = p * per, q1 = q0 + per;
            if (q1 > nq) q1 = nq;
            acc += (q0 < q1) ? mv_col(in, wq, sc, rows, cols, j, q0, q1) : 0.0f;
        }
        out[j] = acc;
    }
}

/* examples/llm/decode.cpp:243-250 (MatvecConfig::split_for with split 4,
 * split_below_cols 2048) and the record_token matvec lambda :1660-1667 */
static void mv_auto(float* out, const float* in, const xo_qweight* w) {
    uint32_t s = 4u;
    if (w->cols >= 2048u) s = 1u;
    else if (s > w->rows / 32u) s = w->rows / 32u;
    if (s > 1u) xo_mv_km4_bs_split(out, in, w->wq, w->sc, w->rows, w->cols, s);
    else xo_mv_km4_bs(out, in, w->wq, w->sc, w->rows, w->cols);
}

/* ------------------------------------------------------------------------ */
/* transformer ops: kernels/llm_transformer.cl                               */
/* ------------------------------------------------------------------------ */
static float rsqrt_f(float x) { return 1.0f / sqrtf(x); }

/* llm_transformer.cl:96-116: strided partial sums of squares, then (1 + w). */
void xo_rmsnorm_gemma(float* out, const float* in, const float* w, uint32_t n, uint32_t nparts,
                      float eps) {
    float ss = 0.0f;
    for (uint32_t p = 0; p < nparts; ++p) {
        float acc = 0.0f;
        for (uint32_t k = p; k < n; k += nparts) acc += in[k] * in[k];
        ss += acc;
    }
    const float scale = rsqrt_f(ss / (float)n + eps);
    for (uint32_t i = 0; i < n; ++i) out[i] = in[i] * scale * (1.0f + w[i]);
}

/* llm_transformer.cl:122-134 */
void xo_rmsnorm_heads_gemma(float* out, const float* in, const float* w, uint32_t n_heads,
                            uint32_t head_dim, float eps) {
    for (uint32_t h = 0; h < n_heads; ++h) {
        const uint32_t base = h * head_dim;
        float ss = 0.0f;
        for (uint32_t k = 0; k < head_dim; ++k) ss += in[base + k] * in[base + k];
        const float scale = rsqrt_f(ss / (float)head_dim + eps);
        for (uint32_t d = 0; d < head_dim; ++d)
            out[base + d] = in[base + d] * scale * (1.0f + w[d]);
    }
}

/* llm_transformer.cl:158-179: rotate-half, inv = exp2(-log2(theta) * 2d/hd) */
void xo_rope(float* x, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float theta) {
    const uint32_t half = head_dim >> 1;
    for (uint32_t h = 0; h < n_heads; ++h)
        for (uint32_t d = 0; d < half; ++d) {
            const uint32_t base = h * head_dim + d;
            /* theta^(-2d/hd) as in the reference, with log2 and exp2 each
             * rounded once from double so every IEEE host and the device
             * agree bit for bit (the reference's fp32 exp2/log2 builtins
             * differ between drivers by an ulp). */
            const float l2 = (float)log2((double)theta);
            const float frac = (float)(2u * d) / (float)head_dim;
            const float inv = (float)exp2((double)(-l2 * frac));
            const float ang = (float)pos * inv;
            const float c = cosf(ang), s = sinf(ang);
            const float lo = x[base], hi = x[base + half];
            x[base] = lo * c - hi * s;
            x[base + half] = lo * s + hi * c;
        }
}

/* llm_transformer.cl:213-231: tanh-approximate GELU with a clamped-exp tanh */
static float tanh_approx(float z) {
    z = fminf(fmaxf(z, -10.0f), 10.0f);
    const float e = expf(-2.0f * z);
    return (1.0f - e) / (1.0f + e);
}
void xo_geglu(float* out, const float* gate, const float* up, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) {
        const float g = gate[i];
        const float inner = 0.7978845608028654f * (g + 0.044715f * g * g * g);
        const float gelu = 0.5f * g * (1.0f + tanh_approx(inner));
        out[i] = gelu * up[i];
    }
}

/* llm_transformer.cl:564-568 */
void xo_add_residual(float* x, const float* y, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) x[i] += y[i];
}

static float kv_at(const void* cache, int fp16, size_t i) {
    return fp16 ? xo_f16_to_f32(((const uint16_t*)cache)[i]) : ((const float*)cache)[i];
}

/* llm_transformer.cl:287-305 (scores), :318-335 (softmax_rows), :478-497
 * (apply), in their serial forms. */
void xo_attention(float* out, const float* q, const void* kc, const void* vc, int kv_fp16,
                  uint32_t n_heads, uint32_t kv_heads, uint32_t head_dim, uint32_t kv_start,
                  uint32_t span, float scale) {
    float* p = (float*)malloc(sizeof(float) * (span ? span : 1u));
    const uint32_t group = n_heads / kv_heads;
    for (uint32_t h = 0; h < n_heads; ++h) {
        const uint32_t kvh = h / group;
        for (uint32_t j = 0; j < span; ++j) {
            const size_t kb = ((size_t)(kv_start + j) * kv_heads + kvh) * head_dim;
            float acc = 0.0f;
            for (uint32_t d = 0; d < head_dim; ++d) acc += q[h * head_dim + d] * kv_at(kc, kv_fp16, kb + d);
            p[j] = acc * scale;
        }
        float m = -INFINITY;
        for (uint32_t j = 0; j < span; ++j) m = fmaxf(m, p[j]);
        float sum = 0.0f;
        for (uint32_t j = 0; j < span; ++j) { const float e = expf(p[j] - m); p[j] = e; sum += e; }
        const float inv = 1.0f / sum;
        for (uint32_t j = 0; j < span; ++j) p[j] *= inv;
        for (uint32_t d = 0; d < head_dim; ++d) {
            const size_t vstride = (size_t)kv_heads * head_dim;
            const size_t vb = ((size_t)kv_start * kv_heads + kvh) * head_dim + d;
            float acc = 0.0f;
            for (uint32_t j = 0; j < span; ++j) acc += p[j] * kv_at(vc, kv_fp16, vb + j * vstride);
            out[h * head_dim + d] = acc;
        }
    }
    free(p);
}

/* ------------------------------------------------------------------------ */
/* sampling: kernels/llm_sampling.cl, examples/llm/decode.cpp:1873-1917      */
/* ------------------------------------------------------------------------ */
/* llm_sampling.cl:57-123: ties -> lowest index */
uint32_t xo_argmax(const float* x, uint32_t n, float* best_val) {
    uint32_t bi = 0;
    float bv = -INFINITY;
    for (uint32_t k = 0; k < n; ++k)
        if (x[k] > bv) { bv = x[k]; bi = k; }
    if (best_val) *best_val = bv;
    return bi;
}

static int better(float va, uint32_t ia, float vb, uint32_t ib) {
    return va > vb || (va == vb && ia < ib);
}

/* llm_sampling.cl:249-286 semantics: the k largest, descending, ties ->
 * lower index (identical to a CPU stable sort). */
uint32_t xo_topk(const float* x, uint32_t n, uint32_t k, float* vals, uint32_t* idx) {
    if (k > n) k = n;
    uint32_t cnt = 0;
    for (uint32_t e = 0; e < n; ++e) {
        const float v = x[e];
        if (cnt == k && !better(v, e, vals[k - 1], idx[k - 1])) continue;
        uint32_t j = cnt < k ? cnt++ : k - 1;
        while (j > 0 && better(v, e, vals[j - 1], idx[j - 1])) {
            vals[j] = vals[j - 1];
            idx[j] = idx[j - 1];
            --j;
        }
        vals[j] = v;
        idx[j] = e;
    }
    return cnt;
}

/* decode.cpp:1873-1917. The candidates are the exact top-k (all of them when
 * top_k == 0), visited in descending order. Weights exp((l - max) / T) in
 * fp32, running sums in double, the crossing token kept by top-p, then the
 * multinomial walk with r = u * sum. */
uint32_t xo_sample(const float* logits, uint32_t n, float temperature, uint32_t top_k,
                   float top_p, float u) {
    const float t = temperature > 0.0f ? temperature : 1.0f;
    uint32_t k = top_k ? (top_k < n ? top_k : n) : n;
    float* v = (float*)malloc(sizeof(float) * k);
    uint32_t* id = (uint32_t*)malloc(sizeof(uint32_t) * k);
    k = xo_topk(logits, n, k, v, id);
    if (k == 0) { free(v); free(id); return 0; }
    const float maxl = v[0];
    double sum = 0.0;
    for (uint32_t i = 0; i < k; ++i) { v[i] = expf((v[i] - maxl) / t); sum += v[i]; }
    if (top_p > 0.0f && top_p < 1.0f && sum > 0.0) {
        double acc = 0.0;
        const double cut = (double)top_p * sum;
        uint32_t keep = 0;
        for (; keep < k; ++keep) { acc += v[keep]; if (acc >= cut) break; }
        k = keep + 1 < k ? keep + 1 : k;
        sum = 0.0;
        for (uint32_t i = 0; i < k; ++i) sum += v[i];
    }
    double r = (double)u * sum;
    uint32_t chosen = id[k - 1];
    for (uint32_t i = 0; i < k; ++i) { r -= v[i]; if (r <= 0.0) { chosen = id[i]; break; } }
    free(v);
    free(id);
    return chosen;
}

/* ------------------------------------------------------------------------ */
/* one token: examples/llm/decode.cpp:1618-1780                              */
/* ------------------------------------------------------------------------ */
/* decode.hpp:327-352: layer i is global iff (i+1) % global_every == 0; a local
 * layer attends the suffix (pos - window, pos]. */
uint32_t xo_layer_kv_start(const xo_model* m, uint32_t layer, uint32_t seq_len) {
    const int global = m->global_every == 0 || (layer + 1u) % m->global_every == 0u;
    const uint32_t w = global ? 0u : m->sliding_window;
    return (w == 0u || seq_len <= w) ? 0u : seq_len - w;
}

int xo_forward(const xo_model* m, xo_state* st, uint32_t token, uint32_t pos, float* logits) {
    const uint32_t H = m->hidden, F = m->ffn;
    const uint32_t qd = m->n_heads * m->head_dim, kvd = m->n_kv_heads * m->head_dim;
    if (token >= m->vocab || pos >= m->max_seq) return -1;
    float* x = (float*)malloc(sizeof(float) * H);
    float* xb = (float*)malloc(sizeof(float) * (H > qd ? H : qd));
    float* xb2 = (float*)malloc(sizeof(float) * H);
    float* qr = (float*)malloc(sizeof(float) * qd);
    float* q = (float*)malloc(sizeof(float) * qd);
    float* kr = (float*)malloc(sizeof(float) * kvd);
    float* k = (float*)malloc(sizeof(float) * kvd);
    float* v = (float*)malloc(sizeof(float) * kvd);
    float* att = (float*)malloc(sizeof(float) * qd);
    float* hg = (float*)malloc(sizeof(float) * F);
    float* hu = (float*)malloc(sizeof(float) * F);
    float* hb = (float*)malloc(sizeof(float) * F);

    /* decode.cpp:1618-1627 -- embedding row times sqrt(hidden) */
    for (uint32_t i = 0; i < H; ++i) x[i] = m->embed[(size_t)token * H + i] * m->embed_scale;
    const uint32_t seq_len = pos + 1u;
    for (uint32_t l = 0; l < m->n_layers; ++l) {
        const xo_layer* w = &m->layers[l];
        const int global = m->global_every == 0 || (l + 1u) % m->global_every == 0u;
        const float theta = global ? m->theta_global : m->theta_local;
        xo_rmsnorm_gemma(xb, x, w->attn_norm, H, m->norm_parts, m->rms_eps);
        mv_auto(qr, xb, &w->wq);
        mv_auto(kr, xb, &w->wk);
        mv_auto(v, xb, &w->wv);
        xo_rmsnorm_heads_gemma(q, qr, w->q_norm, m->n_heads, m->head_dim, m->rms_eps);
        xo_rmsnorm_heads_gemma(k, kr, w->k_norm, m->n_kv_heads, m->head_dim, m->rms_eps);
        xo_rope(q, m->n_heads, m->head_dim, pos, theta);
        xo_rope(k, m->n_kv_heads, m->head_dim, pos, theta);
        for (uint32_t i = 0; i < kvd; ++i) {
            const size_t o = (size_t)pos * kvd + i;
            if (m->kv_fp16) {
                ((uint16_t*)st->kcache[l])[o] = xo_f32_to_f16(k[i]);
                ((uint16_t*)st->vcache[l])[o] = xo_f32_to_f16(v[i]);
            } else {
                ((float*)st->kcache[l])[o] = k[i];
                ((float*)st->vcache[l])[o] = v[i];
            }
        }
        const uint32_t kv_start = xo_layer_kv_start(m, l, seq_len);
        xo_attention(att, q, st->kcache[l], st->vcache[l], m->kv_fp16, m->n_heads,
                     m->n_kv_heads, m->head_dim, kv_start, seq_len - kv_start, m->attn_scale);
        mv_auto(xb, att, &w->wo);
        xo_rmsnorm_gemma(xb2, xb, w->post_attn_norm, H, m->norm_parts, m->rms_eps);
        xo_add_residual(x, xb2, H);
        xo_rmsnorm_gemma(xb, x, w->ffn_norm, H, m->norm_parts, m->rms_eps);
        mv_auto(hg, xb, &w->gate);
        mv_auto(hu, xb, &w->up);
        xo_geglu(hb, hg, hu, F);
        mv_auto(xb, hb, &w->down);
        xo_rmsnorm_gemma(xb2, xb, w->post_ffn_norm, H, m->norm_parts, m->rms_eps);
        xo_add_residual(x, xb2, H);
    }
    xo_rmsnorm_gemma(xb, x, m->final_norm, H, m->norm_parts, m->rms_eps);
    if (logits) mv_auto(logits, xb, &m->lm_head);
    free(x); free(xb); free(xb2); free(qr); free(q); free(kr); free(k); free(v);
    free(att); free(hg); free(hu); free(hb);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* prefill shapes: kernels/llm_sampling.cl:495-736 (row-major [row][col])    */
/* ------------------------------------------------------------------------ */
/* llm_sampling.cl:527-546: per row (max, sum of exp(x - max)); a fully
 * masked row gives (0, 1) */
void xo_softmax_rows_stats(float* stats, const float* x, uint32_t n_rows, uint32_t n_cols) {
    for (uint32_t r = 0; r < n_rows; ++r) {
        const float* row = x + (size_t)r * n_cols;
        float m = -INFINITY;
        for (uint32_t j = 0; j < n_cols; ++j) m = fmaxf(m, row[j]);
        if (!isfinite(m)) { stats[2 * r] = 0.0f; stats[2 * r + 1] = 1.0f; continue; }
        float s = 0.0f;
        for (uint32_t j = 0; j < n_cols; ++j) s += expf(row[j] - m);
        stats[2 * r] = m;
        stats[2 * r + 1] = s;
    }
}

/* llm_sampling.cl:549-556 */
void xo_softmax_rows_apply(float* x, const float* stats, uint32_t n_rows, uint32_t n_cols) {
    for (uint64_t i = 0; i < (uint64_t)n_rows * n_cols; ++i) {
        const uint32_t r = (uint32_t)(i / n_cols);
        x[i] = expf(x[i] - stats[2 * r]) / stats[2 * r + 1];
    }
}

/* llm_sampling.cl:574-602: causal + sliding-window masked scores */
void xo_attention_scores_prefill(float* scores, const float* q, const float* kcache, uint32_t n_heads,
                                 uint32_t kv_heads, uint32_t head_dim, uint32_t n_query,
                                 uint32_t seq_len, uint32_t q_offset, uint32_t window, float scale) {
    const uint32_t group = n_heads / kv_heads;
    for (uint32_t h = 0; h < n_heads; ++h)
        for (uint32_t qi = 0; qi < n_query; ++qi)
            for (uint32_t t = 0; t < seq_len; ++t) {
                const size_t o = ((size_t)h * n_query + qi) * seq_len + t;
                const uint32_t qpos = q_offset + qi;
                if (t > qpos || (window != 0u && t + window <= qpos)) { scores[o] = -INFINITY; continue; }
                const float* qr = q + ((size_t)h * n_query + qi) * head_dim;
                const float* kr = kcache + ((size_t)t * kv_heads + h / group) * head_dim;
                float acc = 0.0f;
                for (uint32_t d = 0; d < head_dim; ++d) acc += qr[d] * kr[d];
                scores[o] = acc * scale;
            }
}

/* llm_sampling.cl:605-630 */
void xo_attention_apply_prefill(float* out, const float* probs, const float* vcache, uint32_t n_heads,
                                uint32_t kv_heads, uint32_t head_dim, uint32_t n_query,
                                uint32_t seq_len) {
    const uint32_t group = n_heads / kv_heads;
    for (uint32_t h = 0; h < n_heads; ++h)
        for (uint32_t qi = 0; qi < n_query; ++qi)
            for (uint32_t d = 0; d < head_dim; ++d) {
                const float* p = probs + ((size_t)h * n_query + qi) * seq_len;
                float acc = 0.0f;
                for (uint32_t t = 0; t < seq_len; ++t)
                    acc += p[t] * vcache[((size_t)t * kv_heads + h / group) * head_dim + d];
                out[((size_t)h * n_query + qi) * head_dim + d] = acc;
            }
}

/* llm_sampling.cl:634-642 */
void xo_rmsnorm_rows_sumsq(float* rowss, const float* in, uint32_t n_rows, uint32_t n) {
    for (uint32_t r = 0; r < n_rows; ++r) {
        float ss = 0.0f;
        for (uint32_t j = 0; j < n; ++j) ss += in[(size_t)r * n + j] * in[(size_t)r * n + j];
        rowss[r] = ss;
    }
}

/* llm_sampling.cl:645-656 */
void xo_rmsnorm_rows_apply_gemma(float* out, const float* in, const float* w, const float* rowss,
                                 uint32_t n_rows, uint32_t n, float eps) {
    for (uint32_t r = 0; r < n_rows; ++r) {
        const float scale = rsqrt_f(rowss[r] / (float)n + eps);
        for (uint32_t j = 0; j < n; ++j)
            out[(size_t)r * n + j] = in[(size_t)r * n + j] * scale * (1.0f + w[j]);
    }
}

/* llm_sampling.cl:659-675 */
void xo_rmsnorm_heads_rows_gemma(float* out, const float* in, const float* w, uint32_t n_tokens,
                                 uint32_t n_heads, uint32_t head_dim, float eps) {
    xo_rmsnorm_heads_gemma(out, in, w, n_tokens * n_heads, head_dim, eps);
}

/* llm_sampling.cl:687-711: token ti at position pos0 + ti, the angle of
 * xo_rope (theta^(-2d/hd) rounded once from double) */
void xo_rope_prefill(float* x, uint32_t n_tokens, uint32_t n_heads, uint32_t head_dim,
                     uint32_t pos0, float theta) {
    const size_t per = (size_t)n_heads * head_dim;
    for (uint32_t t = 0; t < n_tokens; ++t) xo_rope(x + t * per, n_heads, head_dim, pos0 + t, theta);
}

/* llm_sampling.cl:714-722 */
void xo_kv_append_rows(float* cache, const float* src, uint32_t n_tokens, uint32_t row,
                       uint32_t pos0) {
    memcpy(cache + (size_t)pos0 * row, src, (size_t)n_tokens * row * sizeof(float));
}

/* llm_sampling.cl:728-736 */
void xo_embed_lookup_rows(float* out, const float* table, const uint32_t* tokens,
                          uint32_t n_tokens, uint32_t n) {
    for (uint32_t t = 0; t < n_tokens; ++t)
        memcpy(out + (size_t)t * n, table + (size_t)tokens[t] * n, (size_t)n * sizeof(float));
}

/* ------------------------------------------------------------------------ */
/* GGUF tensor types: examples/llm/model/gguf.cpp:448-634 (the ggml blocks)  */
/* ------------------------------------------------------------------------ */
static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }

/* gguf.cpp:431-443: the 6-bit scale and min of Q4_K sub-block j */
static void k4_scale_min(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

int xo_gguf_dequantize(uint32_t type, const void* src, float* dst, uint64_t n) {
    const uint8_t* p = (const uint8_t*)src;
    switch (type) {
        case 0: memcpy(dst, p, n * 4); return 0;
        case 1:
            for (uint64_t i = 0; i < n; ++i) dst[i] = xo_f16_to_f32(rd16(p + 2 * i));
            return 0;
        case 30:
            for (uint64_t i = 0; i < n; ++i) {
                const uint32_t b = (uint32_t)rd16(p + 2 * i) << 16;
                memcpy(dst + i, &b, 4);
            }
            return 0;
        case 2: case 3: case 6: case 7: case 8: {
            if (n % 32) return -1;
            const uint32_t bs = type == 2 ? 18 : type == 3 ? 20 : type == 6 ? 22 : type == 7 ? 24 : 34;
            for (uint64_t b = 0; b < n / 32; ++b) {
                const uint8_t* blk = p + b * bs;
                const float d = xo_f16_to_f32(rd16(blk));
                float* y = dst + b * 32;
                if (type == 8) {
                    for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)blk[2 + j] * d;
                } else if (type == 2 || type == 3) {
                    const float m = type == 3 ? xo_f16_to_f32(rd16(blk + 2)) : 0.0f;
                    const uint8_t* qs = blk + (type == 3 ? 4 : 2);
                    for (int j = 0; j < 16; ++j) {
                        if (type == 2) {
                            y[j] = (float)((int)(qs[j] & 0xF) - 8) * d;
                            y[j + 16] = (float)((int)(qs[j] >> 4) - 8) * d;
                        } else {
                            y[j] = (float)(qs[j] & 0xF) * d + m;
                            y[j + 16] = (float)(qs[j] >> 4) * d + m;
                        }
                    }
                } else {
                    const int one = type == 7;
                    const float m = one ? xo_f16_to_f32(rd16(blk + 2)) : 0.0f;
                    const uint32_t qh = rd32(blk + (one ? 4 : 2));
                    const uint8_t* qs = blk + (one ? 8 : 6);
                    for (int j = 0; j < 16; ++j) {
                        const int q0 = (qs[j] & 0xF) | (int)(((qh >> j) << 4) & 0x10);
                        const int q1 = (qs[j] >> 4) | (int)((qh >> (j + 12)) & 0x10);
                        if (one) {
                            y[j] = (float)q0 * d + m;
                            y[j + 16] = (float)q1 * d + m;
                        } else {
                            y[j] = (float)(q0 - 16) * d;
                            y[j + 16] = (float)(q1 - 16) * d;
                        }
                    }
                }
            }
            return 0;
        }
        case 12:
            if (n % 256) return -1;
            for (uint64_t b = 0; b < n / 256; ++b) {
                const uint8_t* blk = p + b * 144;
                const float d = xo_f16_to_f32(rd16(blk)), dmin = xo_f16_to_f32(rd16(blk + 2));
                const uint8_t* sc = blk + 4;
                for (int e = 0; e < 256; ++e) {
                    const int c = e / 64, w = e % 64, is = 2 * c + (w >= 32), l = w % 32;
                    const uint8_t qb = blk[16 + 32 * c + l];
                    const int q = w < 32 ? (qb & 0xF) : (qb >> 4);
                    uint8_t s, m;
                    k4_scale_min(is, sc, &s, &m);
                    const float d1 = d * (float)s, m1 = dmin * (float)m;
                    dst[b * 256 + e] = d1 * (float)q - m1;
                }
            }
            return 0;
        case 14:
            if (n % 256) return -1;
            for (uint64_t b = 0; b < n / 256; ++b) {
                const uint8_t* blk = p + b * 210;
                const float d = xo_f16_to_f32(rd16(blk + 208));
                for (int e = 0; e < 256; ++e) {
                    const int h = e / 128, r = e % 128, g = r / 32, l = r % 32, is = l / 16;
                    const uint8_t* ql = blk + 64 * h;
                    const uint8_t qh = blk[128 + 32 * h + l];
                    const int8_t s = (int8_t)blk[192 + 8 * h + is + 2 * g];
                    const uint8_t lo = (g & 1) ? ql[l + 32] : ql[l];
                    const int nib = (g < 2) ? (lo & 0xF) : (lo >> 4);
                    const int q = (nib | (((qh >> (2 * g)) & 3) << 4)) - 32;
                    dst[b * 256 + e] = d * (float)s * (float)q;
                }
            }
            return 0;
        default:
            return -1;
    }
}

/* decode.cpp:784-799 */
uint64_t xo_xpack_hash(const void* data, uint64_t nbytes) {
    const uint8_t* p = (const uint8_t*)data;
    uint64_t h = 1469598103934665603ull ^ nbytes;
    uint64_t i = 0;
    for (; i + 8 <= nbytes; i += 8) {
        uint64_t w;
        memcpy(&w, p + i, 8);
        h = (h ^ w) * 1099511628211ull;
        h ^= h >> 29;
    }
    for (; i < nbytes; ++i) h = (h ^ p[i]) * 1099511628211ull;
    h ^= h >> 32;
    h *= 0xff51afd7ed558ccdull;
    h ^= h >> 32;
    return h;
}

/* decode.cpp:803-834: per-4-MiB-chunk hashes folded in chunk order */
uint64_t xo_xpack_hash_chunked(const void* data, uint64_t nbytes) {
    const uint64_t chunk = 4ull << 20;
    const uint8_t* p = (const uint8_t*)data;
    uint64_t acc = 1469598103934665603ull ^ nbytes;
    for (uint64_t off = 0; off < nbytes; off += chunk)
        acc = (acc ^ xo_xpack_hash(p + off, nbytes - off < chunk ? nbytes - off : chunk)) * 1099511628211ull;
    return acc;
}
