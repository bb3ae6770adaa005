// The reference operator surface, one CUDA kernel per entry point of
// kernels/llm_matvec.cl, kernels/llm_transformer.cl and kernels/llm_sampling.cl
// that the reference decode loop (examples/llm/decode.cpp:1634-1780) and its
// harnesses drive. Each keeps the reference entry point's arguments and output
// contract; the work decomposition is this build's own (the registry in
// capi.cu decides CTA shapes from the reference's global-thread grid).
//
// Kernels whose reference form is one serial thread per row or per vector
// (softmax_rows, argmax, *_final, topp_cutoff, multinomial_*) run here as one
// CTA per row with block reductions, producing the same values and the same
// tie rules.
#pragma once
#include "common.cuh"

namespace xp {
namespace ops {

#define GID() (blockIdx.x * blockDim.x + threadIdx.x)

// ---- llm_matvec.cl -----------------------------------------------------------
// mv_reduce (llm_matvec.cl:128-135): out[j] = sum_p partial[p*cols + j]
__global__ void mv_reduce(float* out, const float* partial, uint32_t cols, uint32_t split) {
    const uint32_t j = GID();
    if (j >= cols) return;
    float acc = 0.0f;
    for (uint32_t p = 0; p < split; ++p) acc += partial[(size_t)p * cols + j];
    out[j] = acc;
}

// stream4 (llm_matvec.cl:370-378): pure-load probe; stores only when the sum
// equals a value it cannot take, so every load stays live.
__global__ void stream4(float* out, const uint4* src, uint32_t n, uint32_t threads) {
    const uint32_t i = GID();
    if (i >= threads) return;
    uint4 acc = make_uint4(0, 0, 0, 0);
    for (uint32_t k = i; k < n; k += threads) {
        const uint4 v = __ldg(src + k);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    const uint32_t s = acc.x + acc.y + acc.z + acc.w;
    if (s == 0xDEADBEEFu) out[i & 3u] = (float)s;
}

// ---- llm_transformer.cl ------------------------------------------------------
// rmsnorm / rmsnorm_gemma (llm_transformer.cl:60-84): one CTA computes the
// sum of squares once and applies it, instead of n redundant sums.
template <bool GEMMA>
__global__ void rmsnorm_one(float* out, const float* in, const float* w, uint32_t n, float eps) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (uint32_t k = threadIdx.x; k < n; k += blockDim.x) ss += in[k] * in[k];
    ss = block_sum(ss, red);
    const float scale = rsqrtf(ss / (float)n + eps);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = in[i] * scale * (GEMMA ? 1.0f + w[i] : w[i]);
}

// rmsnorm_sumsq (:96-103): partial[p] = sum_{k = p mod nparts} in[k]^2
__global__ void rmsnorm_sumsq(float* partial, const float* in, uint32_t n, uint32_t nparts) {
    const uint32_t p = GID();
    if (p >= nparts) return;
    float acc = 0.0f;
    for (uint32_t k = p; k < n; k += nparts) acc += in[k] * in[k];
    partial[p] = acc;
}

// rmsnorm_apply_gemma (:106-116)
__global__ void rmsnorm_apply_gemma(float* out, const float* in, const float* w, const float* partial,
                                    uint32_t n, uint32_t nparts, float eps) {
    __shared__ float ssh;
    if (threadIdx.x < 32) {
        float s = 0.0f;
        for (uint32_t p = threadIdx.x; p < nparts; p += 32) s += partial[p];
        s = warp_sum(s);
        if (threadIdx.x == 0) ssh = s;
    }
    __syncthreads();
    const uint32_t i = GID();
    if (i >= n) return;
    const float scale = rsqrtf(ssh / (float)n + eps);
    out[i] = in[i] * scale * (1.0f + w[i]);
}

// rmsnorm_heads_gemma (:122-134): one warp per head.
__global__ void rmsnorm_heads_gemma(float* out, const float* in, const float* w, uint32_t n_heads,
                                    uint32_t head_dim, float eps) {
    const uint32_t h = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const uint32_t lane = threadIdx.x & 31;
    if (h >= n_heads) return;
    const float* x = in + (size_t)h * head_dim;
    float ss = 0.0f;
    for (uint32_t k = lane; k < head_dim; k += 32) ss += x[k] * x[k];
    ss = warp_sum(ss);
    const float scale = rsqrtf(ss / (float)head_dim + eps);
    for (uint32_t d = lane; d < head_dim; d += 32) out[(size_t)h * head_dim + d] = x[d] * scale * (1.0f + w[d]);
}

// RoPE angle for pair index d: pos * theta^(-2d/head_dim), formed as in the
// reference (llm_transformer.cl:158-179) with full-precision exp2/log2/sin/cos.
XP_DEV void rope_cs(uint32_t d, uint32_t head_dim, uint32_t pos, float theta, float& c, float& s) {
    // log2 and exp2 rounded once from double: identical on every IEEE host
    const float l2 = (float)log2((double)theta);
    const float frac = (float)(2u * d) / (float)head_dim;
    const float inv = (float)exp2((double)(-l2 * frac));
    const float ang = (float)pos * inv;
    sincosf(ang, &s, &c);
}

// rope (:158-179): in place, one thread per (head, pair)
__global__ void rope(float* x, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float theta) {
    const uint32_t half = head_dim >> 1;
    const uint32_t i = GID();
    if (i >= n_heads * half) return;
    const uint32_t h = i / half, d = i - h * half;
    const uint32_t base = h * head_dim + d;
    float c, s;
    rope_cs(d, head_dim, pos, theta, c, s);
    const float lo = x[base], hi = x[base + half];
    x[base] = lo * c - hi * s;
    x[base + half] = lo * s + hi * c;
}

// rope_cached (:186-204)
__global__ void rope_cached(float* x, const float* cos_t, const float* sin_t, uint32_t n_heads,
                            uint32_t head_dim) {
    const uint32_t half = head_dim >> 1;
    const uint32_t i = GID();
    if (i >= n_heads * half) return;
    const uint32_t h = i / half, d = i - h * half;
    const uint32_t base = h * head_dim + d;
    const float c = cos_t[d], s = sin_t[d];
    const float lo = x[base], hi = x[base + half];
    x[base] = lo * c - hi * s;
    x[base + half] = lo * s + hi * c;
}

// geglu / swiglu / geglu_fused (:213-256)
__global__ void geglu(float* out, const float* gate, const float* up, uint32_t n) {
    const uint32_t i = GID();
    if (i >= n) return;
    out[i] = gelu_tanh_ref(gate[i]) * up[i];
}
__global__ void swiglu(float* out, const float* gate, const float* up, uint32_t n) {
    const uint32_t i = GID();
    if (i >= n) return;
    const float g = gate[i];
    const float sig = 1.0f / (1.0f + expf(-fminf(fmaxf(g, -30.0f), 30.0f)));
    out[i] = g * sig * up[i];
}
__global__ void geglu_fused(float* out, const float* gate_up, uint32_t n) {
    const uint32_t i = GID();
    if (i >= n) return;
    out[i] = gelu_tanh_ref(gate_up[i]) * gate_up[n + i];
}

// attention_scores (:287-305): scores[h*span + j] = scale * q_h . k[kv_start + j]
// One warp per (head, key).
__global__ void attention_scores(float* scores, const float* q, const float* kcache, uint32_t n_heads,
                                 uint32_t kv_heads, uint32_t head_dim, uint32_t span, float scale,
                                 uint32_t kv_start) {
    const uint32_t w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (w >= n_heads * span) return;
    const uint32_t h = w / span, j = w - h * span, kvh = h / (n_heads / kv_heads);
    const float* qh = q + (size_t)h * head_dim;
    const float* kr = kcache + ((size_t)(kv_start + j) * kv_heads + kvh) * head_dim;
    float acc = 0.0f;
    for (uint32_t d = lane; d < head_dim; d += 32) acc += qh[d] * kr[d];
    acc = warp_sum(acc);
    if (lane == 0) scores[w] = acc * scale;
}

// attention_scores_mq4 (:444-464): 4 heads, 1 kv head, one warp per key.
__global__ void attention_scores_mq4(float* scores, const float* q, const float* kcache, uint32_t head_dim,
                                     uint32_t span, float scale, uint32_t kv_start) {
    const uint32_t j = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
    if (j >= span) return;
    const float* kr = kcache + (size_t)(kv_start + j) * head_dim;
    float a[4] = {0, 0, 0, 0};
    for (uint32_t d = lane; d < head_dim; d += 32) {
        const float k = kr[d];
#pragma unroll
        for (int h = 0; h < 4; ++h) a[h] += q[h * head_dim + d] * k;
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
        const float s = warp_sum(a[h]);
        if (lane == 0) scores[(size_t)h * span + j] = s * scale;
    }
}

// softmax_rows (:318-335): one CTA per row (the reference walks a row with one
// thread; values are the same max-subtracted softmax).
__global__ void softmax_rows(float* x, uint32_t n_rows, uint32_t n_cols) {
    __shared__ float red[32];
    const uint32_t r = blockIdx.x;
    if (r >= n_rows) return;
    float* row = x + (size_t)r * n_cols;
    float m = -INFINITY;
    for (uint32_t j = threadIdx.x; j < n_cols; j += blockDim.x) m = fmaxf(m, row[j]);
    m = warp_max(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = (threadIdx.x & 31) < (blockDim.x >> 5) ? red[threadIdx.x & 31] : -INFINITY;
    m = warp_max(m);
    float s = 0.0f;
    for (uint32_t j = threadIdx.x; j < n_cols; j += blockDim.x) {
        const float e = expf(row[j] - m);
        row[j] = e;
        s += e;
    }
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    for (uint32_t j = threadIdx.x; j < n_cols; j += blockDim.x) row[j] *= inv;
}

// softmax_rows_partial / _finish / _scale (:363-416)
__global__ void softmax_rows_partial(float* pmax, float* psum, const float* x, uint32_t n_rows,
                                     uint32_t n_cols, uint32_t nparts) {
    const uint32_t i = GID();
    if (i >= n_rows * nparts) return;
    const uint32_t r = i / nparts, p = i - r * nparts;
    const float* row = x + (size_t)r * n_cols;
    float m = -INFINITY;
    for (uint32_t j = p; j < n_cols; j += nparts) m = fmaxf(m, row[j]);
    float s = 0.0f;
    if (isfinite(m))
        for (uint32_t j = p; j < n_cols; j += nparts) s += expf(row[j] - m);
    pmax[i] = m;
    psum[i] = s;
}
__global__ void softmax_rows_finish(float* stats, const float* pmax, const float* psum, uint32_t n_rows,
                                    uint32_t nparts) {
    const uint32_t r = GID();
    if (r >= n_rows) return;
    const size_t b = (size_t)r * nparts;
    float M = -INFINITY;
    for (uint32_t p = 0; p < nparts; ++p) M = fmaxf(M, pmax[b + p]);
    if (!isfinite(M)) { stats[2 * r] = 0.0f; stats[2 * r + 1] = 1.0f; return; }
    float S = 0.0f;
    for (uint32_t p = 0; p < nparts; ++p) {
        const float pm = pmax[b + p];
        if (isfinite(pm)) S += psum[b + p] * expf(pm - M);
    }
    stats[2 * r] = M;
    stats[2 * r + 1] = S > 0.0f ? 1.0f / S : 1.0f;
}
__global__ void softmax_rows_scale(float* x, const float* stats, uint32_t n_rows, uint32_t n_cols) {
    const uint32_t i = GID();
    if (i >= n_rows * n_cols) return;
    const uint32_t r = i / n_cols;
    x[i] = expf(x[i] - stats[2 * r]) * stats[2 * r + 1];
}

// attention_apply (:478-497): out[h*hd + d] = sum_j probs[h*span + j] v[kv_start + j][kvh][d]
__global__ void attention_apply(float* out, const float* probs, const float* vcache, uint32_t n_heads,
                                uint32_t kv_heads, uint32_t head_dim, uint32_t span, uint32_t kv_start) {
    const uint32_t i = GID();
    if (i >= n_heads * head_dim) return;
    const uint32_t h = i / head_dim, d = i - h * head_dim, kvh = h / (n_heads / kv_heads);
    const size_t vstride = (size_t)kv_heads * head_dim;
    const float* v = vcache + ((size_t)kv_start * kv_heads + kvh) * head_dim + d;
    const float* p = probs + (size_t)h * span;
    float acc = 0.0f;
    for (uint32_t j = 0; j < span; ++j) acc += p[j] * v[j * vstride];
    out[i] = acc;
}

// attention_apply_mq4 (:515-547) + attention_apply_reduce (:550-557)
__global__ void attention_apply_mq4(float* partial, const float* probs, const float* vcache, uint32_t head_dim,
                                    uint32_t span, uint32_t kv_start, uint32_t split) {
    const uint32_t i = GID();
    if (i >= head_dim * split) return;
    const uint32_t s = i / head_dim, d = i - s * head_dim;
    const uint32_t chunk = (span + split - 1) / split;
    const uint32_t j0 = s * chunk;
    const uint32_t j1 = min(j0 + chunk, span);
    float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    for (uint32_t j = j0; j < j1; ++j) {
        const float v = vcache[(size_t)(kv_start + j) * head_dim + d];
        a0 += probs[j] * v;
        a1 += probs[span + j] * v;
        a2 += probs[2 * span + j] * v;
        a3 += probs[3 * span + j] * v;
    }
    const size_t ob = (size_t)s * 4 * head_dim + d;
    partial[ob] = a0;
    partial[ob + head_dim] = a1;
    partial[ob + 2 * head_dim] = a2;
    partial[ob + 3 * head_dim] = a3;
}
__global__ void attention_apply_reduce(float* out, const float* partial, uint32_t n, uint32_t split) {
    const uint32_t i = GID();
    if (i >= n) return;
    float acc = 0.0f;
    for (uint32_t s = 0; s < split; ++s) acc += partial[(size_t)s * n + i];
    out[i] = acc;
}

// plumbing (:564-608)
__global__ void add_residual(float* x, const float* y, uint32_t n) {
    const uint32_t i = GID();
    if (i < n) x[i] += y[i];
}
__global__ void add_vec(float* out, const float* a, const float* b, uint32_t n) {
    const uint32_t i = GID();
    if (i < n) out[i] = a[i] + b[i];
}
__global__ void mul_scalar(float* x, float s, uint32_t n) {
    const uint32_t i = GID();
    if (i < n) x[i] *= s;
}
__global__ void kv_append(float* cache, const float* src, uint32_t n, uint32_t pos) {
    const uint32_t i = GID();
    if (i < n) cache[(size_t)pos * n + i] = src[i];
}
__global__ void embed_lookup(float* out, const float* table, uint32_t token, uint32_t n) {
    const uint32_t i = GID();
    if (i < n) out[i] = table[(size_t)token * n + i];
}

// ---- argmax family (lowest index wins on ties) ------------------------------
XP_DEV void am_better(float& bv, uint32_t& bi, float v, uint32_t i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}
XP_DEV void am_block(float& bv, uint32_t& bi) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        am_better(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0xFFFFFFFFu;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        am_better(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
}

// argmax (llm_transformer.cl:618-629): out[0] = index as float, out[1] = value
__global__ void argmax(float* out, const float* logits, uint32_t n) {
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t k = threadIdx.x; k < n; k += blockDim.x) am_better(bv, bi, logits[k], k);
    am_block(bv, bi);
    if (threadIdx.x == 0) {
        if (bi == 0xFFFFFFFFu) bi = 0;  // all -inf/NaN: the reference keeps index 0
        out[0] = (float)bi;
        out[1] = bv;
    }
}

// uint index of an argmax result (out[0] holds it as an exact float)
__global__ void argmax_index(uint32_t* idx, const float* out) {
    if (threadIdx.x == 0) idx[0] = (uint32_t)out[0];
}

// argmax_partial (llm_sampling.cl:57-71): strided chains, strict '>'
__global__ void argmax_partial(float* pval, uint32_t* pidx, const float* logits, uint32_t n, uint32_t nparts) {
    const uint32_t p = GID();
    if (p >= nparts) return;
    float bv = -INFINITY;
    uint32_t bi = 0;
    for (uint32_t k = p; k < n; k += nparts) {
        const float v = logits[k];
        if (v > bv) { bv = v; bi = k; }
    }
    pval[p] = bv;
    pidx[p] = bi;
}
// argmax_reduce (:86-100)
__global__ void argmax_reduce(float* oval, uint32_t* oidx, const float* pval, const uint32_t* pidx, uint32_t n,
                              uint32_t nparts) {
    const uint32_t p = GID();
    if (p >= nparts) return;
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t k = p; k < n; k += nparts) am_better(bv, bi, pval[k], pidx[k]);
    oval[p] = bv;
    oidx[p] = bi;
}
// argmax_final (:107-123)
__global__ void argmax_final(float* out, uint32_t* pidx_out, const float* pval, const uint32_t* pidx,
                             uint32_t nparts) {
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t p = threadIdx.x; p < nparts; p += blockDim.x) am_better(bv, bi, pval[p], pidx[p]);
    am_block(bv, bi);
    if (threadIdx.x == 0) {
        out[0] = (float)bi;
        out[1] = bv;
        pidx_out[0] = bi;
    }
}

// apply_temperature (:130-134)
__global__ void apply_temperature(float* logits, float inv_temp, uint32_t n) {
    const uint32_t i = GID();
    if (i < n) logits[i] = logits[i] * inv_temp;
}

// reduce_max_partial / final, softmax_exp_partial, reduce_sum_partial / final,
// softmax_normalize (:157-225)
__global__ void reduce_max_partial(float* pmax, const float* x, uint32_t n, uint32_t nparts) {
    const uint32_t p = GID();
    if (p >= nparts) return;
    float m = -INFINITY;
    for (uint32_t k = p; k < n; k += nparts) m = fmaxf(m, x[k]);
    pmax[p] = m;
}
__global__ void reduce_max_final(float* stats, const float* pmax, uint32_t nparts) {
    __shared__ float red[32];
    float m = -INFINITY;
    for (uint32_t p = threadIdx.x; p < nparts; p += blockDim.x) m = fmaxf(m, pmax[p]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
        m = warp_max(m);
        if (threadIdx.x == 0) stats[0] = m;
    }
}
__global__ void softmax_exp_partial(float* out, float* psum, const float* x, const float* stats, uint32_t n,
                                    uint32_t nparts) {
    const uint32_t p = GID();
    if (p >= nparts) return;
    const float m = stats[0];
    float s = 0.0f;
    for (uint32_t k = p; k < n; k += nparts) {
        const float e = expf(x[k] - m);
        out[k] = e;
        s += e;
    }
    psum[p] = s;
}
__global__ void reduce_sum_partial(float* out, const float* in, uint32_t n, uint32_t nparts) {
    const uint32_t p = GID();
    if (p >= nparts) return;
    float s = 0.0f;
    for (uint32_t k = p; k < n; k += nparts) s += in[k];
    out[p] = s;
}
__global__ void reduce_sum_final(float* stats, const float* psum, uint32_t nparts) {
    // fixed-order serial sum, as the reference: nparts is small
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (uint32_t p = 0; p < nparts; ++p) s += psum[p];
        stats[1] = s;
    }
}
__global__ void softmax_normalize(float* out, const float* stats, uint32_t n) {
    const uint32_t i = GID();
    if (i < n) out[i] = out[i] / stats[1];
}

// ---- top-k family (llm_sampling.cl:249-386) ---------------------------------
constexpr uint32_t TOPK_MAX = 64;

// topk_partial (:257-286): each strided chain keeps its k best (desc, ties -> lower index)
__global__ void topk_partial(float* cval, uint32_t* cidx, const float* x, uint32_t n, uint32_t nparts,
                             uint32_t k) {
    const uint32_t p = GID();
    if (p >= nparts) return;
    if (k > TOPK_MAX) k = TOPK_MAX;
    if (k == 0) return;
    float bv[TOPK_MAX];
    uint32_t bi[TOPK_MAX];
    for (uint32_t j = 0; j < k; ++j) { bv[j] = -INFINITY; bi[j] = 0xFFFFFFFFu; }
    for (uint32_t e = p; e < n; e += nparts) {
        const float v = x[e];
        if (!(v > bv[k - 1])) continue;
        uint32_t j = k - 1;
        while (j > 0 && v > bv[j - 1]) { bv[j] = bv[j - 1]; bi[j] = bi[j - 1]; --j; }
        bv[j] = v;
        bi[j] = e;
    }
    for (uint32_t j = 0; j < k; ++j) { cval[(size_t)p * k + j] = bv[j]; cidx[(size_t)p * k + j] = bi[j]; }
}

// topk4_partial (:318-347): best 4 per chain, kept in registers
__global__ void topk4_partial(float* cval, uint32_t* cidx, const float* x, uint32_t n, uint32_t nparts) {
    const uint32_t p = GID();
    if (p >= nparts) return;
    float v0 = -INFINITY, v1 = -INFINITY, v2 = -INFINITY, v3 = -INFINITY;
    uint32_t i0 = 0xFFFFFFFFu, i1 = i0, i2 = i0, i3 = i0;
    for (uint32_t e = p; e < n; e += nparts) {
        const float v = x[e];
        if (!(v > v3)) continue;
        if (v > v0) { v3 = v2; i3 = i2; v2 = v1; i2 = i1; v1 = v0; i1 = i0; v0 = v; i0 = e; }
        else if (v > v1) { v3 = v2; i3 = i2; v2 = v1; i2 = i1; v1 = v; i1 = e; }
        else if (v > v2) { v3 = v2; i3 = i2; v2 = v; i2 = e; }
        else { v3 = v; i3 = e; }
    }
    const size_t o = (size_t)p * 4;
    cval[o] = v0; cidx[o] = i0;
    cval[o + 1] = v1; cidx[o + 1] = i1;
    cval[o + 2] = v2; cidx[o + 2] = i2;
    cval[o + 3] = v3; cidx[o + 3] = i3;
}

// topk_rank_select (:349-369): rank each candidate; rank < k -> out[rank]
__global__ void topk_rank_select(float* oval, uint32_t* oidx, const float* cval, const uint32_t* cidx,
                                 uint32_t ncand, uint32_t k) {
    const uint32_t i = GID();
    if (i >= ncand) return;
    const float v = cval[i];
    const uint32_t d = cidx[i];
    if (d == 0xFFFFFFFFu) return;
    uint32_t rank = 0;
    for (uint32_t j = 0; j < ncand; ++j) {
        const float w = cval[j];
        const uint32_t e = cidx[j];
        if (e == 0xFFFFFFFFu) continue;
        if (w > v || (w == v && e < d)) ++rank;
    }
    if (rank < k) { oval[rank] = v; oidx[rank] = d; }
}

// topk_mask (:380-386)
__global__ void topk_mask(float* logits, const float* topk_val, uint32_t k, uint32_t n) {
    const uint32_t i = GID();
    if (i >= n) return;
    const float t = topk_val[k - 1];
    if (logits[i] < t) logits[i] = -INFINITY;
}

// topp_cutoff (:407-422): keep the shortest descending prefix reaching p
__global__ void topp_cutoff(float* w, uint32_t k, float p) {
    if (GID() != 0) return;
    float total = 0.0f;
    for (uint32_t j = 0; j < k; ++j) total += w[j];
    if (!(total > 0.0f)) return;
    float cum = 0.0f;
    for (uint32_t j = 0; j < k; ++j) {
        if (cum >= p * total) w[j] = 0.0f;
        else cum += w[j];
    }
}

// multinomial_sample (:432-453)
__global__ void multinomial_sample(float* out, uint32_t* idx_out, const float* w, const uint32_t* idx, uint32_t k,
                                   float u) {
    if (GID() != 0) return;
    float total = 0.0f;
    for (uint32_t j = 0; j < k; ++j) total += w[j];
    const float target = u * total;
    float cum = 0.0f, cw = 0.0f;
    uint32_t chosen = 0;
    for (uint32_t j = 0; j < k; ++j) {
        cum += w[j];
        if (w[j] > 0.0f) { chosen = idx[j]; cw = w[j]; }
        if (cum > target) break;
    }
    out[0] = (float)chosen;
    out[1] = cw;
    idx_out[0] = chosen;
}

// multinomial_strided (:469-494)
__global__ void multinomial_strided(float* out, uint32_t* idx_out, const float* w, const float* psum,
                                    const float* stats, uint32_t n, uint32_t nparts, float u) {
    if (GID() != 0) return;
    const float target = u * stats[1];
    float cum = 0.0f;
    uint32_t chain = nparts - 1;
    for (uint32_t p = 0; p < nparts; ++p) {
        const float s = psum[p];
        if (cum + s > target) { chain = p; break; }
        cum += s;
    }
    uint32_t chosen = chain;
    for (uint32_t k = chain; k < n; k += nparts) {
        chosen = k;
        cum += w[k];
        if (cum > target) break;
    }
    out[0] = (float)chosen;
    out[1] = w[chosen];
    idx_out[0] = chosen;
}

// ---- matvec layouts of the layout study (llm_matvec.cl:25-366, llm.cl:12-117) --
// fp32 scales [block][col]; the nibble of weight (k, j) sits at:
//   COL  word[(k*cols + j) / 8], nibble j % 8                 (llm.cl, mv_ref*)
//   KMN  word[j*(rows/8) + k/8], nibble k % 8                  (mv_kmn)
//   KM   word[((j/64)*(rows/8) + k/8)*64 + j%64], nibble k % 8  (mv_km)
//   KM4  uint4[((j/64)*(rows/32) + k/32)*64 + j%64], word (k/8)%4, nibble k % 8
//                                                    (mv_km4 and its variants)
// One warp per (output column, K split); lanes take 32-row blocks in turn, each
// block's (sum in*(nibble - 8)) * scale added to the lane's sum, then a warp sum.
XP_DEV uint32_t warp_gid() { return blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); }
enum MvLayout : int { MVL_COL = 0, MVL_KMN = 1, MVL_KM = 2, MVL_KM4 = 3 };
template <int L>
XP_DEV uint32_t mvl_nibble(const uint32_t* w, uint32_t k, uint32_t j, uint32_t rows, uint32_t cols) {
    if (L == MVL_COL) return (w[((size_t)k * cols + j) >> 3] >> ((j & 7u) * 4u)) & 15u;
    const uint32_t sh = (k & 7u) * 4u;
    if (L == MVL_KMN) return (w[(size_t)j * (rows >> 3) + (k >> 3)] >> sh) & 15u;
    if (L == MVL_KM) return (w[(((size_t)(j >> 6) * (rows >> 3) + (k >> 3)) << 6) + (j & 63u)] >> sh) & 15u;
    return (w[((((size_t)(j >> 6) * (rows >> 5) + (k >> 5)) << 6) + (j & 63u)) * 4 + ((k >> 3) & 3u)] >> sh) & 15u;
}
template <int L>
__global__ void mv_layout(float* out, const float* in, const uint32_t* wq, const float* scale, uint32_t rows,
                          uint32_t cols, uint32_t split) {
    const uint32_t w = warp_gid(), lane = threadIdx.x & 31;
    if (w >= cols * split) return;
    const uint32_t j = w % cols, p = w / cols, nblk = rows / 32;
    const uint32_t per = (nblk + split - 1) / split, b0 = p * per, b1 = min(b0 + per, nblk);
    float acc = 0.0f;
    for (uint32_t b = b0 + lane; b < b1; b += 32) {
        float part = 0.0f;
        for (uint32_t t = 0; t < 32; ++t) {
            const uint32_t k = b * 32 + t;
            part += in[k] * ((float)mvl_nibble<L>(wq, k, j, rows, cols) - 8.0f);
        }
        acc += part * scale[(size_t)b * cols + j];
    }
    acc = warp_sum(acc);
    if (lane == 0) out[(size_t)p * cols + j] = acc;
}

// matvec_f32 (llm.cl:12-19): out[j] = sum_k in[k] w[k*cols + j]; thread per
// column (consecutive threads read consecutive w)
__global__ void matvec_f32(float* out, const float* in, const float* w, uint32_t rows, uint32_t cols) {
    const uint32_t j = GID();
    if (j >= cols) return;
    float acc = 0.0f;
    for (uint32_t k = 0; k < rows; ++k) acc += in[k] * w[(size_t)k * cols + j];
    out[j] = acc;
}
// stream_read (llm.cl:60-66): a load probe over 65536 strided lanes; out[0]
// = lane 0's sum (src[0] + src[65536] + ...), as the reference writes it. The
// other lanes store only on a sum they cannot reach, so their loads stay live.
__global__ void stream_read(float* out, const uint32_t* src, uint32_t n) {
    const uint32_t i = GID();
    if (i >= 65536u) return;
    uint32_t acc = 0;
    for (uint32_t k = i; k < n; k += 65536u) acc += __ldg(src + k);
    if (i == 0) out[0] = (float)acc;
    else if (acc == 0xDEADBEEFu && n == 0u) out[1] = 0.0f;
}

// ---- prefill shapes (llm_sampling.cl:495-736) -------------------------------
// Row-major [row][col] everywhere, as in the reference. Row reductions run one
// warp per row (the reference walks a row with one thread); elementwise work is
// one thread per element.

// softmax_rows_stats (:527-546): stats[2r] = row max, stats[2r + 1] = row sum
// of exp(x - max); a fully masked row gives (0, 1).
__global__ void softmax_rows_stats(float* stats, const float* x, uint32_t n_rows, uint32_t n_cols) {
    const uint32_t r = warp_gid(), lane = threadIdx.x & 31;
    if (r >= n_rows) return;
    const float* row = x + (size_t)r * n_cols;
    float m = -INFINITY;
    for (uint32_t j = lane; j < n_cols; j += 32) m = fmaxf(m, row[j]);
    m = warp_max(m);
    if (!isfinite(m)) {
        if (lane == 0) { stats[2 * r] = 0.0f; stats[2 * r + 1] = 1.0f; }
        return;
    }
    float s = 0.0f;
    for (uint32_t j = lane; j < n_cols; j += 32) s += expf(row[j] - m);
    s = warp_sum(s);
    if (lane == 0) { stats[2 * r] = m; stats[2 * r + 1] = s; }
}

// softmax_rows_apply (:549-556)
__global__ void softmax_rows_apply(float* x, const float* stats, uint32_t n_rows, uint32_t n_cols) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_rows * n_cols) return;
    const uint32_t r = (uint32_t)(i / n_cols);
    x[i] = expf(x[i] - stats[2 * r]) / stats[2 * r + 1];
}

// attention_scores_prefill (:574-602): scores[(h*n_query + qi)*seq_len + t],
// causal (t <= q_offset + qi) and sliding-window (t > qpos - window) masks
// folded in as -inf. One warp per score; lanes split head_dim.
__global__ void attention_scores_prefill(float* scores, const float* q, const float* kcache, uint32_t n_heads,
                                         uint32_t kv_heads, uint32_t head_dim, uint32_t n_query,
                                         uint32_t seq_len, uint32_t q_offset, uint32_t window, float scale) {
    const uint64_t i = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31;
    if (i >= (uint64_t)n_heads * n_query * seq_len) return;
    const uint32_t t = (uint32_t)(i % seq_len);
    const uint32_t hq = (uint32_t)(i / seq_len);
    const uint32_t qi = hq % n_query, h = hq / n_query;
    const uint32_t qpos = q_offset + qi;
    if (t > qpos || (window != 0u && t + window <= qpos)) {
        if (lane == 0) scores[i] = -INFINITY;
        return;
    }
    const uint32_t kvh = h / (n_heads / kv_heads);
    const float* qr = q + (size_t)hq * head_dim;
    const float* kr = kcache + ((size_t)t * kv_heads + kvh) * head_dim;
    float acc = 0.0f;
    for (uint32_t d = lane; d < head_dim; d += 32) acc += qr[d] * kr[d];
    acc = warp_sum(acc);
    if (lane == 0) scores[i] = acc * scale;
}

// attention_apply_prefill (:605-630): out[(h*n_query + qi)*head_dim + d] =
// sum_t probs[(h*n_query + qi)*seq_len + t] v[t][kvh][d]; one thread per output
// (a warp shares one probability row and reads 32 consecutive v values).
__global__ void attention_apply_prefill(float* out, const float* probs, const float* vcache, uint32_t n_heads,
                                        uint32_t kv_heads, uint32_t head_dim, uint32_t n_query,
                                        uint32_t seq_len) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_heads * n_query * head_dim) return;
    const uint32_t d = (uint32_t)(i % head_dim);
    const uint32_t hq = (uint32_t)(i / head_dim);
    const uint32_t h = hq / n_query;
    const uint32_t kvh = h / (n_heads / kv_heads);
    const float* p = probs + (size_t)hq * seq_len;
    const size_t vstride = (size_t)kv_heads * head_dim;
    const float* v = vcache + (size_t)kvh * head_dim + d;
    float acc = 0.0f;
    for (uint32_t t = 0; t < seq_len; ++t) acc += p[t] * v[t * vstride];
    out[i] = acc;
}

// rmsnorm_rows_sumsq (:634-642): one warp per row
__global__ void rmsnorm_rows_sumsq(float* rowss, const float* in, uint32_t n_rows, uint32_t n) {
    const uint32_t r = warp_gid(), lane = threadIdx.x & 31;
    if (r >= n_rows) return;
    const float* row = in + (size_t)r * n;
    float ss = 0.0f;
    for (uint32_t j = lane; j < n; j += 32) ss += row[j] * row[j];
    ss = warp_sum(ss);
    if (lane == 0) rowss[r] = ss;
}

// rmsnorm_rows_apply_gemma (:645-656): Gemma's (1 + w), w shared across rows
__global__ void rmsnorm_rows_apply_gemma(float* out, const float* in, const float* w, const float* rowss,
                                         uint32_t n_rows, uint32_t n, float eps) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_rows * n) return;
    const uint32_t r = (uint32_t)(i / n), j = (uint32_t)(i - (uint64_t)r * n);
    const float scale = rsqrtf(rowss[r] / (float)n + eps);
    out[i] = in[i] * scale * (1.0f + w[j]);
}

// rmsnorm_heads_rows_gemma (:659-675): QK-norm over [token][head][head_dim];
// one warp per (token, head) writes its whole head.
__global__ void rmsnorm_heads_rows_gemma(float* out, const float* in, const float* w, uint32_t n_tokens,
                                         uint32_t n_heads, uint32_t head_dim, float eps) {
    const uint32_t th = warp_gid(), lane = threadIdx.x & 31;
    if (th >= n_tokens * n_heads) return;
    const float* x = in + (size_t)th * head_dim;
    float ss = 0.0f;
    for (uint32_t k = lane; k < head_dim; k += 32) ss += x[k] * x[k];
    ss = warp_sum(ss);
    const float scale = rsqrtf(ss / (float)head_dim + eps);
    for (uint32_t d = lane; d < head_dim; d += 32) out[(size_t)th * head_dim + d] = x[d] * scale * (1.0f + w[d]);
}

// rope_prefill (:687-711): rotate-half RoPE over [token][head][head_dim], the
// position of token ti being pos0 + ti; one thread per (token, head, pair),
// the same angle and expressions as the decode `rope` at that position, so a
// position rotates bit-identically through either entry point.
__global__ void rope_prefill(float* x, uint32_t n_tokens, uint32_t n_heads, uint32_t head_dim, uint32_t pos0,
                             float theta) {
    const uint32_t half = head_dim >> 1;
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_tokens * n_heads * half) return;
    const uint32_t d = (uint32_t)(i % half);
    const uint32_t th = (uint32_t)(i / half);
    const uint32_t ti = th / n_heads;
    const size_t base = (size_t)th * head_dim + d;
    float c, s;
    rope_cs(d, head_dim, pos0 + ti, theta, c, s);
    const float lo = x[base], hi = x[base + half];
    x[base] = lo * c - hi * s;
    x[base + half] = lo * s + hi * c;
}

// kv_append_rows (:714-722): n_tokens rows of `row` floats at row pos0
__global__ void kv_append_rows(float* cache, const float* src, uint32_t n_tokens, uint32_t row, uint32_t pos0) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_tokens * row) return;
    cache[(size_t)pos0 * row + i] = src[i];
}

// embed_lookup_rows (:728-736): out[ti][j] = table[tokens[ti]][j]
__global__ void embed_lookup_rows(float* out, const float* table, const uint32_t* tokens, uint32_t n_tokens,
                                  uint32_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_tokens * n) return;
    const uint32_t ti = (uint32_t)(i / n), j = (uint32_t)(i - (uint64_t)ti * n);
    out[i] = table[(size_t)tokens[ti] * n + j];
}

#undef GID
}  // namespace ops
}  // namespace xp
