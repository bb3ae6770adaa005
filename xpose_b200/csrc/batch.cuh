// Batched decode: B independent sequences advance one position per step over
// the same weights. The int4 matvecs run on the tensor cores (bmm.cuh); the
// per-sequence work between them runs here, one CTA per sequence. Arithmetic
// follows the reference's per-token ops (examples/llm/decode.cpp:1634-1780,
// kernels/llm_transformer.cl) exactly as the batch-1 path does: gemma RMSNorm
// x * rsqrt(mean(x^2) + eps) * (1 + w), QK-norm per head, rotate-half RoPE with
// theta^(-2d/256) rounded once from double, fp16 KV cache, max-subtracted
// softmax, tanh-approximate GeGLU.
#pragma once
#include <cooperative_groups.h>
#include "attention.cuh"
#include "bmm.cuh"
#include "common.cuh"

namespace xp {

constexpr int BK_THREADS = 512;

// Matvec results arrive as fp32 partial sums, one per K range of the
// tensor-core launch ([ks][B][cols], plain stores); the consuming kernel adds
// them in K-range order, so the result is deterministic. Loads are issued in
// groups (all of a group in flight together) before any add.
struct BkSums {
    const float* p;
    uint32_t ks;       // K ranges (partials)
    uint32_t stride;   // floats between consecutive partials (B x cols)
};
// v[j] = element idx[j] (< 0: none, v = 0) summed over the partials
template <int J, int KU>
XP_DEV void bk_gather(const BkSums& s, const long long (&idx)[J], float (&v)[J]) {
#pragma unroll
    for (int j = 0; j < J; ++j) v[j] = 0.0f;
#pragma unroll 1
    for (uint32_t k0 = 0; k0 < s.ks; k0 += KU) {
        float t[KU][J];
#pragma unroll
        for (int k = 0; k < KU; ++k)
#pragma unroll
            for (int j = 0; j < J; ++j)
                t[k][j] = (k0 + k < s.ks && idx[j] >= 0) ? __ldcg(s.p + (size_t)(k0 + k) * s.stride + idx[j]) : 0.0f;
#pragma unroll
        for (int k = 0; k < KU; ++k)
#pragma unroll
            for (int j = 0; j < J; ++j) v[j] += t[k][j];
    }
}

// Every kernel of a batched step may be launched programmatically (its
// launch overlapping the previous kernel's tail): each one lets its
// dependents launch at once and reads nothing the previous kernels write
// before griddepcontrol.wait.

// x[b] = embed[token[b]] * scale
__global__ void bk_embed_kernel(const uint32_t* tokens, const float* embed, float scale, float* x, uint32_t H) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t b = blockIdx.x;
    const float* row = embed + (size_t)tokens[b] * H;
    for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) x[(size_t)b * H + i] = row[i] * scale;
}

// Where a kernel leaves a matvec input: the tensor-core operand of its
// sequence (bmm_put_seq), padded to Npad sequences.
struct BkOperand {
    float* xs;
    unsigned char* xb;
    uint32_t Npad;
};

// mode 0: xn = rmsnorm_gemma(x, w_pre)
// mode 1: x += rmsnorm_gemma(y, w_post); xn = rmsnorm_gemma(x, w_pre)  (y: partial sums)
// xn goes out as the next matvec's operand. One block reduction serves both
// norms: with u = y (1 + w_post) and s1 = rsqrt(sum y^2 / H + eps), the
// residual is r = x + s1 u and sum r^2 = sum x^2 + 2 s1 sum x u + s1^2 sum u^2;
// x is loaded beside the partial sums.
__global__ void __launch_bounds__(BK_THREADS) bk_resid_norm_kernel(float* x, BkSums y, const float* w_post,
                                                                 const float* w_pre, BkOperand xn, uint32_t H, float eps,
                                                                 int mode) {
    __shared__ float4 red4[BK_THREADS / 32];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t b = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* xb = x + (size_t)b * H;
    constexpr int J = 4;  // H <= 2048
    float xv[J], uv[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const uint32_t i = threadIdx.x + j * BK_THREADS;
        xv[j] = i < H ? xb[i] : 0.0f;
    }
    float4 s4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // y^2, x^2, x u, u^2
    if (mode == 1) {
        float yv[J];
        long long idx[J];
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const uint32_t i = threadIdx.x + j * BK_THREADS;
            idx[j] = i < H ? (long long)b * H + i : -1;
        }
        bk_gather<J, 8>(y, idx, yv);
#pragma unroll
        for (int j = 0; j < J; ++j) {
            const uint32_t i = threadIdx.x + j * BK_THREADS;
            uv[j] = i < H ? yv[j] * (1.0f + w_post[i]) : 0.0f;
            s4.x += yv[j] * yv[j];
            s4.z += xv[j] * uv[j];
            s4.w += uv[j] * uv[j];
        }
    } else {
#pragma unroll
        for (int j = 0; j < J; ++j) uv[j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < J; ++j) s4.y += xv[j] * xv[j];
    s4.x = warp_sum(s4.x);
    s4.y = warp_sum(s4.y);
    s4.z = warp_sum(s4.z);
    s4.w = warp_sum(s4.w);
    if (lane == 0) red4[warp] = s4;
    __syncthreads();
    float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < BK_THREADS / 32; ++w) {
        const float4 q = red4[w];
        t.x += q.x;
        t.y += q.y;
        t.z += q.z;
        t.w += q.w;
    }
    const float s1 = mode == 1 ? rsqrtf(t.x / (float)H + eps) : 0.0f;
    const float sc2 = rsqrtf((t.y + 2.0f * s1 * t.z + s1 * s1 * t.w) / (float)H + eps);
    float o[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const uint32_t i = threadIdx.x + j * BK_THREADS;
        const float r = xv[j] + s1 * uv[j];
        if (mode == 1 && i < H) xb[i] = r;
        o[j] = i < H ? r * sc2 * (1.0f + w_pre[i]) : 0.0f;
    }
    bmm_put_seq(o, H, b, xn.Npad, xn.xs, xn.xb);
}

__global__ void bk_pos_inc_kernel(uint32_t* pos, uint32_t B) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x < B) pos[threadIdx.x] += 1;
}

// hb = gelu(g) * u, left as the down-proj operand (F <= BK_THREADS * BK_GJ).
// One cluster of BK_GC CTAs per sequence: CTA rank r takes elements
// t + (r * BK_GJC + j) * BK_THREADS, and the operand's power-of-two scale
// comes from the exact maximum of |hb| over the cluster (each CTA's block
// maximum read from the others' shared memory), so every stored value is the
// same as one CTA per sequence would store, on a quarter of the latency chain.
constexpr int BK_GJ = 16;
constexpr int BK_GC = 4;
constexpr int BK_GJC = BK_GJ / BK_GC;
static_assert(BK_GJ % BK_GC == 0, "elements per thread split over the cluster");
__global__ void __launch_bounds__(BK_THREADS) bk_geglu_kernel(BkSums g, BkSums u, BkOperand hb, uint32_t F) {
    namespace cg = cooperative_groups;
    __shared__ float wmax[BK_THREADS / 32];
    __shared__ float cmax;
    cg::cluster_group cl = cg::this_cluster();
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t b = blockIdx.x / BK_GC, r = cl.block_rank();
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    long long idx[BK_GJC];
#pragma unroll
    for (int j = 0; j < BK_GJC; ++j) {
        const uint32_t i = tid + (r * BK_GJC + j) * BK_THREADS;
        idx[j] = i < F ? (long long)b * F + i : -1;
    }
    float gv[BK_GJC], uv[BK_GJC];
    bk_gather<BK_GJC, 2>(g, idx, gv);
    bk_gather<BK_GJC, 2>(u, idx, uv);
    float h[BK_GJC];
    float am = 0.0f;
#pragma unroll
    for (int j = 0; j < BK_GJC; ++j) {
        h[j] = idx[j] >= 0 ? gelu_tanh_ref(gv[j]) * uv[j] : 0.0f;
        am = fmaxf(am, fabsf(h[j]));
    }
    am = warp_max(am);
    if (lane == 0) wmax[warp] = am;
    __syncthreads();
    if (warp == 0) {
        am = warp_max(lane < BK_THREADS / 32 ? wmax[lane] : 0.0f);
        if (lane == 0) cmax = am;
    }
    cl.sync();  // every CTA's maximum is in its shared memory
    float m = 0.0f;
#pragma unroll
    for (int q = 0; q < BK_GC; ++q) m = fmaxf(m, *cl.map_shared_rank(&cmax, q));
    cl.sync();  // no CTA leaves while a peer may still read its maximum
    const int eb = (int)((__float_as_uint(m) >> 23) & 0xFFu);
    const float sc = eb > 0 && eb < 253 ? __uint_as_float((uint32_t)(eb + 1) << 23) : 1.0f;
    if (r == 0 && tid == 0) hb.xs[b] = sc;
#pragma unroll
    for (int j = 0; j < BK_GJC; ++j) {
        const uint32_t i = tid + (r * BK_GJC + j) * BK_THREADS;
        if (i < F) bmm_xput(hb.xb, hb.Npad, b, i, h[j] / sc);  // exact: power of two
    }
}

// One CTA per sequence: QK-norm + RoPE of the raw q (4 heads) and k, fp16 KV
// append at pos[b], then 4-head attention over [kv_start, pos] of this
// sequence's cache (window 0 = global). Dynamic smem: 4 * span_max floats.
struct BkAttnArgs {
    BkSums q;              // [B][1024] raw q, partial sums
    BkSums k;              // [B][256]
    BkSums v;              // [B][256]
    const float* qn;       // [256] q_norm weights
    const float* kn;       // [256] k_norm weights
    __half* kc;            // [B][max_seq][256]
    __half* vc;
    const uint32_t* pos;   // [B]
    BkOperand att;         // [B][1024] as the o-proj operand
    uint32_t max_seq, window;
    float theta, eps, scale;
    float inv_freq[128];   // RoPE theta^(-2d/256), from rope_table_host
    // Batched decode: mode 0, sequence b's cache at kc + b * seq_stride.
    // Chunked prefill (rows = consecutive positions of one sequence, one
    // shared cache, seq_stride 0): mode 1 appends every row's k and v (the
    // q|k|v sums stay), then mode 2 attends with the rows' own k and v read
    // back from the cache and clears the sums.
    size_t seq_stride;
    int mode;
    // CTAs per sequence (1, or 2 as a cluster): with 2, each CTA attends to
    // half of the keys and the cluster's rank 0 merges the two partials
    // (max, sum, unnormalised P.V) from its peer's shared memory
    uint32_t split;
};
constexpr uint32_t BK_ATT_SPLIT = 2;  // CTAs (one cluster) per attending sequence
__global__ void __launch_bounds__(BK_THREADS) bk_attn_kernel(const __grid_constant__ BkAttnArgs a) {
    extern __shared__ __align__(16) float bsm_f[];
    __shared__ float qs[4 * 256];
    __shared__ float red[4 * 4 * 256];  // P.V partials [4 groups][4 heads][256]
    __shared__ __align__(16) __half knew[256], vnew[256];
    __shared__ float cs[256];           // cos | sin for this position
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t split = a.split, b = blockIdx.x / split, rk = blockIdx.x % split;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t pos = a.pos[b];
    const uint32_t seq = pos + 1;
    const uint32_t kv_start = (a.window == 0 || seq <= a.window) ? 0 : seq - a.window;
    const uint32_t span = seq - kv_start;
    float* sc = bsm_f;  // [4][max_span]
    const uint32_t ms = a.window ? min(a.window, a.max_seq) : a.max_seq;
    if (tid < 128) {
        float s, c;
        rope_sincos((float)pos * a.inv_freq[tid], &s, &c);
        cs[tid] = c;
        cs[128 + tid] = s;
    }
    // this sequence's q|k|v: every thread gathers three of the 1536 sums (all
    // partial loads in flight together) into shared memory (the P.V partials'
    // buffer, free until the scores are done)
    float* qkv_s = red;
    {
        const bool want_q = a.mode != 1, want_kv = a.mode != 2;
        long long idx[3];
        const BkSums* src[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const uint32_t i = tid + r * BK_THREADS;  // 0..1023 q, 1024..1279 k, 1280..1535 v
            const bool isq = i < 1024;
            src[r] = isq ? &a.q : (i < 1280 ? &a.k : &a.v);
            idx[r] = (isq ? want_q : want_kv) ? (isq ? (long long)b * 1024 + i : (long long)b * 256 + ((i - 1024) & 255)) : -1;
        }
        // q, k and v come from one launch: the same K ranges, their own strides
        float v3[3] = {0.0f, 0.0f, 0.0f};
        const uint32_t ks = a.q.ks;
#pragma unroll 1
        for (uint32_t k0 = 0; k0 < ks; k0 += 16) {
            float t[3][16];
#pragma unroll
            for (int r = 0; r < 3; ++r)
#pragma unroll
                for (int k = 0; k < 16; ++k)
                    t[r][k] = (k0 + k < ks && idx[r] >= 0) ? __ldcg(src[r]->p + (size_t)(k0 + k) * src[r]->stride + idx[r]) : 0.0f;
#pragma unroll
            for (int r = 0; r < 3; ++r)
#pragma unroll
                for (int k = 0; k < 16; ++k) v3[r] += t[r][k];
        }
#pragma unroll
        for (int r = 0; r < 3; ++r) qkv_s[tid + r * BK_THREADS] = v3[r];
    }
    __syncthreads();
    __half* kcb = a.kc + (size_t)b * a.seq_stride;
    __half* vcb = a.vc + (size_t)b * a.seq_stride;
    const bool want_q = a.mode != 1, want_kv = a.mode != 2;
    if (warp < 6 && (warp < 4 ? want_q : want_kv)) {
        // warps 0-3: q heads, 4: k, 5: v; lane holds dims 4 lane..+3 and 128 + 4 lane..+3
        const float* src = qkv_s + (warp < 4 ? warp * 256 : (warp == 4 ? 1024 : 1280));
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = src[i < 4 ? 4 * lane + i : 128 + 4 * lane + (i - 4)];
        if (warp < 5) {
            const float* w = warp < 4 ? a.qn : a.kn;
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
            ss = warp_sum(ss);
            const float s = rsqrtf(ss / 256.0f + a.eps);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t d = 4 * lane + i;
                const float lo = v[i] * s * (1.0f + w[d]);
                const float hi = v[4 + i] * s * (1.0f + w[128 + d]);
                v[i] = lo * cs[d] - hi * cs[128 + d];
                v[4 + i] = lo * cs[128 + d] + hi * cs[d];
            }
        }
        if (warp < 4) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                qs[warp * 256 + 4 * lane + i] = v[i] * a.scale;
                qs[warp * 256 + 128 + 4 * lane + i] = v[4 + i] * a.scale;
            }
        } else {
            __half* dst = warp == 4 ? knew : vnew;
            __half* cache = warp == 4 ? kcb : vcb;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __half lo = __float2half_rn(v[i]), hi = __float2half_rn(v[4 + i]);
                dst[4 * lane + i] = lo;
                dst[128 + 4 * lane + i] = hi;
                if (rk == 0) {
                    cache[(size_t)pos * 256 + 4 * lane + i] = lo;
                    cache[(size_t)pos * 256 + 128 + 4 * lane + i] = hi;
                }
            }
        }
    }
    if (a.mode == 1) return;
    const uint32_t pnew = a.mode == 0 ? pos : 0xFFFFFFFFu;  // mode 2 reads row pos from the cache
    __syncthreads();
    // this CTA's keys: [k_lo, k_hi) of the window
    const uint32_t half = (span + split - 1) / split;
    const uint32_t k_lo = min(span, rk * half), k_hi = min(span, k_lo + half);
    // scores: one key per warp, lane holds 8 dims of every head; four keys'
    // loads in flight per warp
#pragma unroll 4
    for (uint32_t jj = k_lo + warp; jj < k_hi; jj += BK_THREADS / 32) {
        const uint32_t j = kv_start + jj;
        const uint4 raw = j == pnew ? *reinterpret_cast<const uint4*>(knew + 8 * lane)
                                   : *reinterpret_cast<const uint4*>(kcb + (size_t)j * 256 + 8 * lane);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
        float kf[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h2[i]);
            kf[2 * i] = f.x;
            kf[2 * i + 1] = f.y;
        }
        float s4[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = fmaf(qs[h * 256 + 8 * lane + i], kf[i], acc);
            s4[h] = acc;
        }
        const float tot = reduce4(s4[0], s4[1], s4[2], s4[3]);
        if ((lane & 7) == 0) sc[(((lane >> 4) & 1) * 2 + ((lane >> 3) & 1)) * ms + jj] = tot;
    }
    __syncthreads();
    __shared__ float sums[4], mh[4];
    if (warp < 4) {
        float m = -INFINITY;
        for (uint32_t jj = k_lo + lane; jj < k_hi; jj += 32) m = fmaxf(m, sc[warp * ms + jj]);
        m = warp_max(m);
        float sum = 0.0f;
        for (uint32_t jj = k_lo + lane; jj < k_hi; jj += 32) {
            const float p = expf(sc[warp * ms + jj] - m);
            sc[warp * ms + jj] = p;
            sum += p;
        }
        sum = warp_sum(sum);
        if (lane == 0) {
            sums[warp] = sum;
            mh[warp] = m;
        }
    }
    __syncthreads();
    {
        const uint32_t dp = tid & 127, qr = tid >> 7;
        float acc[4][2] = {};
#pragma unroll 8
        for (uint32_t jj = k_lo + qr; jj < k_hi; jj += 4) {
            const uint32_t j = kv_start + jj;
            const __half2 hv = j == pnew ? reinterpret_cast<const __half2*>(vnew)[dp]
                                        : reinterpret_cast<const __half2*>(vcb + (size_t)j * 256)[dp];
            const float2 vf = __half22float2(hv);
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float p = sc[h * ms + jj];
                acc[h][0] = fmaf(p, vf.x, acc[h][0]);
                acc[h][1] = fmaf(p, vf.y, acc[h][1]);
            }
        }
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            red[(qr * 4 + h) * 256 + 2 * dp] = acc[h][0];
            red[(qr * 4 + h) * 256 + 2 * dp + 1] = acc[h][1];
        }
    }
    __syncthreads();
    float o[1024 / BK_THREADS];
#pragma unroll
    for (int j = 0; j < 1024 / BK_THREADS; ++j) {
        const uint32_t i = tid + j * BK_THREADS;
        o[j] = red[i] + red[1024 + i] + red[2048 + i] + red[3072 + i];
    }
    if (split == 1) {
#pragma unroll
        for (int j = 0; j < 1024 / BK_THREADS; ++j) o[j] /= sums[(tid + j * BK_THREADS) >> 8];
    } else {
        // flash merge of the two halves: weights e^(m_r - M) per head (a half
        // with no keys has m = -inf and weight 0)
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        float* part = qs;  // the scaled q is no longer read: this CTA's unnormalised P.V
#pragma unroll
        for (int j = 0; j < 1024 / BK_THREADS; ++j) part[tid + j * BK_THREADS] = o[j];
        cl.sync();
        if (rk == 0) {
            const float* ppart = cl.map_shared_rank(part, 1);
            const float* psums = cl.map_shared_rank(sums, 1);
            const float* pmh = cl.map_shared_rank(mh, 1);
#pragma unroll
            for (int j = 0; j < 1024 / BK_THREADS; ++j) {
                const uint32_t i = tid + j * BK_THREADS, h = i >> 8;
                const float m0 = mh[h], m1 = pmh[h], M = fmaxf(m0, m1);
                const float w0 = m0 == -INFINITY ? 0.0f : expf(m0 - M);
                const float w1 = m1 == -INFINITY ? 0.0f : expf(m1 - M);
                o[j] = (o[j] * w0 + ppart[i] * w1) / (sums[h] * w0 + psums[h] * w1);
            }
        }
        cl.sync();  // the peer's shared memory stays until rank 0 has read it
        if (rk != 0) return;
    }
    bmm_put_seq(o, 1024, b, a.att.Npad, a.att.xs, a.att.xb);
}

}  // namespace xp
