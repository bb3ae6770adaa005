// Fused single-query GQA attention for one decode position (sm_100a).
//
// Replaces the reference's per-layer chain rmsnorm_heads_gemma(q), (k) -> rope
// (q), (k) -> kv_append(k), (v) -> attention_scores(_mq4) -> softmax_rows(_*) ->
// attention_apply(_mq4/_reduce) (examples/llm/decode.cpp:1676-1731) with one
// split-K flash-decode kernel:
//   * every CTA applies QK-norm (llm_transformer.cl:122-134) and rotate-half
//     RoPE (:158-179) to q and k itself (1280 values, cheaper than a launch);
//   * CTA 0 appends k and v to the fp16 cache at `pos` (read from device
//     memory, so one captured graph serves every position);
//   * the attended window [kv_start, pos] (sliding-window suffix on local
//     layers, decode.hpp:327-352) is cut into `gridDim.x` contiguous chunks;
//     each CTA computes scores, an online-softmax partial (max, sum) and the
//     unnormalised P.V for its chunk;
//   * the last CTA to finish (atomic ticket) combines the partials in a fixed
//     order and writes the attention output and its matvec limbs.
// Shape: n_heads = NH query heads sharing one kv head, head_dim = 256.
#pragma once
#include "common.cuh"
#include "xq.cuh"

namespace xp {

constexpr int ATT_THREADS = 256;
constexpr int ATT_HD = 256;

struct AttnArgs {
    const float* q_raw;    // [NH][256]
    const float* k_raw;    // [256]
    const float* v_raw;    // [256]
    const float* q_norm;   // [256] (Gemma 1+w)
    const float* k_norm;   // [256]
    __half* kcache;        // [max_seq][256]
    __half* vcache;
    const uint32_t* pos;   // device-resident position
    uint32_t window;       // 0 = global layer
    float theta, eps, scale;
    uint32_t chunk_max;    // smem capacity in positions per CTA
    float* part;           // [grid][NH][256]
    float* pstat;          // [grid][NH][2] (max, sum)
    uint32_t* ticket;      // zero between launches
    float* att;            // [NH][256]
    XBlk* att_xq;          // [NH*256/32]
    uint32_t* err;         // error word (chunk overflow)
};

// RoPE inverse frequency theta^(-2d/hd), rounded once from double so host and
// device agree bit for bit.
XP_DEV float rope_inv_freq(uint32_t d, uint32_t head_dim, float theta) {
    const float l2 = (float)log2((double)theta);
    const float frac = (float)(2u * d) / (float)head_dim;
    const float e = -l2 * frac;
    return (float)exp2((double)e);
}

// Warp-level: normalise one 256-wide head held as 8 values per lane (lane
// owns dims 4*lane..4*lane+3 and 128+4*lane..+3), then rotate-half.
XP_DEV void qk_post(float v[8], const float* w, float eps, uint32_t pos, float theta) {
    const int lane = threadIdx.x & 31;
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
    ss = warp_sum(ss);
    const float sc = rsqrtf(ss / 256.0f + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t d = 4 * lane + i;
        v[i] = v[i] * sc * (1.0f + w[d]);
        v[4 + i] = v[4 + i] * sc * (1.0f + w[128 + d]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t d = 4 * lane + i;
        const float inv = rope_inv_freq(d, 256, theta);
        const float ang = (float)pos * inv;
        float s, c;
        sincosf(ang, &s, &c);
        const float lo = v[i], hi = v[4 + i];
        v[i] = lo * c - hi * s;
        v[4 + i] = lo * s + hi * c;
    }
}

// Sum four per-lane values across the warp with 6 shuffles; afterwards lane L
// holds the total of head ((L >> 4) & 1) * 2 + ((L >> 3) & 1).
XP_DEV float reduce4(float v0, float v1, float v2, float v3) {
    const int lane = threadIdx.x & 31;
    const bool up = lane & 16;
    float k0 = up ? v2 : v0, k1 = up ? v3 : v1;
    const float t0 = up ? v0 : v2, t1 = up ? v1 : v3;
    k0 += __shfl_xor_sync(0xffffffffu, t0, 16);
    k1 += __shfl_xor_sync(0xffffffffu, t1, 16);
    const bool b8 = lane & 8;
    float kk = b8 ? k1 : k0;
    const float t = b8 ? k0 : k1;
    kk += __shfl_xor_sync(0xffffffffu, t, 8);
    kk += __shfl_xor_sync(0xffffffffu, kk, 4);
    kk += __shfl_xor_sync(0xffffffffu, kk, 2);
    kk += __shfl_xor_sync(0xffffffffu, kk, 1);
    return kk;
}

template <int NH>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const AttnArgs a) {
    static_assert(NH == 4, "the reduce4 score path is written for 4 query heads");
    extern __shared__ __align__(16) unsigned char smem[];
    float* qs = reinterpret_cast<float*>(smem);          // [NH][256], pre-scaled
    __half* kn = reinterpret_cast<__half*>(qs + NH * 256);  // [256] new k (fp16)
    __half* vn = kn + 256;                                // [256] new v (fp16)
    float* sc = reinterpret_cast<float*>(vn + 256);       // [NH][chunk_max] scores / probs
    float* accs = sc + NH * a.chunk_max;                  // [2][NH][256] P.V halves
    float* stat = accs + 2 * NH * 256;                    // [NH][2]
    __shared__ uint32_t s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_launch_dependents();
    pdl_wait();

    const uint32_t pos = *a.pos;
    const uint32_t seq = pos + 1;
    const uint32_t kv_start = (a.window == 0 || seq <= a.window) ? 0 : seq - a.window;
    const uint32_t span = seq - kv_start;
    const uint32_t nblk = gridDim.x;
    uint32_t chunk = (span + nblk - 1) / nblk;
    chunk = (chunk + 7) & ~7u;
    if (chunk > a.chunk_max) {  // host sized the grid wrong: flag and produce zeros
        if (tid == 0 && a.err) atomicOr(a.err, 1u);
        chunk = a.chunk_max;
    }
    const uint32_t j0 = kv_start + min(blockIdx.x * chunk, span);
    const uint32_t j1 = kv_start + min((blockIdx.x + 1) * chunk, span);
    const uint32_t n = j1 - j0;

    // ---- q, k, v post-processing -------------------------------------------------
    if (warp < NH || warp == NH || warp == NH + 1) {
        const float* src = warp < NH ? a.q_raw + warp * 256 : (warp == NH ? a.k_raw : a.v_raw);
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[i] = src[4 * lane + i];
            v[4 + i] = src[128 + 4 * lane + i];
        }
        if (warp < NH) {
            qk_post(v, a.q_norm, a.eps, pos, a.theta);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                qs[warp * 256 + 4 * lane + i] = v[i] * a.scale;
                qs[warp * 256 + 128 + 4 * lane + i] = v[4 + i] * a.scale;
            }
        } else {
            if (warp == NH) qk_post(v, a.k_norm, a.eps, pos, a.theta);
            __half* dst = warp == NH ? kn : vn;
            __half* cache = warp == NH ? a.kcache : a.vcache;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __half lo = __float2half_rn(v[i]), hi = __float2half_rn(v[4 + i]);
                dst[4 * lane + i] = lo;
                dst[128 + 4 * lane + i] = hi;
                if (blockIdx.x == 0) {
                    cache[(size_t)pos * 256 + 4 * lane + i] = lo;
                    cache[(size_t)pos * 256 + 128 + 4 * lane + i] = hi;
                }
            }
        }
    }
    __syncthreads();

    // ---- scores: one warp per key, lane owns dims 8*lane..8*lane+7 ----------------
    float q[NH][8];
#pragma unroll
    for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int i = 0; i < 8; ++i) q[h][i] = qs[h * 256 + 8 * lane + i];
    for (uint32_t jj = warp; jj < n; jj += ATT_THREADS / 32) {
        const uint32_t j = j0 + jj;
        uint4 raw;
        if (j == pos) raw = *reinterpret_cast<const uint4*>(kn + 8 * lane);
        else raw = __ldg(reinterpret_cast<const uint4*>(a.kcache + (size_t)j * 256) + lane);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
        float kf[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h2[i]);
            kf[2 * i] = f.x;
            kf[2 * i + 1] = f.y;
        }
        float s[NH];
#pragma unroll
        for (int h = 0; h < NH; ++h) {
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = fmaf(q[h][i], kf[i], acc);
            s[h] = acc;
        }
        const float tot = reduce4(s[0], s[1], s[2], s[3]);
        if ((lane & 7) == 0) {
            const int h = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
            sc[h * a.chunk_max + jj] = tot;
        }
    }
    __syncthreads();

    // ---- chunk softmax statistics ---------------------------------------------------
    if (warp < NH) {
        float m = -INFINITY;
        for (uint32_t jj = lane; jj < n; jj += 32) m = fmaxf(m, sc[warp * a.chunk_max + jj]);
        m = warp_max(m);
        float l = 0.0f;
        for (uint32_t jj = lane; jj < n; jj += 32) {
            const float p = expf(sc[warp * a.chunk_max + jj] - m);
            sc[warp * a.chunk_max + jj] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) { stat[warp * 2] = m; stat[warp * 2 + 1] = l; }
    }
    __syncthreads();

    // ---- P.V: thread owns a dim pair, two halves of the chunk ---------------------------
    {
        const uint32_t dp = tid & 127, half = tid >> 7;
        float acc[NH][2];
#pragma unroll
        for (int h = 0; h < NH; ++h) acc[h][0] = acc[h][1] = 0.0f;
        for (uint32_t jj = half; jj < n; jj += 2) {
            const uint32_t j = j0 + jj;
            __half2 hv;
            if (j == pos) hv = reinterpret_cast<const __half2*>(vn)[dp];
            else hv = __ldg(reinterpret_cast<const __half2*>(a.vcache + (size_t)j * 256) + dp);
            const float2 vf = __half22float2(hv);
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                const float p = sc[h * a.chunk_max + jj];
                acc[h][0] = fmaf(p, vf.x, acc[h][0]);
                acc[h][1] = fmaf(p, vf.y, acc[h][1]);
            }
        }
#pragma unroll
        for (int h = 0; h < NH; ++h) {
            accs[(half * NH + h) * 256 + 2 * dp] = acc[h][0];
            accs[(half * NH + h) * 256 + 2 * dp + 1] = acc[h][1];
        }
    }
    __syncthreads();
    float* mypart = a.part + (size_t)blockIdx.x * NH * 256;
    for (uint32_t i = tid; i < NH * 256; i += ATT_THREADS) mypart[i] = accs[i] + accs[NH * 256 + i];
    if (tid < NH * 2) a.pstat[(size_t)blockIdx.x * NH * 2 + tid] = stat[tid];

    // ---- last CTA combines -----------------------------------------------------------------
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(a.ticket, 1u) == nblk - 1) ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid < NH) {
        float M = -INFINITY;
        for (uint32_t b = 0; b < nblk; ++b) M = fmaxf(M, a.pstat[(size_t)b * NH * 2 + tid * 2]);
        float L = 0.0f;
        for (uint32_t b = 0; b < nblk; ++b) {
            const float bm = a.pstat[(size_t)b * NH * 2 + tid * 2];
            const float bl = a.pstat[(size_t)b * NH * 2 + tid * 2 + 1];
            if (bl > 0.0f) L += bl * expf(bm - M);
        }
        stat[tid * 2] = M;
        stat[tid * 2 + 1] = 1.0f / L;
    }
    __syncthreads();
    for (uint32_t i = tid; i < NH * 256; i += ATT_THREADS) {
        const uint32_t h = i >> 8;
        const float M = stat[h * 2], invL = stat[h * 2 + 1];
        float o = 0.0f;
        for (uint32_t b = 0; b < nblk; ++b) {
            const float bl = a.pstat[(size_t)b * NH * 2 + h * 2 + 1];
            if (bl > 0.0f) o += a.part[(size_t)b * NH * 256 + i] * expf(a.pstat[(size_t)b * NH * 2 + h * 2] - M);
        }
        o *= invL;
        a.att[i] = o;
        accs[i] = o;
    }
    __syncthreads();
    if (a.att_xq)
        for (uint32_t bb = warp; bb < NH * 256 / 32; bb += ATT_THREADS / 32)
            xq_prep_block(accs[bb * 32 + lane], &a.att_xq[bb]);
    if (tid == 0) *a.ticket = 0;
}

}  // namespace xp
