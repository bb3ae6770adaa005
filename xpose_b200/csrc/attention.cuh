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
//     each CTA streams its chunk's K rows, then its V rows, through a ring of
//     bulk copies (cp.async.bulk, 32 positions = 16 KB a stage) issued before
//     the q/k work, and computes scores, a softmax partial (max, sum) and the
//     unnormalised P.V for its chunk;
//   * the combine is two-level: the CTAs of a thread-block cluster (up to 8)
//     leave their partials in shared memory and the cluster's first CTA
//     merges them through distributed shared memory; with more than one
//     cluster, the last cluster to finish (atomic ticket) merges the cluster
//     results in cluster order and writes the attention output and its matvec
//     limbs. Fixed merge order: deterministic.
// Shape: n_heads = NH query heads sharing one kv head, head_dim = 256.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"
#include "tk_primitives.cuh"
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
    uint32_t cache_rows;   // rows the K and V caches hold (a position at or past it is refused)
    uint32_t window;       // 0 = global layer
    float theta, eps, scale;
    uint32_t chunk_max;    // smem capacity in positions per CTA
    float* part;           // [clusters][NH][256] cluster partials
    float* pstat;          // [clusters][NH][2] (max, sum)
    uint32_t* ticket;      // zero between launches
    float* att;            // [NH][256]
    XBlk* att_xq;          // [NH*256/32]
    uint32_t* err;         // error word (TK_ERR_ATTN_CHUNK, TK_ERR_MBAR)
    float inv_freq[128];   // RoPE theta^(-2d/256), from rope_table_host
};

// RoPE inverse frequency theta^(-2d/hd), rounded once from double so host and
// device agree bit for bit.
XP_DEV float rope_inv_freq(uint32_t d, uint32_t head_dim, float theta) {
    const float l2 = (float)log2((double)theta);
    const float frac = (float)(2u * d) / (float)head_dim;
    const float e = -l2 * frac;
    return (float)exp2((double)e);
}

// sin and cos of a RoPE angle. CUDA's sincosf takes a slow reduction path for
// the angles of long contexts (pos * theta^0 is the position itself), and
// fp64 is slow on this part, so reduce in fp32 first: Cody-Waite reduction by
// pi/2 with pi/2 split into C1 + C2 + C3 (11-bit significands each, so k * Ci
// is exact for |k| < 2^13) + C4 (the rest), one FMA per part, then sincosf of
// the reduced argument (|r| <= pi/4) and the quadrant's signs. Within 2 ulp of
// sin/cos of the float angle (the bound CUDA states for sincosf); angles past
// 8192 * pi/2 take sincosf directly.
XP_DEV void rope_sincos(float ang, float* s, float* c) {
    if (!(fabsf(ang) < 12867.0f)) {
        sincosf(ang, s, c);
        return;
    }
    const float k = rintf(ang * 0.636619772f);  // 2/pi
    float r = fmaf(-k, 0x1.92p+0f, ang);
    r = fmaf(-k, 0x1.fb4p-12f, r);
    r = fmaf(-k, 0x1.444p-24f, r);
    r = fmaf(-k, 0x1.68c234p-39f, r);
    float sr, cr;
    sincosf(r, &sr, &cr);
    switch ((int)k & 3) {
        case 0: *s = sr; *c = cr; break;
        case 1: *s = cr; *c = -sr; break;
        case 2: *s = -sr; *c = -cr; break;
        default: *s = -cr; *c = sr; break;
    }
}

// Warp-level: normalise one 256-wide head held as 8 values per lane (lane
// owns dims 4*lane..4*lane+3 and 128+4*lane..+3) with its (1 + w) weights wv
// (same layout), then rotate-half with the position's table rcs = cos[128] |
// sin[128].
XP_DEV void qk_norm_rope(float v[8], const float wv[8], float eps, const float* rcs) {
    const int lane = threadIdx.x & 31;
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
    ss = warp_sum(ss);
    const float sc = rsqrtf(ss / 256.0f + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t d = 4 * lane + i;
        const float lo = v[i] * sc * (1.0f + wv[i]), hi = v[4 + i] * sc * (1.0f + wv[4 + i]);
        const float c = rcs[d], s = rcs[128 + d];
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

constexpr uint32_t ATT_TILE = 32;    // positions per bulk-copy stage (16 KB of K or V)
constexpr uint32_t ATT_STAGES = 4;

// Shared-memory layout of attn_decode_kernel (bytes from the dynamic base).
struct AttnSmem {
    static constexpr size_t bar = 0;
    static constexpr size_t ring = 128;
    static constexpr size_t qs = ring + (size_t)ATT_STAGES * ATT_TILE * 512;
    static constexpr size_t knv = qs + 4 * 256 * 4;
    static constexpr size_t accs = knv + 2 * 256 * 2;
    static constexpr size_t sc = accs + 2 * 4 * 256 * 4;
    static constexpr size_t bytes(uint32_t chunk_max) { return sc + (size_t)4 * chunk_max * 4; }
};

// Merge `cnt` flash-decode partials (unnormalised P.V [NH][256] and (max, sum)
// per head) in index order; part(b) and stat(b) give partial b's arrays (global
// memory, or a cluster peer's shared memory when DSMEM). Each thread owns four
// consecutive outputs of one head and recomputes that head's max, weights
// e^(m_b - M) and sum itself, so the merge needs no block synchronisation.
// final: out = (sum_b P_b e^(m_b - M)) / L, with matvec limbs when xq is set
// (accs: 1024 floats of staging); else the merged partial and its (M, L).
template <int NH, bool DSMEM, class PF, class SF>
__device__ __noinline__ void attn_merge(PF part, SF stat, uint32_t cnt, float* out, float* ostat, XBlk* xq, bool final,
                                        float* accs) {
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    static_assert(NH * 256 == 4 * ATT_THREADS, "one float4 of outputs per thread");
    const uint32_t h = (4 * tid) >> 8;
    auto ld4 = [&](uint32_t b) {
        const float4* p = reinterpret_cast<const float4*>(part(b)) + tid;
        return DSMEM ? *p : __ldcg(p);
    };
    auto ld2 = [&](uint32_t b) {
        const float2* p = reinterpret_cast<const float2*>(stat(b)) + h;
        return DSMEM ? *p : __ldcg(p);
    };
    float M = -INFINITY, L = 0.0f;
    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (DSMEM) {
        // a cluster holds at most 8 partials: every load in one round trip
        float4 v[8];
        float2 st[8];
#pragma unroll
        for (int b = 0; b < 8; ++b)
            if ((uint32_t)b < cnt) { v[b] = ld4(b); st[b] = ld2(b); }
#pragma unroll
        for (int b = 0; b < 8; ++b)
            if ((uint32_t)b < cnt && st[b].y > 0.0f) M = fmaxf(M, st[b].x);
#pragma unroll
        for (int b = 0; b < 8; ++b)
            if ((uint32_t)b < cnt) {
                const float w = st[b].y > 0.0f ? expf(st[b].x - M) : 0.0f;
                L += st[b].y * w;
                o.x += v[b].x * w; o.y += v[b].y * w; o.z += v[b].z * w; o.w += v[b].w * w;
            }
    } else {
#pragma unroll 4
        for (uint32_t b = 0; b < cnt; ++b) {
            const float2 st = ld2(b);
            if (st.y > 0.0f) M = fmaxf(M, st.x);
        }
#pragma unroll 4
        for (uint32_t b = 0; b < cnt; ++b) {
            const float4 v = ld4(b);
            const float2 st = ld2(b);
            const float w = st.y > 0.0f ? expf(st.x - M) : 0.0f;
            L += st.y * w;
            o.x += v.x * w; o.y += v.y * w; o.z += v.z * w; o.w += v.w * w;
        }
    }
    if (!final) {
        reinterpret_cast<float4*>(out)[tid] = o;
        if ((tid & 63) == 0) { ostat[h * 2] = M; ostat[h * 2 + 1] = L; }
        return;
    }
    const float inv = 1.0f / L;
    o.x *= inv; o.y *= inv; o.z *= inv; o.w *= inv;
    reinterpret_cast<float4*>(out)[tid] = o;
    if (xq) {
        reinterpret_cast<float4*>(accs)[tid] = o;
        __syncthreads();
        for (uint32_t bb = warp; bb < NH * 256 / 32; bb += ATT_THREADS / 32) xq_prep_block(accs[bb * 32 + lane], &xq[bb]);
    }
}

template <int NH>
__global__ void __launch_bounds__(ATT_THREADS, 1) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    static_assert(NH == 4, "the reduce4 score path is written for 4 query heads");
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + AttnSmem::bar);
    __half* ring = reinterpret_cast<__half*>(smem + AttnSmem::ring);  // [stage][32][256]
    float* qs = reinterpret_cast<float*>(smem + AttnSmem::qs);         // [NH][256], pre-scaled
    __half* kn = reinterpret_cast<__half*>(smem + AttnSmem::knv);     // [256] new k (fp16)
    __half* vn = kn + 256;                                            // [256] new v (fp16)
    float* accs = reinterpret_cast<float*>(smem + AttnSmem::accs);     // [2][NH][256] P.V halves
    float* sc = reinterpret_cast<float*>(smem + AttnSmem::sc);         // [chunk_max][NH] scores / probs
    __shared__ __align__(16) float stat[NH * 2];  // (max, sum) per head, read as float2 by the merge
    __shared__ float rcs[256];  // RoPE cos | sin of this position
    __shared__ uint32_t s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (uint32_t s = 0; s < ATT_STAGES; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    pdl_launch_dependents();
    pdl_wait();

    const uint32_t pos = *a.pos;
    if (pos >= a.cache_rows) {  // the append would land past the caches: flag, write nothing
        if (tid == 0 && blockIdx.x == 0 && a.err) atomicOr(a.err, TK_ERR_POS);
        return;
    }
    const uint32_t seq = pos + 1;
    const uint32_t kv_start = (a.window == 0 || seq <= a.window) ? 0 : seq - a.window;
    const uint32_t span = seq - kv_start;
    const uint32_t nblk = gridDim.x;
    uint32_t chunk = (span + nblk - 1) / nblk;
    chunk = (chunk + 7) & ~7u;
    if (chunk > a.chunk_max) {  // host sized the grid wrong: flag and attend to a prefix
        if (tid == 0 && a.err) atomicOr(a.err, TK_ERR_ATTN_CHUNK);
        chunk = a.chunk_max;
    }
    const uint32_t j0 = kv_start + min(blockIdx.x * chunk, span);
    const uint32_t j1 = kv_start + min((blockIdx.x + 1) * chunk, span);
    const uint32_t n = j1 - j0;
    const uint32_t nt = (n + ATT_TILE - 1) / ATT_TILE;  // tiles of K, then as many of V
    // copy u (< 2 nt) into stage u % ATT_STAGES
    auto issue = [&](uint32_t u) {
        const bool isv = u >= nt;
        const uint32_t t = isv ? u - nt : u;
        const uint32_t rows = min(ATT_TILE, n - t * ATT_TILE);
        const __half* src = (isv ? a.vcache : a.kcache) + (size_t)(j0 + t * ATT_TILE) * 256;
        uint64_t* b = &bar[u % ATT_STAGES];
        mbar_expect_tx(b, rows * 512);
        bulk_g2s(ring + (size_t)(u % ATT_STAGES) * ATT_TILE * 256, src, rows * 512, b);
    };
    __syncthreads();  // barriers initialised
    if (tid == 0)
        for (uint32_t u = 0; u < min(2 * nt, ATT_STAGES); ++u) issue(u);

    // ---- q, k, v post-processing (overlaps the first copies) ------------------------------
    // The position's RoPE table is computed once (one angle per thread); the
    // q, k, v loads are in flight meanwhile.
    float v[8], wv[8];
    if (warp <= NH + 1) {
        const float* src = warp < NH ? a.q_raw + warp * 256 : (warp == NH ? a.k_raw : a.v_raw);
        const float* wsrc = warp < NH ? a.q_norm : a.k_norm;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[i] = src[4 * lane + i];
            v[4 + i] = src[128 + 4 * lane + i];
            wv[i] = wsrc[4 * lane + i];
            wv[4 + i] = wsrc[128 + 4 * lane + i];
        }
    }
    if (tid < 128) rope_sincos((float)pos * a.inv_freq[tid], &rcs[128 + tid], &rcs[tid]);
    __syncthreads();
    if (warp <= NH) qk_norm_rope(v, wv, a.eps, rcs);
    if (warp < NH) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            qs[warp * 256 + 4 * lane + i] = v[i] * a.scale;
            qs[warp * 256 + 128 + 4 * lane + i] = v[4 + i] * a.scale;
        }
    } else if (warp <= NH + 1) {
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
    __syncthreads();

    // ---- scores: one warp per key, lane owns dims 8*lane..8*lane+7 ----------------
    float q[NH][8];
#pragma unroll
    for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int i = 0; i < 8; ++i) q[h][i] = qs[h * 256 + 8 * lane + i];
    for (uint32_t u = 0; u < nt; ++u) {
        mbar_wait(&bar[u % ATT_STAGES], (u / ATT_STAGES) & 1, a.err);
        const __half* tile = ring + (size_t)(u % ATT_STAGES) * ATT_TILE * 256;
        const uint32_t rows = min(ATT_TILE, n - u * ATT_TILE);
        static_assert(ATT_TILE == 4 * (ATT_THREADS / 32), "four rows of a tile per warp");
        // rows 4 warp .. 4 warp + 3: four independent dot products and reductions
        float tot[4];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const uint32_t r = 4 * warp + rr;
            const uint32_t jj = u * ATT_TILE + r;
            uint4 raw = make_uint4(0u, 0u, 0u, 0u);
            if (r < rows)
                raw = (j0 + jj == pos) ? *reinterpret_cast<const uint4*>(kn + 8 * lane)
                                       : *reinterpret_cast<const uint4*>(tile + r * 256 + 8 * lane);
            const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
            float kf[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(h2[i]);
                kf[2 * i] = f.x;
                kf[2 * i + 1] = f.y;
            }
            float sh[NH];
#pragma unroll
            for (int h = 0; h < NH; ++h) {
                float acc = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; ++i) acc = fmaf(q[h][i], kf[i], acc);
                sh[h] = acc;
            }
            tot[rr] = reduce4(sh[0], sh[1], sh[2], sh[3]);
        }
        if ((lane & 7) == 0) {
            const int h = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
#pragma unroll
            for (int rr = 0; rr < 4; ++rr)
                if (4 * warp + rr < rows) sc[(u * ATT_TILE + 4 * warp + rr) * NH + h] = tot[rr];
        }
        __syncthreads();  // stage consumed
        if (tid == 0 && u + ATT_STAGES < 2 * nt) issue(u + ATT_STAGES);
    }

    // ---- chunk softmax statistics ---------------------------------------------------
    if (warp < NH) {
        float m = -INFINITY;
        for (uint32_t jj = lane; jj < n; jj += 32) m = fmaxf(m, sc[jj * NH + warp]);
        m = warp_max(m);
        float l = 0.0f;
        for (uint32_t jj = lane; jj < n; jj += 32) {
            const float p = expf(sc[jj * NH + warp] - m);
            sc[jj * NH + warp] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) { stat[warp * 2] = m; stat[warp * 2 + 1] = l; }
    }
    __syncthreads();

    // ---- P.V: thread owns a dim pair, alternate rows of each tile ------------------------
    {
        const uint32_t dp = tid & 127, half = tid >> 7;
        float acc[NH][2];
#pragma unroll
        for (int h = 0; h < NH; ++h) acc[h][0] = acc[h][1] = 0.0f;
        for (uint32_t t = 0; t < nt; ++t) {
            const uint32_t u = nt + t;
            mbar_wait(&bar[u % ATT_STAGES], (u / ATT_STAGES) & 1, a.err);
            const __half* tile = ring + (size_t)(u % ATT_STAGES) * ATT_TILE * 256;
            const uint32_t rows = min(ATT_TILE, n - t * ATT_TILE);
            auto row = [&](uint32_t r) {
                const uint32_t jj = t * ATT_TILE + r;
                const __half2 hv = (j0 + jj == pos) ? reinterpret_cast<const __half2*>(vn)[dp]
                                                    : reinterpret_cast<const __half2*>(tile + r * 256)[dp];
                const float2 vf = __half22float2(hv);
                const float4 p4 = reinterpret_cast<const float4*>(sc)[jj];
                const float p[NH] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
                for (int h = 0; h < NH; ++h) {
                    acc[h][0] = fmaf(p[h], vf.x, acc[h][0]);
                    acc[h][1] = fmaf(p[h], vf.y, acc[h][1]);
                }
            };
            if (rows == ATT_TILE) {
#pragma unroll
                for (uint32_t r0 = 0; r0 < ATT_TILE; r0 += 2) row(r0 + half);
            } else {
#pragma unroll 1
                for (uint32_t r = half; r < rows; r += 2) row(r);
            }
            __syncthreads();  // stage consumed
            if (tid == 0 && u + ATT_STAGES < 2 * nt) issue(u + ATT_STAGES);
        }
#pragma unroll
        for (int h = 0; h < NH; ++h) {
            accs[(half * NH + h) * 256 + 2 * dp] = acc[h][0];
            accs[(half * NH + h) * 256 + 2 * dp + 1] = acc[h][1];
        }
    }
    __syncthreads();
    // ---- combine: cluster peers through DSMEM, then clusters through global memory ----------------
    for (uint32_t i = tid; i < NH * 256; i += ATT_THREADS) accs[i] += accs[NH * 256 + i];
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const uint32_t csize = cl.num_blocks(), crank = cl.block_rank();
    const uint32_t ncl = nblk / csize, ci = blockIdx.x / csize;
    cl.sync();  // every CTA's partial (accs, stat) is in its shared memory
    if (crank == 0) {
        auto ppart = [&](uint32_t b) { return cl.map_shared_rank(accs, b); };
        auto pstat = [&](uint32_t b) { return cl.map_shared_rank(&stat[0], b); };
        // the merged cluster partial goes to the second half of accs (unused by peers)
        if (ncl == 1)
            attn_merge<NH, true>(ppart, pstat, csize, a.att, nullptr, a.att_xq, true, accs + NH * 256);
        else
            attn_merge<NH, true>(ppart, pstat, csize, a.part + (size_t)ci * NH * 256, a.pstat + (size_t)ci * NH * 2,
                                 nullptr, false, accs + NH * 256);
    }
    cl.sync();  // peers keep their shared memory until the first CTA has read it
    if (ncl == 1 || crank != 0) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(a.ticket, 1u) == ncl - 1) ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    auto gpart = [&](uint32_t b) { return a.part + (size_t)b * NH * 256; };
    auto gstat = [&](uint32_t b) { return a.pstat + (size_t)b * NH * 2; };
    attn_merge<NH, false>(gpart, gstat, ncl, a.att, nullptr, a.att_xq, true, accs);
    if (tid == 0) *a.ticket = 0;
}

}  // namespace xp
