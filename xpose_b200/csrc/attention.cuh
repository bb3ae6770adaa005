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
//   * the combine is two-level: within a thread-block cluster (up to 16
//     CTAs) the output is cut into one slice per CTA; every CTA pushes slice
//     k of its partial into CTA k's shared memory (st.async, completing on
//     CTA k's mbarrier; no cluster-wide barrier after the work) and each CTA
//     merges its slice; with more than one cluster, the last CTA to finish
//     (atomic ticket) merges the cluster results in cluster order and writes
//     the attention output and its matvec limbs. Fixed merge order:
//     deterministic.
// Shape: n_heads = NH query heads sharing one kv head, head_dim = 256.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"
#include "tk_primitives.cuh"
#include "xq.cuh"

namespace xp {

#ifndef XP_ATT_THREADS
#define XP_ATT_THREADS 256
#endif
constexpr int ATT_THREADS = XP_ATT_THREADS;  // 256 or 512
constexpr int ATT_MT = 256;                  // threads of the combine and merge: one float4 of outputs each
constexpr int ATT_PVG = ATT_THREADS / 128;   // P.V row groups (a thread owns a dim pair)
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

// Phase timestamps for latency studies, compiled only with XP_ATT_TRACE:
// [launch][cta][10] globaltimer values (entry, after the grid dependency,
// position read, q/k ready, scores, softmax, P.V, partials published, cluster
// merged, final merge).
#ifdef XP_ATT_TRACE
__device__ unsigned long long g_att_trace[64 * 160 * 16];
__device__ uint32_t g_att_launch;
#define ATT_STAMP(i) do { if (threadIdx.x == 0) tr_[i] = globaltimer_ns(); } while (0)
#else
#define ATT_STAMP(i) do { } while (0)
#endif

// Cluster primitives of the push merge: each CTA stores a slice of its
// partial into the shared memory of the CTA that merges that slice with
// st.async, which completes bytes on the receiver's mbarrier, so only
// receivers wait and no cluster-wide barrier follows the merge.
XP_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
XP_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
XP_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
XP_DEV void st_async_v4(uint32_t addr, float4 v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
                 ::"r"(addr), "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
                   "r"(__float_as_uint(v.w)), "r"(bar)
                 : "memory");
}

constexpr uint32_t ATT_TILE = 32;    // positions per bulk-copy stage (16 KB of K or V)
#ifndef XP_ATT_STAGES
#define XP_ATT_STAGES 4
#endif
constexpr uint32_t ATT_STAGES = XP_ATT_STAGES;  // copies in flight per CTA
static_assert(ATT_STAGES + 1 <= 16, "the ring and merge barriers fit the 128-byte barrier area");
constexpr size_t ATT_SMEM_MAX = 225 * 1024;  // dynamic shared memory a launch may ask for

// Shared-memory layout of attn_decode_kernel (bytes from the dynamic base).
struct AttnSmem {
    static constexpr size_t bar = 0;
    static constexpr size_t ring = 128;
    static constexpr size_t qs = ring + (size_t)ATT_STAGES * ATT_TILE * 512;
    static constexpr size_t knv = qs + 4 * 256 * 4;
    static constexpr size_t accs = knv + 2 * 256 * 2;
    static constexpr size_t sc = accs + (size_t)ATT_PVG * 4 * 256 * 4;
    // merge slots: one per cluster CTA, its slice of this CTA's part of the
    // output (4 KB / cluster) | (max, sum) x NH
    static constexpr size_t slot_bytes(uint32_t cluster) { return 4 * 256 * 4 / cluster + 4 * 2 * 4; }
    __host__ __device__ static constexpr size_t slots(uint32_t chunk_max) { return sc + (size_t)4 * chunk_max * 4; }
    static constexpr size_t bytes(uint32_t chunk_max, uint32_t cluster) {
        return slots(chunk_max) + (cluster > 1 ? (size_t)cluster * slot_bytes(cluster) : 0);
    }
};

// Finish a merged flash-decode partial (thread's float4 o of [NH][256], its
// head's max M and sum L). final: out = o / L, with matvec limbs when xq is set
// (accs: 1024 floats of staging); else the partial and its (M, L). Run by
// threads 0..ATT_MT-1 only.
template <int NH>
XP_DEV void attn_finish(float4 o, float M, float L, float* out, float* ostat, XBlk* xq, bool final, float* accs) {
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t h = (4 * tid) >> 8;
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
        asm volatile("bar.sync 1, %0;" ::"n"(ATT_MT) : "memory");  // the merging threads only
        for (uint32_t bb = warp; bb < NH * 256 / 32; bb += ATT_MT / 32) xq_prep_block(accs[bb * 32 + lane], &xq[bb]);
    }
}

// Merge `cnt` flash-decode partials (unnormalised P.V [NH][256] and (max, sum)
// per head) in index order: M = max of the non-empty partials' maxima, then
// o = sum_b P_b e^(m_b - M) and L = sum_b l_b e^(m_b - M). Each thread owns
// four consecutive outputs of one head and recomputes that head's M itself,
// so the merge needs no block synchronisation.
//
// Cluster partials in global memory (the last cluster merges them): a loop.
template <int NH>
__device__ __noinline__ void attn_merge_global(const float* part, const float* stat, uint32_t cnt, float* out,
                                               XBlk* xq, float* accs) {
    const uint32_t tid = threadIdx.x;
    static_assert(NH * 256 == 4 * ATT_MT, "one float4 of outputs per merging thread");
    const uint32_t h = (4 * tid) >> 8;
    float M = -INFINITY, L = 0.0f;
    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 4
    for (uint32_t b = 0; b < cnt; ++b) {
        const float2 st = __ldcg(reinterpret_cast<const float2*>(stat + (size_t)b * NH * 2) + h);
        if (st.y > 0.0f) M = fmaxf(M, st.x);
    }
#pragma unroll 4
    for (uint32_t b = 0; b < cnt; ++b) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(part + (size_t)b * NH * 256) + tid);
        const float2 st = __ldcg(reinterpret_cast<const float2*>(stat + (size_t)b * NH * 2) + h);
        const float w = st.y > 0.0f ? expf(st.x - M) : 0.0f;
        L += st.y * w;
        o.x += v.x * w; o.y += v.y * w; o.z += v.z * w; o.w += v.w * w;
    }
    attn_finish<NH>(o, M, L, out, nullptr, xq, true, accs);
}

// The RoPE table again when the position changed after the speculative one
// (rare: out of line, so its code is not fetched on the common path).
__device__ __noinline__ void rope_table_again(float ang, float* s, float* c) { rope_sincos(ang, s, c); }

template <int NH>
__global__ void __launch_bounds__(ATT_THREADS, 1) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    static_assert(NH == 4, "the reduce4 score path is written for 4 query heads");
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + AttnSmem::bar);
    __half* ring = reinterpret_cast<__half*>(smem + AttnSmem::ring);  // [stage][32][256]
    float* qs = reinterpret_cast<float*>(smem + AttnSmem::qs);         // [NH][256], pre-scaled
    __half* kn = reinterpret_cast<__half*>(smem + AttnSmem::knv);     // [256] new k (fp16)
    __half* vn = kn + 256;                                            // [256] new v (fp16)
    float* accs = reinterpret_cast<float*>(smem + AttnSmem::accs);     // [ATT_PVG][NH][256] P.V by row group
    float* sc = reinterpret_cast<float*>(smem + AttnSmem::sc);         // [chunk_max][NH] scores / probs
    __shared__ __align__(16) float stat[NH * 2];  // (max, sum) per head, read as float2 by the merge
    __shared__ float rcs[256];  // RoPE cos | sin of this position
    __shared__ uint32_t s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
#ifdef XP_ATT_TRACE
    unsigned long long tr_[16] = {};
    ATT_STAMP(0);
#endif
    if (tid == 0) {
        for (uint32_t s = 0; s <= ATT_STAGES; ++s) mbar_init(&bar[s], 1);  // copy ring + merge
        fence_mbar_init();
    }
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const uint32_t csize = cl.num_blocks(), crank = cl.block_rank();
    if (csize > 1) cluster_arrive_relaxed();  // this CTA's merge barrier is initialised
    pdl_launch_dependents();
    // Before the grid dependency resolves (this launch may overlap the tail
    // of the kernel before it): the position read here may be stale, so it
    // only steers an L2 prefetch of this CTA's K and V rows (a hint: what the
    // copies below read is unaffected) and a RoPE table that is recomputed
    // if the position turns out different.
    const uint32_t pos_early = __ldcg(a.pos);
    if (pos_early < a.cache_rows) {
        const uint32_t seq_e = pos_early + 1;
        const uint32_t ks_e = (a.window == 0 || seq_e <= a.window) ? 0 : seq_e - a.window;
        const uint32_t span_e = seq_e - ks_e;
        uint32_t ch = (span_e + gridDim.x - 1) / gridDim.x;
        ch = min((ch + 7) & ~7u, a.chunk_max);
        const uint32_t r0 = ks_e + min(blockIdx.x * ch, span_e), r1 = ks_e + min((blockIdx.x + 1) * ch, span_e);
        if (tid == 0 && r1 > r0) {
            bulk_prefetch_l2(a.kcache + (size_t)r0 * 256, (r1 - r0) * 512);
            bulk_prefetch_l2(a.vcache + (size_t)r0 * 256, (r1 - r0) * 512);
        }
        if (tid < 128) rope_sincos((float)pos_early * a.inv_freq[tid], &rcs[128 + tid], &rcs[tid]);
    }
    pdl_wait();
    ATT_STAMP(1);
#ifdef XP_ATT_TRACE
    const uint32_t launch_ = *(volatile uint32_t*)&g_att_launch & 63;
    auto flush_ = [&]() {
        if (tid == 0 && blockIdx.x < 160)
            for (int i = 0; i < 16; ++i) g_att_trace[((size_t)launch_ * 160 + blockIdx.x) * 16 + i] = tr_[i];
    };
#endif

    // q, k, v and the norm weights load together with the position (they do
    // not depend on it)
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
    const uint32_t pos = *a.pos;
    ATT_STAMP(2);
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
    // thread 0 initialised the barriers, so it issues the first copies at once;
    // every other thread's first wait comes after the block barrier below
    if (tid == 0)
        for (uint32_t u = 0; u < min(2 * nt, ATT_STAGES); ++u) issue(u);
    ATT_STAMP(10);

    // ---- q, k, v post-processing (overlaps the first copies) ------------------------------
    // The position's RoPE table is computed once (one angle per thread); the
    // q, k, v loads are in flight meanwhile.
    if (tid < 128 && pos != pos_early) rope_table_again((float)pos * a.inv_freq[tid], &rcs[128 + tid], &rcs[tid]);
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
    ATT_STAMP(3);


    // ---- scores: one warp per key, lane owns dims 8*lane..8*lane+7 ----------------
    float q[NH][8];
#pragma unroll
    for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int i = 0; i < 8; ++i) q[h][i] = qs[h * 256 + 8 * lane + i];
    for (uint32_t u = 0; u < nt; ++u) {
        mbar_wait(&bar[u % ATT_STAGES], (u / ATT_STAGES) & 1, a.err);
#ifdef XP_ATT_TRACE
        if (u < 2) ATT_STAMP(11 + u);
#endif
        const __half* tile = ring + (size_t)(u % ATT_STAGES) * ATT_TILE * 256;
        const uint32_t rows = min(ATT_TILE, n - u * ATT_TILE);
        constexpr int RPW = ATT_TILE / (ATT_THREADS / 32);  // rows of a tile per warp
        static_assert(RPW * (ATT_THREADS / 32) == ATT_TILE, "whole rows per warp");
        // rows RPW warp .. RPW warp + RPW - 1: independent dot products and reductions
        float tot[RPW];
#pragma unroll
        for (int rr = 0; rr < RPW; ++rr) {
            const uint32_t r = RPW * warp + rr;
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
            for (int rr = 0; rr < RPW; ++rr)
                if (RPW * warp + rr < rows) sc[(u * ATT_TILE + RPW * warp + rr) * NH + h] = tot[rr];
        }
        __syncthreads();  // stage consumed
        if (tid == 0 && u + ATT_STAGES < 2 * nt) issue(u + ATT_STAGES);
    }

    ATT_STAMP(4);
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
    ATT_STAMP(5);

    // ---- P.V: thread owns a dim pair and every ATT_PVG-th row of each tile -----------------
    {
        const uint32_t dp = tid & 127, grp = tid >> 7;
        float acc[NH][2];
#pragma unroll
        for (int h = 0; h < NH; ++h) acc[h][0] = acc[h][1] = 0.0f;
        for (uint32_t t = 0; t < nt; ++t) {
            const uint32_t u = nt + t;
            mbar_wait(&bar[u % ATT_STAGES], (u / ATT_STAGES) & 1, a.err);
#ifdef XP_ATT_TRACE
            if (t < 2) ATT_STAMP(13 + t);
#endif
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
                for (uint32_t r0 = 0; r0 < ATT_TILE; r0 += ATT_PVG) row(r0 + grp);
            } else {
#pragma unroll 1
                for (uint32_t r = grp; r < rows; r += ATT_PVG) row(r);
            }
            __syncthreads();  // stage consumed
            if (tid == 0 && u + ATT_STAGES < 2 * nt) issue(u + ATT_STAGES);
        }
#pragma unroll
        for (int h = 0; h < NH; ++h) {
            accs[(grp * NH + h) * 256 + 2 * dp] = acc[h][0];
            accs[(grp * NH + h) * 256 + 2 * dp + 1] = acc[h][1];
        }
    }
    __syncthreads();
    ATT_STAMP(6);
    // ---- combine: slices pushed to the CTAs that merge them, then clusters through global memory ----
    // threads 0..ATT_MT-1 own one float4 of the [NH][256] partial each
    const uint32_t ncl = nblk / csize, ci = blockIdx.x / csize;
    float* slots = reinterpret_cast<float*>(smem + AttnSmem::slots(a.chunk_max));
    const bool mt = tid < ATT_MT;
    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (mt)
#pragma unroll
        for (int g = 0; g < ATT_PVG; ++g) {
            const float4 x = reinterpret_cast<const float4*>(accs)[g * NH * 64 + tid];
            o.x += x.x; o.y += x.y; o.z += x.z; o.w += x.w;
        }
    // Distributed merge: the cluster's [NH][256] output is cut into csize
    // slices of S4 float4s; slice k is merged by cluster CTA k. Every CTA
    // stores slice k of its partial (and its per-head statistics) into CTA
    // k's slot for it with st.async, which completes bytes on CTA k's merge
    // barrier, so each CTA receives 4 KB in total (plus 32 B of statistics
    // per peer) instead of one CTA receiving every partial.
    const uint32_t S4 = (uint32_t)ATT_MT / csize;      // float4s per slice
    const uint32_t SLOT4 = S4 + 2;                      // slice + (max, sum) x NH
    float4* slots4 = reinterpret_cast<float4*>(slots);  // [csize][SLOT4]
    if (csize > 1) {
        cluster_wait();  // every CTA's merge barrier is initialised
        if (mt) {
            const uint32_t k = tid / S4;
            const uint32_t dst = mapa_shared(smem_u32(slots4 + crank * SLOT4), k);
            const uint32_t rb = mapa_shared(smem_u32(&bar[ATT_STAGES]), k);
            st_async_v4(dst + 16 * (tid % S4), o, rb);
            if (tid % S4 == 0) {
                st_async_v4(dst + 16 * S4, reinterpret_cast<const float4*>(stat)[0], rb);
                st_async_v4(dst + 16 * S4 + 16, reinterpret_cast<const float4*>(stat)[1], rb);
            }
        }
        if (tid == 0) mbar_expect_tx(&bar[ATT_STAGES], csize * SLOT4 * 16);
        mbar_wait(&bar[ATT_STAGES], 0, a.err);
    }
    ATT_STAMP(7);
    // This CTA's merged slice (a lone CTA's own partial as it stands: the
    // merge of one partial is the identity), in partial order: M = max of the
    // non-empty partials' maxima, w_b = e^(m_b - M), L = sum l_b w_b,
    // o = sum P_b w_b.
    const uint32_t nmine = csize > 1 ? S4 : (uint32_t)ATT_MT;  // float4s this CTA finishes
    const uint32_t e4 = (csize > 1 ? crank * S4 : 0u) + tid;    // float4 index in [NH][256]
    const bool fin = tid < nmine;
    float M = -INFINITY, L = 0.0f;
    if (fin) {
        const uint32_t h = (4 * e4) >> 8;
        if (csize > 1) {
            const float* sf = reinterpret_cast<const float*>(slots4);
            for (uint32_t b = 0; b < csize; ++b) {
                const float2 st = reinterpret_cast<const float2*>(sf + (b * SLOT4 + S4) * 4)[h];
                if (st.y > 0.0f) M = fmaxf(M, st.x);
            }
            o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (uint32_t b = 0; b < csize; ++b) {
                const float2 st = reinterpret_cast<const float2*>(sf + (b * SLOT4 + S4) * 4)[h];
                const float w = st.y > 0.0f ? expf(st.x - M) : 0.0f;
                const float4 v = slots4[b * SLOT4 + tid];
                L += st.y * w;
                o.x += v.x * w; o.y += v.y * w; o.z += v.z * w; o.w += v.w * w;
            }
        } else {
            const float2 st = reinterpret_cast<const float2*>(stat)[h];
            const bool live = st.y > 0.0f;
            M = live ? st.x : -INFINITY;
            L = live ? st.y : 0.0f;
            if (!live) o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        if (ncl > 1) {
            // the cluster's partial slice and, once per head, its (M, L)
            reinterpret_cast<float4*>(a.part + (size_t)ci * NH * 256)[e4] = o;
            if ((e4 & 63) == 0) { a.pstat[((size_t)ci * NH + h) * 2] = M; a.pstat[((size_t)ci * NH + h) * 2 + 1] = L; }
        } else {
            const float inv = 1.0f / L;
            o.x *= inv; o.y *= inv; o.z *= inv; o.w *= inv;
            reinterpret_cast<float4*>(a.att)[e4] = o;
            if (a.att_xq) reinterpret_cast<float4*>(accs + NH * 256)[e4] = o;
        }
    }
    if (ncl == 1 && a.att_xq) {
        // matvec limbs of this CTA's output blocks (32 floats each)
        __syncthreads();
        const uint32_t b0 = (csize > 1 ? crank * S4 : 0u) / 8, nb = nmine / 8;
        for (uint32_t bb = warp; bb < nb; bb += ATT_THREADS / 32)
            xq_prep_block(accs[NH * 256 + (b0 + bb) * 32 + lane], &a.att_xq[b0 + bb]);
    }
#ifdef XP_ATT_TRACE
    if (tid == 0) tr_[14] = globaltimer_ns();
#endif
    ATT_STAMP(8);
#ifdef XP_ATT_TRACE
    flush_();
    if (ncl == 1 && tid == 0) { __threadfence(); atomicAdd(&g_att_launch, 1u); }
#endif
    if (ncl == 1) return;
    // every CTA of every cluster wrote a slice: the last of them merges the
    // clusters
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(a.ticket, 1u) == nblk - 1) ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (mt) attn_merge_global<NH>(a.part, a.pstat, ncl, a.att, a.att_xq, accs);
    if (tid == 0) *a.ticket = 0;
#ifdef XP_ATT_TRACE
    ATT_STAMP(9);
    flush_();
    if (tid == 0) { __threadfence(); atomicAdd(&g_att_launch, 1u); }
#endif
}

}  // namespace xp
