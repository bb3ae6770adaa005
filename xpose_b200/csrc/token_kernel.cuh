// Persistent token kernel: one cooperative launch decodes `ntok` positions
// back to back (one per graph replay for decode_step(), up to 512 for a
// greedy generate() on one GPU).
//
// Grid = one CTA per SM, all co-resident; each CTA is 16 compute warps plus
// one producer warp. The reference's per-token op order
// (examples/llm/decode.cpp:1634-1780) runs as four steps per layer, then one
// LM-head step:
//
//   QKV  : residual + post-FFN norm of layer l-1 (or the embedding), attention
//          norm, then a K-split int4 matvec unit -> q|k|v sums. For l >= 1
//          the norm is split: the part of the input known a step early is
//          dotted during the previous barrier wait.
//   ATTN : QK-norm + RoPE, fp16 KV append (CTA 0), one contiguous chunk of the
//          attended window per CTA -> flash partials
//   O    : combine the flash partials of this CTA's 128-dim K range, o-proj
//          unit -> sums
//   GU   : residual + post-attention norm, FFN norm, gate|up units of 16
//          columns over all K -> GeGLU -> hb rows of this CTA, then the
//          down-proj of exactly those rows for every output column -> sums
//          (the CTA that makes an hb row is the one that consumes it, so the
//          down-proj needs no grid barrier of its own)
//   HEAD : residual + post-FFN + final norm, LM-head tiles, per-CTA argmax;
//          then the lowest-index maximum (greedy).
//
// Grid barriers follow QKV, O and GU; one follows ATTN only when the window
// has more than TK_LL_SPLITS splits, otherwise the partials reach O as
// flagged 8-byte words and polling them is the wait.
//
// Design rules of this kernel, each measured on B200:
//   * Code size. Every step's code runs once per layer and is fetched cold
//     every layer, so the layer loop is ONE phase machine (the norm prologue,
//     the limb prep and the 64-column tile loop exist once), and the timeline
//     instrumentation lives only in the TRACE instance: even predicated-off
//     instructions cost their fetch.
//   * Grid barriers (~0.75 us from the last arrival to the release) are the
//     dearest thing in a layer: three per layer at most.
//   * K-split sums go through int64 fixed-point accumulators (2^-32 units,
//     red.add): integer addition is order-independent, so the result is
//     deterministic, and a consumer loads one vector instead of every partial.
//   * Everything a step reads that does not depend on this token is in shared
//     memory before the step starts: weights live in unit-major images (one
//     bulk copy per CTA and step), per-step norm vectors are contiguous, the
//     KV rows a CTA attends to are staged ahead, per-layer facts are copied
//     once per launch. The producer warp issues all of those copies, so no
//     compute thread ever blocks on issuing one.
#pragma once
#include "attention.cuh"
#include "common.cuh"
#include "tk_primitives.cuh"
#include "xq.cuh"

namespace xp {

#ifndef XP_TK_THREADS
#define XP_TK_THREADS 512
#endif
constexpr int TK_THREADS = XP_TK_THREADS;    // compute threads
#ifndef XP_TK_FIX_PER_UNIT
#define XP_TK_FIX_PER_UNIT 0
#endif
constexpr bool TK_FIX_PER_UNIT = XP_TK_FIX_PER_UNIT;
constexpr int TK_WARPS = TK_THREADS / 32;
constexpr int TK_BLOCK = TK_THREADS + 32;      // + one producer warp that issues every bulk copy
constexpr int TK_MAXJ = (1536 + TK_THREADS - 1) / TK_THREADS;  // hidden and q|k|v width <= 1536
constexpr int TK_GROUPS = TK_THREADS / 128;  // 128-thread groups (attention P.V, O combine)
static_assert(TK_THREADS % 128 == 0 && TK_THREADS >= 256 && TK_THREADS <= 512, "compute threads");
constexpr int TK_NMB = 32;   // mbarriers
// "full" mbarriers: complete once per fill of a slot
constexpr int TK_MB_QKV = 0, TK_MB_O = 1, TK_MB_GU = 2, TK_MB_DOWN = 3, TK_MB_KV = 4;
constexpr int TK_MB_CQKV = 5, TK_MB_CATT = 6, TK_MB_CGU = 7, TK_MB_HEAD = 8;  // head ring: 8..15
constexpr int TK_MAX_RING = 8;
// "empty" mbarriers: the compute warps arrive once they are done reading a
// slot; the producer waits on them before refilling it
constexpr int TK_ME_QKV = 16, TK_ME_ATT = 17, TK_ME_O = 18, TK_ME_GU = 19, TK_ME_DOWN = 20, TK_ME_HEAD = 21;
constexpr int TK_MB_STAGE = 29;  // flash partials staged for the O combine
constexpr int TK_ME_HEADGO = 30;  // HEAD's input sums are loaded: the LM-head stream may start
static_assert(TK_ME_HEAD + TK_MAX_RING <= TK_MB_STAGE && TK_MB_STAGE < TK_NMB, "mbarrier count");
constexpr int TK_SPLIT_CAP = 128;
// Layers attended in at most TK_LL_SPLITS splits hand the flash partials to
// the O step as flagged words (no grid barrier between ATTN and O)
constexpr uint32_t TK_LL_SPLITS = 32;
constexpr uint32_t TK_XR = 2048;  // x1 kept in red[TK_XR .. TK_XR + H) from GU to the next QKV
constexpr int TK_HEAD_GROUPS = TK_WARPS / 4;  // LM-head tiles in flight per CTA (4 warps each)  // attention splits per layer (the O stage holds 512 B each)

// steps of the phase machine
constexpr uint32_t TK_S_QKV = 0, TK_S_ATTN = 1, TK_S_O = 2, TK_S_GU = 3, TK_S_HEAD = 5;
constexpr uint32_t TK_STEPS = 4;  // steps per layer

// Trace layout (u64 words, %globaltimer ns): [0] barriers, [1] start,
// [2k, 2k+1] CTA 0 arrive/leave of barrier k, [512 + 8k + i] CTA 0 marks in
// step k ([508] the previous launch's end, [509] this launch's end, [510] its
// entry), then per CTA c and barrier k < TK_TRACE_MAXBAR its arrive/leave at
// TK_TRACE_CTA + (c * TK_TRACE_MAXBAR + k) * 2.
constexpr uint32_t TK_TRACE_CTA = 512 + 8 * 1024, TK_TRACE_MAXBAR = 160, TK_TRACE_MAXCTA = 160;
constexpr uint32_t TK_TRACE_WORDS = TK_TRACE_CTA + 2 * TK_TRACE_MAXBAR * TK_TRACE_MAXCTA;

struct TkPhase {
    uint32_t units;      // units in the phase
    uint32_t nb;         // 32-row blocks per unit
    uint32_t cw;         // columns per unit
    uint32_t nmat;       // matrices per unit image (2 for gate|up)
    uint32_t ks;         // K chunks per column tile (unit = tile * ks + chunk)
    uint32_t img_bytes;  // bytes of one unit image
    uint32_t per_cta;    // most units any CTA takes
};

struct TkLayer {
    const unsigned char* qkv;
    const unsigned char* o;
    const unsigned char* gu;
    const unsigned char* down;
    const float* c_qkv;   // [post_ffn of layer l-1 (zeros for l = 0) | attn_norm]   2H floats
    const float* c_attn;  // [q_norm | k_norm]                                       512 floats
    const float* c_gu;    // [post_attn_norm | ffn_norm]                              2H floats
    __half* kc;
    __half* vc;
    uint32_t window;      // 0 = global layer
    uint32_t global;      // RoPE table: 1 = global theta, 0 = local
};


// Tensor-parallel LM head: every rank's best (value, index) lands in one slot
// of every rank's exchange buffer; flag = the launch counter + 1.
struct TkTpSlot {
    float val;
    uint32_t idx;
    uint32_t flag;
    uint32_t pad;
};
constexpr uint32_t TK_TP_MAX = 8;
// Two banks of TK_TP_MAX slots, chosen by the parity of the launch's flag. A
// peer can run at most one launch ahead of a rank that is still reading its
// entry (its next-but-one launch needs this rank's next entry), so the entry
// being read is never the one being rewritten.
constexpr uint32_t TK_TP_SLOTS = 2 * TK_TP_MAX;

struct TkArgs {
    const TkLayer* layers;
    uint32_t n_layers, H, F, QD, KVD, V;
    float eps, embed_scale, attn_scale, theta_global, theta_local;
    TkPhase qkv, o, gu, head;
    TkPhase down;         // down-proj rows of each gate|up unit: units = gu.units, img = H x (uint2 + bf16)
    const unsigned char* head_img;
    const float* c_head;  // [post_ffn of the last layer | final_norm]  2H floats
    const float* embed;
    float* x0;            // residual after the FFN sublayer (written in QKV)
    float* x1;            // residual after the attention sublayer (written in GU)
    long long* acc_qkv;   // [QD + 2 KVD] fixed-point q|k|v sums
    long long* acc_o;     // [H] fixed-point o-proj sums
    long long* acc_dn;    // [H] fixed-point down-proj sums
    float* att_part;      // [QD / 128][grid][128] flash partials, one 128-dim slice per O unit
    float* att_stat;      // [grid][4][2] (max, sum) per split and head
    unsigned long long* att_ll;     // [QD / 128][TK_LL_SPLITS][128] flagged partials
    unsigned long long* att_ll_st;  // [TK_LL_SPLITS][4][2] flagged (max, sum)
    float* logits;        // [V]
    float* am_val;        // [grid]
    uint32_t* am_idx;     // [grid]
    uint32_t* token;
    uint32_t* pos;
    uint32_t* hist;
    float* sample_out;
    uint64_t* bar;
    uint64_t* epoch;
    uint32_t* err;
    uint64_t* trace;      // optional timeline (XP_TRACE)
    int want_logits;
    int greedy;
    uint32_t ntok;        // tokens this launch decodes back to back (> 1: greedy, one rank)
    uint32_t chunk_max;   // most KV rows one CTA attends to
    uint32_t chunk_min;   // fewest KV rows per split
    uint32_t off_qkv, off_o, off_gu, off_down, off_kv, off_cqkv, off_catt, off_cgu, off_rope;
    uint32_t off_xn, off_xq, off_q, off_sc, off_red, off_misc;
    uint32_t off_lay;     // TkLayInfo per layer, copied to shared memory at launch
    uint32_t head_ring;   // LM-head ring buffers laid from off_ring on
    uint32_t off_ring;    // off_qkv, or off_o when the ring fits without the QKV slot
    int qkv_free;         // the ring leaves the QKV slot alone (it is refilled during HEAD)
    uint32_t head_u0, head_u1;          // this rank's LM-head units [u0, u1)
    uint32_t tp_rank, tp_world;         // tensor-parallel group of the LM head (world 1 = none)
    TkTpSlot* tp_slots[TK_TP_MAX];      // every rank's exchange buffer (peer mappings), TK_TP_SLOTS slots each
    uint32_t* tp_count;                 // [0] launches so far (the argmax exchange flag), [1] down-sum exchanges so far
    // FFN row shard (tensor parallel): this rank's gate|up units [gu_u0, gu_u1)
    // (16 GeGLU rows each) and the matching down-proj K rows. Each rank's
    // down-proj sums then cover only its rows; after the GU barrier every CTA
    // sends its stripe of them to each peer as flagged 32-bit halves
    // (dn_rx of the peer: [bank][sender][H][2] words, bank = layer parity)
    // and every reader adds the peers' parts to its own (int64, exact, so the
    // result is bit-identical to one GPU).
    uint32_t gu_u0, gu_u1;
    int ffn_shard;
    unsigned long long* dn_rx[TK_TP_MAX];  // every rank's receive area (peer mappings)
};
// words of the down-sum receive area: 2 banks x TK_TP_MAX senders x H x 2
constexpr size_t tk_dn_rx_words(uint32_t H) { return (size_t)2 * TK_TP_MAX * H * 2; }

// ---- helpers -------------------------------------------------------------------
// CTA barrier of the 16 compute warps only (named barrier 1); the producer
// warp never joins it.
XP_DEV void tk_sync() { asm volatile("bar.sync 1, %0;" ::"n"(TK_THREADS) : "memory"); }

XP_DEV float tk_block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    v = warp_sum(v);
    tk_sync();
    if (lane == 0) red[wid] = v;
    tk_sync();
    const float t = lane < TK_WARPS ? red[lane] : 0.0f;
    return warp_sum(t);
}
XP_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// generic-proxy global writes of other CTAs (ordered before this thread by an
// acquire) before this thread's async-proxy (bulk copy) reads
XP_DEV void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

// Fixed point in units of 2^-32: |v| < 2^31 is exact to 2^-33. An
// out-of-range (or NaN) value sets TK_ERR_RANGE and contributes 0.
XP_DEV long long tk_fix(float v, uint32_t* err) {
    const float s = v * 4294967296.0f;
    if (!(fabsf(s) < 9.2e18f)) {
        atomicOr(err, TK_ERR_RANGE);
        return 0;
    }
    return __float2ll_rn(s);
}
// tk_fix without a 64-bit conversion instruction: v * 2^32 is an integer
// already once |v * 2^32| >= 2^23 (its mantissa shifted left), and fits a
// 32-bit round-to-nearest conversion below that, so the result equals
// tk_fix's. Out of range (|v| >= 2^31, or NaN): 0 and *bad = true.
XP_DEV long long tk_fix_fast(float v, bool& bad) {
    const float f = v * 4294967296.0f;
    const uint32_t u = __float_as_uint(f), e = (u >> 23) & 0xFFu;
    if (e < 150u) return (long long)__float2int_rn(f);
    const bool ok = e < 190u;
    bad |= !ok;
    const long long m = (long long)((u & 0x7FFFFFu) | 0x800000u) << (ok ? e - 150u : 0u);
    return ok ? ((u >> 31) ? -m : m) : 0;
}
XP_DEV float tk_unfix(long long x) { return __ll2float_rn(x) * 2.3283064365386963e-10f; }
XP_DEV void red_add_s64(long long* p, long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

XP_DEV float tk_dot(const uint4 w, uint16_t s, const XBlk& X) {
    const int d = xq_dot(w, reinterpret_cast<const int4*>(X.w), X.bias);
    return (float)d * (X.f * __uint_as_float((uint32_t)s << 16));
}

// Down-proj of one gate|up unit: its 16 rows are one half of a KM4 block
// (words 0-1 of the uint4 hold rows 0-15, words 2-3 rows 16-31, and the half
// image keeps the right pair), dotted against limbs whose block carries the
// 16 values in rows 0-15 and zeros in rows 16-31.
XP_DEV float tk_dot_half(const uint2 w, uint16_t s, const XBlk& X) {
    int a0 = 0, a1 = 0, a2 = X.bias;
    const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int lo = (int)(ws[i] & 0x0F0F0F0Fu);
        const int hi = (int)((ws[i] >> 4) & 0x0F0F0F0Fu);
        a0 = __dp4a(lo, X.w[0][i], a0);
        a0 = __dp4a(hi, X.w[0][4 + i], a0);
        a1 = __dp4a(lo, X.w[1][i], a1);
        a1 = __dp4a(hi, X.w[1][4 + i], a1);
        a2 = __dp4a(lo, X.w[2][i], a2);
        a2 = __dp4a(hi, X.w[2][4 + i], a2);
    }
    const int d = (a0 * 128 + a1) * 128 + a2;
    return (float)d * (X.f * __uint_as_float((uint32_t)s << 16));
}

// A unit image of 64 columns over nb blocks: warp w takes blocks w, w+16, ...;
// lane handles columns lane and lane+32. Column sums -> red[0..64).
XP_DEV void tk_tile64(const unsigned char* img, uint32_t nb, const XBlk* xq, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint4* nib = reinterpret_cast<const uint4*>(img);
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(img + (size_t)nb * 64 * 16);
    float a0 = 0.0f, a1 = 0.0f;
    for (uint32_t b = warp; b < nb; b += TK_WARPS) {
        const XBlk& X = xq[b];
        a0 += tk_dot(nib[b * 64 + lane], sc[b * 64 + lane], X);
        a1 += tk_dot(nib[b * 64 + lane + 32], sc[b * 64 + lane + 32], X);
    }
    float* wr = red + 64;  // [16][64] warp partials
    wr[warp * 64 + lane] = a0;
    wr[warp * 64 + lane + 32] = a1;
    tk_sync();
    if (threadIdx.x < 64) {
        float s = 0.0f;
        const uint32_t nw = nb < (uint32_t)TK_WARPS ? nb : (uint32_t)TK_WARPS;
#pragma unroll 1
        for (uint32_t w = 0; w < nw; ++w) s += wr[w * 64 + threadIdx.x];
        red[threadIdx.x] = s;
    }
    tk_sync();
}

// Issue the bulk copies of this CTA's units of a phase into its slot
// (producer lane). Returns whether anything was armed on `bar`.
// Units [u0, u1) of the phase (all of them unless the phase is sharded): CTA
// c takes u0 + c, u0 + c + G, ...
__device__ __noinline__ bool tk_issue(const unsigned char* imgs, const TkPhase& P, unsigned char* slot, uint64_t* bar,
                                      uint32_t u0 = 0, uint32_t u1 = 0xFFFFFFFFu) {
    const uint32_t G = gridDim.x, c = blockIdx.x;
    if (u1 > P.units) u1 = P.units;
    if (u0 + c >= u1) return false;
    uint32_t n = 0;
    for (uint32_t u = u0 + c; u < u1; u += G) ++n;
    fence_proxy_async();
    mbar_expect_tx(bar, n * P.img_bytes);
    uint32_t i = 0;
    for (uint32_t u = u0 + c; u < u1; u += G, ++i)
        bulk_g2s(slot + (size_t)i * P.img_bytes, imgs + (size_t)u * P.img_bytes, P.img_bytes, bar);
    return true;
}

// ---- FFN shard: the down-proj sums across ranks ---------------------------------
XP_DEV void st_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
XP_DEV unsigned long long ld_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Send this CTA's stripe of the local down-proj sums (complete after the GU
// barrier) to every peer: element i as two flagged words (low, high half).
XP_DEV void tk_dn_send(const TkArgs& a, uint32_t bank, uint32_t flag) {
    const uint32_t G = gridDim.x, c = blockIdx.x, W = a.tp_world;
    const uint32_t per = (a.H + G - 1) / G;
    for (uint32_t t = threadIdx.x; t < per * W; t += TK_THREADS) {
        const uint32_t r = t % W, i = c * per + t / W;
        if (r == a.tp_rank || i >= a.H) continue;
        const unsigned long long v = (unsigned long long)a.acc_dn[i];
        unsigned long long* dst = a.dn_rx[r] + (((size_t)bank * TK_TP_MAX + a.tp_rank) * a.H + i) * 2;
        st_sys_u64(dst, ((unsigned long long)flag << 32) | (v & 0xFFFFFFFFull));
        st_sys_u64(dst + 1, ((unsigned long long)flag << 32) | (v >> 32));
    }
}
// The full down-proj sum of element i: the local part plus every peer's part
// (polled: the flag is the wait; bounded).
XP_DEV long long tk_dn(const TkArgs& a, uint32_t i, uint32_t bank, uint32_t flag) {
    long long v = a.acc_dn[i];
    if (!a.ffn_shard) return v;
    const unsigned long long* rx = a.dn_rx[a.tp_rank] + (size_t)bank * TK_TP_MAX * a.H * 2;
    for (uint32_t r = 0; r < a.tp_world; ++r) {
        if (r == a.tp_rank) continue;
        const unsigned long long* p = rx + ((size_t)r * a.H + i) * 2;
        unsigned long long lo, hi;
        uint32_t it = 0;
        do {
            lo = ld_sys_u64(p);
            hi = ld_sys_u64(p + 1);
            if (++it > TK_SPIN_LIMIT) { atomicOr(a.err, TK_ERR_TP_WAIT); break; }
        } while ((uint32_t)(lo >> 32) != flag || (uint32_t)(hi >> 32) != flag);
        v += (long long)(((hi & 0xFFFFFFFFull) << 32) | (lo & 0xFFFFFFFFull));
    }
    return v;
}
XP_DEV bool tk_issue_vec(const float* src, uint32_t n, unsigned char* slot, uint64_t* bar) {
    fence_proxy_async();
    mbar_expect_tx(bar, n * 4);
    bulk_g2s(slot, src, n * 4, bar);
    return true;
}

// The attended window of one layer and this CTA's split of it: chunks of at
// least chunk_min rows (a multiple of 8), at most TK_SPLIT_CAP splits.
struct TkWin {
    uint32_t kv_start, span, chunk, nsplit, j0, j1;
};
XP_DEV TkWin tk_window(uint32_t pos, uint32_t window, uint32_t chunk_min) {
    TkWin w;
    const uint32_t seq = pos + 1;
    w.kv_start = (window == 0 || seq <= window) ? 0 : seq - window;
    w.span = seq - w.kv_start;
    uint32_t ch = (w.span + TK_SPLIT_CAP - 1) / TK_SPLIT_CAP;
    ch = ch > chunk_min ? ch : chunk_min;
    w.chunk = (ch + 7) & ~7u;
    w.nsplit = (w.span + w.chunk - 1) / w.chunk;
    w.j0 = w.kv_start + min(blockIdx.x * w.chunk, w.span);
    w.j1 = w.kv_start + min((blockIdx.x + 1) * w.chunk, w.span);
    return w;
}

// What the compute warps need of a layer in every step, kept in shared
// memory: global loads there would each cost an L2 round trip after the grid
// barrier's acquire.
struct TkLayInfo {
    __half* kc;
    __half* vc;
    uint32_t window;
    uint32_t global;
    TkWin w;  // this position's window and this CTA's split of it (set per position)
};
constexpr uint32_t TK_MAX_LAYERS = 64;

// Stage the KV rows [j0, min(j1, pos)) of one layer (producer lane).
__device__ __noinline__ bool tk_issue_kv(const TkArgs& a, const TkLayer& L, uint32_t pos, unsigned char* kvs, uint64_t* bar) {
    const TkWin w = tk_window(pos, L.window, a.chunk_min);
    const uint32_t end = min(w.j1, pos);
    if (w.j1 - w.j0 > a.chunk_max) { atomicOr(a.err, TK_ERR_ATTN_CHUNK); return false; }
    if (end <= w.j0) return false;
    const uint32_t rows = end - w.j0;
    const uint32_t bytes = rows * a.KVD * 2;
    fence_proxy_async();
    mbar_expect_tx(bar, 2 * bytes);
    bulk_g2s(kvs, L.kc + (size_t)w.j0 * a.KVD, bytes, bar);
    bulk_g2s(kvs + (size_t)a.chunk_max * a.KVD * 2, L.vc + (size_t)w.j0 * a.KVD, bytes, bar);
    return true;
}

// ---------------------------------------------------------------------------------
// TRACE: record the phase timeline into a.trace (XP_TRACE); the production
// instance carries none of that code.
template <bool TRACE, bool TP>
__global__ void __launch_bounds__(TK_BLOCK, 1) token_kernel(const __grid_constant__ TkArgs a) {
    uint64_t* const trace = TRACE ? a.trace : nullptr;
    // tensor-parallel code exists only in the TP instance (code size: every
    // layer's code is fetched cold)
    const bool ffn = TP && a.ffn_shard;
    extern __shared__ __align__(128) unsigned char sm[];
    const uint32_t G = gridDim.x, c = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint64_t* mb = reinterpret_cast<uint64_t*>(sm + a.off_misc);
    float* red32 = reinterpret_cast<float*>(sm + a.off_misc + 8 * TK_NMB);
    float* xn = reinterpret_cast<float*>(sm + a.off_xn);
    XBlk* xq = reinterpret_cast<XBlk*>(sm + a.off_xq);
    float* red = reinterpret_cast<float*>(sm + a.off_red);
    unsigned char* s_qkv = sm + a.off_qkv;
    unsigned char* s_o = sm + a.off_o;
    unsigned char* s_gu = sm + a.off_gu;
    unsigned char* s_down = sm + a.off_down;
    unsigned char* s_kv = sm + a.off_kv;  // KV rows in ATTN, the flash-partial stage in O
    const float* cq = reinterpret_cast<const float*>(sm + a.off_cqkv);
    const float* ca = reinterpret_cast<const float*>(sm + a.off_catt);
    const float* cg = reinterpret_cast<const float*>(sm + a.off_cgu);
    float* rope = reinterpret_cast<float*>(sm + a.off_rope);  // [local | global][cos 128 | sin 128], inv freqs
    TkLayInfo* lay = reinterpret_cast<TkLayInfo*>(sm + a.off_lay);

    const uint32_t pos0 = *a.pos;
    const uint64_t base = *a.epoch;
    const uint32_t L = a.n_layers, H = a.H;
    const uint32_t QKVW = a.QD + 2 * a.KVD;
    uint32_t nbar = 0;
    uint32_t par = 0;  // parity bit per "full" mbarrier, identical in every compute thread

    if (trace && c == 0 && tid == 0) {
        trace[508] = trace[509];  // the previous launch's end
        trace[510] = globaltimer_ns();
    }
    if (tid == 0) {
        for (int i = 0; i < TK_NMB; ++i) mbar_init(&mb[i], 1);
        fence_mbar_init();
    }
    __syncthreads();

    // ---------------- producer warp: every weight/constant/KV copy ----------------
    // Each "full" mbarrier completes exactly once per fill, with the copy's
    // bytes or, when this CTA has nothing to load, with a plain arrive, so the
    // compute warps wait on every fill unconditionally. A slot is refilled
    // for layer l+1 once the compute warps have arrived on its "empty"
    // mbarrier at the grid barrier that closes the step reading it. The KV
    // slot doubles as the O step's stage, so its refill waits for O.
    if (warp == TK_WARPS) {
        if (lane != 0) return;
        uint32_t epar = 0;  // parity bit per "empty" mbarrier
        auto fill = [&](bool issued, int i) {
            if (!issued) mbar_arrive(&mb[i]);
        };
        auto wait_empty = [&](int i) {
            mbar_wait(&mb[i], (epar >> i) & 1u, a.err);
            epar ^= 1u << i;
        };
        const uint32_t ring_used = min(a.head_ring, (a.head_u1 - a.head_u0 + G - 1 - c) / G);
        for (uint32_t tk = 0; tk < a.ntok; ++tk) {
        const uint32_t pos = pos0 + tk;
        const TkLayer& L0 = a.layers[0];
        if (tk > 0) {
            // the previous token's last uses of every slot: the HEAD
            // constants, its last layer's ATTN, GU and O steps and the ring
            // (the QKV weights of layer 0 went in while the ring streamed)
            wait_empty(TK_ME_QKV);
            fill(tk_issue_vec(L0.c_qkv, 2 * H, (unsigned char*)cq, &mb[TK_MB_CQKV]), TK_MB_CQKV);
            wait_empty(TK_ME_ATT);
            fill(tk_issue_vec(L0.c_attn, 512, (unsigned char*)ca, &mb[TK_MB_CATT]), TK_MB_CATT);
            wait_empty(TK_ME_GU);
            fill(tk_issue_vec(L0.c_gu, 2 * H, (unsigned char*)cg, &mb[TK_MB_CGU]), TK_MB_CGU);
            wait_empty(TK_ME_O);
            for (uint32_t r = 0; r < ring_used; ++r) wait_empty(TK_ME_HEAD + r);
            if (!a.qkv_free) fill(tk_issue(L0.qkv, a.qkv, s_qkv, &mb[TK_MB_QKV]), TK_MB_QKV);
        } else {
            fill(tk_issue_vec(L0.c_qkv, 2 * H, (unsigned char*)cq, &mb[TK_MB_CQKV]), TK_MB_CQKV);
            fill(tk_issue(L0.qkv, a.qkv, s_qkv, &mb[TK_MB_QKV]), TK_MB_QKV);
            fill(tk_issue_vec(L0.c_attn, 512, (unsigned char*)ca, &mb[TK_MB_CATT]), TK_MB_CATT);
            fill(tk_issue_vec(L0.c_gu, 2 * H, (unsigned char*)cg, &mb[TK_MB_CGU]), TK_MB_CGU);
        }
        {
            fill(tk_issue_kv(a, L0, pos, s_kv, &mb[TK_MB_KV]), TK_MB_KV);
            fill(tk_issue(L0.o, a.o, s_o, &mb[TK_MB_O]), TK_MB_O);
            fill(tk_issue(L0.gu, a.gu, s_gu, &mb[TK_MB_GU], a.gu_u0, a.gu_u1), TK_MB_GU);
            fill(tk_issue(L0.down, a.down, s_down, &mb[TK_MB_DOWN], a.gu_u0, a.gu_u1), TK_MB_DOWN);
        }
        for (uint32_t l = 0; l + 1 < L; ++l) {
            const TkLayer& Ln = a.layers[l + 1];
            wait_empty(TK_ME_QKV);
            fill(tk_issue(Ln.qkv, a.qkv, s_qkv, &mb[TK_MB_QKV]), TK_MB_QKV);
            fill(tk_issue_vec(Ln.c_qkv, 2 * H, (unsigned char*)cq, &mb[TK_MB_CQKV]), TK_MB_CQKV);
            wait_empty(TK_ME_ATT);
            fill(tk_issue_vec(Ln.c_attn, 512, (unsigned char*)ca, &mb[TK_MB_CATT]), TK_MB_CATT);
            wait_empty(TK_ME_O);
            fill(tk_issue(Ln.o, a.o, s_o, &mb[TK_MB_O]), TK_MB_O);
            fill(tk_issue_kv(a, Ln, pos, s_kv, &mb[TK_MB_KV]), TK_MB_KV);
            wait_empty(TK_ME_GU);
            fill(tk_issue(Ln.gu, a.gu, s_gu, &mb[TK_MB_GU], a.gu_u0, a.gu_u1), TK_MB_GU);
            fill(tk_issue_vec(Ln.c_gu, 2 * H, (unsigned char*)cg, &mb[TK_MB_CGU]), TK_MB_CGU);
            wait_empty(TK_ME_DOWN);
            fill(tk_issue(Ln.down, a.down, s_down, &mb[TK_MB_DOWN], a.gu_u0, a.gu_u1), TK_MB_DOWN);
        }
        if (!a.want_logits) return;
        // last layer: the head constants once QKV is done with its slot, the
        // LM-head ring over every weight slot once DOWN is done with them
        wait_empty(TK_ME_QKV);
        fill(tk_issue_vec(a.c_head, 2 * H, (unsigned char*)cq, &mb[TK_MB_CQKV]), TK_MB_CQKV);
        wait_empty(TK_ME_DOWN);
        // start the 170 MB stream once HEAD's prologue has its sums: issued
        // earlier, it queues those L2 loads behind the HBM traffic
        wait_empty(TK_ME_HEADGO);
        uint32_t i = 0;
        for (uint32_t t = a.head_u0 + c; t < a.head_u1; t += G, ++i) {
            const uint32_t r = i & (a.head_ring - 1);  // head_ring: 4 or 8
            if (i >= a.head_ring) wait_empty(TK_ME_HEAD + r);
            fence_proxy_async();
            mbar_expect_tx(&mb[TK_MB_HEAD + r], a.head.img_bytes);
            bulk_g2s(sm + a.off_ring + (size_t)r * a.head.img_bytes, a.head_img + (size_t)t * a.head.img_bytes,
                     a.head.img_bytes, &mb[TK_MB_HEAD + r]);
        }
        // the next position's layer-0 QKV weights, into the slot the ring
        // leaves alone (its last reader, QKV of the last layer, is done)
        if (a.qkv_free && tk + 1 < a.ntok)
            fill(tk_issue(a.layers[0].qkv, a.qkv, s_qkv, &mb[TK_MB_QKV]), TK_MB_QKV);
        }  // token
        return;
    }

    // ---------------- compute warps ----------------
    auto wait_slot = [&](int i) {
        mbar_wait(&mb[i], (par >> i) & 1u, a.err);
        par ^= 1u << i;
    };

    const uint32_t base_g = (uint32_t)(base / G);  // barriers before this launch
    // FFN shard: flags of this launch's down-sum exchanges (one per layer;
    // a tensor-parallel launch decodes one position)
    // FFN shard: exchanges are numbered across launches (tp_count[1] counts
    // them), so consecutive exchanges alternate between the two banks and a
    // peer can never be more than one exchange ahead of a reader
    const uint32_t dn_flag0 = ffn ? a.tp_count[1] + 1u : 0u;
    const float inv_h = 1.0f / (float)H;
    __shared__ uint32_t s_tok;  // the input token of the next position (multi-token launches)
    // this CTA's unit coordinates, fixed for the launch (no divisions in the steps)
    __shared__ uint32_t s_qkv_b0, s_qkv_col0, s_o_kc, s_o_col0, s_gu_nu;
    if (tid == 0) {
        s_qkv_b0 = (c % a.qkv.ks) * a.qkv.nb;
        s_qkv_col0 = (c / a.qkv.ks) * 64;
        s_o_kc = c % a.o.ks;
        s_o_col0 = (c / a.o.ks) * 64;
        uint32_t nu = 0;
        for (uint32_t u = a.gu_u0 + c; u < a.gu_u1; u += G) ++nu;
        s_gu_nu = nu;
    }
    if ((uint32_t)tid < a.n_layers) {
        const TkLayer& Li = a.layers[tid];
        lay[tid] = TkLayInfo{Li.kc, Li.vc, Li.window, Li.global};
    }
    if (tid == 0) s_tok = *a.token;
    // RoPE inverse frequencies theta^(-2d/256), rounded once from double, once
    // per launch (rope[512..768): local 128 | global 128)
    if (tid < 256) rope[512 + tid] = rope_inv_freq(tid & 127, 256, (tid >> 7) ? a.theta_global : a.theta_local);
#pragma unroll 1
    for (uint32_t tk = 0; tk < a.ntok; ++tk) {
    const uint32_t pos = pos0 + tk;
    if ((uint32_t)tid < a.n_layers) lay[tid].w = tk_window(pos, lay[tid].window, a.chunk_min);
    // RoPE table for this position: angle pos * inv in fp32, sin/cos after an
    // exact reduction (llm_transformer.cl:158-179)
    if (tid < 256) {
        const uint32_t t = tid >> 7, d = tid & 127;
        const float inv = rope[512 + tid];
        float s, co;
        rope_sincos((float)pos * inv, &s, &co);
        rope[t * 256 + d] = co;
        rope[t * 256 + 128 + d] = s;
    }
    if (trace && c == 0 && tid == 0) trace[1] = globaltimer_ns();
    tk_sync();

#define TK_MARK(k) \
    if (trace && c == 0 && tid == 0) trace[512 + nbar * 8 + (k)] = globaltimer_ns();

    const uint32_t nstep = TK_STEPS * L + (a.want_logits ? 1u : 0u);
    float bv = -INFINITY;  // HEAD: this thread's best logit and its index (warp 0)
    uint32_t bi = 0xFFFFFFFFu;
    // split-norm QKV: dot(W, A) of the next layer's unit (warps 1..nb, made
    // during the GU barrier wait) and sum x1^2 of the residual it starts from
    float aq0 = 0.0f, aq1 = 0.0f, ss_x1 = 0.0f;
    float* xr = red + TK_XR;  // x1 (residual after attention), GU -> next QKV
#pragma unroll 1
    for (uint32_t step = 0; step < nstep; ++step) {
        const uint32_t l = step / TK_STEPS;
        const uint32_t k = l == L ? TK_S_HEAD : step - TK_STEPS * l;
        const TkLayInfo& Ly = lay[l < L ? l : L - 1];

        const bool split_qkv = k == TK_S_QKV && l > 0;
        // flag of this layer's flagged words: unique per launch and layer
        const uint32_t llf = base_g + nbar + 1;
        if (k == TK_S_QKV && c == G - 1) {
            // the o-proj sums were consumed by the previous layer's GU step;
            // the QKV -> ATTN barrier orders this before this layer's O red.adds
#pragma unroll 1
            for (uint32_t i = tid; i < H; i += TK_THREADS) a.acc_o[i] = 0;
        }
        if (split_qkv) {
            // ---------------- QKV of layers >= 1: split norm ----------------
            // The unit's input is x = sc2 (1 + w_attn) (x1 + s1 u) with
            // u = y (1 + w_post) and y the down-proj sums, so its dot is
            // sc2 [dot(W, A) + s1 dot(W, B)], A = (1 + w_attn) x1 (dotted during
            // the previous barrier wait) and B = (1 + w_attn) u. B's limbs need
            // only y, not the norms, so the B dot runs beside the block
            // reduction of the norm sums instead of after it.
            const TkPhase& P = a.qkv;
            const bool mine = c < P.units && warp >= 1 && (uint32_t)(warp - 1) < P.nb;
            // FFN shard: the previous layer's down-proj sums, completed by the peers' parts
            const uint32_t dn_flag = dn_flag0 + l - 1, dn_bank = dn_flag & 1u;
            if (ffn) tk_dn_send(a, dn_bank, dn_flag);
            const uint32_t bw = warp - 1, b0 = s_qkv_b0;
            float uv[TK_MAXJ], xb[TK_MAXJ];
            float sy = 0.0f, sbu = 0.0f, suu = 0.0f;
#pragma unroll
            for (int j = 0; j < TK_MAXJ; ++j) {
                const uint32_t i = tid + j * TK_THREADS;
                const float y = i < H ? tk_unfix(ffn ? tk_dn(a, i, dn_bank, dn_flag) : a.acc_dn[i]) : 0.0f;
                xb[j] = i < H ? xr[i] : 0.0f;
                uv[j] = i < H ? y * (1.0f + cq[i]) : 0.0f;
                sy += y * y;
                sbu += xb[j] * uv[j];
                suu += uv[j] * uv[j];
            }
            float bq0 = 0.0f, bq1 = 0.0f;
            if (mine) {
                const uint32_t i = (b0 + bw) * 32 + lane;
                const float yb = tk_unfix(ffn ? tk_dn(a, i, dn_bank, dn_flag) : a.acc_dn[i]);
                xq_prep_block(yb * (1.0f + cq[i]) * (1.0f + cq[H + i]), &xq[bw]);
                __syncwarp();
                const uint4* nib = reinterpret_cast<const uint4*>(s_qkv);
                const uint16_t* scl = reinterpret_cast<const uint16_t*>(s_qkv + (size_t)P.nb * 64 * 16);
                bq0 = tk_dot(nib[bw * 64 + lane], scl[bw * 64 + lane], xq[bw]);
                bq1 = tk_dot(nib[bw * 64 + lane + 32], scl[bw * 64 + lane + 32], xq[bw]);
            }
            TK_MARK(4)
            {
                const float q4 = reduce4(sy, sbu, suu, 0.0f);
                if ((lane & 7) == 0) red32[warp * 4 + (lane >> 3)] = q4;
            }
            tk_sync();
            TK_MARK(5)
            float t4 = 0.0f;
#pragma unroll
            for (int q = lane; q < 4 * TK_WARPS; q += 32) t4 += red32[q];
            t4 += __shfl_xor_sync(0xffffffffu, t4, 4);
            t4 += __shfl_xor_sync(0xffffffffu, t4, 8);
            t4 += __shfl_xor_sync(0xffffffffu, t4, 16);
            const float tx = __shfl_sync(0xffffffffu, t4, 0), ty = __shfl_sync(0xffffffffu, t4, 1);
            const float tz = __shfl_sync(0xffffffffu, t4, 2);
            const float s1 = rsqrtf(tx * inv_h + a.eps);
            const float sc2 = rsqrtf((ss_x1 + 2.0f * s1 * ty + s1 * s1 * tz) * inv_h + a.eps);
            if (c == 0) {
#pragma unroll
                for (int j = 0; j < TK_MAXJ; ++j) {
                    const uint32_t i = tid + j * TK_THREADS;
                    if (i < H) a.x0[i] = xb[j] + s1 * uv[j];
                }
            }
            float* wr = red;  // [nb][64] per-block partials
            if (mine) {
                wr[bw * 64 + lane] = aq0 + s1 * bq0;
                wr[bw * 64 + lane + 32] = aq1 + s1 * bq1;
            }
            tk_sync();
            if (c < P.units && tid < 64) {
                float sum = 0.0f;
#pragma unroll 1
                for (uint32_t w = 0; w < P.nb; ++w) sum += wr[w * 64 + tid];
                const uint32_t col = s_qkv_col0 + tid;
                if (col < QKVW) red_add_s64(&a.acc_qkv[col], tk_fix(sum * sc2, a.err));
            }
            TK_MARK(2)
        } else if (k == TK_S_QKV || k == TK_S_GU || k == TK_S_HEAD) {
            // ---------------- input of the step -> xn ----------------
            // r = base + rmsnorm_gemma(sum, w_post) (or the scaled embedding
            // row); x_out = r (CTA 0); xn = rmsnorm_gemma(r, w_pre)
            wait_slot(k == TK_S_GU ? TK_MB_CGU : TK_MB_CQKV);
            const float* wv = k == TK_S_GU ? cg : cq;
            const float* bsrc = k == TK_S_GU ? a.x0 : a.x1;
            const long long* acc = k == TK_S_GU ? a.acc_o : a.acc_dn;
            float* x_out = k == TK_S_QKV ? a.x0 : (k == TK_S_GU ? a.x1 : nullptr);
            // One block reduction for both norms: with u = y (1 + w_post) and
            // s1 = rsqrt(sum y^2 / H + eps), r = b + s1 u and
            // sum r^2 = sum b^2 + 2 s1 sum b u + s1^2 sum u^2.
            float rv[TK_MAXJ], uv[TK_MAXJ];
            float4 sums = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // y^2, b^2, b u, u^2
            const bool emb = k == TK_S_QKV && l == 0;
            if (emb) {
                const float* row = a.embed + (size_t)s_tok * H;
#pragma unroll
                for (int j = 0; j < TK_MAXJ; ++j) {
                    const uint32_t i = tid + j * TK_THREADS;
                    rv[j] = i < H ? row[i] * a.embed_scale : 0.0f;
                    uv[j] = 0.0f;
                    sums.y += rv[j] * rv[j];
                }
            } else {
                const bool head_dn = k == TK_S_HEAD && ffn;
                const uint32_t dn_flag = dn_flag0 + L - 1, dn_bank = dn_flag & 1u;
                if (head_dn) tk_dn_send(a, dn_bank, dn_flag);
#pragma unroll
                for (int j = 0; j < TK_MAXJ; ++j) {
                    const uint32_t i = tid + j * TK_THREADS;
                    const float y = i < H ? tk_unfix(head_dn ? tk_dn(a, i, dn_bank, dn_flag) : acc[i]) : 0.0f;
                    rv[j] = i < H ? bsrc[i] : 0.0f;
                    uv[j] = i < H ? y * (1.0f + wv[i]) : 0.0f;
                    sums.x += y * y;
                    sums.y += rv[j] * rv[j];
                    sums.z += rv[j] * uv[j];
                    sums.w += uv[j] * uv[j];
                }
            }
            // one reduction for the four sums: reduce4 leaves sum q in lanes
            // with (lane >> 3) == q; then lane l adds its sum l % 4 over the
            // warps l / 4, l / 4 + 8, ... and three shuffles finish it
            {
                const float q4 = reduce4(sums.x, sums.y, sums.z, sums.w);
                if ((lane & 7) == 0) red32[warp * 4 + (lane >> 3)] = q4;
            }
            if (k == TK_S_HEAD && tid == 0) mbar_arrive(&mb[TK_ME_HEADGO]);
            TK_MARK(4)
            tk_sync();
            TK_MARK(5)
            float t4 = 0.0f;
#pragma unroll
            for (int q = lane; q < 4 * TK_WARPS; q += 32) t4 += red32[q];
            t4 += __shfl_xor_sync(0xffffffffu, t4, 4);
            t4 += __shfl_xor_sync(0xffffffffu, t4, 8);
            t4 += __shfl_xor_sync(0xffffffffu, t4, 16);
            const float tx = __shfl_sync(0xffffffffu, t4, 0), ty = __shfl_sync(0xffffffffu, t4, 1);
            const float tz = __shfl_sync(0xffffffffu, t4, 2), tw = __shfl_sync(0xffffffffu, t4, 3);
            const float s1 = emb ? 0.0f : rsqrtf(tx * inv_h + a.eps);
            const float ssr = ty + 2.0f * s1 * tz + s1 * s1 * tw;  // sum r^2
            const float sc2 = rsqrtf(ssr * inv_h + a.eps);
            if (k == TK_S_GU) ss_x1 = ssr;
            // normalised input -> xn; the shared limb prep below reads it
#pragma unroll
            for (int j = 0; j < TK_MAXJ; ++j) {
                const uint32_t i = tid + j * TK_THREADS;
                if (i < H) {
                    const float r = rv[j] + s1 * uv[j];
                    if (x_out && c == 0) x_out[i] = r;
                    if (k == TK_S_GU) xr[i] = r;
                    else xn[i] = r * sc2 * (1.0f + wv[H + i]);
                }
            }
            if (k == TK_S_GU && s_gu_nu) {
                // GU's limbs straight from registers: block warp + 16 j holds
                // exactly this warp's element j, and the gate|up dot reads only
                // the blocks its own warp made (no xn round trip, no CTA barrier)
#pragma unroll
                for (int j = 0; j < TK_MAXJ; ++j) {
                    const uint32_t i = tid + j * TK_THREADS;
                    if (i < H) xq_prep_block((rv[j] + s1 * uv[j]) * sc2 * (1.0f + wv[H + i]), &xq[warp + j * TK_WARPS]);
                }
            }
            TK_MARK(6)
        } else if (k == TK_S_O) {
            // flash combine of this CTA's 128-dim slice over the splits: the
            // slice of every split arrives in one bulk copy while each warp
            // reduces the splits' statistics itself
            const TkWin w = Ly.w;
            const bool ll = w.nsplit <= TK_LL_SPLITS;
            if (c < a.o.units) {
                const uint32_t kc = s_o_kc, h = kc * 128 / 256;
                float* stage = reinterpret_cast<float*>(s_kv);  // [nsplit][128]
                float* mst = red + 1024 + TK_SPLIT_CAP;        // [nsplit][2] (max, sum) of head h
                if (ll) {
                    // no grid barrier: polling the flagged partials is the wait;
                    // warp w takes splits w and w + 16, loads in flight together
                    const uint32_t s0 = warp, s1 = warp + TK_WARPS;
                    const bool h0 = s0 < w.nsplit, h1 = s1 < w.nsplit;
                    const unsigned long long* p0 = a.att_ll + (kc * TK_LL_SPLITS + s0) * 128 + 4 * lane;
                    const unsigned long long* p1 = a.att_ll + (kc * TK_LL_SPLITS + s1) * 128 + 4 * lane;
                    const unsigned long long* q0 = a.att_ll_st + (s0 * 4 + h) * 2 + (lane & 1);
                    const unsigned long long* q1 = a.att_ll_st + (s1 * 4 + h) * 2 + (lane & 1);
                    ulonglong2 a0 = {}, a1 = {}, b0 = {}, b1 = {};
                    unsigned long long t0 = 0, t1 = 0;
                    uint32_t it = 0;
                    for (;;) {
                        bool ok = true;
                        if (h0) {
                            a0 = ld_flagged2(p0);
                            a1 = ld_flagged2(p0 + 2);
                            t0 = ld_flagged(q0);
                        }
                        if (h1) {
                            b0 = ld_flagged2(p1);
                            b1 = ld_flagged2(p1 + 2);
                            t1 = ld_flagged(q1);
                        }
                        if (h0) ok = flag_is(a0.x, llf) && flag_is(a0.y, llf) && flag_is(a1.x, llf) && flag_is(a1.y, llf) && flag_is(t0, llf);
                        if (h1) ok = ok && flag_is(b0.x, llf) && flag_is(b0.y, llf) && flag_is(b1.x, llf) && flag_is(b1.y, llf) && flag_is(t1, llf);
                        if (__all_sync(0xffffffffu, ok)) break;
                        if (++it > TK_SPIN_LIMIT) {
                            if (lane == 0) atomicOr(a.err, TK_ERR_LL_WAIT);
                            break;
                        }
                    }
                    if (h0) {
                        *reinterpret_cast<float4*>(stage + s0 * 128 + 4 * lane) =
                            make_float4(flag_val(a0.x), flag_val(a0.y), flag_val(a1.x), flag_val(a1.y));
                        if (lane < 2) mst[s0 * 2 + lane] = flag_val(t0);
                    }
                    if (h1) {
                        *reinterpret_cast<float4*>(stage + s1 * 128 + 4 * lane) =
                            make_float4(flag_val(b0.x), flag_val(b0.y), flag_val(b1.x), flag_val(b1.y));
                        if (lane < 2) mst[s1 * 2 + lane] = flag_val(t1);
                    }
                } else {
                    // after the grid barrier: one bulk copy of every split's slice,
                    // the statistics by plain loads
                    if (tid == 0) {
                        fence_proxy_async_all();
                        mbar_expect_tx(&mb[TK_MB_STAGE], w.nsplit * 512);
                        bulk_g2s(s_kv, a.att_part + (size_t)kc * G * 128, w.nsplit * 512, &mb[TK_MB_STAGE]);
                    }
                    if ((uint32_t)tid < 2 * w.nsplit) mst[tid] = a.att_stat[((size_t)(tid >> 1) * 4 + h) * 2 + (tid & 1)];
                    wait_slot(TK_MB_STAGE);
                }
                tk_sync();
                TK_MARK(5)
                float M = -INFINITY;
#pragma unroll 1
                for (uint32_t s_ = lane; s_ < w.nsplit; s_ += 32) M = fmaxf(M, mst[s_ * 2]);
                M = warp_max(M);
                float Ls = 0.0f;
                float* wts = red + 1024;  // [TK_SPLIT_CAP]
#pragma unroll 1
                for (uint32_t s_ = lane; s_ < w.nsplit; s_ += 32) {
                    const float e = expf(mst[s_ * 2] - M);
                    Ls += mst[s_ * 2 + 1] * e;
                    if (warp == 0) wts[s_] = e;
                }
                Ls = warp_sum(Ls);
                tk_sync();
                TK_MARK(4)
                // warp w < 4 combines dims 32w..32w+31 over every split and
                // makes that block's limbs straight from registers
                if (warp < 4) {
                    const uint32_t d = warp * 32 + lane;
                    float acc = 0.0f;
#pragma unroll 4
                    for (uint32_t s_ = 0; s_ < w.nsplit; ++s_) acc += stage[s_ * 128 + d] * wts[s_];
                    xq_prep_block(acc / Ls, &xq[warp]);
                }
                TK_MARK(6)
            }
        } else {
            // ================= ATTN =================
            const TkWin w = Ly.w;
            const bool ll = w.nsplit <= TK_LL_SPLITS;
            wait_slot(TK_MB_CATT);
            if (c < w.nsplit) {
                const uint32_t n = w.j1 - w.j0;
                float* qs = reinterpret_cast<float*>(sm + a.off_q);   // [4][256] pre-scaled
                __half* kn = reinterpret_cast<__half*>(qs + 4 * 256);  // [256]
                __half* vn = kn + 256;                                 // [256]
                float* sc = reinterpret_cast<float*>(sm + a.off_sc);   // [4][chunk_max]
                if (warp < 6) {
                    // warps 0-3: q heads, 4: k, 5: v, each loading its head's
                    // fixed-point sums itself; lane holds dims 4l..4l+3 and
                    // 128+4l..+3 (the rotate-half pairs)
                    const uint32_t off = warp < 4 ? warp * 256 : (warp == 4 ? a.QD : a.QD + a.KVD);
                    const longlong2* src = reinterpret_cast<const longlong2*>(a.acc_qkv + off + 4 * lane);
                    const longlong2 r0 = src[0], r1 = src[1], r2 = src[64], r3 = src[65];
                    float v[8] = {tk_unfix(r0.x), tk_unfix(r0.y), tk_unfix(r1.x), tk_unfix(r1.y),
                                  tk_unfix(r2.x), tk_unfix(r2.y), tk_unfix(r3.x), tk_unfix(r3.y)};
                    TK_MARK(0)
                    if (warp < 5) {
                        // QK-norm + rotate-half RoPE
                        const float* wq = (warp < 4 ? ca : ca + 256) + 4 * lane;
                        const float* cosT = rope + (Ly.global ? 256 : 0) + 4 * lane;
                        const float4 wl = *reinterpret_cast<const float4*>(wq);
                        const float4 wh = *reinterpret_cast<const float4*>(wq + 128);
                        const float4 cs = *reinterpret_cast<const float4*>(cosT);
                        const float4 sn = *reinterpret_cast<const float4*>(cosT + 128);
                        const float wlo[4] = {wl.x, wl.y, wl.z, wl.w}, whi[4] = {wh.x, wh.y, wh.z, wh.w};
                        const float co[4] = {cs.x, cs.y, cs.z, cs.w}, si[4] = {sn.x, sn.y, sn.z, sn.w};
                        float ss = 0.0f;
#pragma unroll
                        for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
                        ss = warp_sum(ss);
                        const float scl = rsqrtf(ss / 256.0f + a.eps);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float lo = v[i] * scl * (1.0f + wlo[i]);
                            const float hi = v[4 + i] * scl * (1.0f + whi[i]);
                            v[i] = lo * co[i] - hi * si[i];
                            v[4 + i] = lo * si[i] + hi * co[i];
                        }
                    }
                    if (warp < 4) {
                        // q in the key-lane order of the score loop: dim d sits at
                        // [(d & 7) >> 2][d >> 3][d & 3] of the head's 256 floats, so
                        // lane l's dims 8l..8l+7 are two conflict-free float4 loads
                        const float sq = a.attn_scale;
                        float* qh = qs + warp * 256 + (lane & 1) * 128 + (lane >> 1) * 4;
                        *reinterpret_cast<float4*>(qh) = make_float4(v[0] * sq, v[1] * sq, v[2] * sq, v[3] * sq);
                        *reinterpret_cast<float4*>(qh + 64) = make_float4(v[4] * sq, v[5] * sq, v[6] * sq, v[7] * sq);
                    } else {
                        const __half2 l01 = __floats2half2_rn(v[0], v[1]), l23 = __floats2half2_rn(v[2], v[3]);
                        const __half2 h01 = __floats2half2_rn(v[4], v[5]), h23 = __floats2half2_rn(v[6], v[7]);
                        uint2 lo, hi;
                        lo.x = *reinterpret_cast<const uint32_t*>(&l01);
                        lo.y = *reinterpret_cast<const uint32_t*>(&l23);
                        hi.x = *reinterpret_cast<const uint32_t*>(&h01);
                        hi.y = *reinterpret_cast<const uint32_t*>(&h23);
                        __half* dst = warp == 4 ? kn : vn;
                        reinterpret_cast<uint2*>(dst + 4 * lane)[0] = lo;
                        reinterpret_cast<uint2*>(dst + 128 + 4 * lane)[0] = hi;
                        if (c == 0) {
                            __half* cache = (warp == 4 ? Ly.kc : Ly.vc) + (size_t)pos * 256;
                            reinterpret_cast<uint2*>(cache + 4 * lane)[0] = lo;
                            reinterpret_cast<uint2*>(cache + 128 + 4 * lane)[0] = hi;
                        }
                    }
                }
                wait_slot(TK_MB_KV);
                tk_sync();
                TK_MARK(1)
                const __half* ks = reinterpret_cast<const __half*>(s_kv);
                const __half* vs = ks + (size_t)a.chunk_max * 256;
                // scores: a warp per key, lane l holds dims 8l..8l+7 of every
                // head's q in registers (loaded once per warp), so each key costs
                // one conflict-free row load; about two keys per warp keeps the
                // q loads few when the chunk is short
                {
                    const uint32_t nwk = min((uint32_t)TK_WARPS, max(1u, (n + 1) / 2));
                    if ((uint32_t)warp < nwk) {
                        float4 qa[4], qb[4];
#pragma unroll
                        for (int hh = 0; hh < 4; ++hh) {
                            qa[hh] = *reinterpret_cast<const float4*>(qs + hh * 256 + 4 * lane);
                            qb[hh] = *reinterpret_cast<const float4*>(qs + hh * 256 + 128 + 4 * lane);
                        }
#pragma unroll 1
                        for (uint32_t jj = warp; jj < n; jj += nwk) {
                            const uint32_t j = w.j0 + jj;
                            const uint4 raw = j == pos ? *reinterpret_cast<const uint4*>(kn + 8 * lane)
                                                       : *reinterpret_cast<const uint4*>(ks + (size_t)jj * 256 + 8 * lane);
                            const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
                            const float2 k0 = __half22float2(h2[0]), k1 = __half22float2(h2[1]);
                            const float2 k2 = __half22float2(h2[2]), k3 = __half22float2(h2[3]);
                            float s4[4];
#pragma unroll
                            for (int hh = 0; hh < 4; ++hh) {
                                float acc = qa[hh].x * k0.x;
                                acc = fmaf(qa[hh].y, k0.y, acc);
                                acc = fmaf(qa[hh].z, k1.x, acc);
                                acc = fmaf(qa[hh].w, k1.y, acc);
                                acc = fmaf(qb[hh].x, k2.x, acc);
                                acc = fmaf(qb[hh].y, k2.y, acc);
                                acc = fmaf(qb[hh].z, k3.x, acc);
                                acc = fmaf(qb[hh].w, k3.y, acc);
                                s4[hh] = acc;
                            }
                            const float tot = reduce4(s4[0], s4[1], s4[2], s4[3]);
                            if ((lane & 7) == 0) sc[(((lane >> 4) & 1) * 2 + ((lane >> 3) & 1)) * a.chunk_max + jj] = tot;
                        }
                    }
                }
                tk_sync();
                TK_MARK(2)
                if (warp < 4) {
                    float m = -INFINITY;
#pragma unroll 1
                    for (uint32_t jj = lane; jj < n; jj += 32) m = fmaxf(m, sc[warp * a.chunk_max + jj]);
                    m = warp_max(m);
                    float sum = 0.0f;
#pragma unroll 1
                    for (uint32_t jj = lane; jj < n; jj += 32) {
                        const float p = expf(sc[warp * a.chunk_max + jj] - m);
                        sc[warp * a.chunk_max + jj] = p;
                        sum += p;
                    }
                    sum = warp_sum(sum);
                    if (lane == 0) {
                        if (ll) {
                            st_flagged(a.att_ll_st + (c * 4 + warp) * 2, m, llf);
                            st_flagged(a.att_ll_st + (c * 4 + warp) * 2 + 1, sum, llf);
                        } else {
                            a.att_stat[((size_t)c * 4 + warp) * 2] = m;
                            a.att_stat[((size_t)c * 4 + warp) * 2 + 1] = sum;
                        }
                    }
                }
                tk_sync();
                {
                    const uint32_t dp = tid & 127, qr = tid >> 7;
                    float acc[4][2] = {};
#pragma unroll 2
                    for (uint32_t jj = qr; jj < n; jj += TK_GROUPS) {
                        const uint32_t j = w.j0 + jj;
                        const __half2 hv = j == pos ? reinterpret_cast<const __half2*>(vn)[dp]
                                                    : reinterpret_cast<const __half2*>(vs + (size_t)jj * 256)[dp];
                        const float2 vf = __half22float2(hv);
#pragma unroll
                        for (int hh = 0; hh < 4; ++hh) {
                            const float p = sc[hh * a.chunk_max + jj];
                            acc[hh][0] = fmaf(p, vf.x, acc[hh][0]);
                            acc[hh][1] = fmaf(p, vf.y, acc[hh][1]);
                        }
                    }
#pragma unroll
                    for (int hh = 0; hh < 4; ++hh) {
                        red[(qr * 4 + hh) * 256 + 2 * dp] = acc[hh][0];
                        red[(qr * 4 + hh) * 256 + 2 * dp + 1] = acc[hh][1];
                    }
                }
                tk_sync();
                // slice i / 128 of the partial goes where the O unit of that
                // K range reads it: att_part[slice][c][i % 128]
#pragma unroll 1
                for (uint32_t i = tid; i < 4 * 256; i += TK_THREADS)
                {
                    float t = 0.0f;
#pragma unroll
                    for (int q = 0; q < TK_GROUPS; ++q) t += red[q * 1024 + i];
                    if (ll)
                        st_flagged(a.att_ll + ((i >> 7) * TK_LL_SPLITS + c) * 128 + (i & 127), t, llf);
                    else
                        a.att_part[((size_t)(i >> 7) * G + c) * 128 + (i & 127)] = t;
                }
                TK_MARK(3)
            } else {
                wait_slot(TK_MB_KV);
            }
            // the down-proj sums were consumed by this layer's QKV step (and
            // the O -> GU barrier orders this before GU's red.adds)
            if (c == G - 1) {
#pragma unroll 1
                for (uint32_t i = tid; i < H; i += TK_THREADS) a.acc_dn[i] = 0;
            }
        }

        if (k != TK_S_ATTN && !split_qkv) {
            // ---------------- limbs of xn: one shared prep ----------------
            const TkPhase& P = k == TK_S_QKV ? a.qkv : k == TK_S_O ? a.o : k == TK_S_GU ? a.gu : a.head;
            const bool has = c < (k == TK_S_GU ? a.gu_u1 - a.gu_u0 : P.units);
            if (k != TK_S_GU) tk_sync();  // xn complete (O: its limbs, made by the combine)
            if (k != TK_S_O && k != TK_S_GU) {
                if (has) {
                    const uint32_t b0 = k == TK_S_QKV ? s_qkv_b0 : 0;
#pragma unroll 1
                    for (uint32_t b = warp; b < P.nb; b += TK_WARPS) xq_prep_block(xn[(b0 + b) * 32 + lane], &xq[b]);
                }
                // QKV (layer 0) and GU dot exactly the blocks each warp just
                // prepared (block b on warp b mod 16); the LM head's warp
                // groups read every block
                if (k == TK_S_HEAD) tk_sync();
                else __syncwarp();
            } else if (k == TK_S_GU) {
                __syncwarp();
            }
            TK_MARK(0)

            if (k == TK_S_GU) {
                // ---------------- gate|up units -> GeGLU -> hb -> down-proj ----------------
                wait_slot(TK_MB_GU);
                TK_MARK(1)
                if (has) {
                    const uint32_t nb = P.nb;
                    const uint32_t nu = s_gu_nu;
                    // warp w takes blocks w, w + 16, ... and holds that block's limbs
                    // in registers for every unit; lane = (matrix lane / 16,
                    // column lane % 16), so the limb loads are warp-wide broadcasts
                    // and a quarter-warp's nibble load is one contiguous 128 B
                    const uint32_t m = lane >> 4, col = lane & 15;
                    float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f;
#pragma unroll 1
                    for (uint32_t b = warp; b < nb; b += TK_WARPS) {
                        const XBlk X = xq[b];
#pragma unroll
                        for (uint32_t ui = 0; ui < 3; ++ui) {
                            if (ui < nu) {
                                const unsigned char* img = s_gu + (size_t)ui * P.img_bytes;
                                const uint32_t e = (m * nb + b) * 16 + col;
                                const float d = tk_dot(reinterpret_cast<const uint4*>(img)[e],
                                                       reinterpret_cast<const uint16_t*>(img + (size_t)2 * nb * 16 * 16)[e], X);
                                if (ui == 0) acc0 += d;
                                else if (ui == 1) acc1 += d;
                                else acc2 += d;
                            }
                        }
                    }
                    float* wp = red;  // [warp][unit][32]
                    wp[(warp * 3 + 0) * 32 + lane] = acc0;
                    wp[(warp * 3 + 1) * 32 + lane] = acc1;
                    wp[(warp * 3 + 2) * 32 + lane] = acc2;
                    tk_sync();
                    TK_MARK(2)
                    // warp ui: lanes 0-15 sum unit ui's gate partials, lanes 16-31
                    // its up partials; hb = GeGLU in lanes 0-15 (zeros above),
                    // whose limbs the same warp makes (rows 0-15 of a block)
                    if ((uint32_t)warp < nu) {
                        const uint32_t nw = nb < (uint32_t)TK_WARPS ? nb : (uint32_t)TK_WARPS;
                        float t = 0.0f;
#pragma unroll 4
                        for (uint32_t q = 0; q < nw; ++q) t += wp[(q * 3 + warp) * 32 + lane];
                        const float upv = __shfl_down_sync(0xffffffffu, t, 16);
                        xq_prep_block(lane < 16 ? gelu_tanh_ref(t) * upv : 0.0f, &xq[warp]);  // hb rows (c + warp G) * 16 + lane
                    }
                    tk_sync();
                }
                // down-proj of this CTA's hb rows for every output column
                wait_slot(TK_MB_DOWN);
                TK_MARK(3)
                if (has) {
                    const uint32_t nu = s_gu_nu;
                    const uint32_t ib = a.down.img_bytes;
                    // unit-outer: each unit's limbs are loaded once per thread.
                    // Each unit's partial is fixed-point on its own and the
                    // units are added as integers, so the sums do not depend
                    // on which CTA (or rank) holds which unit.
                    long long s[TK_MAXJ];
                    float f[TK_MAXJ];
                    bool bad = false;
#pragma unroll
                    for (int jj = 0; jj < TK_MAXJ; ++jj) {
                        s[jj] = 0;
                        f[jj] = 0.0f;
                    }
#pragma unroll
                    for (uint32_t ui = 0; ui < 3; ++ui) {
                        if (ui >= nu) break;
                        const XBlk& X = xq[ui];
                        const unsigned char* img = s_down + (size_t)ui * ib;
#pragma unroll
                        for (int jj = 0; jj < TK_MAXJ; ++jj) {
                            const uint32_t j = tid + jj * TK_THREADS;
                            if (j < H) {
                                const float d = tk_dot_half(reinterpret_cast<const uint2*>(img)[j],
                                                            reinterpret_cast<const uint16_t*>(img + (size_t)H * 8)[j], X);
                                if (TK_FIX_PER_UNIT || TP) s[jj] += tk_fix_fast(d, bad);
                                else f[jj] += d;
                            }
                        }
                    }
                    if (!(TK_FIX_PER_UNIT || TP)) {
#pragma unroll
                        for (int jj = 0; jj < TK_MAXJ; ++jj) s[jj] = tk_fix_fast(f[jj], bad);
                    }
                    if (bad) atomicOr(a.err, TK_ERR_RANGE);
#pragma unroll
                    for (int jj = 0; jj < TK_MAXJ; ++jj) {
                        const uint32_t j = tid + jj * TK_THREADS;
                        if (j < H) red_add_s64(&a.acc_dn[j], s[jj]);
                    }
                }
                // the q|k|v sums were consumed by this layer's ATTN step
                if (c == G - 1) {
#pragma unroll 1
                    for (uint32_t i = tid; i < QKVW; i += TK_THREADS) a.acc_qkv[i] = 0;
                }
            } else {
                if (k == TK_S_HEAD) {
                    // ---------------- LM head: ring of 64-column tiles, four at a time ----------------
                    // warp group g (4 warps) takes tiles i = g, g + 4, ... from ring
                    // slot i % head_ring (a multiple of 4, so a group's slots are its
                    // own), splits the blocks over its warps and reduces through a
                    // double-buffered [4][64] partial with a 128-thread named barrier
                    const uint32_t hu = a.head_u1 - a.head_u0;
                    const uint32_t ntile = hu > c ? (hu - c + G - 1) / G : 0;
                    const uint32_t grp = warp >> 2, gw = warp & 3;
                    TK_MARK(1)
#pragma unroll 1
                    for (uint32_t i = grp, it = 0; i < ntile; i += TK_HEAD_GROUPS, ++it) {
                        const uint32_t r = i & (a.head_ring - 1);  // head_ring: 4 or 8
                        wait_slot(TK_MB_HEAD + r);
                        const unsigned char* img = sm + a.off_ring + (size_t)r * P.img_bytes;
                        const uint4* nib = reinterpret_cast<const uint4*>(img);
                        const uint16_t* scl = reinterpret_cast<const uint16_t*>(img + (size_t)P.nb * 64 * 16);
                        float a0 = 0.0f, a1 = 0.0f;
                        for (uint32_t b = gw; b < P.nb; b += 4) {
                            const XBlk& X = xq[b];
                            a0 += tk_dot(nib[b * 64 + lane], scl[b * 64 + lane], X);
                            a1 += tk_dot(nib[b * 64 + lane + 32], scl[b * 64 + lane + 32], X);
                        }
                        float* wr = red + grp * 512 + (it & 1) * 256;
                        wr[gw * 64 + lane] = a0;
                        wr[gw * 64 + lane + 32] = a1;
                        asm volatile("bar.sync %0, 128;" ::"r"(2 + grp) : "memory");
                        if (gw == 0 && lane == 0) mbar_arrive(&mb[TK_ME_HEAD + r]);  // the producer refills it
                        if (gw < 2) {
                            const uint32_t col = gw * 32 + lane;
                            const float v = (wr[col] + wr[64 + col]) + (wr[128 + col] + wr[192 + col]);
                            const uint32_t t = a.head_u0 + c + i * G;
                            a.logits[(size_t)t * 64 + col] = v;
                            const uint32_t ix = t * 64 + col;
                            if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
                        }
                    }
                    TK_MARK(2)
                    // lowest-index maximum of the CTA
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                    }
                    if (lane == 0) {
                        red32[warp] = bv;
                        reinterpret_cast<uint32_t*>(red32)[TK_WARPS + warp] = bi;
                    }
                    tk_sync();
                    if (warp == 0) {
                        bv = lane < TK_WARPS ? red32[lane] : -INFINITY;
                        bi = lane < TK_WARPS ? reinterpret_cast<const uint32_t*>(red32)[TK_WARPS + lane] : 0xFFFFFFFFu;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                        }
                        if (lane == 0) { a.am_val[c] = bv; a.am_idx[c] = bi; }
                    }
                } else {
                    // ---------------- one 64-column tile: QKV, O ----------------
                    const int full = k == TK_S_QKV ? TK_MB_QKV : TK_MB_O;
                    long long* acc = k == TK_S_QKV ? a.acc_qkv : a.acc_o;
                    const uint32_t accw = k == TK_S_QKV ? QKVW : H;
                    const unsigned char* slot = k == TK_S_QKV ? s_qkv : s_o;
                    wait_slot(full);
                    TK_MARK(1)
                    if (has) {
                        tk_tile64(slot, P.nb, xq, red);
                        if (tid < 64) {
                            const uint32_t col = (k == TK_S_QKV ? s_qkv_col0 : s_o_col0) + tid;
                            if (col < accw) red_add_s64(&acc[col], tk_fix(red[tid], a.err));
                        }
                    }
                    TK_MARK(2)
                }
            }
        }

        // ---------------- grid barrier; the step's slots go back to the producer ----------------
        // (none after ATTN when its partials travel as flagged words)
        const bool gbar = k != TK_S_ATTN || Ly.w.nsplit > TK_LL_SPLITS;
        if (gbar) ++nbar;
        tk_sync();
        if (tid == 0) {
            if (trace && gbar) {
                const uint64_t t = globaltimer_ns();
                if (c == 0) trace[2 * nbar] = t;
                if (nbar < TK_TRACE_MAXBAR && c < TK_TRACE_MAXCTA)
                    trace[TK_TRACE_CTA + ((size_t)c * TK_TRACE_MAXBAR + nbar) * 2] = t;
            }
            if (gbar) red_release_add_u64(a.bar, 1ull);
            mbar_arrive(&mb[TK_ME_QKV + (k == TK_S_HEAD ? 0u : k)]);  // HEAD: its constants were in the QKV slot
            if (k == TK_S_GU) mbar_arrive(&mb[TK_ME_DOWN]);
        }
        if (k == TK_S_GU && l + 1 < L) {
            // while thread 0 waits: dot(W, A) of the next layer's QKV unit,
            // A = (1 + w_attn) x1 for this warp's block (warps 1..nb)
            wait_slot(TK_MB_CQKV);
            wait_slot(TK_MB_QKV);
            const TkPhase& P = a.qkv;
            const uint32_t bw = warp - 1;
            if (c < P.units && warp >= 1 && bw < P.nb) {
                const uint32_t i = (s_qkv_b0 + bw) * 32 + lane;
                xq_prep_block(xr[i] * (1.0f + cq[H + i]), &xq[bw]);
                __syncwarp();
                const uint4* nib = reinterpret_cast<const uint4*>(s_qkv);
                const uint16_t* scl = reinterpret_cast<const uint16_t*>(s_qkv + (size_t)P.nb * 64 * 16);
                aq0 = tk_dot(nib[bw * 64 + lane], scl[bw * 64 + lane], xq[bw]);
                aq1 = tk_dot(nib[bw * 64 + lane + 32], scl[bw * 64 + lane + 32], xq[bw]);
            }
        }
        if (tid == 0 && gbar) {
            const uint64_t target = base + (uint64_t)nbar * G;
            uint32_t it = 0;
            // acquire load + the closing bar.sync order every thread's later
            // reads after the other CTAs' released writes
            while (ld_acquire_u64(a.bar) < target) {
                if (++it > TK_SPIN_LIMIT) {
                    atomicOr(a.err, TK_ERR_GRID_BAR);
                    break;
                }
            }
            if (trace) {
                const uint64_t t = globaltimer_ns();
                if (c == 0) trace[2 * nbar + 1] = t;
                if (nbar < TK_TRACE_MAXBAR && c < TK_TRACE_MAXCTA)
                    trace[TK_TRACE_CTA + ((size_t)c * TK_TRACE_MAXBAR + nbar) * 2 + 1] = t;
            }
        }
        tk_sync();
    }

    // ---------------- sample (greedy): lowest-index maximum over the CTAs ----------------
    if (a.want_logits) {
        // one CTA publishes the token; with more tokens to go every CTA picks
        // it too (the same lowest-index maximum) for the next embedding row
        if (a.greedy && warp == 0 && (c == 0 || a.ntok > 1)) {
            float v = -INFINITY;
            uint32_t ix = 0xFFFFFFFFu;
            for (uint32_t p = lane; p < G; p += 32) {
                const float pv = a.am_val[p];
                const uint32_t pi = a.am_idx[p];
                if (pv > v || (pv == v && pi < ix)) { v = pv; ix = pi; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, ix, o);
                if (ov > v || (ov == v && oi < ix)) { v = ov; ix = oi; }
            }
            if (TP && a.tp_world > 1) {
                // lane r publishes this rank's best into rank r's slot
                // [tp_rank] over NVLink, then waits for rank r's entry in our
                // own buffer (bounded) and the warp keeps the lowest-index max
                const uint32_t flag = *a.tp_count + 1;
                const uint32_t bank = (flag & 1u) * TK_TP_MAX;
                if ((uint32_t)lane < a.tp_world) {
                    TkTpSlot* dst = a.tp_slots[lane] + bank + a.tp_rank;
                    dst->val = v;
                    dst->idx = ix;
                    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(&dst->flag), "r"(flag) : "memory");
                }
                float rv = -INFINITY;
                uint32_t ri = 0xFFFFFFFFu;
                if ((uint32_t)lane < a.tp_world) {
                    const TkTpSlot* src = a.tp_slots[a.tp_rank] + bank + lane;
                    uint32_t f = 0, it = 0;
                    do {
                        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(&src->flag) : "memory");
                        if (++it > TK_SPIN_LIMIT) { atomicOr(a.err, TK_ERR_TP_WAIT); break; }
                    } while (f != flag);
                    rv = *reinterpret_cast<const volatile float*>(&src->val);
                    ri = *reinterpret_cast<const volatile uint32_t*>(&src->idx);
                }
                v = rv;
                ix = ri;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                    const uint32_t oi = __shfl_xor_sync(0xffffffffu, ix, o);
                    if (ov > v || (ov == v && oi < ix)) { v = ov; ix = oi; }
                }
                if (lane == 0) *a.tp_count = flag;
            }
            if (lane == 0) {
                if (ix == 0xFFFFFFFFu) ix = 0;
                s_tok = ix;
                if (c == 0) {
                    *a.token = ix;
                    if (a.sample_out) { a.sample_out[0] = (float)ix; a.sample_out[1] = v; }
                    *a.pos = pos + 1;
                    if (a.hist) a.hist[pos + 1] = ix;
                }
            }
        }
    } else if (c == 0 && tid == 0) {
        *a.pos = pos + 1;
    }
    tk_sync();  // s_tok before the next position's embedding row
    }  // token
    if (c == 0 && tid == 0) {
        *a.epoch = base + (uint64_t)nbar * G;
        // this launch's down-sum exchanges: one per layer consumed (L - 1, or
        // L when HEAD ran); every CTA read tp_count[1] before the first barrier
        if (ffn) a.tp_count[1] += a.want_logits ? L : L - 1;
        if (trace) {
            trace[0] = nbar;
            trace[509] = trace[2 * nbar + 2] = globaltimer_ns();
        }
    }
#undef TK_MARK
}

// ---- load-time repack: reference KM4 + bf16-scale planes -> unit images ----------------
// Unit u of a phase holds, for matrices m < nmat, nibbles[m][b][c] (uint4)
// then scales[m][b][c] (bf16) for blocks b < nb and columns c < cw. The
// dequantised weight of every (k, j) is unchanged: same nibble, same bf16.
struct RepackArgs {
    const uint4* words;    // reference nibble plane
    const uint32_t* sc;    // reference scale plane (uint2 per quad and column)
    uint32_t rows, cols;
    unsigned char* dst;
    uint32_t img_bytes, cw, nb, nmat, mat, ks, tile0;
};
__global__ void repack_units_kernel(const RepackArgs r) {
    const uint32_t nblk = r.rows / 32;
    const uint64_t total = (uint64_t)nblk * r.cols;
    for (uint64_t id = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; id < total;
         id += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t j = (uint32_t)(id % r.cols), b = (uint32_t)(id / r.cols);
        const uint4 w = r.words[((size_t)(j / 64) * nblk + b) * 64 + (j % 64)];
        const uint32_t sw = r.sc[((size_t)(b / 4) * r.cols + j) * 2 + ((b % 4) >> 1)];
        const uint16_t s = (uint16_t)((b & 1) ? (sw >> 16) : (sw & 0xFFFFu));
        const uint32_t u = (r.tile0 + j / r.cw) * r.ks + b / r.nb;
        const uint32_t bl = b % r.nb, cl = j % r.cw;
        unsigned char* img = r.dst + (size_t)u * r.img_bytes;
        const size_t e = ((size_t)r.mat * r.nb + bl) * r.cw + cl;
        reinterpret_cast<uint4*>(img)[e] = w;
        reinterpret_cast<uint16_t*>(img + (size_t)r.nmat * r.nb * r.cw * 16)[e] = s;
    }
}

// Down-proj images for the fused GU step: gate|up unit U (rows 16U..16U+15
// of the [rows = F][cols = H] down matrix, one half of KM4 block U / 2) gets
// [cols] uint2 (the half's two nibble words) then [cols] bf16 (the block's
// scale). The nibbles and scales are the reference's, unchanged.
__global__ void repack_half_kernel(const uint4* words, const uint32_t* sc, uint32_t rows, uint32_t cols,
                                   unsigned char* dst) {
    const uint32_t nblk = rows / 32;
    const uint64_t total = (uint64_t)(rows / 16) * cols;
    for (uint64_t id = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; id < total;
         id += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t j = (uint32_t)(id % cols), U = (uint32_t)(id / cols), b = U / 2;
        const uint4 w = words[((size_t)(j / 64) * nblk + b) * 64 + (j % 64)];
        const uint32_t sw = sc[((size_t)(b / 4) * cols + j) * 2 + ((b % 4) >> 1)];
        unsigned char* img = dst + (size_t)U * cols * 10;
        reinterpret_cast<uint2*>(img)[j] = (U & 1) ? make_uint2(w.z, w.w) : make_uint2(w.x, w.y);
        reinterpret_cast<uint16_t*>(img + (size_t)cols * 8)[j] = (uint16_t)((b & 1) ? (sw >> 16) : (sw & 0xFFFFu));
    }
}

}  // namespace xp
