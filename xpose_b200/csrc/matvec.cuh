// int4 KM4 + bf16-scale matvec for sm_100a, with fused prologues/epilogues.
//
// Weight layout is the reference's, unchanged (examples/llm/decode.cpp:157-229,
// kernels/llm_matvec.cl:37-50 and :380-405): nibble plane uint4[(g*nblk + b)*64
// + t] for column j = 64g + t and 32-row block b; scale plane uint2[(b/4)*cols
// + j], four bf16 block scales per uint2. For one 64-column group the nibbles
// of a block are 1 KB contiguous, so a warp reading columns t and t+32 of a
// block issues two fully coalesced 512-byte LDG.128s.
//
// Work decomposition: a TILE is one 64-column group of one matrix (two
// matrices for the GeGLU epilogue, gate and up of the same columns). A tile's
// K range may be split across a thread-block cluster of `ksplit` CTAs; their
// partial column sums are reduced through distributed shared memory by the
// cluster's rank-0 CTA in a fixed order, so results are deterministic.
// Inside a CTA the 8 warps take the tile's (unit, block) items round robin and
// keep PF items of loads in flight per lane.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"
#include "xq.cuh"

namespace xp {

enum MvPro : int {
    PRO_XQ = 0,          // activation limbs precomputed in global memory (xq)
    PRO_PLAIN = 1,       // fp32 x, converted in the CTA
    PRO_NORM = 2,        // x = rmsnorm_gemma(in, w_pre)
    PRO_RESID_NORM = 3,  // r = x + rmsnorm_gemma(y, w_post); x_out = r; x = rmsnorm_gemma(r, w_pre)
    PRO_EMBED_NORM = 4,  // r = embed[token] * embed_scale; x_out = r; x = rmsnorm_gemma(r, w_pre)
};
enum MvEpi : int {
    EPI_STORE = 0,   // out[j] = y_j
    EPI_GEGLU = 1,   // hb[j] = gelu_tanh(gate_j) * up_j (+ hb limbs)
    EPI_ARGMAX = 2,  // out[j] = y_j and per-tile (max, lowest index)
    EPI_PARTIAL = 3, // out[crank*cols + j] = this CTA's K-range partial (no reduction)
};

struct MvMat {
    const uint4* wq;
    const uint2* sc;
    float* out;
    uint32_t cols;
    uint32_t tile0;  // first tile index of this matrix
};

struct MvArgs {
    MvMat m[3];
    int nmat;
    uint32_t ntiles;   // total tiles (groups) over all matrices; GEGLU: groups of m[0]
    uint32_t K;        // input length (rows), multiple of 128
    uint32_t ksplit;   // CTAs per tile (cluster size); 1 = persistent over tiles
    int pro, epi;
    const XBlk* xq_in;      // PRO_XQ
    const float* x;         // PLAIN/NORM input, RESID residual stream
    const float* y;         // RESID sublayer output
    const float* w_post;
    const float* w_pre;
    float* x_out;           // RESID/EMBED new residual stream (tile 0 writes)
    float eps;
    const float* embed;     // EMBED
    const uint32_t* token;  // EMBED (device-resident token id)
    float embed_scale;
    float* hb;              // GEGLU output
    XBlk* xq_out;           // GEGLU: limbs of hb for the next matvec (may be null)
    float* am_val;          // ARGMAX partials, one per tile
    uint32_t* am_idx;
    uint32_t hidden;        // length of x/y for the norm prologues (== K)
    int quad_split;         // K ranges aligned to groups of 4 blocks (reference split-k)
};

constexpr int MV_THREADS = 256;
constexpr int MV_WARPS = MV_THREADS / 32;
constexpr int MV_PF = 4;

// Shared memory: [xbuf: K floats (norm prologues) | xq: nbc XBlk | red: warps*2*64 floats | misc]
struct MvSmem {
    static size_t bytes(const MvArgs& a, uint32_t nbc_max) {
        size_t s = 0;
        if (a.pro >= PRO_NORM) s += (size_t)a.K * 4;
        s = (s + 127) & ~(size_t)127;
        s += (size_t)nbc_max * sizeof(XBlk);
        s += (size_t)MV_WARPS * 2 * 64 * 4;  // warp partials
        s += 2 * 64 * 4;                     // CTA result (read by the cluster leader)
        s += 64 * 4;                         // block_sum scratch
        return s;
    }
};

// Which matrix a tile belongs to (non-GEGLU, tiles are laid out matrix after matrix).
XP_DEV int mv_mat_of(const MvArgs& a, uint32_t tile) {
    int m = 0;
    if (a.nmat > 1 && tile >= a.m[1].tile0) m = 1;
    if (a.nmat > 2 && tile >= a.m[2].tile0) m = 2;
    return m;
}

XP_DEV void mv_load_item(const MvArgs& a, uint32_t tile, int u, uint32_t b, int lane, uint4& w0,
                         uint4& w1, uint2& s0, uint2& s1) {
    const MvMat& M = a.m[a.epi == EPI_GEGLU ? u : mv_mat_of(a, tile)];
    const uint32_t nblk = a.K >> 5;
    const uint32_t g = tile - M.tile0;
    const uint4* p = M.wq + ((size_t)g * nblk + b) * 64 + lane;
    w0 = __ldg(p);
    w1 = __ldg(p + 32);
    const uint2* q = M.sc + (size_t)(b >> 2) * M.cols + (size_t)g * 64 + lane;
    s0 = __ldg(q);
    s1 = __ldg(q + 32);
}

// rmsnorm_gemma over `n` values in smem (in place): v * rsqrt(mean(v^2)+eps) * (1+w).
XP_DEV void smem_rmsnorm(float* v, const float* w, uint32_t n, float eps, float* red) {
    float ss = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += v[i] * v[i];
    ss = block_sum(ss, red);
    const float scale = rsqrtf(ss / (float)n + eps);
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) v[i] = v[i] * scale * (1.0f + w[i]);
    __syncthreads();
}

__global__ void __launch_bounds__(MV_THREADS, 2) mv_kernel(const MvArgs a) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t nblk = a.K >> 5;
    const uint32_t ksplit = a.ksplit;
    const uint32_t crank = ksplit > 1 ? (blockIdx.x % ksplit) : 0;
    const uint32_t per = a.quad_split ? 4 * ((nblk / 4 + ksplit - 1) / ksplit) : (nblk + ksplit - 1) / ksplit;
    const uint32_t kb0 = min(crank * per, nblk);
    const uint32_t kb1 = min(kb0 + per, nblk);
    const uint32_t nbc = kb1 - kb0;
    const int U = a.epi == EPI_GEGLU ? 2 : 1;

    size_t off = 0;
    float* xbuf = reinterpret_cast<float*>(smem);
    if (a.pro >= PRO_NORM) off += (size_t)a.K * 4;
    off = (off + 127) & ~(size_t)127;
    XBlk* xq = reinterpret_cast<XBlk*>(smem + off);
    off += (size_t)per * sizeof(XBlk);
    float* wred = reinterpret_cast<float*>(smem + off);
    off += (size_t)MV_WARPS * 2 * 64 * 4;
    float* cres = reinterpret_cast<float*>(smem + off);
    off += 2 * 64 * 4;
    float* red = reinterpret_cast<float*>(smem + off);

    uint32_t tile = ksplit > 1 ? blockIdx.x / ksplit : blockIdx.x;
    // cluster mode: one tile per cluster (the stride ends the loop after it)
    const uint32_t tstride = ksplit > 1 ? a.ntiles : gridDim.x;

    // ---- prefetch this CTA's first weights before waiting on the producer ----
    const uint32_t nitems = (uint32_t)U * nbc;
    uint32_t cnt = nitems > (uint32_t)warp ? (nitems - warp + MV_WARPS - 1) / MV_WARPS : 0;
    uint4 bw0[MV_PF], bw1[MV_PF];
    uint2 bs0[MV_PF], bs1[MV_PF];
    if (tile < a.ntiles) {
#pragma unroll
        for (int p = 0; p < MV_PF; ++p)
            if ((uint32_t)p < cnt) {
                const uint32_t it = warp + MV_WARPS * p;
                mv_load_item(a, tile, (int)(it / nbc), kb0 + it % nbc, lane, bw0[p], bw1[p], bs0[p], bs1[p]);
            }
    }

    // Let the next kernel's CTAs launch and start their own weight prefetch
    // as soon as every CTA of this grid is resident.
    pdl_launch_dependents();
    pdl_wait();

    // ---- prologue: build this CTA's activation limbs ---------------------------
    if (a.pro == PRO_XQ) {
        const int4* src = reinterpret_cast<const int4*>(a.xq_in + kb0);
        int4* dst = reinterpret_cast<int4*>(xq);
        for (uint32_t i = tid; i < nbc * 8; i += MV_THREADS) dst[i] = src[i];
        __syncthreads();
    } else if (a.pro == PRO_PLAIN) {
        for (uint32_t bb = warp; bb < nbc; bb += MV_WARPS)
            xq_prep_block(a.x[(size_t)(kb0 + bb) * 32 + lane], &xq[bb]);
        __syncthreads();
    } else {
        const uint32_t n = a.hidden;
        if (a.pro == PRO_NORM) {
            for (uint32_t i = tid; i < n; i += MV_THREADS) xbuf[i] = a.x[i];
        } else if (a.pro == PRO_RESID_NORM) {
            for (uint32_t i = tid; i < n; i += MV_THREADS) xbuf[i] = a.y[i];
            __syncthreads();
            smem_rmsnorm(xbuf, a.w_post, n, a.eps, red);
            for (uint32_t i = tid; i < n; i += MV_THREADS) xbuf[i] = a.x[i] + xbuf[i];
        } else {  // PRO_EMBED_NORM
            const uint32_t t = *a.token;
            const float* row = a.embed + (size_t)t * n;
            for (uint32_t i = tid; i < n; i += MV_THREADS) xbuf[i] = row[i] * a.embed_scale;
        }
        __syncthreads();
        if ((a.pro == PRO_RESID_NORM || a.pro == PRO_EMBED_NORM) && blockIdx.x == 0 && a.x_out)
            for (uint32_t i = tid; i < n; i += MV_THREADS) a.x_out[i] = xbuf[i];
        smem_rmsnorm(xbuf, a.w_pre, n, a.eps, red);
        for (uint32_t bb = warp; bb < nbc; bb += MV_WARPS)
            xq_prep_block(xbuf[(kb0 + bb) * 32 + lane], &xq[bb]);
        __syncthreads();
    }

    // ---- main loop over tiles ------------------------------------------------------
    for (; tile < a.ntiles; tile += tstride) {
        float acc00 = 0.f, acc01 = 0.f, acc10 = 0.f, acc11 = 0.f;
        for (uint32_t i0 = 0; i0 < cnt; i0 += MV_PF) {
#pragma unroll
            for (int p = 0; p < MV_PF; ++p) {
                const uint32_t i = i0 + p;
                if (i < cnt) {
                    const uint32_t it = warp + MV_WARPS * i;
                    const int u = (int)(it / nbc);
                    const uint32_t bl = it % nbc;
                    const uint32_t b = kb0 + bl;
                    const XBlk& X = xq[bl];
                    const int4* Xw = reinterpret_cast<const int4*>(X.w);
                    const int bias = X.bias;
                    const float f = X.f;
                    const int d0 = xq_dot(bw0[p], Xw, bias);
                    const int d1 = xq_dot(bw1[p], Xw, bias);
                    const uint32_t sw0 = (b & 2) ? bs0[p].y : bs0[p].x;
                    const uint32_t sw1 = (b & 2) ? bs1[p].y : bs1[p].x;
                    const float ws0 = (b & 1) ? bf16_hi(sw0) : bf16_lo(sw0);
                    const float ws1 = (b & 1) ? bf16_hi(sw1) : bf16_lo(sw1);
                    if (u == 0) {
                        acc00 = fmaf((float)d0, f * ws0, acc00);
                        acc01 = fmaf((float)d1, f * ws1, acc01);
                    } else {
                        acc10 = fmaf((float)d0, f * ws0, acc10);
                        acc11 = fmaf((float)d1, f * ws1, acc11);
                    }
                    const uint32_t inext = i + MV_PF;
                    if (inext < cnt) {
                        const uint32_t itn = warp + MV_WARPS * inext;
                        mv_load_item(a, tile, (int)(itn / nbc), kb0 + itn % nbc, lane, bw0[p], bw1[p],
                                     bs0[p], bs1[p]);
                    }
                }
            }
        }
        // prefetch the next tile (persistent mode) before reducing this one
        const uint32_t ntile = tile + tstride;
        if (ksplit == 1 && ntile < a.ntiles) {
#pragma unroll
            for (int p = 0; p < MV_PF; ++p)
                if ((uint32_t)p < cnt) {
                    const uint32_t it = warp + MV_WARPS * p;
                    mv_load_item(a, ntile, (int)(it / nbc), kb0 + it % nbc, lane, bw0[p], bw1[p], bs0[p], bs1[p]);
                }
        }

        // ---- reduce: warps -> CTA -> cluster ----------------------------------------
        wred[(warp * 2 + 0) * 64 + lane] = acc00;
        wred[(warp * 2 + 0) * 64 + lane + 32] = acc01;
        wred[(warp * 2 + 1) * 64 + lane] = acc10;
        wred[(warp * 2 + 1) * 64 + lane + 32] = acc11;
        __syncthreads();
        if (tid < U * 64) {
            const int u = tid >> 6, c = tid & 63;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < MV_WARPS; ++w) s += wred[(w * 2 + u) * 64 + c];
            cres[u * 64 + c] = s;
        }
        if (ksplit > 1 && a.epi != EPI_PARTIAL) {
            cg::cluster_group cl = cg::this_cluster();
            cl.sync();
            if (crank == 0 && tid < U * 64) {
                float s = 0.0f;
                for (uint32_t r = 0; r < ksplit; ++r) s += cl.map_shared_rank(cres, r)[tid];
                cres[tid] = s;
            }
            cl.sync();
            if (crank != 0) return;
        }
        __syncthreads();

        // ---- epilogue ---------------------------------------------------------------
        if (a.epi == EPI_GEGLU) {
            const uint32_t g = tile;
            if (tid < 64) {
                const float h = gelu_tanh_ref(cres[tid]) * cres[64 + tid];
                a.hb[(size_t)g * 64 + tid] = h;
                wred[tid] = h;  // warp partials are consumed; reuse for the limbs
            }
            if (a.xq_out) {
                __syncthreads();
                if (warp < 2) xq_prep_block(wred[warp * 32 + lane], &a.xq_out[g * 2 + warp]);
            }
        } else {
            const int m = mv_mat_of(a, tile);
            const MvMat& M = a.m[m];
            const uint32_t g = tile - M.tile0;
            const size_t ob = a.epi == EPI_PARTIAL ? (size_t)crank * M.cols : 0;
            if (tid < 64) M.out[ob + (size_t)g * 64 + tid] = cres[tid];
            if (a.epi == EPI_ARGMAX && warp == 0) {
                float v0 = cres[lane], v1 = cres[lane + 32];
                float bv = v0;
                uint32_t bi = g * 64 + lane;
                if (v1 > bv) { bv = v1; bi = g * 64 + lane + 32; }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                }
                if (lane == 0) { a.am_val[tile] = bv; a.am_idx[tile] = bi; }
            }
        }
        __syncthreads();
    }
}

}  // namespace xp
