// DecodeSession on sm_100a: the reference's per-token op order
// (examples/llm/decode.cpp:1634-1780) as five fused kernels per layer,
// captured once into a CUDA graph with programmatic dependent launch.
//
//   qkv    : [residual + post-FFN norm of the previous layer] + attn norm ->
//            int4 matvec q|k|v (cluster K-split)
//   attn   : QK-norm + RoPE + fp16 KV append + split-K flash-decode + combine
//   o      : int4 matvec (cluster K-split) on the attention output's limbs
//   gateup : residual + post-attn norm + FFN norm -> gate|up matvec -> GeGLU
//   down   : int4 matvec (cluster K-split) on hb's limbs
// then final norm -> LM head (per-tile argmax) -> sampler. The token id and
// the position live in device memory, so the same graph replays for every
// position; a local layer's window is computed on the device from `pos`.
#pragma once
#include <cmath>
#include <cstdlib>
#include <initializer_list>
#include <string>
#include <unordered_map>
#include <vector>

#include "runtime.cuh"
#include "batch.cuh"
#include "token_kernel.cuh"

namespace xp {

struct QW {
    uint4* wq = nullptr;
    uint2* sc = nullptr;
    uint32_t rows = 0, cols = 0;
};
struct LayerDev {
    QW m[7];          // q, k, v, o, gate, up, down
    float* norm[6];   // attn, post_attn, ffn, post_ffn, q_norm, k_norm
    __half* kc = nullptr;
    __half* vc = nullptr;
};

inline int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return v && *v ? std::atoi(v) : dflt;
}

// Smallest K-split (cluster size <= 8) that puts at least ~0.9 CTAs per SM
// on the GPU, preferring splits that divide the block count evenly.
inline uint32_t pick_ksplit(uint32_t tiles, uint32_t nblk) {
    const uint32_t want = (uint32_t)(0.9 * sm_count());
    uint32_t best = 1;
    for (uint32_t ks = 1; ks <= 8; ++ks) {
        if (nblk / ks < 2) break;
        best = ks;
        if (tiles * ks >= want && nblk % ks == 0) return ks;
    }
    for (uint32_t ks = 1; ks <= 8; ++ks)
        if (tiles * ks >= want && nblk / ks >= 2) return ks;
    return best;
}

}  // namespace xp

using namespace xp;

struct xp_session {
    int device = 0;
    cudaStream_t st = nullptr;
    xp_model_config cfg{};
    xp_sampling sp{};
    std::vector<LayerDev> L;
    QW lm;
    float* final_norm = nullptr;
    float* embed = nullptr;
    // activations
    float *xa = nullptr, *xb = nullptr, *qr = nullptr, *kr = nullptr, *vr = nullptr, *att = nullptr;
    float *oo = nullptr, *hb = nullptr, *dn = nullptr, *logits = nullptr, *amv = nullptr, *sample_out = nullptr;
    uint32_t *ami = nullptr, *token = nullptr, *pos = nullptr, *hist = nullptr;
    XBlk *att_xq = nullptr, *hb_xq = nullptr, *lm_xq = nullptr;
    void* attn_scratch = nullptr;
    void* samp_scratch = nullptr;
    uint32_t* h_in = nullptr;
    uint32_t* h_out = nullptr;
    xp_bdec* pre = nullptr;     // chunked prefill (64 prompt positions per pass), made on first use
    bool pre_failed = false;
    cudaGraphExec_t g_dev = nullptr, g_io = nullptr, g_prefill = nullptr;
    uint32_t* tp_buf = nullptr;              // this rank's exchange area (IPC-exported): argmax slots, then the down-sum receive area
    // [argmax slots | down-sum receive area | candidate area (2 banks) | candidate flags (2 x 8)]
    size_t tp_off_cand() const { return TK_TP_SLOTS * sizeof(TkTpSlot) + tk_dn_rx_words(cfg.hidden) * 8; }
    size_t tp_cand_keys() const { return (size_t)((cfg.vocab + TOPK_SLICE - 1) / TOPK_SLICE) * TOPK_TK; }
    size_t tp_off_cflags() const { return tp_off_cand() + 2 * tp_cand_keys() * 8; }
    size_t tp_buf_bytes() const { return tp_off_cflags() + 2 * 8 * 4; }
    std::vector<void*> tp_peers;             // opened peer mappings
    cudaEvent_t ev_done = nullptr, ev_a = nullptr, ev_b = nullptr;
    uint32_t host_pos = 0;
    bool have_logits = false;
    bool tk_tp_instance = false;             // run the tensor-parallel token kernel (also at one rank)
    std::string load_info;                   // how the weights were loaded (GGUF sessions)
    int load_from_cache = 0, load_cache_written = 0;
    uint32_t kernels_per_token = 0;
    uint64_t weight_bytes = 0;
    uint32_t nsplit_global = 0, nsplit_local = 0;
    uint32_t ks_qkv = 1, ks_o = 1, ks_gu = 1, ks_down = 1;
    bool pdl = true;
    std::vector<void*> allocs;
    uint32_t launches = 0;  // counted while recording
    // ---- persistent token kernel ----
    bool use_tk = false;
    TkArgs tk{};
    size_t tk_smem = 0;
    uint32_t tk_grid = 0;
    TkLayer* tk_layers_dev = nullptr;
    std::vector<TkLayer> tk_layers;
    unsigned char* tk_head = nullptr;
    uint64_t* tk_bar = nullptr;
    uint32_t mv_launches = 0;
    uint64_t mv_token_bytes = 0;

    ~xp_session() {
        cudaSetDevice(device);
        if (st) cudaStreamSynchronize(st);
        for (cudaGraphExec_t g : {g_dev, g_io, g_prefill, g_mv})
            if (g) cudaGraphExecDestroy(g);
        if (mv_plan) xp_mv_plan_destroy(mv_plan);
        for (void* p : tp_peers) cudaIpcCloseMemHandle(p);
        for (cudaEvent_t e : {ev_done, ev_a, ev_b})
            if (e) cudaEventDestroy(e);
        for (void* p : allocs) cudaFree(p);
        if (h_in) cudaFreeHost(h_in);
        if (h_out) cudaFreeHost(h_out);
        if (st) cudaStreamDestroy(st);
    }

    template <class T> xp_status alloc(T** p, size_t count) {
        void* d = nullptr;
        cudaError_t e = cudaMalloc(&d, count * sizeof(T) + 16);
        if (e != cudaSuccess) return fail(XP_ERR_OOM, "decode: cudaMalloc(%zu) failed: %s", count * sizeof(T),
                                          cudaGetErrorString(e));
        if ((e = zero_fill_sync(d, count * sizeof(T) + 16)) != cudaSuccess) {
            cudaFree(d);
            return fail(XP_ERR_CUDA, "decode: zero fill failed: %s", cudaGetErrorString(e));
        }
        allocs.push_back(d);
        *p = static_cast<T*>(d);
        return XP_OK;
    }

    uint32_t q_dim() const { return cfg.n_heads * cfg.head_dim; }
    uint32_t kv_dim() const { return cfg.n_kv_heads * cfg.head_dim; }
    bool is_global(uint32_t l) const { return cfg.global_every == 0 || (l + 1) % cfg.global_every == 0; }

    // ---- recording one token ----------------------------------------------------------
    cudaError_t rec_mv(const MvArgs& a, bool pdl_here, uint32_t max_ctas = 0) {
        ++launches;
        return launch_mv(a, st, pdl_here, max_ctas);
    }

    bool mv_only = false;       // record only the int4 matvecs (roofline profiling)
    uint64_t mv_bytes = 0;      // algorithmic bytes of the recorded matvecs
    cudaGraphExec_t g_mv = nullptr;
    xp_mv_plan* mv_plan = nullptr;  // the token's matvecs as one streaming plan (profiling)
    float* mv_out = nullptr;

    void count_mv(uint32_t rows, uint32_t cols, uint32_t nmat_same = 1) {
        // nibbles + bf16 scales + activation read (4 B/elt) + output (4 B/elt)
        mv_bytes += nmat_same * ((uint64_t)rows * cols / 2 + (uint64_t)rows * cols / 16 + (uint64_t)cols * 4);
        mv_bytes += (uint64_t)rows * 4;
    }

    cudaError_t record_forward(bool want_logits, bool first_after_copy, bool advance_only_hist) {
        const uint32_t H = cfg.hidden, F = cfg.ffn, QD = q_dim(), KVD = kv_dim();
        const float embed_scale = cfg.embed_scale > 0 ? cfg.embed_scale : std::sqrt((float)H);
        const float attn_scale = cfg.attn_scale > 0 ? cfg.attn_scale : 1.0f / std::sqrt((float)cfg.head_dim);
        cudaError_t e = cudaSuccess;
        bool pdl_next = pdl && !first_after_copy;
        for (uint32_t l = 0; l < cfg.n_layers; ++l) {
            LayerDev& w = L[l];
            // qkv
            MvArgs a{};
            a.m[0] = MvMat{w.m[0].wq, w.m[0].sc, qr, QD, 0};
            a.m[1] = MvMat{w.m[1].wq, w.m[1].sc, kr, KVD, QD / 64};
            a.m[2] = MvMat{w.m[2].wq, w.m[2].sc, vr, KVD, QD / 64 + KVD / 64};
            a.nmat = 3;
            a.ntiles = (QD + 2 * KVD) / 64;
            a.K = H;
            a.hidden = H;
            a.ksplit = ks_qkv;
            a.epi = EPI_STORE;
            a.eps = cfg.rms_eps;
            a.w_pre = w.norm[0];
            a.x_out = xb;
            if (l == 0) {
                a.pro = PRO_EMBED_NORM;
                a.embed = embed;
                a.token = token;
                a.embed_scale = embed_scale;
            } else {
                a.pro = PRO_RESID_NORM;
                a.x = xa;
                a.y = dn;
                a.w_post = L[l - 1].norm[3];
            }
            if (mv_only) { a.pro = PRO_XQ; a.xq_in = lm_xq; }
            if ((e = rec_mv(a, pdl_next)) != cudaSuccess) return e;
            count_mv(H, QD); mv_bytes += (uint64_t)H * KVD * 2 * 9 / 16 + 2 * KVD * 4;
            pdl_next = pdl;
            // attention
            AttnArgs t{};
            t.q_raw = qr; t.k_raw = kr; t.v_raw = vr;
            t.q_norm = w.norm[4]; t.k_norm = w.norm[5];
            t.kcache = w.kc; t.vcache = w.vc;
            t.pos = pos;
            t.cache_rows = cfg.max_seq;
            const bool glob = is_global(l);
            t.window = glob ? 0 : cfg.sliding_window;
            t.theta = glob ? cfg.rope_theta_global : cfg.rope_theta_local;
            t.eps = cfg.rms_eps;
            t.scale = attn_scale;
            t.att = att;
            t.att_xq = att_xq;
            const uint32_t ns = glob ? nsplit_global : nsplit_local;
            const uint32_t span_max = glob ? cfg.max_seq : std::min(cfg.max_seq, cfg.sliding_window);
            if (!mv_only) {
                ++launches;
                if ((e = launch_attn(t, attn_scratch, ns, span_max, st, pdl)) != cudaSuccess) return e;
            }
            // o
            MvArgs o{};
            o.m[0] = MvMat{w.m[3].wq, w.m[3].sc, oo, H, 0};
            o.nmat = 1;
            o.ntiles = H / 64;
            o.K = QD;
            o.hidden = QD;
            o.ksplit = ks_o;
            o.pro = PRO_XQ;
            o.xq_in = att_xq;
            o.epi = EPI_STORE;
            if ((e = rec_mv(o, pdl)) != cudaSuccess) return e;
            count_mv(QD, H);
            // gate / up + GeGLU
            MvArgs g{};
            g.m[0] = MvMat{w.m[4].wq, w.m[4].sc, nullptr, F, 0};
            g.m[1] = MvMat{w.m[5].wq, w.m[5].sc, nullptr, F, 0};
            g.nmat = 2;
            g.ntiles = F / 64;
            g.K = H;
            g.hidden = H;
            g.ksplit = ks_gu;
            g.pro = PRO_RESID_NORM;
            g.x = xb;
            g.y = oo;
            g.w_post = w.norm[1];
            g.w_pre = w.norm[2];
            g.x_out = xa;
            g.eps = cfg.rms_eps;
            g.epi = EPI_GEGLU;
            g.hb = hb;
            g.xq_out = hb_xq;
            if (mv_only) { g.pro = PRO_XQ; g.xq_in = lm_xq; g.xq_out = nullptr; }
            if ((e = rec_mv(g, pdl)) != cudaSuccess) return e;
            count_mv(H, F, 2);
            // down
            MvArgs d{};
            d.m[0] = MvMat{w.m[6].wq, w.m[6].sc, dn, H, 0};
            d.nmat = 1;
            d.ntiles = H / 64;
            d.K = F;
            d.hidden = F;
            d.ksplit = ks_down;
            d.pro = PRO_XQ;
            d.xq_in = hb_xq;
            d.epi = EPI_STORE;
            if ((e = rec_mv(d, pdl)) != cudaSuccess) return e;
            count_mv(F, H);
        }
        if (!want_logits) {
            ++launches;
            return launch_ex(advance_kernel, dim3(1), dim3(32), 0, st, 1, pdl, pos);
        }
        // final norm -> LM head -> sampler
        if (!mv_only) ++launches;
        if (!mv_only && (e = launch_ex(final_norm_xq_kernel, dim3(1), dim3(1024), (size_t)H * 4, st, 1, pdl, (const float*)xa,
                           (const float*)dn, (const float*)L[cfg.n_layers - 1].norm[3], (const float*)final_norm, H,
                           cfg.rms_eps, (float*)nullptr, lm_xq)) != cudaSuccess)
            return e;
        MvArgs h{};
        h.m[0] = MvMat{lm.wq, lm.sc, logits, cfg.vocab, 0};
        h.nmat = 1;
        h.ntiles = cfg.vocab / 64;
        h.K = H;
        h.hidden = H;
        h.ksplit = 1;
        h.pro = PRO_XQ;
        h.xq_in = lm_xq;
        h.epi = EPI_ARGMAX;
        h.am_val = amv;
        h.am_idx = ami;
        if ((e = rec_mv(h, pdl)) != cudaSuccess) return e;
        count_mv(H, cfg.vocab);
        if (mv_only) return cudaSuccess;
        uint32_t* hp = advance_only_hist ? hist : hist;
        if (sp.greedy) {
            ++launches;
            return launch_ex(greedy_final_kernel, dim3(1), dim3(1024), 0, st, 1, pdl, (const float*)amv,
                             (const uint32_t*)ami, h.ntiles, token, sample_out, pos, hp);
        }
        launches += 2;
        return launch_sample_topk(token, sample_out, pos, nullptr, nullptr, logits, cfg.vocab, sp.top_k,
                                  sp.temperature, sp.top_p, sp.seed, sp.seq_id, samp_scratch, st, pdl, true, hp);
    }

    xp_status capture(cudaGraphExec_t* out, bool want_logits, bool io) {
        cudaGraph_t graph = nullptr;
        launches = 0;
        XP_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = cudaSuccess;
        if (io) e = cudaMemcpyAsync(token, h_in, 4, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = (use_tk && !mv_only) ? record_token_kernel(want_logits)
                                                       : record_forward(want_logits, io, false);
        if (e == cudaSuccess && io) e = cudaMemcpyAsync(h_out, token, 4, cudaMemcpyDeviceToHost, st);
        cudaError_t ce = cudaStreamEndCapture(st, &graph);
        if (e != cudaSuccess || ce != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            return fail(XP_ERR_CUDA, "decode: graph capture failed: %s",
                        cudaGetErrorString(e != cudaSuccess ? e : ce));
        }
        cudaError_t ie = cudaGraphInstantiate(out, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) return fail(XP_ERR_CUDA, "decode: cudaGraphInstantiate: %s", cudaGetErrorString(ie));
        return XP_OK;
    }

    // ---- token kernel plan -------------------------------------------------------------
    static uint32_t largest_divisor_upto(uint32_t n, uint32_t cap) {
        uint32_t best = 1;
        for (uint32_t d = 1; d <= n && d <= cap; ++d)
            if (n % d == 0) best = d;
        return best;
    }
    static TkPhase mk_phase(uint32_t units, uint32_t nb, uint32_t cw, uint32_t nmat, uint32_t ks, uint32_t G) {
        TkPhase p{};
        p.units = units;
        p.nb = nb;
        p.cw = cw;
        p.nmat = nmat;
        p.ks = ks;
        p.img_bytes = nmat * nb * cw * 18;
        p.per_cta = (units + G - 1) / G;
        return p;
    }
    static uint32_t al128(uint32_t v) { return (v + 127u) & ~127u; }

    // Returns false (and leaves the multi-kernel graph in charge) when the
    // model does not fit the token kernel's one-unit-per-CTA phases.
    bool plan_token_kernel() {
        if (env_int("XP_ENGINE_MULTI", 0)) return false;
        const uint32_t G = (uint32_t)sm_count();
        const uint32_t H = cfg.hidden, F = cfg.ffn, QD = q_dim(), KVD = kv_dim();
        const uint32_t nbH = H / 32, nbQ = QD / 32;
        if (H > 512 * TK_MAXJ || (H / 64) > G || QD + 2 * KVD > 512 * TK_MAXJ) return false;
        if (cfg.vocab % 64) return false;
        const uint32_t tq = (QD + 2 * KVD) / 64;
        const uint32_t kmax = 8;  // K splits per column tile
        const uint32_t ksq = largest_divisor_upto(nbH, std::min<uint32_t>(kmax, G / tq));
        const uint32_t kso = nbQ / 4;  // 128-dim K ranges (inside one 256-dim head)
        const uint32_t to = H / 64;
        if (tq * ksq > G || to * kso > G || tq == 0 || QD % 128 || F % 16) return false;
        tk.qkv = mk_phase(tq * ksq, nbH / ksq, 64, 1, ksq, G);
        tk.o = mk_phase(to * kso, 4, 64, 1, kso, G);
        tk.gu = mk_phase(F / 16, nbH, 16, 2, 1, G);
        // down-proj rows of every gate|up unit (fused into the GU step)
        tk.down = TkPhase{};
        tk.down.units = tk.gu.units;
        tk.down.cw = H;
        tk.down.nmat = 1;
        tk.down.ks = 1;
        tk.down.img_bytes = H * 10;
        tk.down.per_cta = tk.gu.per_cta;
        tk.head = mk_phase(cfg.vocab / 64, nbH, 64, 1, 1, G);
        if (tk.gu.per_cta > 3 || tk.gu.per_cta * 16 > std::max<uint32_t>(H, 128)) return false;
        // attention: at most TK_SPLIT_CAP splits of at least chunk_min rows
        tk.chunk_min = (uint32_t)std::max(8, env_int("XP_TK_CHUNK_MIN", 32));
        tk.chunk_max = (std::max<uint32_t>(tk.chunk_min, (cfg.max_seq + TK_SPLIT_CAP - 1) / TK_SPLIT_CAP) + 7) & ~7u;
        uint32_t off = 0;
        tk.off_qkv = off; off += al128(tk.qkv.img_bytes);
        tk.off_o = off; off += al128(tk.o.img_bytes);
        tk.off_gu = off; off += al128(tk.gu.per_cta * tk.gu.img_bytes);
        tk.off_down = off; off += al128(tk.down.per_cta * tk.down.img_bytes);
        // KV rows of ATTN, then the flash-partial stage of O (512 B per split)
        tk.off_kv = off; off += al128(std::max<uint32_t>(2 * tk.chunk_max * KVD * 2, TK_SPLIT_CAP * 512));
        // a multiple of the LM-head warp groups: each group owns its ring slots
        auto ring_slots = [&](uint32_t from) {
            return std::min<uint32_t>(TK_MAX_RING, (off - from) / tk.head.img_bytes) / TK_HEAD_GROUPS * TK_HEAD_GROUPS;
        };
        tk.head_ring = ring_slots(tk.off_qkv);
        if (tk.head_ring == 0) return false;
        // keep the QKV slot out of the ring when that costs no ring slot: the
        // next position's layer-0 QKV weights then load while HEAD streams
        tk.qkv_free = ring_slots(tk.off_o) == tk.head_ring ? 1 : 0;
        tk.off_ring = tk.qkv_free ? tk.off_o : tk.off_qkv;
        tk.off_cqkv = off; off += al128(2 * H * 4);
        tk.off_catt = off; off += al128(512 * 4);
        tk.off_cgu = off; off += al128(2 * H * 4);
        tk.off_rope = off; off += al128(768 * 4);
        tk.off_xn = off; off += al128(std::max<uint32_t>(H, 128) * 4);
        const uint32_t maxnb = std::max(std::max(std::max(tk.qkv.nb, tk.o.nb), std::max(tk.gu.nb, tk.gu.per_cta)), tk.head.nb);
        tk.off_xq = off; off += al128(maxnb * (uint32_t)sizeof(XBlk));
        tk.off_q = off; off += al128(4 * 256 * 4 + 2 * 256 * 2);
        tk.off_sc = off; off += al128(4 * tk.chunk_max * 4);
        tk.off_red = off; off += al128(std::max<uint32_t>(4096, 64 + 16 * 64) * 4);
        tk.off_misc = off; off += 512;
        if (cfg.n_layers > TK_MAX_LAYERS) return false;
        tk.off_lay = off; off += al128(cfg.n_layers * (uint32_t)sizeof(TkLayInfo));
        tk_smem = off;
        if (tk_smem + 1024 > 227 * 1024) return false;
        tk_grid = G;
        return true;
    }

    xp_status repack(const QW& q, unsigned char* dst, const TkPhase& P, uint32_t mat, uint32_t tile0) {
        RepackArgs r{};
        r.words = q.wq;
        r.sc = reinterpret_cast<const uint32_t*>(q.sc);
        r.rows = q.rows;
        r.cols = q.cols;
        r.dst = dst;
        r.img_bytes = P.img_bytes;
        r.cw = P.cw;
        r.nb = P.nb;
        r.nmat = P.nmat;
        r.mat = mat;
        r.ks = P.ks;
        r.tile0 = tile0;
        const uint64_t total = (uint64_t)(q.rows / 32) * q.cols;
        const unsigned blocks = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 32);
        repack_units_kernel<<<blocks, 256, 0, st>>>(r);
        XP_CUDA_TRY(cudaGetLastError());
        return XP_OK;
    }

    xp_status setup_token_kernel() {
        use_tk = plan_token_kernel();
        if (!use_tk) return XP_OK;
        const uint32_t G = tk_grid, H = cfg.hidden, QD = q_dim(), KVD = kv_dim();
        xp_status e;
        tk_layers.resize(cfg.n_layers);
        for (uint32_t l = 0; l < cfg.n_layers; ++l) {
            LayerDev& w = L[l];
            TkLayer& t = tk_layers[l];
            unsigned char *iq, *io, *ig, *id;
            if ((e = alloc(&iq, (size_t)tk.qkv.units * tk.qkv.img_bytes)) != XP_OK) return e;
            if ((e = alloc(&io, (size_t)tk.o.units * tk.o.img_bytes)) != XP_OK) return e;
            if ((e = alloc(&ig, (size_t)tk.gu.units * tk.gu.img_bytes)) != XP_OK) return e;
            if ((e = alloc(&id, (size_t)tk.down.units * tk.down.img_bytes)) != XP_OK) return e;
            if ((e = repack(w.m[0], iq, tk.qkv, 0, 0)) != XP_OK) return e;
            if ((e = repack(w.m[1], iq, tk.qkv, 0, QD / 64)) != XP_OK) return e;
            if ((e = repack(w.m[2], iq, tk.qkv, 0, (QD + KVD) / 64)) != XP_OK) return e;
            if ((e = repack(w.m[3], io, tk.o, 0, 0)) != XP_OK) return e;
            if ((e = repack(w.m[4], ig, tk.gu, 0, 0)) != XP_OK) return e;
            if ((e = repack(w.m[5], ig, tk.gu, 1, 0)) != XP_OK) return e;
            repack_half_kernel<<<sm_count() * 8, 256, 0, st>>>(w.m[6].wq, reinterpret_cast<const uint32_t*>(w.m[6].sc),
                                                              w.m[6].rows, w.m[6].cols, id);
            XP_CUDA_TRY(cudaGetLastError());
            t.qkv = iq; t.o = io; t.gu = ig; t.down = id;
            // per-phase constant vectors, contiguous for one bulk copy each
            float *cq, *ca, *cgu;
            if ((e = alloc(&cq, 2 * H)) != XP_OK) return e;
            if ((e = alloc(&ca, 512)) != XP_OK) return e;
            if ((e = alloc(&cgu, 2 * H)) != XP_OK) return e;
            if (l > 0) XP_CUDA_TRY(cudaMemcpyAsync(cq, L[l - 1].norm[3], H * 4, cudaMemcpyDeviceToDevice, st));
            XP_CUDA_TRY(cudaMemcpyAsync(cq + H, w.norm[0], H * 4, cudaMemcpyDeviceToDevice, st));
            XP_CUDA_TRY(cudaMemcpyAsync(ca, w.norm[4], 256 * 4, cudaMemcpyDeviceToDevice, st));
            XP_CUDA_TRY(cudaMemcpyAsync(ca + 256, w.norm[5], 256 * 4, cudaMemcpyDeviceToDevice, st));
            XP_CUDA_TRY(cudaMemcpyAsync(cgu, w.norm[1], H * 4, cudaMemcpyDeviceToDevice, st));
            XP_CUDA_TRY(cudaMemcpyAsync(cgu + H, w.norm[2], H * 4, cudaMemcpyDeviceToDevice, st));
            t.c_qkv = cq; t.c_attn = ca; t.c_gu = cgu;
            t.kc = w.kc;
            t.vc = w.vc;
            const bool glob = is_global(l);
            t.window = glob ? 0 : cfg.sliding_window;
            t.global = glob ? 1 : 0;
        }
        float* ch;
        if ((e = alloc(&ch, 2 * H)) != XP_OK) return e;
        XP_CUDA_TRY(cudaMemcpyAsync(ch, L[cfg.n_layers - 1].norm[3], H * 4, cudaMemcpyDeviceToDevice, st));
        XP_CUDA_TRY(cudaMemcpyAsync(ch + H, final_norm, H * 4, cudaMemcpyDeviceToDevice, st));
        tk.c_head = ch;
        if ((e = alloc(&tk_head, (size_t)tk.head.units * tk.head.img_bytes)) != XP_OK) return e;
        if ((e = repack(lm, tk_head, tk.head, 0, 0)) != XP_OK) return e;
        if ((e = alloc(&tk_layers_dev, cfg.n_layers)) != XP_OK) return e;
        XP_CUDA_TRY(h2d_sync(tk_layers_dev, tk_layers.data(), sizeof(TkLayer) * cfg.n_layers));
        float *attp, *atts, *amv2;
        long long *aq, *ao, *ad;
        uint32_t* ami2;
        if ((e = alloc(&aq, (size_t)(QD + 2 * KVD))) != XP_OK) return e;
        if ((e = alloc(&ao, (size_t)H)) != XP_OK) return e;
        if ((e = alloc(&ad, (size_t)H)) != XP_OK) return e;
        if ((e = alloc(&attp, (size_t)G * QD)) != XP_OK) return e;
        if ((e = alloc(&atts, (size_t)G * 8)) != XP_OK) return e;
        if ((e = alloc(&tk.att_ll, (size_t)(QD / 128) * TK_LL_SPLITS * 128)) != XP_OK) return e;
        if ((e = alloc(&tk.att_ll_st, (size_t)TK_LL_SPLITS * 8)) != XP_OK) return e;
        if ((e = alloc(&amv2, G)) != XP_OK) return e;
        if ((e = alloc(&ami2, G)) != XP_OK) return e;
        if ((e = alloc(&tk_bar, 4)) != XP_OK) return e;
        if (env_int("XP_TRACE", 0)) {
            if ((e = alloc(&tk.trace, TK_TRACE_WORDS)) != XP_OK) return e;
        }
        tk.layers = tk_layers_dev;
        tk.n_layers = cfg.n_layers;
        tk.H = H; tk.F = cfg.ffn; tk.QD = QD; tk.KVD = KVD; tk.V = cfg.vocab;
        tk.eps = cfg.rms_eps;
        tk.embed_scale = cfg.embed_scale > 0 ? cfg.embed_scale : std::sqrt((float)H);
        tk.attn_scale = cfg.attn_scale > 0 ? cfg.attn_scale : 1.0f / std::sqrt((float)cfg.head_dim);
        tk.head_img = tk_head;
        tk.theta_global = cfg.rope_theta_global;
        tk.theta_local = cfg.rope_theta_local;
        tk.embed = embed;
        tk.x0 = xa; tk.x1 = xb;
        tk.acc_qkv = aq; tk.acc_o = ao; tk.acc_dn = ad;
        tk.att_part = attp; tk.att_stat = atts;
        tk.logits = logits; tk.am_val = amv2; tk.am_idx = ami2;
        tk.token = token; tk.pos = pos; tk.hist = hist; tk.sample_out = sample_out;
        tk.bar = tk_bar; tk.epoch = tk_bar + 1;
        tk.err = static_cast<uint32_t*>(attn_scratch) + 1;
        tk.greedy = sp.greedy;
        // LM head unsharded until xp_session_tp_attach
        tk.head_u0 = 0;
        tk.head_u1 = tk.head.units;
        tk.gu_u0 = 0;
        tk.gu_u1 = tk.gu.units;
        tk.ffn_shard = 0;
        tk.tp_rank = 0;
        tk.tp_world = 1;
        if ((e = alloc(&tp_buf, tp_buf_bytes() / 4)) != XP_OK) return e;
        if ((e = alloc(&tk.tp_count, 8)) != XP_OK) return e;
        tk.tp_slots[0] = reinterpret_cast<TkTpSlot*>(tp_buf);
        XP_CUDA_TRY(cudaFuncSetAttribute(token_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tk_smem));
        XP_CUDA_TRY(cudaFuncSetAttribute(token_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tk_smem));
        XP_CUDA_TRY(cudaFuncSetAttribute(token_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tk_smem));
        XP_CUDA_TRY(cudaStreamSynchronize(st));
        return XP_OK;
    }

    cudaError_t record_token_kernel(bool want_logits, uint32_t ntok = 1) {
        TkArgs a = tk;
        a.want_logits = want_logits ? 1 : 0;
        a.ntok = ntok;
        cudaLaunchConfig_t c = {};
        c.gridDim = dim3(tk_grid);
        c.blockDim = dim3(TK_BLOCK);
        c.dynamicSmemBytes = tk_smem;
        c.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeCooperative;
        at[0].val.cooperative = 1;
        c.attrs = at;
        c.numAttrs = 1;
        ++launches;
        cudaError_t e = a.trace              ? cudaLaunchKernelEx(&c, token_kernel<true, false>, a)
                        : (a.tp_world > 1 || tk_tp_instance) ? cudaLaunchKernelEx(&c, token_kernel<false, true>, a)
                                         : cudaLaunchKernelEx(&c, token_kernel<false, false>, a);
        if (e != cudaSuccess || !want_logits || sp.greedy) return e;
        launches += 2;
        TpCandArgs tpa{};
        const bool tp = tk.tp_world > 1;
        if (tp) {  // this rank's logits are its LM-head shard: gather the candidates
            tpa.s0 = tk.head_u0 * 64 / TOPK_SLICE;
            tpa.s1 = tk.head_u1 * 64 / TOPK_SLICE;
            tpa.rank = tk.tp_rank;
            tpa.world = tk.tp_world;
            for (uint32_t r = 0; r < tk.tp_world; ++r) {
                unsigned char* b = reinterpret_cast<unsigned char*>(tk.tp_slots[r]);
                tpa.area[r] = reinterpret_cast<uint64_t*>(b + tp_off_cand());
                tpa.flags[r] = reinterpret_cast<uint32_t*>(b + tp_off_cflags());
            }
            tpa.count = tk.tp_count;
            tpa.err = tk.err;
        }
        return launch_sample_topk(token, sample_out, pos, nullptr, nullptr, logits, cfg.vocab, sp.top_k,
                                  sp.temperature, sp.top_p, sp.seed, sp.seq_id, samp_scratch, st, false, true, hist,
                                  tp ? &tpa : nullptr);
    }

    xp_status validate_cfg() {
        const xp_model_config& c = cfg;
        if (!c.n_layers || !c.hidden || !c.ffn || !c.vocab || !c.max_seq)
            return fail(XP_ERR_INVALID, "decode: zero dimension in model config");
        if (c.head_dim != 256 || c.n_heads != 4 || c.n_kv_heads != 1)
            return fail(XP_ERR_UNSUPPORTED,
                        "decode: the fused attention kernel implements Gemma-3-1B heads (4 q, 1 kv, head_dim 256); got %u/%u/%u",
                        c.n_heads, c.n_kv_heads, c.head_dim);
        if (c.hidden % 128 || c.ffn % 128 || c.vocab % 64)
            return fail(XP_ERR_INVALID, "decode: hidden and ffn must be multiples of 128, vocab of 64");
        if (!sp.greedy && (sp.top_k > 64 || c.vocab < 64 || c.vocab > TOPK_MAX_CAND / TOPK_TK * TOPK_SLICE))
            return fail(XP_ERR_UNSUPPORTED, "decode: the device sampler supports top_k <= 64");
        return XP_OK;
    }

    xp_status init_common() {
        XP_CUDA_TRY(cudaSetDevice(device));
        XP_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        XP_CUDA_TRY(cudaEventCreateWithFlags(&ev_done, cudaEventDisableTiming));
        XP_CUDA_TRY(cudaEventCreate(&ev_a));
        XP_CUDA_TRY(cudaEventCreate(&ev_b));
        XP_CUDA_TRY(cudaHostAlloc(&h_in, 64, cudaHostAllocDefault));
        XP_CUDA_TRY(cudaHostAlloc(&h_out, 64, cudaHostAllocDefault));
        std::memset(h_in, 0, 64);
        std::memset(h_out, 0, 64);
        pdl = env_int("XP_PDL", 1) != 0;
        const uint32_t H = cfg.hidden, F = cfg.ffn, QD = q_dim(), KVD = kv_dim();
        xp_status s;
#define A(p, n) if ((s = alloc(&p, n)) != XP_OK) return s
        A(xa, H); A(xb, H); A(qr, QD); A(kr, KVD); A(vr, KVD); A(att, QD); A(oo, H); A(hb, F); A(dn, H);
        A(logits, cfg.vocab); A(amv, cfg.vocab / 64); A(ami, cfg.vocab / 64); A(sample_out, 2);
        A(token, 1); A(pos, 1); A(hist, (size_t)cfg.max_seq + 1);
        A(att_xq, QD / 32); A(hb_xq, F / 32); A(lm_xq, H / 32);
        nsplit_global = std::max<uint32_t>(1, std::min<uint32_t>((cfg.max_seq + 63) / 64, 2 * sm_count()));
        const uint32_t lspan = std::min(cfg.max_seq, cfg.sliding_window ? cfg.sliding_window : cfg.max_seq);
        nsplit_local = std::max<uint32_t>(1, std::min<uint32_t>((lspan + 31) / 32, 2 * sm_count()));
        nsplit_global = (uint32_t)env_int("XP_NSPLIT_GLOBAL", (int)nsplit_global);
        nsplit_local = (uint32_t)env_int("XP_NSPLIT_LOCAL", (int)nsplit_local);
        unsigned char* scr = nullptr;
        A(scr, attn_scratch_bytes(std::max(nsplit_global, nsplit_local)));
        attn_scratch = scr;
        unsigned char* ss = nullptr;
        A(ss, sample_scratch_bytes(cfg.vocab));
        samp_scratch = ss;
        for (uint32_t l = 0; l < cfg.n_layers; ++l) {
            A(L[l].kc, (size_t)cfg.max_seq * KVD);
            A(L[l].vc, (size_t)cfg.max_seq * KVD);
        }
#undef A
        ks_qkv = (uint32_t)env_int("XP_KS_QKV", (int)pick_ksplit((QD + 2 * KVD) / 64, H / 32));
        ks_o = (uint32_t)env_int("XP_KS_O", (int)pick_ksplit(H / 64, QD / 32));
        ks_gu = (uint32_t)env_int("XP_KS_GU", (int)pick_ksplit(F / 64, H / 32));
        ks_down = (uint32_t)env_int("XP_KS_DOWN", (int)pick_ksplit(H / 64, F / 32));
        return XP_OK;
    }

    xp_status alloc_weights() {
        const uint32_t H = cfg.hidden, F = cfg.ffn, QD = q_dim(), KVD = kv_dim();
        const uint32_t shapes[7][2] = {{H, QD}, {H, KVD}, {H, KVD}, {QD, H}, {H, F}, {H, F}, {F, H}};
        xp_status s;
        weight_bytes = 0;
        for (uint32_t l = 0; l < cfg.n_layers; ++l) {
            for (int m = 0; m < 7; ++m) {
                QW& q = L[l].m[m];
                q.rows = shapes[m][0];
                q.cols = shapes[m][1];
                if ((s = alloc(&q.wq, (size_t)q.rows * q.cols / 32)) != XP_OK) return s;
                if ((s = alloc(&q.sc, (size_t)q.rows * q.cols / 128)) != XP_OK) return s;
                weight_bytes += (size_t)q.rows * q.cols / 2 + (size_t)q.rows * q.cols / 16;
            }
            for (int n = 0; n < 6; ++n)
                if ((s = alloc(&L[l].norm[n], n < 4 ? H : cfg.head_dim)) != XP_OK) return s;
        }
        lm.rows = H;
        lm.cols = cfg.vocab;
        if ((s = alloc(&lm.wq, (size_t)lm.rows * lm.cols / 32)) != XP_OK) return s;
        if ((s = alloc(&lm.sc, (size_t)lm.rows * lm.cols / 128)) != XP_OK) return s;
        weight_bytes += (size_t)lm.rows * lm.cols / 2 + (size_t)lm.rows * lm.cols / 16;
        if ((s = alloc(&final_norm, H)) != XP_OK) return s;
        if ((s = alloc(&embed, (size_t)cfg.vocab * H)) != XP_OK) return s;
        return XP_OK;
    }

    xp_status build_graphs() {
        xp_status s;
        if ((s = capture(&g_dev, true, false)) != XP_OK) return s;
        kernels_per_token = launches;
        if ((s = capture(&g_io, true, true)) != XP_OK) return s;
        if ((s = capture(&g_prefill, false, true)) != XP_OK) return s;
        return XP_OK;
    }

    xp_status wait_prev() {
        cudaError_t e = cudaEventSynchronize(ev_done);
        if (e != cudaSuccess) return fail(XP_ERR_DEVICE, "decode: device error: %s", cudaGetErrorString(e));
        return XP_OK;
    }
};

extern "C" {

uint64_t xp_session_tensor_stream(uint32_t layer, uint32_t which) { return 0x1000ull + layer * 32ull + which; }

static xp_status session_common(int device, const xp_model_config* cfg, const xp_sampling* sp, xp_session** out,
                                xp_session** made) {
    if (!cfg || !out) return fail(XP_ERR_INVALID, "decode: null config or out");
    if (device < 0 || device >= xp_device_count()) return fail(XP_ERR_NO_DEVICE, "decode: no CUDA device %d", device);
    auto* s = new xp_session;
    s->device = device;
    s->cfg = *cfg;
    if (sp) s->sp = *sp;
    else { s->sp.greedy = 1; s->sp.temperature = 1.0f; s->sp.top_p = 1.0f; s->sp.seed = 1234; }
    xp_status st = s->validate_cfg();
    if (st == XP_OK) {
        s->L.resize(cfg->n_layers);
        st = s->init_common();
    }
    if (st == XP_OK) st = s->alloc_weights();
    if (st != XP_OK) { delete s; return st; }
    *made = s;
    return XP_OK;
}

xp_status xp_session_create_random(int device, const xp_model_config* cfg, const xp_sampling* sp, uint64_t seed,
                                   xp_session** out) {
    xp_session* s = nullptr;
    xp_status st = session_common(device, cfg, sp, out, &s);
    if (st != XP_OK) return st;
    const uint32_t H = s->cfg.hidden;
    float* tmp = nullptr;
    size_t maxe = 0;
    for (int m = 0; m < 7; ++m) maxe = std::max(maxe, (size_t)s->L[0].m[m].rows * s->L[0].m[m].cols);
    if ((st = s->alloc(&tmp, maxe)) != XP_OK) { delete s; return st; }
    auto gen = [&](float* dst, size_t n, uint64_t stream) {
        return xp_gen_normal(s->st, dst, n, 0, seed, stream, 0.02f);
    };
    for (uint32_t l = 0; l < s->cfg.n_layers && st == XP_OK; ++l) {
        for (int m = 0; m < 7 && st == XP_OK; ++m) {
            QW& q = s->L[l].m[m];
            st = gen(tmp, (size_t)q.rows * q.cols, xp_session_tensor_stream(l, m));
            if (st == XP_OK)
                st = xp_pack_km4bf16(s->st, tmp, q.rows, q.cols, reinterpret_cast<uint32_t*>(q.wq),
                                     reinterpret_cast<uint32_t*>(q.sc));
        }
        for (int n = 0; n < 6 && st == XP_OK; ++n)
            st = gen(s->L[l].norm[n], n < 4 ? H : s->cfg.head_dim, xp_session_tensor_stream(l, 7 + n));
    }
    const uint32_t NL = s->cfg.n_layers;
    if (st == XP_OK) st = gen(s->embed, (size_t)s->cfg.vocab * H, xp_session_tensor_stream(NL, 0));
    if (st == XP_OK)
        st = xp_pack_km4bf16(s->st, s->embed, H, s->cfg.vocab, reinterpret_cast<uint32_t*>(s->lm.wq),
                             reinterpret_cast<uint32_t*>(s->lm.sc));
    if (st == XP_OK) st = gen(s->final_norm, H, xp_session_tensor_stream(NL, 7));
    if (st == XP_OK && cudaStreamSynchronize(s->st) != cudaSuccess) st = fail(XP_ERR_CUDA, "decode: weight init failed");
    if (st == XP_OK) st = s->setup_token_kernel();
    if (st == XP_OK) st = s->build_graphs();
    if (st != XP_OK) { delete s; return st; }
    *out = s;
    return XP_OK;
}

xp_status xp_session_create(int device, const xp_model_config* cfg, const xp_sampling* sp,
                            const xp_layer_weights* layers, const uint32_t* lm_words, const uint32_t* lm_scales,
                            const float* final_norm, const float* embed, xp_session** out) {
    if (!layers || !lm_words || !lm_scales || !final_norm || !embed)
        return fail(XP_ERR_INVALID, "decode: null weight pointer");
    xp_session* s = nullptr;
    xp_status st = session_common(device, cfg, sp, out, &s);
    if (st != XP_OK) return st;
    const uint32_t H = s->cfg.hidden;
    auto up = [&](void* dst, const void* src, size_t bytes) -> xp_status {
        if (!src) return fail(XP_ERR_INVALID, "decode: null weight pointer");
        XP_CUDA_TRY(h2d_sync(dst, src, bytes));
        return XP_OK;
    };
    for (uint32_t l = 0; l < s->cfg.n_layers && st == XP_OK; ++l) {
        for (int m = 0; m < 7 && st == XP_OK; ++m) {
            QW& q = s->L[l].m[m];
            st = up(q.wq, layers[l].words[m], (size_t)q.rows * q.cols / 2);
            if (st == XP_OK) st = up(q.sc, layers[l].scales[m], (size_t)q.rows * q.cols / 16);
        }
        const float* nsrc[6] = {layers[l].attn_norm, layers[l].post_attn_norm, layers[l].ffn_norm,
                                layers[l].post_ffn_norm, layers[l].q_norm, layers[l].k_norm};
        for (int n = 0; n < 6 && st == XP_OK; ++n)
            st = up(s->L[l].norm[n], nsrc[n], (size_t)(n < 4 ? H : s->cfg.head_dim) * 4);
    }
    if (st == XP_OK) st = up(s->lm.wq, lm_words, (size_t)H * s->cfg.vocab / 2);
    if (st == XP_OK) st = up(s->lm.sc, lm_scales, (size_t)H * s->cfg.vocab / 16);
    if (st == XP_OK) st = up(s->final_norm, final_norm, (size_t)H * 4);
    if (st == XP_OK) st = up(s->embed, embed, (size_t)s->cfg.vocab * H * 4);
    if (st == XP_OK) st = s->setup_token_kernel();
    if (st == XP_OK) st = s->build_graphs();
    if (st != XP_OK) { delete s; return st; }
    *out = s;
    return XP_OK;
}

xp_status xp_session_destroy(xp_session* s) {
    if (s && s->pre) xp_bdec_destroy(s->pre);
    delete s;
    return XP_OK;
}

xp_status xp_session_reset(xp_session* s) {
    if (!s) return fail(XP_ERR_INVALID, "null session");
    cudaSetDevice(s->device);
    XP_CUDA_TRY(cudaStreamSynchronize(s->st));
    XP_CUDA_TRY(cudaMemsetAsync(s->pos, 0, 4, s->st));
    if (s->tk_bar) XP_CUDA_TRY(cudaMemsetAsync(s->tk_bar, 0, 16, s->st));
    // the flagged attention words carry flags derived from the barrier count
    // just reset: clear them so no stale word can match a new flag
    if (s->tk.att_ll) {
        XP_CUDA_TRY(cudaMemsetAsync(s->tk.att_ll, 0, (size_t)(s->q_dim() / 128) * TK_LL_SPLITS * 128 * 8, s->st));
        XP_CUDA_TRY(cudaMemsetAsync(s->tk.att_ll_st, 0, (size_t)TK_LL_SPLITS * 8 * 8, s->st));
    }
    XP_CUDA_TRY(cudaStreamSynchronize(s->st));
    s->host_pos = 0;
    s->have_logits = false;
    return XP_OK;
}

static xp_status prefill_chunked(xp_session* s, const uint32_t* tokens, uint32_t n);

xp_status xp_session_prefill(xp_session* s, const uint32_t* tokens, uint32_t n) {
    if (!s) return fail(XP_ERR_INVALID, "null session");
    if (n == 0) return XP_OK;
    if (!tokens) return fail(XP_ERR_INVALID, "decode: null token array");
    cudaSetDevice(s->device);
    if (n >= (uint32_t)env_int("XP_PREFILL_CHUNK_MIN", 32) && s->use_tk && !s->mv_only && !s->tk_tp_instance &&
        !s->tk.trace && !s->pre_failed && s->host_pos + n <= s->cfg.max_seq) {
        bool ok = true;
        for (uint32_t i = 0; i < n && ok; ++i) ok = tokens[i] < s->cfg.vocab;
        if (ok) {
            xp_status st = prefill_chunked(s, tokens, n);
            if (st != XP_ERR_UNSUPPORTED) return st;
        }
    }
    for (uint32_t i = 0; i < n; ++i) {
        if (s->host_pos >= s->cfg.max_seq)
            return fail(XP_ERR_KV_FULL, "decode: prompt exceeds max_seq (%u)", s->cfg.max_seq);
        if (tokens[i] >= s->cfg.vocab)
            return fail(XP_ERR_INVALID, "decode: token id %u is outside the vocabulary", tokens[i]);
        xp_status st = s->wait_prev();
        if (st != XP_OK) return st;
        *s->h_in = tokens[i];
        const bool last = i + 1 == n;
        XP_CUDA_TRY(cudaGraphLaunch(last ? s->g_io : s->g_prefill, s->st));
        XP_CUDA_TRY(cudaEventRecord(s->ev_done, s->st));
        ++s->host_pos;
    }
    s->have_logits = true;
    return s->wait_prev();
}

xp_status xp_session_decode_step(xp_session* s, uint32_t* token) {
    if (!s) return fail(XP_ERR_INVALID, "null session");
    if (s->host_pos == 0)
        return fail(XP_ERR_STATE, "decode: decode_step() before prefill() — there is no context to condition on");
    if (s->host_pos >= s->cfg.max_seq)
        return fail(XP_ERR_KV_FULL, "decode: KV cache is full (max_seq %u)", s->cfg.max_seq);
    cudaSetDevice(s->device);
    xp_status st = s->wait_prev();
    if (st != XP_OK) return st;
    const uint32_t t = *s->h_out;  // sampled from the previous pass's logits
    *s->h_in = t;
    XP_CUDA_TRY(cudaGraphLaunch(s->g_io, s->st));
    XP_CUDA_TRY(cudaEventRecord(s->ev_done, s->st));
    ++s->host_pos;
    if (token) *token = t;
    return XP_OK;
}

xp_status xp_session_generate(xp_session* s, uint32_t n, uint32_t* tokens, float* ms) {
    if (!s) return fail(XP_ERR_INVALID, "null session");
    if (s->host_pos == 0) return fail(XP_ERR_STATE, "decode: generate() before prefill()");
    if (s->host_pos + n > s->cfg.max_seq)
        return fail(XP_ERR_KV_FULL, "decode: %u steps from position %u exceed max_seq %u", n, s->host_pos,
                    s->cfg.max_seq);
    cudaSetDevice(s->device);
    xp_status st = s->wait_prev();
    if (st != XP_OK) return st;
    const uint32_t p0 = s->host_pos;
    XP_CUDA_TRY(cudaEventRecord(s->ev_a, s->st));
    if (s->use_tk && !s->mv_only && s->sp.greedy && s->tk.tp_world == 1 && !s->tk.trace) {
        // greedy on one GPU: the token kernel decodes up to 512 positions per
        // launch, each position's input token picked on the device
        for (uint32_t i = 0; i < n;) {
            const uint32_t m = std::min<uint32_t>(n - i, 512);
            XP_CUDA_TRY(s->record_token_kernel(true, m));
            i += m;
        }
    } else {
        for (uint32_t i = 0; i < n; ++i) XP_CUDA_TRY(cudaGraphLaunch(s->g_dev, s->st));
    }
    XP_CUDA_TRY(cudaEventRecord(s->ev_b, s->st));
    XP_CUDA_TRY(cudaMemcpyAsync(s->h_out, s->token, 4, cudaMemcpyDeviceToHost, s->st));
    XP_CUDA_TRY(cudaEventRecord(s->ev_done, s->st));
    XP_CUDA_TRY(cudaEventSynchronize(s->ev_done));
    s->host_pos += n;
    if (ms) XP_CUDA_TRY(cudaEventElapsedTime(ms, s->ev_a, s->ev_b));
    if (tokens && n) {
        // hist[p] holds the token sampled at the step that advanced to p; the
        // first generated step consumed the token sampled before it (h_out of
        // the previous pass), so tokens[i] = the input of step i.
        std::vector<uint32_t> h(n + 1);
        XP_CUDA_TRY(cudaMemcpy(h.data(), s->hist + p0, (size_t)(n + 1) * 4, cudaMemcpyDeviceToHost));
        for (uint32_t i = 0; i < n; ++i) tokens[i] = h[i];
    }
    return XP_OK;
}

xp_status xp_session_profile_matvec(xp_session* s, uint32_t iters, float* ms_per_token, uint64_t* bytes_per_token,
                                    uint32_t* launches_per_token) {
    if (!s || iters == 0) return fail(XP_ERR_INVALID, "profile: bad arguments");
    cudaSetDevice(s->device);
    xp_status st = s->wait_prev();
    if (st != XP_OK) return st;
    if (!s->mv_plan) {
        // the token's int4 matvecs as one streaming plan: 26 x (q, k, v, o,
        // gate, up, down) + LM head, on the session's packed planes
        const uint32_t H = s->cfg.hidden, F = s->cfg.ffn, QD = s->q_dim();
        std::vector<xp_mv_job> jobs;
        size_t outs = s->cfg.vocab;
        for (uint32_t l = 0; l < s->cfg.n_layers; ++l)
            for (int m = 0; m < 7; ++m) outs += s->L[l].m[m].cols;
        if ((st = s->alloc(&s->mv_out, outs)) != XP_OK) return st;
        size_t off = 0;
        auto add = [&](const QW& q) {
            const float* in = q.rows == H ? s->xa : (q.rows == F ? s->hb : s->att);
            jobs.push_back(xp_mv_job{s->mv_out + off, in, reinterpret_cast<const uint32_t*>(q.wq),
                                     reinterpret_cast<const uint32_t*>(q.sc), q.rows, q.cols});
            off += q.cols;
        };
        for (uint32_t l = 0; l < s->cfg.n_layers; ++l)
            for (int m = 0; m < 7; ++m) add(s->L[l].m[m]);
        add(s->lm);
        (void)QD;
        if ((st = xp_mv_plan_create(jobs.data(), (uint32_t)jobs.size(), &s->mv_plan)) != XP_OK) return st;
    }
    if ((st = xp_mv_plan_run(s->mv_plan, s->st)) != XP_OK) return st;
    XP_CUDA_TRY(cudaEventRecord(s->ev_a, s->st));
    for (uint32_t i = 0; i < iters; ++i)
        if ((st = xp_mv_plan_run(s->mv_plan, s->st)) != XP_OK) return st;
    XP_CUDA_TRY(cudaEventRecord(s->ev_b, s->st));
    XP_CUDA_TRY(cudaEventRecord(s->ev_done, s->st));
    XP_CUDA_TRY(cudaEventSynchronize(s->ev_b));
    float ms = 0;
    XP_CUDA_TRY(cudaEventElapsedTime(&ms, s->ev_a, s->ev_b));
    uint64_t b = 0;
    xp_mv_plan_bytes(s->mv_plan, &b);
    if (ms_per_token) *ms_per_token = ms / iters;
    if (bytes_per_token) *bytes_per_token = b;
    if (launches_per_token) *launches_per_token = 2;  // limbs + the streaming matvec
    return XP_OK;
}

xp_status xp_session_trace(xp_session* s, uint64_t* out, uint32_t n) {
    if (!s || !out) return fail(XP_ERR_INVALID, "null argument");
    if (!s->use_tk || !s->tk.trace) return fail(XP_ERR_STATE, "trace: set XP_TRACE=1 before creating the session");
    cudaSetDevice(s->device);
    xp_status st = s->wait_prev();
    if (st != XP_OK) return st;
    XP_CUDA_TRY(cudaMemcpy(out, s->tk.trace, (size_t)std::min<uint32_t>(n, TK_TRACE_WORDS) * 8, cudaMemcpyDeviceToHost));
    return XP_OK;
}

xp_status xp_session_timer(xp_session* s, int stop, float* ms) {
    if (!s) return fail(XP_ERR_INVALID, "null session");
    cudaSetDevice(s->device);
    if (!stop) {
        XP_CUDA_TRY(cudaEventRecord(s->ev_a, s->st));
        return XP_OK;
    }
    XP_CUDA_TRY(cudaEventRecord(s->ev_b, s->st));
    XP_CUDA_TRY(cudaEventSynchronize(s->ev_b));
    if (ms) XP_CUDA_TRY(cudaEventElapsedTime(ms, s->ev_a, s->ev_b));
    return XP_OK;
}

xp_status xp_session_position(xp_session* s, uint32_t* p) {
    if (!s || !p) return fail(XP_ERR_INVALID, "null argument");
    *p = s->host_pos;
    return XP_OK;
}
xp_status xp_session_logits(xp_session* s, float* out, uint32_t n) {
    if (!s || !out) return fail(XP_ERR_INVALID, "null argument");
    if (n != s->cfg.vocab) return fail(XP_ERR_INVALID, "decode: logits buffer holds %u, vocab is %u", n, s->cfg.vocab);
    if (!s->have_logits) return fail(XP_ERR_STATE, "decode: no forward pass with logits yet");
    cudaSetDevice(s->device);
    xp_status st = s->wait_prev();
    if (st != XP_OK) return st;
    XP_CUDA_TRY(cudaMemcpy(out, s->logits, (size_t)n * 4, cudaMemcpyDeviceToHost));
    return XP_OK;
}
xp_status xp_session_stats(xp_session* s, uint32_t* kpt, uint64_t* wb) {
    if (!s) return fail(XP_ERR_INVALID, "null session");
    if (kpt) *kpt = s->kernels_per_token;
    if (wb) *wb = s->weight_bytes;
    return XP_OK;
}
xp_status xp_session_debug_ptr(xp_session* s, const char* name, void** d, size_t* bytes) {
    if (!s || !name || !d) return fail(XP_ERR_INVALID, "null argument");
    const std::string n(name);
    const uint32_t H = s->cfg.hidden;
    size_t b = 0;
    void* p = nullptr;
    if (n == "xa") { p = s->xa; b = H * 4; }
    else if (n == "xb") { p = s->xb; b = H * 4; }
    else if (n == "logits") { p = s->logits; b = (size_t)s->cfg.vocab * 4; }
    else if (n == "att") { p = s->att; b = (size_t)s->q_dim() * 4; }
    else if (n == "embed") { p = s->embed; b = (size_t)s->cfg.vocab * H * 4; }
    else if (n == "token") { p = s->token; b = 4; }
    else if (n == "pos") { p = s->pos; b = 4; }
    else if (n.rfind("kcache", 0) == 0 || n.rfind("vcache", 0) == 0) {
        const uint32_t l = (uint32_t)std::atoi(n.c_str() + 6);
        if (l >= s->cfg.n_layers) return fail(XP_ERR_INVALID, "no layer %u", l);
        p = n[0] == 'k' ? (void*)s->L[l].kc : (void*)s->L[l].vc;
        b = (size_t)s->cfg.max_seq * s->kv_dim() * 2;
    } else if (n.rfind("w", 0) == 0 && n.size() >= 3) {
        // "w<m>_<l>" words of matrix m (0..6, 7 = lm head) in layer l; "s<m>_<l>" scales
        return fail(XP_ERR_INVALID, "unknown buffer '%s'", name);
    } else return fail(XP_ERR_INVALID, "unknown buffer '%s'", name);
    *d = p;
    if (bytes) *bytes = b;
    return XP_OK;
}
xp_status xp_session_error_word(xp_session* s, uint32_t* w) {
    if (!s || !w) return fail(XP_ERR_INVALID, "null argument");
    cudaSetDevice(s->device);
    XP_CUDA_TRY(cudaStreamSynchronize(s->st));
    // the attention error word follows the ticket at the head of the scratch
    uint32_t* err = static_cast<uint32_t*>(s->attn_scratch) + 1;
    XP_CUDA_TRY(cudaMemcpy(w, err, 4, cudaMemcpyDeviceToHost));
    XP_CUDA_TRY(zero_fill_sync(err, 4));
    return XP_OK;
}

}  // extern "C"

// ============================================================================
// Batched decode: B sequences over one session's weights (tensor-core matvecs)
// ============================================================================
struct xp_bdec {
    xp_session* s = nullptr;
    int device = 0;
    cudaStream_t st = nullptr;
    uint32_t B = 0, max_seq = 0;
    xp_sampling sp{};
    uint64_t seq0 = 0;
    std::vector<void*> allocs;
    float *x = nullptr, *logits = nullptr;
    // matvec inputs, written as tensor-core operands by the kernels that make them
    BkOperand op_xn{}, op_att{}, op_hb{};
    // matvec results as fp32 partial sums, one per K range of the tensor-core
    // launch ([ks][B][cols]); the consuming kernel adds them
    float *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *g = nullptr, *u = nullptr, *dn = nullptr;
    uint32_t ks_qkv = 1, ks_o = 1, ks_gu = 1, ks_dn = 1;
    BkSums sums(const float* p, uint32_t ks, uint32_t cols) const { return BkSums{p, ks, B * cols}; }
    std::vector<__half*> kc, vc;
    uint32_t *tokens = nullptr, *pos = nullptr, *h_tok = nullptr;
    // one tensor-core scratch per matrix shape: a call leaves its fixed-point
    // sums zero only where its own shape keeps them
    std::vector<std::pair<uint64_t, unsigned char*>> bscratch;
    uint64_t* cand = nullptr;
    uint32_t ns = 0, nc = 0;
    // per scale plane: every scale in the fp16-exact range, so its matvecs use
    // the tensor-core kernel's scaled operand mode (checked once at creation)
    std::unordered_map<const void*, bool> s16;
    int mode_of(const QW& w) const {
        auto it = s16.find(w.sc);
        return it != s16.end() && it->second ? BMM_MODE_SCALED : BMM_MODE_INTEGER;
    }
    cudaGraphExec_t g_fwd = nullptr, g_step = nullptr, g_nohead = nullptr;
    cudaEvent_t ev_a = nullptr, ev_b = nullptr;
    uint32_t h_pos = 0;  // every sequence is at the same position
    // chunked prefill of the session's own sequence: row b is position
    // pos[b] of one sequence, the caches are the session's
    bool chunk = false;
    // Programmatic dependent launch (XP_BDEC_PDL bit 0: tensor-core launches,
    // which then request their first weights under the previous kernel's tail;
    // bit 1: the per-sequence kernels, measured slightly slower, so off)
    bool pdl_mm = (env_int("XP_BDEC_PDL", 1) & 1) != 0, pdl_k = (env_int("XP_BDEC_PDL", 1) & 2) != 0;

    ~xp_bdec() {
        cudaSetDevice(device);
        if (st) cudaStreamSynchronize(st);
        for (cudaGraphExec_t ge : {g_fwd, g_step, g_nohead})
            if (ge) cudaGraphExecDestroy(ge);
        for (cudaEvent_t e : {ev_a, ev_b})
            if (e) cudaEventDestroy(e);
        for (void* p : allocs) cudaFree(p);
        if (h_tok) cudaFreeHost(h_tok);
        if (st) cudaStreamDestroy(st);
    }
    template <class T> xp_status alloc(T** p, size_t count) {
        void* d = nullptr;
        cudaError_t e = cudaMalloc(&d, count * sizeof(T) + 256);
        if (e != cudaSuccess) return fail(XP_ERR_OOM, "batch: cudaMalloc(%zu) failed: %s", count * sizeof(T),
                                          cudaGetErrorString(e));
        if ((e = zero_fill_sync(d, count * sizeof(T) + 256)) != cudaSuccess) {
            cudaFree(d);
            return fail(XP_ERR_CUDA, "batch: zero fill failed: %s", cudaGetErrorString(e));
        }
        allocs.push_back(d);
        *p = static_cast<T*>(d);
        return XP_OK;
    }
    unsigned char* scratch_for(uint32_t rows, uint32_t cols) {
        const uint64_t key = ((uint64_t)rows << 32) | cols;
        for (auto& kv : bscratch)
            if (kv.first == key) return kv.second;
        return nullptr;
    }
    // out (fp32) = in x W for every sequence
    cudaError_t mm(float* out, const BkOperand& in, const QW& w) {
        unsigned char* scr = scratch_for(w.rows, w.cols);
        if (!scr) return cudaErrorInvalidValue;
        const BmmMat m{reinterpret_cast<const uint32_t*>(w.wq), reinterpret_cast<const uint32_t*>(w.sc), w.cols, out, nullptr};
        const BmmPrep pr{in.xs, in.xb};
        return bmm_run(st, &m, 1, false, nullptr, w.rows, B, scr, &pr, pdl_mm, mode_of(w)) == XP_OK ? cudaSuccess
                                                                                                   : cudaErrorUnknown;
    }
    // raw[i] (fixed-point sums, zero on entry) = in x W[i] for every sequence:
    // matrices with the same rows in one launch
    cudaError_t mm_raw(std::initializer_list<std::pair<float*, const QW*>> parts, const BkOperand& in) {
        BmmMat m[BMM_MAXPARTS];
        uint32_t n = 0, cols = 0, rows = 0;
        int mode = BMM_MODE_SCALED;
        for (auto& pr : parts) {
            const QW& w = *pr.second;
            if (mode_of(w) != BMM_MODE_SCALED) mode = BMM_MODE_INTEGER;
            m[n++] = BmmMat{reinterpret_cast<const uint32_t*>(w.wq), reinterpret_cast<const uint32_t*>(w.sc), w.cols,
                            nullptr, pr.first};  // partials [ks][B][cols]
            cols += w.cols;
            rows = w.rows;
        }
        unsigned char* scr = scratch_for(rows, cols);
        if (!scr) return cudaErrorInvalidValue;
        const BmmPrep pr{in.xs, in.xb};
        return bmm_run(st, m, n, true, nullptr, rows, B, scr, &pr, pdl_mm, mode) == XP_OK ? cudaSuccess : cudaErrorUnknown;
    }
    // one position for every sequence: tokens -> logits, pos += 1
    cudaError_t resid_norm(BkSums y, const float* w_post, const float* w_pre, int mode) {
        return launch_ex(bk_resid_norm_kernel, dim3(B), dim3(BK_THREADS), 0, st, 1, pdl_k, x, y, w_post, w_pre, op_xn,
                         s->cfg.hidden, s->cfg.rms_eps, mode);
    }
    cudaError_t forward(bool head = true) {
        const xp_model_config& c = s->cfg;
        const uint32_t H = c.hidden, F = c.ffn, L = c.n_layers;
        const float escale = c.embed_scale > 0 ? c.embed_scale : std::sqrt((float)H);
        const float ascale = c.attn_scale > 0 ? c.attn_scale : 1.0f / std::sqrt((float)c.head_dim);
        cudaError_t e;
        if ((e = launch_ex(bk_embed_kernel, dim3(B), dim3(256), 0, st, 1, pdl_k, (const uint32_t*)tokens, (const float*)s->embed,
                           escale, x, H)) != cudaSuccess)
            return e;
        for (uint32_t l = 0; l < L; ++l) {
            const LayerDev& W = s->L[l];
            if ((e = resid_norm(sums(dn, ks_dn, H), l == 0 ? nullptr : s->L[l - 1].norm[3], W.norm[0], l == 0 ? 0 : 1)) !=
                cudaSuccess)
                return e;
            if ((e = mm_raw({{q, &W.m[0]}, {k, &W.m[1]}, {v, &W.m[2]}}, op_xn)) != cudaSuccess) return e;
            BkAttnArgs aa{};
            aa.q = sums(q, ks_qkv, 1024); aa.k = sums(k, ks_qkv, 256); aa.v = sums(v, ks_qkv, 256);
            aa.qn = W.norm[4]; aa.kn = W.norm[5];
            aa.kc = kc[l]; aa.vc = vc[l]; aa.pos = pos; aa.att = op_att; aa.max_seq = max_seq;
            const bool glob = s->is_global(l);
            aa.window = glob ? 0 : c.sliding_window;
            aa.theta = glob ? c.rope_theta_global : c.rope_theta_local;
            rope_table_host(aa.theta, aa.inv_freq);
            aa.eps = c.rms_eps;
            aa.scale = ascale;
            const uint32_t ms = aa.window ? std::min(aa.window, max_seq) : max_seq;
            aa.seq_stride = chunk ? 0 : (size_t)max_seq * 256;
            aa.mode = chunk ? 1 : 0;
            aa.split = chunk ? 1 : BK_ATT_SPLIT;  // decode steps only (prefill passes keep one CTA per row)
            if ((e = launch_ex(bk_attn_kernel, dim3(B * aa.split), dim3(BK_THREADS), (size_t)4 * ms * 4, st, aa.split, pdl_k,
                               aa)) != cudaSuccess)
                return e;
            if (chunk) {
                // every row's k and v are in the cache before any row attends
                aa.mode = 2;
                aa.split = 1;  // prefill rows: the 2-CTA split measured slower here
                if ((e = launch_ex(bk_attn_kernel, dim3(B * aa.split), dim3(BK_THREADS), (size_t)4 * ms * 4, st, aa.split,
                                   pdl_k, aa)) != cudaSuccess)
                    return e;
            }
            if ((e = mm_raw({{o, &W.m[3]}}, op_att)) != cudaSuccess) return e;
            if ((e = resid_norm(sums(o, ks_o, H), W.norm[1], W.norm[2], 1)) != cudaSuccess) return e;
            if ((e = mm_raw({{g, &W.m[4]}, {u, &W.m[5]}}, op_xn)) != cudaSuccess) return e;
            if ((e = launch_ex(bk_geglu_kernel, dim3(B * BK_GC), dim3(BK_THREADS), 0, st, BK_GC, pdl_k, sums(g, ks_gu, F),
                               sums(u, ks_gu, F), op_hb, F)) != cudaSuccess)
                return e;
            if ((e = mm_raw({{dn, &W.m[6]}}, op_hb)) != cudaSuccess) return e;
        }
        if (!head) {
            // a prompt position (or chunk) before the last: no LM head
            return launch_ex(bk_pos_inc_kernel, dim3(1), dim3(64), 0, st, 1, false, pos, B);
        }
        if ((e = resid_norm(sums(dn, ks_dn, H), s->L[L - 1].norm[3], s->final_norm, 1)) != cudaSuccess) return e;
        if ((e = mm(logits, op_xn, s->lm)) != cudaSuccess) return e;
        if ((e = launch_ex(bk_pos_inc_kernel, dim3(1), dim3(64), 0, st, 1, pdl_k, pos, B)) != cudaSuccess) return e;
        return cudaGetLastError();
    }
    // tokens[b] = sample(logits[b]) with the uniform of (seed, seq0 + b, pos[b])
    cudaError_t sample() {
        const uint32_t V = s->cfg.vocab;
        TopkDrawArgs da{};
        da.top_k = sp.greedy ? 1u : sp.top_k;
        da.temperature = sp.temperature;
        da.top_p = sp.top_p;
        da.seed = sp.seed;
        da.seq0 = seq0;
        da.token = tokens;
        da.pos_read = pos;
        cudaError_t e = launch_topk(logits, V, B, cand, da, st, true);
        if (e != cudaSuccess) return e;
        return cudaGetLastError();
    }
    xp_status capture(cudaGraphExec_t* out, bool with_sample, bool head = true) {
        cudaGraph_t gr = nullptr;
        XP_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = with_sample ? sample() : cudaSuccess;
        if (e == cudaSuccess) e = forward(head);
        cudaError_t e2 = cudaStreamEndCapture(st, &gr);
        if (e != cudaSuccess || e2 != cudaSuccess) {
            if (gr) cudaGraphDestroy(gr);
            return fail(XP_ERR_CUDA, "batch: graph capture failed: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
        }
        e = cudaGraphInstantiate(out, gr, 0);
        cudaGraphDestroy(gr);
        if (e != cudaSuccess) return fail(XP_ERR_CUDA, "batch: graph instantiate failed: %s", cudaGetErrorString(e));
        return XP_OK;
    }
};

extern "C" {

static xp_status bdec_create(xp_session* s, uint32_t nseq, uint32_t max_seq, const xp_sampling* sp, uint64_t seq0,
                             bool chunk, xp_bdec** out);
xp_status xp_bdec_create(xp_session* s, uint32_t nseq, uint32_t max_seq, const xp_sampling* sp, uint64_t seq0,
                          xp_bdec** out) {
    return bdec_create(s, nseq, max_seq, sp, seq0, false, out);
}
static xp_status bdec_create(xp_session* s, uint32_t nseq, uint32_t max_seq, const xp_sampling* sp, uint64_t seq0,
                             bool chunk, xp_bdec** out) {
    if (!s || !sp || !out) return fail(XP_ERR_INVALID, "xp_bdec_create: null argument");
    *out = nullptr;
    if (nseq == 0 || nseq > BMM_MAXN) return fail(XP_ERR_INVALID, "xp_bdec_create: 1..%d sequences (got %u)", BMM_MAXN, nseq);
    if (max_seq == 0 || max_seq > s->cfg.max_seq)
        return fail(XP_ERR_INVALID, "xp_bdec_create: max_seq %u (1..%u)", max_seq, s->cfg.max_seq);
    if (s->cfg.hidden > 4 * BK_THREADS || s->cfg.ffn > BK_GJ * BK_THREADS || s->cfg.hidden % 128 || s->cfg.ffn % 128 ||
        s->cfg.vocab % 128)
        return fail(XP_ERR_UNSUPPORTED, "xp_bdec_create: hidden <= 2048, ffn <= 8192, and hidden, ffn, vocab multiples of 128");
    if ((size_t)4 * max_seq * 4 > 200 * 1024)
        return fail(XP_ERR_UNSUPPORTED, "xp_bdec_create: max_seq %u exceeds the attention kernel's score buffer", max_seq);
    auto* b = new xp_bdec();
    b->s = s;
    b->device = s->device;
    b->B = nseq;
    b->max_seq = max_seq;
    b->sp = *sp;
    b->seq0 = seq0;
    b->chunk = chunk;
    cudaSetDevice(b->device);
    auto bail = [&](xp_status st) { delete b; return st; };
    if (cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreate(&b->ev_a) != cudaSuccess || cudaEventCreate(&b->ev_b) != cudaSuccess)
        return bail(fail(XP_ERR_CUDA, "xp_bdec_create: stream/event creation failed"));
    const xp_model_config& c = s->cfg;
    const size_t H = c.hidden, F = c.ffn, QD = s->q_dim(), KVD = s->kv_dim(), V = c.vocab;
    xp_status e;
#define BA(p, n) if ((e = b->alloc(&b->p, (n))) != XP_OK) return bail(e)
    // partial-sum buffers: one per K range of the launch that fills them
    b->ks_qkv = bmm_ksplit((uint32_t)H, (uint32_t)(QD + 2 * KVD), nseq);
    b->ks_o = bmm_ksplit((uint32_t)QD, (uint32_t)H, nseq);
    b->ks_gu = bmm_ksplit((uint32_t)H, (uint32_t)(2 * F), nseq);
    b->ks_dn = bmm_ksplit((uint32_t)F, (uint32_t)H, nseq);
    BA(x, nseq * H); BA(q, b->ks_qkv * nseq * QD); BA(k, b->ks_qkv * nseq * KVD); BA(v, b->ks_qkv * nseq * KVD);
    BA(o, b->ks_o * nseq * H); BA(g, b->ks_gu * nseq * F); BA(u, b->ks_gu * nseq * F); BA(dn, b->ks_dn * nseq * H);
    BA(logits, nseq * V);
    for (auto pr : {std::make_pair(&b->op_xn, H), std::make_pair(&b->op_att, QD), std::make_pair(&b->op_hb, F)}) {
        BkOperand& op = *pr.first;
        op.Npad = bmm_npad(nseq);
        if ((e = b->alloc(&op.xs, 64)) != XP_OK) return bail(e);
        if ((e = b->alloc(&op.xb, bmm_xb_bytes(pr.second, nseq))) != XP_OK) return bail(e);
    }
    BA(tokens, nseq); BA(pos, nseq);
#undef BA
    b->kc.resize(c.n_layers);
    b->vc.resize(c.n_layers);
    for (uint32_t l = 0; l < c.n_layers; ++l) {
        if (chunk) {
            b->kc[l] = s->L[l].kc;
            b->vc[l] = s->L[l].vc;
            continue;
        }
        if ((e = b->alloc(&b->kc[l], (size_t)nseq * max_seq * 256)) != XP_OK) return bail(e);
        if ((e = b->alloc(&b->vc[l], (size_t)nseq * max_seq * 256)) != XP_OK) return bail(e);
    }
    // launch shapes (rows, total columns): q|k|v, o, gate|up, down, LM head
    const uint32_t shapes[5][2] = {{(uint32_t)H, (uint32_t)(QD + 2 * KVD)}, {(uint32_t)QD, (uint32_t)H},
                                   {(uint32_t)H, (uint32_t)(2 * F)}, {(uint32_t)F, (uint32_t)H}, {(uint32_t)H, (uint32_t)V}};
    for (auto& sh : shapes) {
        const uint64_t key = ((uint64_t)sh[0] << 32) | sh[1];
        bool have = false;
        for (auto& kv : b->bscratch) have = have || kv.first == key;
        if (have) continue;
        const size_t sb = xp_mv_km4_bs_batch_scratch_bytes(sh[0], sh[1], nseq);
        if (sb == 0) return bail(fail(XP_ERR_UNSUPPORTED, "xp_bdec_create: a matrix shape is not supported by the batched matvec"));
        unsigned char* scr = nullptr;
        if ((e = b->alloc(&scr, sb)) != XP_OK) return bail(e);
        b->bscratch.push_back({key, scr});
    }
    {
        // operand mode per matrix: scan each scale plane once
        uint32_t* dflag = nullptr;
        if ((e = b->alloc(&dflag, 1)) != XP_OK) return bail(e);
        auto check = [&](const QW& w) -> cudaError_t {
            if (!w.sc || b->s16.count(w.sc)) return cudaSuccess;
            bool ok = false;
            const cudaError_t ce = bmm_scales_exact16(b->st, w.sc, w.rows, w.cols, dflag, &ok);
            b->s16[w.sc] = ok;
            return ce;
        };
        cudaError_t ce = check(s->lm);
        for (uint32_t l = 0; l < c.n_layers && ce == cudaSuccess; ++l)
            for (const QW& w : s->L[l].m)
                if (ce == cudaSuccess) ce = check(w);
        if (ce != cudaSuccess)
            return bail(fail(XP_ERR_CUDA, "xp_bdec_create: scale-range check failed: %s", cudaGetErrorString(ce)));
    }
    b->ns = (uint32_t)((V + TOPK_SLICE - 1) / TOPK_SLICE);
    b->nc = b->ns * TOPK_TK;
    if ((e = b->alloc(&b->cand, (size_t)nseq * b->nc)) != XP_OK) return bail(e);
    if (cudaHostAlloc(&b->h_tok, (size_t)nseq * 4, cudaHostAllocDefault) != cudaSuccess)
        return bail(fail(XP_ERR_OOM, "xp_bdec_create: pinned buffer"));
    XP_CUDA_TRY(cudaFuncSetAttribute(bk_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    // warm every kernel once outside capture (attributes, lazy loading); a
    // chunk object must not touch the session's caches here
    if (chunk) {
        // every row at the last position: the only cache row written is the
        // last one, which a real pass at that position writes before reading
        std::vector<uint32_t> hp(nseq, max_seq - 1);
        XP_CUDA_TRY(h2d_sync(b->pos, hp.data(), (size_t)nseq * 4));
    }
    if (b->forward() != cudaSuccess) return bail(fail(XP_ERR_CUDA, "xp_bdec_create: warm-up forward failed"));
    XP_CUDA_TRY(cudaMemsetAsync(b->pos, 0, (size_t)nseq * 4, b->st));
    XP_CUDA_TRY(cudaStreamSynchronize(b->st));
    if ((e = b->capture(&b->g_fwd, false)) != XP_OK) return bail(e);
    if ((e = b->capture(&b->g_step, true)) != XP_OK) return bail(e);
    if ((e = b->capture(&b->g_nohead, false, false)) != XP_OK) return bail(e);
    *out = b;
    return XP_OK;
}

void xp_bdec_destroy(xp_bdec* b) { delete b; }

xp_status xp_bdec_prefill(xp_bdec* b, const uint32_t* tokens, uint32_t n) {
    if (!b || (!tokens && n)) return fail(XP_ERR_INVALID, "xp_bdec_prefill: null argument");
    if (b->h_pos + n > b->max_seq) return fail(XP_ERR_KV_FULL, "xp_bdec_prefill: %u + %u > max_seq %u", b->h_pos, n, b->max_seq);
    cudaSetDevice(b->device);
    for (uint32_t t = 0; t < n; ++t) {
        std::memcpy(b->h_tok, tokens + (size_t)t * b->B, (size_t)b->B * 4);
        XP_CUDA_TRY(cudaMemcpyAsync(b->tokens, b->h_tok, (size_t)b->B * 4, cudaMemcpyHostToDevice, b->st));
        // only the last prompt position's logits are kept
        XP_CUDA_TRY(cudaGraphLaunch(t + 1 < n ? b->g_nohead : b->g_fwd, b->st));
        XP_CUDA_TRY(cudaStreamSynchronize(b->st));  // h_tok is reused
        ++b->h_pos;
    }
    return XP_OK;
}

xp_status xp_bdec_step(xp_bdec* b, uint32_t* tokens_out) {
    if (!b) return fail(XP_ERR_INVALID, "xp_bdec_step: null batch");
    if (b->h_pos == 0) return fail(XP_ERR_STATE, "xp_bdec_step: prefill at least one token first");
    if (b->h_pos + 1 > b->max_seq) return fail(XP_ERR_KV_FULL, "xp_bdec_step: position %u at max_seq", b->h_pos);
    cudaSetDevice(b->device);
    XP_CUDA_TRY(cudaGraphLaunch(b->g_step, b->st));
    ++b->h_pos;
    if (tokens_out) {
        XP_CUDA_TRY(cudaMemcpyAsync(b->h_tok, b->tokens, (size_t)b->B * 4, cudaMemcpyDeviceToHost, b->st));
        XP_CUDA_TRY(cudaStreamSynchronize(b->st));
        std::memcpy(tokens_out, b->h_tok, (size_t)b->B * 4);
    }
    return XP_OK;
}

xp_status xp_bdec_generate(xp_bdec* b, uint32_t n, float* ms) {
    if (!b) return fail(XP_ERR_INVALID, "xp_bdec_generate: null batch");
    if (b->h_pos == 0) return fail(XP_ERR_STATE, "xp_bdec_generate: prefill at least one token first");
    if (b->h_pos + n > b->max_seq) return fail(XP_ERR_KV_FULL, "xp_bdec_generate: %u + %u > max_seq", b->h_pos, n);
    cudaSetDevice(b->device);
    XP_CUDA_TRY(cudaEventRecord(b->ev_a, b->st));
    for (uint32_t i = 0; i < n; ++i) XP_CUDA_TRY(cudaGraphLaunch(b->g_step, b->st));
    XP_CUDA_TRY(cudaEventRecord(b->ev_b, b->st));
    XP_CUDA_TRY(cudaEventSynchronize(b->ev_b));
    b->h_pos += n;
    float t = 0;
    XP_CUDA_TRY(cudaEventElapsedTime(&t, b->ev_a, b->ev_b));
    if (ms) *ms = t;
    return XP_OK;
}

xp_status xp_bdec_logits(xp_bdec* b, float* out, size_t n) {
    if (!b || !out) return fail(XP_ERR_INVALID, "xp_bdec_logits: null argument");
    const size_t all = (size_t)b->B * b->s->cfg.vocab;
    cudaSetDevice(b->device);
    XP_CUDA_TRY(cudaStreamSynchronize(b->st));
    XP_CUDA_TRY(cudaMemcpy(out, b->logits, std::min(n, all) * 4, cudaMemcpyDeviceToHost));
    return XP_OK;
}

xp_status xp_bdec_position(xp_bdec* b, uint32_t* pos) {
    if (!b || !pos) return fail(XP_ERR_INVALID, "xp_bdec_position: null argument");
    *pos = b->h_pos;
    return XP_OK;
}

}  // extern "C"

extern "C" {

xp_status xp_session_tp_handle(xp_session* s, void* handle) {
    if (!s || !handle) return fail(XP_ERR_INVALID, "xp_session_tp_handle: null argument");
    if (!s->use_tk) return fail(XP_ERR_UNSUPPORTED, "xp_session_tp_handle: needs the persistent token kernel path");
    cudaSetDevice(s->device);
    cudaIpcMemHandle_t h;
    XP_CUDA_TRY(cudaIpcGetMemHandle(&h, s->tp_buf));
    std::memcpy(handle, &h, sizeof(h));
    return XP_OK;
}

xp_status xp_session_tp_attach(xp_session* s, uint32_t rank, uint32_t world, const void* handles) {
    return xp_session_tp_attach_ex(s, rank, world, handles, 0u);
}

xp_status xp_session_tp_attach_ex(xp_session* s, uint32_t rank, uint32_t world, const void* handles, uint32_t flags) {
    if (!s || !handles) return fail(XP_ERR_INVALID, "xp_session_tp_attach: null argument");
    if (!s->use_tk) return fail(XP_ERR_UNSUPPORTED, "xp_session_tp_attach: needs the persistent token kernel path");
    if (world == 0 || world > TK_TP_MAX || rank >= world)
        return fail(XP_ERR_INVALID, "xp_session_tp_attach: rank %u of %u (world 1..%u)", rank, world, TK_TP_MAX);
    cudaSetDevice(s->device);
    xp_status st = s->wait_prev();
    if (st != XP_OK) return st;
    for (void* p : s->tp_peers) cudaIpcCloseMemHandle(p);
    s->tp_peers.clear();
    const unsigned char* hb = static_cast<const unsigned char*>(handles);
    for (uint32_t r = 0; r < world; ++r) {
        if (r == rank) {
            s->tk.tp_slots[r] = reinterpret_cast<TkTpSlot*>(s->tp_buf);
            s->tk.dn_rx[r] = reinterpret_cast<unsigned long long*>(s->tk.tp_slots[r] + TK_TP_SLOTS);
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)r * sizeof(h), sizeof(h));
        void* p = nullptr;
        XP_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        s->tp_peers.push_back(p);
        s->tk.tp_slots[r] = static_cast<TkTpSlot*>(p);
        s->tk.dn_rx[r] = reinterpret_cast<unsigned long long*>(s->tk.tp_slots[r] + TK_TP_SLOTS);
    }
    // units of 64 vocabulary rows split evenly; every rank runs the same launches
    const uint32_t U = s->tk.head.units;
    s->tk.head_u0 = (uint32_t)((uint64_t)U * rank / world);
    s->tk.head_u1 = (uint32_t)((uint64_t)U * (rank + 1) / world);
    // sampling draws from every shard's candidate lists, made per sampler
    // slice: the shards must split the vocabulary on slice boundaries
    if (!s->sp.greedy && world > 1 &&
        ((s->tk.head_u0 * 64) % TOPK_SLICE || (s->tk.head_u1 * 64) % TOPK_SLICE))
        return fail(XP_ERR_UNSUPPORTED,
                    "xp_session_tp_attach: sampled decoding needs the vocabulary (%u) split on %u-row slices over %u ranks",
                    s->cfg.vocab, TOPK_SLICE, world);
    s->tk.tp_rank = rank;
    s->tk.tp_world = world;
    // FFN row shard: gate|up units of 16 GeGLU rows split evenly, the
    // down-proj K rows with them (its sums exchanged inside the launch)
    const bool ffn = (flags & XP_TP_SHARD_FFN) && world > 1;
    const uint32_t GU = s->tk.gu.units;
    s->tk.gu_u0 = ffn ? (uint32_t)((uint64_t)GU * rank / world) : 0u;
    s->tk.gu_u1 = ffn ? (uint32_t)((uint64_t)GU * (rank + 1) / world) : GU;
    s->tk.ffn_shard = ffn ? 1 : 0;
    // The tensor-parallel kernel fixes every down-proj unit's partial sum on
    // its own, so its results do not depend on how units fall on ranks; one
    // rank attached with XP_TP_SHARD_FFN runs it too (the reference for the
    // sharded runs, bit for bit).
    s->tk_tp_instance = world > 1 || (flags & XP_TP_SHARD_FFN);
    XP_CUDA_TRY(zero_fill_sync(s->tp_buf, s->tp_buf_bytes()));
    XP_CUDA_TRY(zero_fill_sync(s->tk.tp_count, 8));
    for (cudaGraphExec_t* g : {&s->g_dev, &s->g_io, &s->g_prefill})
        if (*g) { cudaGraphExecDestroy(*g); *g = nullptr; }
    return s->build_graphs();
}

}  // extern "C"

// Chunked prefill: the prompt as tensor-core GEMMs. Up to 64 prompt
// positions per pass run as the rows of the batched engine over the
// session's own KV caches: tensor-core matvecs for all rows at once, then
// per layer every row's k and v appended before any row attends (causal over
// the cache, the window rule per layer). Only the last position's logits are
// kept; the next token comes from them as after a per-token prefill.
static xp_status prefill_chunked(xp_session* s, const uint32_t* tokens, uint32_t n) {
    xp_status st = s->wait_prev();
    if (st != XP_OK) return st;
    if (!s->pre) {
        const xp_sampling sp = s->sp;
        st = bdec_create(s, BMM_MAXN, s->cfg.max_seq, &sp, 0, true, &s->pre);
        if (st != XP_OK) {
            s->pre = nullptr;
            s->pre_failed = true;
            return XP_ERR_UNSUPPORTED;  // the caller falls back to one pass per token
        }
    }
    xp_bdec* b = s->pre;
    const uint32_t B = b->B;
    std::vector<uint32_t> tk(B), ps(B);
    uint32_t last = 0;
    for (uint32_t p = 0; p < n; p += B) {
        const uint32_t m = std::min(B, n - p);
        for (uint32_t r = 0; r < B; ++r) {
            const uint32_t q = p + std::min(r, m - 1);  // rows past the chunk repeat its last position
            tk[r] = tokens[q];
            ps[r] = s->host_pos + q;
        }
        XP_CUDA_TRY(cudaMemcpyAsync(b->tokens, tk.data(), (size_t)B * 4, cudaMemcpyHostToDevice, b->st));
        XP_CUDA_TRY(cudaMemcpyAsync(b->pos, ps.data(), (size_t)B * 4, cudaMemcpyHostToDevice, b->st));
        XP_CUDA_TRY(cudaGraphLaunch(p + m < n ? b->g_nohead : b->g_fwd, b->st));
        XP_CUDA_TRY(cudaStreamSynchronize(b->st));  // tk / ps are reused
        last = m - 1;
    }
    // the last position's logits become the session's; then what the last
    // token-kernel pass would have done: the position advances and the next
    // token is picked (greedy: lowest-index maximum) or sampled
    const uint32_t V = s->cfg.vocab;
    const uint32_t endpos = s->host_pos + n;
    XP_CUDA_TRY(cudaMemcpyAsync(s->logits, b->logits + (size_t)last * V, (size_t)V * 4, cudaMemcpyDeviceToDevice, s->st));
    // both pickers advance the position from the last prompt position
    const uint32_t p_last = endpos - 1;
    XP_CUDA_TRY(cudaMemcpyAsync(s->pos, &p_last, 4, cudaMemcpyHostToDevice, s->st));
    if (s->sp.greedy) {
        XP_CUDA_TRY(launch_ex(greedy_final_kernel, dim3(1), dim3(1024), 0, s->st, 1, false, (const float*)s->logits,
                              (const uint32_t*)nullptr, V, s->token, s->sample_out, s->pos, s->hist));
    } else {
        XP_CUDA_TRY(launch_sample_topk(s->token, s->sample_out, s->pos, nullptr, nullptr, s->logits, V, s->sp.top_k,
                                       s->sp.temperature, s->sp.top_p, s->sp.seed, s->sp.seq_id, s->samp_scratch, s->st,
                                       false, true, s->hist));
    }
    XP_CUDA_TRY(cudaMemcpyAsync(s->h_out, s->token, 4, cudaMemcpyDeviceToHost, s->st));
    XP_CUDA_TRY(cudaStreamSynchronize(s->st));
    s->host_pos = endpos;
    s->have_logits = true;
    return XP_OK;
}
