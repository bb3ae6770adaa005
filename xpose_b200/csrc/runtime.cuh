// Host runtime pieces shared by the C ABI and the decode engine: error
// state, device properties, and launch helpers for the fused kernels.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstring>
#include <cstdio>
#include <cstdlib>
#include <string>

#include "../../include/xp_cuda.h"
#include "attention.cuh"
#include "aux_kernels.cuh"
#include "matvec.cuh"

namespace xp {

inline thread_local std::string g_err;

inline xp_status fail(xp_status s, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return s;
}

#define XP_CUDA_TRY(expr)                                                                          \
    do {                                                                                           \
        cudaError_t e_ = (expr);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            return ::xp::fail(e_ == cudaErrorMemoryAllocation ? XP_ERR_OOM : XP_ERR_CUDA,          \
                              "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                              __LINE__);                                                           \
    } while (0)

constexpr int kMaxDevices = 64;

inline int sm_count() {
    static std::atomic<int> per_dev[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) dev = 0;
    int n = per_dev[dev].load(std::memory_order_relaxed);
    if (!n) {
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
        per_dev[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Function attributes are held per device: raise `kern`'s dynamic shared
// memory limit (and optionally allow non-portable cluster sizes) on the
// current device the first time it launches there. `done` is the call site's
// per-device flag array.
template <typename Kern>
inline cudaError_t smem_attr_once(std::atomic<bool>* done, Kern* kern, int bytes, bool nonportable_cluster = false) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool track = dev >= 0 && dev < kMaxDevices;
    if (track && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && nonportable_cluster)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess && track) done[dev].store(true, std::memory_order_release);
    return e;
}

// Zero-fill device memory and wait for it. cudaMemset runs on the legacy
// default stream, which the library's non-blocking streams do not order
// against: without the wait, a fill could land after the first uploads or
// kernels on those streams. Set-up paths only.
inline cudaError_t zero_fill_sync(void* d, size_t bytes) {
    cudaError_t e = cudaMemset(d, 0, bytes);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    return e;
}
// Host -> device copy that has landed when it returns: a plain cudaMemcpy from
// pageable memory may return once the data is staged, before the DMA that
// work on the non-blocking streams would not wait for. Set-up paths only.
inline cudaError_t h2d_sync(void* dst, const void* src, size_t bytes) {
    cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    return e;
}

// Launch with optional cluster size and programmatic dependent launch.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             unsigned cluster_x, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    unsigned na = 0;
    if (cluster_x > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cluster_x;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

// ---- int4 matvec -------------------------------------------------------------------
inline uint32_t mv_per(const MvArgs& a) {
    const uint32_t nblk = a.K / 32;
    if (a.quad_split) return 4 * ((nblk / 4 + a.ksplit - 1) / a.ksplit);
    return (nblk + a.ksplit - 1) / a.ksplit;
}

inline cudaError_t launch_mv(const MvArgs& a, cudaStream_t st, bool pdl, uint32_t max_ctas = 0) {
    static std::atomic<bool> attr_set[kMaxDevices];
    if (cudaError_t e = smem_attr_once(attr_set, mv_kernel, 200 * 1024, true); e != cudaSuccess) return e;
    const size_t smem = MvSmem::bytes(a, mv_per(a));
    uint32_t grid;
    unsigned cluster = 1;
    if (a.ksplit > 1) {
        grid = a.ntiles * a.ksplit;
        if (a.epi != EPI_PARTIAL) cluster = a.ksplit;
    } else {
        grid = a.ntiles;
        if (max_ctas && grid > max_ctas) grid = max_ctas;
    }
    return launch_ex(mv_kernel, dim3(grid), dim3(MV_THREADS), smem, st, cluster, pdl, a);
}

// ---- attention -------------------------------------------------------------------------
// CTAs per split launch: nsplit, rounded up to a multiple of 8 above 64 so
// that large grids form clusters of 8 (else 4, 2 or 1 CTAs). A grid that is a
// multiple of 16 forms clusters of 16 (a non-portable size: one GPC), one
// merge level fewer at 16 and 128 splits; XP_ATTN_CLUSTER=8 keeps clusters
// within the portable 8.
constexpr uint32_t attn_grid(uint32_t nsplit) { return nsplit <= 64 ? nsplit : (nsplit + 7) & ~7u; }
inline uint32_t attn_cluster_max() {
    static const uint32_t c = [] {
        const char* e = std::getenv("XP_ATTN_CLUSTER");
        return (e && std::atoi(e) == 8) ? 8u : 16u;
    }();
    return c;
}
inline uint32_t attn_cluster(uint32_t grid) {
    if (attn_cluster_max() == 16 && grid % 16 == 0) return 16;
    return grid % 8 == 0 ? 8 : grid % 4 == 0 ? 4 : grid % 2 == 0 ? 2 : 1;
}
// scratch: [ticket u32 | error word u32 | pad to 512][cluster partials | cluster stats]
constexpr size_t ATT_SCRATCH_HDR = 512;
constexpr size_t attn_scratch_bytes(uint32_t nsplit) {
    return ATT_SCRATCH_HDR + (size_t)attn_grid(nsplit) * (4 * 256 * 4 + 8 * 4);
}
// Longest span one call attends: the window of a sliding-window layer, else
// every row the caches hold.
constexpr uint32_t attn_span_max(uint32_t window, uint32_t max_seq) {
    return (window != 0 && window < max_seq) ? window : max_seq;
}
inline uint32_t attn_chunk_max(uint32_t nsplit, uint32_t max_seq) {
    uint32_t c = (max_seq + nsplit - 1) / nsplit;
    return (c + 7) & ~7u;
}
inline size_t attn_smem(uint32_t chunk_max, uint32_t cluster) { return AttnSmem::bytes(chunk_max, cluster); }
// RoPE inverse frequencies theta^(-2d/256), d < 128, with log2 and exp2 each
// rounded once from double (the oracle's formula, computed on the host so the
// device table matches it bit for bit). Small per-thread cache: decode
// alternates between two thetas.
inline void rope_table_host(float theta, float* out) {
    thread_local float cache_theta[4] = {-1.0f, -1.0f, -1.0f, -1.0f};
    thread_local float cache[4][128];
    thread_local int next = 0;
    for (int c = 0; c < 4; ++c)
        if (cache_theta[c] == theta) {
            std::memcpy(out, cache[c], 128 * sizeof(float));
            return;
        }
    const float l2 = (float)std::log2((double)theta);
    for (uint32_t d = 0; d < 128; ++d) {
        const float frac = (float)(2u * d) / 256.0f;
        out[d] = (float)std::exp2((double)(-l2 * frac));
    }
    cache_theta[next] = theta;
    std::memcpy(cache[next], out, 128 * sizeof(float));
    next = (next + 1) & 3;
}
inline cudaError_t launch_attn(AttnArgs a, void* scratch, uint32_t nsplit, uint32_t max_seq, cudaStream_t st,
                               bool pdl) {
    static std::atomic<bool> attr_set[kMaxDevices];
    if (cudaError_t e = smem_attr_once(attr_set, attn_decode_kernel<4>, (int)ATT_SMEM_MAX, true); e != cudaSuccess) return e;
    char* s = static_cast<char*>(scratch);
    const uint32_t grid = attn_grid(nsplit), cl = attn_cluster(grid);
    a.ticket = reinterpret_cast<uint32_t*>(s);
    a.err = a.ticket + 1;
    a.part = reinterpret_cast<float*>(s + ATT_SCRATCH_HDR);
    a.pstat = a.part + (size_t)(grid / cl) * 4 * 256;
    a.chunk_max = attn_chunk_max(grid, max_seq);
    rope_table_host(a.theta, a.inv_freq);
    return launch_ex(attn_decode_kernel<4>, dim3(grid), dim3(ATT_THREADS), attn_smem(a.chunk_max, cl), st, cl, pdl, a);
}

// ---- sampling ----------------------------------------------------------------------------
constexpr uint32_t TOPK_SLICE = TOPK_THREADS * 8;
constexpr uint32_t TOPK_TK = 64;
constexpr uint32_t TOPK_MAX_CAND = 200 * 1024 / 8;  // phase-2 candidates held in shared memory
inline size_t sample_scratch_bytes(uint32_t n) {
    const uint32_t ns = (n + TOPK_SLICE - 1) / TOPK_SLICE;
    return (size_t)ns * TOPK_TK * 8 + 64;
}
// Two launches over nseq sequences of n logits each: slice candidates, then
// one drawing CTA per sequence. `cand` holds nseq * slices * TOPK_TK keys.
inline cudaError_t launch_topk(const float* logits, uint32_t n, uint32_t nseq, uint64_t* cand,
                               const TopkDrawArgs& da_in, cudaStream_t st, bool pdl,
                               const TpCandArgs* tp = nullptr) {
    static std::atomic<bool> attr_set[kMaxDevices];
    if (cudaError_t e = smem_attr_once(attr_set, topk_draw_kernel, 200 * 1024); e != cudaSuccess) return e;
    const uint32_t ns = (n + TOPK_SLICE - 1) / TOPK_SLICE;
    const uint32_t s0 = tp ? tp->s0 : 0u, s1 = tp ? tp->s1 : ns;
    cudaError_t e = launch_ex(topk_cand_kernel, dim3(s1 - s0, nseq), dim3(TOPK_THREADS), 0, st, 1, pdl, logits, n, cand,
                              s0, ns);
    if (e != cudaSuccess) return e;
    TopkDrawArgs da = da_in;
    da.cand = cand;
    if (tp) {  // sharded logits: gather every rank's candidate lists into cand, then draw from them
        TpCandArgs x = *tp;
        x.cand = cand;
        x.ns = ns;
        e = launch_ex(tp_cand_exchange_kernel, dim3(1), dim3(1024), 0, st, 1, true, x);
        if (e != cudaSuccess) return e;
    }
    da.ncand = ns * TOPK_TK;
    if (da.top_k == 0 || da.top_k > TOPK_TK) da.top_k = TOPK_TK;
    return launch_ex(topk_draw_kernel, dim3(nseq), dim3(TOPK_THREADS), (size_t)da.ncand * 8, st, 1, true, da);
}
inline cudaError_t launch_sample_topk(uint32_t* token, float* sample_out, uint32_t* pos_dev, float* out_vals,
                                      uint32_t* out_idx, const float* logits, uint32_t n, uint32_t top_k,
                                      float temperature, float top_p, uint64_t seed, uint64_t seq_id, void* scratch,
                                      cudaStream_t st, bool pdl, bool advance, uint32_t* hist = nullptr,
                                      const TpCandArgs* tp = nullptr) {
    TopkDrawArgs da{};
    da.top_k = top_k;
    da.temperature = temperature;
    da.top_p = top_p;
    da.seed = seed;
    da.seq0 = seq_id;
    da.token = token;
    da.sample_out = sample_out;
    // the sampler reads *pos for the uniform's index; it advances it only in
    // the engine (advance == true)
    da.pos_adv = advance ? pos_dev : nullptr;
    da.pos_read = advance ? nullptr : pos_dev;
    da.out_vals = out_vals;
    da.out_idx = out_idx;
    da.hist = hist;
    return launch_topk(logits, n, 1, static_cast<uint64_t*>(scratch), da, st, pdl, tp);
}

}  // namespace xp
