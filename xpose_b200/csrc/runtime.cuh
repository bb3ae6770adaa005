// Host runtime pieces shared by the C ABI and the decode engine: error
// state, device properties, and launch helpers for the fused kernels.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
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

inline int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
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
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(mv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        cudaFuncSetAttribute(mv_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        attr_set = true;
    }
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
inline size_t attn_scratch_bytes(uint32_t nsplit) {
    return (size_t)nsplit * 4 * 256 * 4 + (size_t)nsplit * 8 * 4 + 64;
}
inline uint32_t attn_chunk_max(uint32_t nsplit, uint32_t max_seq) {
    uint32_t c = (max_seq + nsplit - 1) / nsplit;
    return (c + 7) & ~7u;
}
inline size_t attn_smem(uint32_t chunk_max) {
    return 4 * 256 * 4 + 2 * 256 * 2 + 4 * (size_t)chunk_max * 4 + 2 * 4 * 256 * 4 + 8 * 4;
}
inline cudaError_t launch_attn(AttnArgs a, void* scratch, uint32_t nsplit, uint32_t max_seq, cudaStream_t st,
                               bool pdl) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(attn_decode_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_set = true;
    }
    // scratch: [ticket u32 | error word u32 | pad to 64 B | partials | stats]
    char* s = static_cast<char*>(scratch);
    a.ticket = reinterpret_cast<uint32_t*>(s);
    a.err = a.ticket + 1;
    a.part = reinterpret_cast<float*>(s + 64);
    a.pstat = reinterpret_cast<float*>(s + 64 + (size_t)nsplit * 4 * 256 * 4);
    a.chunk_max = attn_chunk_max(nsplit, max_seq);
    return launch_ex(attn_decode_kernel<4>, dim3(nsplit), dim3(ATT_THREADS), attn_smem(a.chunk_max), st, 1, pdl,
                     a);
}

// ---- sampling ----------------------------------------------------------------------------
constexpr uint32_t TOPK_SLICE = 2048;
constexpr uint32_t TOPK_TK = 64;
inline uint32_t pow2_ceil(uint32_t v) {
    uint32_t p = 1;
    while (p < v) p <<= 1;
    return p;
}
inline size_t sample_scratch_bytes(uint32_t n) {
    const uint32_t ns = (n + TOPK_SLICE - 1) / TOPK_SLICE;
    return (size_t)ns * TOPK_TK * 8 + 64;
}
inline cudaError_t launch_sample_topk(uint32_t* token, float* sample_out, uint32_t* pos_dev, float* out_vals,
                                      uint32_t* out_idx, const float* logits, uint32_t n, uint32_t top_k,
                                      float temperature, float top_p, uint64_t seed, uint64_t seq_id, void* scratch,
                                      cudaStream_t st, bool pdl, bool advance, uint32_t* hist = nullptr) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(topk_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr_set = true;
    }
    const uint32_t ns = (n + TOPK_SLICE - 1) / TOPK_SLICE;
    uint64_t* cand = static_cast<uint64_t*>(scratch);
    cudaError_t e = launch_ex(topk_slice_kernel, dim3(ns), dim3(256), TOPK_SLICE * 8, st, 1, pdl, logits, n,
                              TOPK_SLICE, TOPK_TK, cand);
    if (e != cudaSuccess) return e;
    const uint32_t nc = ns * TOPK_TK;
    const uint32_t p2 = pow2_ceil(nc);
    if (top_k == 0 || top_k > TOPK_TK) top_k = TOPK_TK;
    // the sampler reads *pos for the uniform's index; it advances it only in
    // the engine (advance == true)
    return launch_ex(topk_sample_kernel, dim3(1), dim3(1024), (size_t)p2 * 8, st, 1, pdl, (const uint64_t*)cand,
                     p2, nc, top_k, temperature, top_p, seed, seq_id, token, sample_out,
                     advance ? pos_dev : (uint32_t*)nullptr, out_vals, out_idx,
                     advance ? (const uint32_t*)nullptr : (const uint32_t*)pos_dev, hist);
}

}  // namespace xp
