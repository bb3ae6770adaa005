// C ABI: runtime (context, buffers), kernel registry with the reference's
// launch validation, Batch -> CUDA graph, Fence, and the typed entry points.
#pragma once
#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <unordered_map>
#include <utility>
#include <vector>

#include "bmm.cuh"
#include "mv_stream.cuh"
#include "ops.cuh"
#include "quant.cuh"
#include "runtime.cuh"

using namespace xp;

// ============================================================================
// Registry
// ============================================================================
namespace {

enum Geo : int {
    GEO_THREADS = 0,   // one thread per global id, 256-thread CTAs
    GEO_WARPS = 1,     // one warp per global id
    GEO_ROWS = 2,      // one CTA per global id
    GEO_ONE = 3,       // one CTA of 1024 threads regardless of grid
    GEO_CUSTOM = 4,    // launcher picks (matvec family)
    GEO_HEADS = 5,     // rmsnorm_heads: one warp per head; grid = heads * head_dim
};

struct ArgSpec {
    int kind;       // 1 buffer, 0 pod
    uint32_t size;  // pod size
};

using Launcher = cudaError_t (*)(const xp_arg* a, xp_grid g, cudaStream_t st);

struct Entry {
    const char* module;
    const char* name;
    const char* arg_names;  // comma separated, from the reference prototype
    std::vector<ArgSpec> args;
    Launcher launch;
};

template <class T> T arg_as(const xp_arg& a) {
    if constexpr (std::is_pointer_v<T>) {
        return (T)(const_cast<void*>(a.ptr));
    } else {
        T v{};
        std::memcpy(&v, a.ptr, sizeof(T));
        return v;
    }
}
template <class T> constexpr ArgSpec spec_of() {
    if constexpr (std::is_pointer_v<T>) return ArgSpec{1, 0};
    else return ArgSpec{0, (uint32_t)sizeof(T)};
}

template <auto K, int G> struct Gen;
template <class... P, void (*K)(P...), int G> struct Gen<K, G> {
    template <size_t... I>
    static cudaError_t go(const xp_arg* a, dim3 grid, dim3 block, cudaStream_t st, std::index_sequence<I...>) {
        K<<<grid, block, 0, st>>>(arg_as<P>(a[I])...);
        return cudaGetLastError();
    }
    static cudaError_t launch(const xp_arg* a, xp_grid g, cudaStream_t st) {
        const uint64_t n = (uint64_t)g.x * g.y * g.z;
        dim3 grid, block;
        switch (G) {
            case GEO_THREADS: block = dim3(256); grid = dim3((unsigned)((n + 255) / 256)); break;
            case GEO_WARPS: block = dim3(256); grid = dim3((unsigned)((n * 32 + 255) / 256)); break;
            case GEO_ROWS: block = dim3(256); grid = dim3((unsigned)n); break;
            case GEO_ONE: block = dim3(1024); grid = dim3(1); break;
            default: block = dim3(256); grid = dim3((unsigned)((n + 255) / 256)); break;
        }
        return go(a, grid, block, st, std::index_sequence_for<P...>{});
    }
    static std::vector<ArgSpec> specs() { return {spec_of<P>()...}; }
};

// rmsnorm_heads_gemma: grid = n_heads * head_dim in the reference; here one warp per head.
cudaError_t launch_heads(const xp_arg* a, xp_grid, cudaStream_t st) {
    const uint32_t nh = arg_as<uint32_t>(a[3]);
    ops::rmsnorm_heads_gemma<<<(nh + 7) / 8, 256, 0, st>>>(arg_as<float*>(a[0]), arg_as<const float*>(a[1]),
                                                           arg_as<const float*>(a[2]), nh, arg_as<uint32_t>(a[4]),
                                                           arg_as<float>(a[5]));
    return cudaGetLastError();
}
// rmsnorm / rmsnorm_gemma (one-pass forms): one CTA computes the sum, all apply
template <bool GEMMA>
cudaError_t launch_rms1(const xp_arg* a, xp_grid, cudaStream_t st) {
    ops::rmsnorm_one<GEMMA><<<1, 1024, 0, st>>>(arg_as<float*>(a[0]), arg_as<const float*>(a[1]),
                                                arg_as<const float*>(a[2]), arg_as<uint32_t>(a[3]),
                                                arg_as<float>(a[4]));
    return cudaGetLastError();
}
// mv_km4_bs(out, in, wq, sc, rows, cols) on the fused B200 matvec
MvArgs mv_plain_args(float* out, const float* in, const void* wq, const void* sc, uint32_t rows, uint32_t cols) {
    MvArgs m{};
    m.m[0] = MvMat{(const uint4*)wq, (const uint2*)sc, out, cols, 0};
    m.nmat = 1;
    m.ntiles = cols / 64;
    m.K = rows;
    m.hidden = rows;
    m.pro = PRO_PLAIN;
    m.epi = EPI_STORE;
    m.x = in;
    const uint32_t nblk = rows / 32;
    uint32_t ks = 1;
    // narrow outputs: split K across a cluster so the whole GPU streams
    while (ks < 8 && m.ntiles * ks * 2 <= (uint32_t)sm_count() * 2 && nblk / (ks * 2) >= 4) ks *= 2;
    m.ksplit = ks;
    return m;
}
cudaError_t launch_mv_plain(const xp_arg* a, xp_grid, cudaStream_t st) {
    MvArgs m = mv_plain_args(arg_as<float*>(a[0]), arg_as<const float*>(a[1]), a[2].ptr, a[3].ptr,
                             arg_as<uint32_t>(a[4]), arg_as<uint32_t>(a[5]));
    return launch_mv(m, st, false, (uint32_t)sm_count() * 4);
}
cudaError_t launch_mv_split(const xp_arg* a, xp_grid, cudaStream_t st) {
    const uint32_t rows = arg_as<uint32_t>(a[4]), cols = arg_as<uint32_t>(a[5]), split = arg_as<uint32_t>(a[6]);
    MvArgs m = mv_plain_args(arg_as<float*>(a[0]), arg_as<const float*>(a[1]), a[2].ptr, a[3].ptr, rows, cols);
    m.ksplit = split;
    m.quad_split = 1;
    m.epi = EPI_PARTIAL;
    return launch_mv(m, st, false);
}
// argmax tree collapsed: the same out[2] contract as argmax / argmax_final
// rmsnorm_heads_rows_gemma: grid = n_tokens * n_heads * head_dim in the
// reference; here one warp per (token, head).
cudaError_t launch_heads_rows(const xp_arg* a, xp_grid, cudaStream_t st) {
    const uint32_t nth = arg_as<uint32_t>(a[3]) * arg_as<uint32_t>(a[4]);
    ops::rmsnorm_heads_rows_gemma<<<(nth + 7) / 8, 256, 0, st>>>(
        arg_as<float*>(a[0]), arg_as<const float*>(a[1]), arg_as<const float*>(a[2]), arg_as<uint32_t>(a[3]),
        arg_as<uint32_t>(a[4]), arg_as<uint32_t>(a[5]), arg_as<float>(a[6]));
    return cudaGetLastError();
}
// The layout-study matvecs: one warp per (column, split); the reference grid
// (a thread per column, per column pair or per (column, split)) is ignored.
template <int L, bool SPLIT>
cudaError_t launch_mv_layout(const xp_arg* a, xp_grid, cudaStream_t st) {
    const uint32_t cols = arg_as<uint32_t>(a[5]), split = SPLIT ? arg_as<uint32_t>(a[6]) : 1u;
    const uint64_t warps = (uint64_t)cols * split;
    ops::mv_layout<L><<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
        arg_as<float*>(a[0]), arg_as<const float*>(a[1]), arg_as<const uint32_t*>(a[2]), arg_as<const float*>(a[3]),
        arg_as<uint32_t>(a[4]), cols, split);
    return cudaGetLastError();
}
cudaError_t launch_stream_read(const xp_arg* a, xp_grid, cudaStream_t st) {
    ops::stream_read<<<65536 / 256, 256, 0, st>>>(arg_as<float*>(a[0]), arg_as<const uint32_t*>(a[1]),
                                                  arg_as<uint32_t>(a[2]));
    return cudaGetLastError();
}
cudaError_t launch_argmax(const xp_arg* a, xp_grid, cudaStream_t st) {
    ops::argmax<<<1, 1024, 0, st>>>(arg_as<float*>(a[0]), arg_as<const float*>(a[1]), arg_as<uint32_t>(a[2]));
    return cudaGetLastError();
}
cudaError_t launch_stream4(const xp_arg* a, xp_grid g, cudaStream_t st) {
    const uint32_t threads = arg_as<uint32_t>(a[3]);
    ops::stream4<<<(threads + 255) / 256, 256, 0, st>>>(arg_as<float*>(a[0]), arg_as<const uint4*>(a[1]),
                                                        arg_as<uint32_t>(a[2]), threads);
    (void)g;
    return cudaGetLastError();
}

// kernels/llm_quant.cl: element-wise dequant on the ggml element decoder,
// native-layout matvecs a warp per row, repacked matvecs a CTA per 64-row group
template <uint32_t TYPE>
cudaError_t launch_dequant(const xp_arg* a, xp_grid, cudaStream_t st) {
    return gguf_dequant(st, TYPE, a[1].ptr, arg_as<float*>(a[0]), arg_as<uint32_t>(a[2]));
}
template <void (*K)(float*, const float*, const uint32_t*, uint32_t, uint32_t)>
cudaError_t launch_mvq(const xp_arg* a, xp_grid, cudaStream_t st) {
    const uint32_t rows = arg_as<uint32_t>(a[3]);
    K<<<(rows + 7) / 8, 256, 0, st>>>(arg_as<float*>(a[0]), arg_as<const float*>(a[1]), arg_as<const uint32_t*>(a[2]),
                                      rows, arg_as<uint32_t>(a[4]));
    return cudaGetLastError();
}
template <int F, bool SPLIT>
cudaError_t launch_rqv(const xp_arg* a, xp_grid, cudaStream_t st) {
    quant::RqArgs r{};
    r.out = arg_as<float*>(a[0]);
    r.x = arg_as<const float4*>(a[1]);
    r.q = arg_as<const uint4*>(a[2]);
    uint32_t i = 3;
    if (F == quant::RQ50 || F == quant::RQ6K) r.hi = arg_as<const uint32_t*>(a[i++]);
    r.scale = arg_as<const float*>(a[i++]);
    if (F == quant::RQ4K) r.bias = arg_as<const float*>(a[i++]);
    r.rows = arg_as<uint32_t>(a[i++]);
    r.cols = arg_as<uint32_t>(a[i++]);
    r.split = SPLIT ? arg_as<uint32_t>(a[i]) : 1u;
    if (r.split == 0 || r.rows == 0) return cudaErrorInvalidValue;
    return quant::launch_rq(F, r, st);
}
__global__ void proto_rq4k(float*, const float4*, const uint4*, const float*, const float*, uint32_t, uint32_t) {}
__global__ void proto_rq4k_split(float*, const float4*, const uint4*, const float*, const float*, uint32_t, uint32_t,
                                 uint32_t) {}
__global__ void proto_rqhi(float*, const float4*, const uint4*, const uint32_t*, const float*, uint32_t, uint32_t) {}
__global__ void proto_rqhi_split(float*, const float4*, const uint4*, const uint32_t*, const float*, uint32_t,
                                 uint32_t, uint32_t) {}
__global__ void proto_rq80(float*, const float4*, const uint4*, const float*, uint32_t, uint32_t) {}
__global__ void proto_rq80_split(float*, const float4*, const uint4*, const float*, uint32_t, uint32_t, uint32_t) {}

#define LLM "kernels/llm.spv"
#define MV "kernels/llm_matvec.spv"
#define TF "kernels/llm_transformer.spv"
#define SM "kernels/llm_sampling.spv"
#define QT "kernels/llm_quant.spv"
#define E(mod, fn, geo, names) Entry{mod, #fn, names, Gen<&ops::fn, geo>::specs(), &Gen<&ops::fn, geo>::launch}
#define EC(mod, fn, proto, launcher, names) Entry{mod, fn, names, Gen<proto, GEO_CUSTOM>::specs(), launcher}

// prototypes for entries with custom launchers
__global__ void proto_mv(float*, const float*, const uint4*, const uint2*, uint32_t, uint32_t) {}
__global__ void proto_mv_split(float*, const float*, const uint4*, const uint2*, uint32_t, uint32_t, uint32_t) {}
__global__ void proto_heads(float*, const float*, const float*, uint32_t, uint32_t, float) {}
__global__ void proto_rms(float*, const float*, const float*, uint32_t, float) {}
__global__ void proto_mvl(float*, const float*, const uint32_t*, const float*, uint32_t, uint32_t) {}
__global__ void proto_mvl4(float*, const float*, const uint4*, const float*, uint32_t, uint32_t) {}
__global__ void proto_mvl_split(float*, const float*, const uint32_t*, const float*, uint32_t, uint32_t, uint32_t) {}
__global__ void proto_mvl4_split(float*, const float*, const uint4*, const float*, uint32_t, uint32_t, uint32_t) {}

const std::vector<Entry>& registry() {
    static const std::vector<Entry> t = {
        // kernels/llm.cl (the first, column-nibble matvec module)
        E(LLM, matvec_f32, GEO_THREADS, "out,in,w,rows,cols"),
        EC(LLM, "matvec_q4", &proto_mvl, (&launch_mv_layout<ops::MVL_COL, false>), "out,in,wq,scale,rows,cols"),
        EC(LLM, "stream_read", &ops::stream_read, &launch_stream_read, "out,src,n"),
        EC(LLM, "matvec_q4_split", &proto_mvl_split, (&launch_mv_layout<ops::MVL_COL, true>),
           "partial,in,wq,scale,rows,cols,split"),
        Entry{LLM, "matvec_reduce", "out,partial,cols,split", Gen<&ops::mv_reduce, GEO_THREADS>::specs(),
              &Gen<&ops::mv_reduce, GEO_THREADS>::launch},
        // kernels/llm_matvec.cl
        EC(MV, "mv_ref", &proto_mvl, (&launch_mv_layout<ops::MVL_COL, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_ref_split", &proto_mvl_split, (&launch_mv_layout<ops::MVL_COL, true>),
           "partial,in,wq,scale,rows,cols,split"),
        EC(MV, "mv_kmn", &proto_mvl, (&launch_mv_layout<ops::MVL_KMN, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km", &proto_mvl, (&launch_mv_layout<ops::MVL_KM, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km4", &proto_mvl4, (&launch_mv_layout<ops::MVL_KM4, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km4_wg128", &proto_mvl4, (&launch_mv_layout<ops::MVL_KM4, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km4_wg256", &proto_mvl4, (&launch_mv_layout<ops::MVL_KM4, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km4_wg32", &proto_mvl4, (&launch_mv_layout<ops::MVL_KM4, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km4_c2", &proto_mvl4, (&launch_mv_layout<ops::MVL_KM4, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km4_c2_wg32", &proto_mvl4, (&launch_mv_layout<ops::MVL_KM4, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km4_c4", &proto_mvl4, (&launch_mv_layout<ops::MVL_KM4, false>), "out,in,wq,scale,rows,cols"),
        EC(MV, "mv_km4_split", &proto_mvl4_split, (&launch_mv_layout<ops::MVL_KM4, true>),
           "partial,in,wq,scale,rows,cols,split"),
        EC(MV, "mv_km4_bs", &proto_mv, &launch_mv_plain, "out,in,wq,sc,rows,cols"),
        EC(MV, "mv_km4_bs_split", &proto_mv_split, &launch_mv_split, "partial,in,wq,sc,rows,cols,split"),
        E(MV, mv_reduce, GEO_THREADS, "out,partial,cols,split"),
        EC(MV, "stream4", &ops::stream4, &launch_stream4, "out,src,n,threads"),
        // kernels/llm_transformer.cl
        EC(TF, "rmsnorm", &proto_rms, &launch_rms1<false>, "out,in,w,n,eps"),
        EC(TF, "rmsnorm_gemma", &proto_rms, &launch_rms1<true>, "out,in,w,n,eps"),
        E(TF, rmsnorm_sumsq, GEO_THREADS, "partial,in,n,nparts"),
        E(TF, rmsnorm_apply_gemma, GEO_THREADS, "out,in,w,partial,n,nparts,eps"),
        EC(TF, "rmsnorm_heads_gemma", &proto_heads, &launch_heads, "out,in,w,n_heads,head_dim,eps"),
        E(TF, rope, GEO_THREADS, "x,n_heads,head_dim,pos,theta"),
        E(TF, rope_cached, GEO_THREADS, "x,cos_t,sin_t,n_heads,head_dim"),
        E(TF, geglu, GEO_THREADS, "out,gate,up,n"),
        E(TF, swiglu, GEO_THREADS, "out,gate,up,n"),
        E(TF, geglu_fused, GEO_THREADS, "out,gate_up,n"),
        E(TF, attention_scores, GEO_WARPS, "scores,q,kcache,n_heads,kv_heads,head_dim,span,scale,kv_start"),
        E(TF, attention_scores_mq4, GEO_WARPS, "scores,q,kcache,head_dim,span,scale,kv_start"),
        E(TF, softmax_rows, GEO_ROWS, "x,n_rows,n_cols"),
        E(TF, softmax_rows_partial, GEO_THREADS, "pmax,psum,x,n_rows,n_cols,nparts"),
        E(TF, softmax_rows_finish, GEO_THREADS, "stats,pmax,psum,n_rows,nparts"),
        E(TF, softmax_rows_scale, GEO_THREADS, "x,stats,n_rows,n_cols"),
        E(TF, attention_apply, GEO_THREADS, "out,probs,vcache,n_heads,kv_heads,head_dim,span,kv_start"),
        E(TF, attention_apply_mq4, GEO_THREADS, "partial,probs,vcache,head_dim,span,kv_start,split"),
        E(TF, attention_apply_reduce, GEO_THREADS, "out,partial,n,split"),
        E(TF, add_residual, GEO_THREADS, "x,y,n"),
        E(TF, add_vec, GEO_THREADS, "out,a,b,n"),
        E(TF, mul_scalar, GEO_THREADS, "x,s,n"),
        E(TF, kv_append, GEO_THREADS, "cache,src,n,pos"),
        E(TF, embed_lookup, GEO_THREADS, "out,table,token,n"),
        EC(TF, "argmax", &ops::argmax, &launch_argmax, "out,logits,n"),
        // kernels/llm_sampling.cl
        E(SM, argmax_partial, GEO_THREADS, "pval,pidx,logits,n,nparts"),
        E(SM, argmax_reduce, GEO_THREADS, "oval,oidx,pval,pidx,n,nparts"),
        E(SM, argmax_final, GEO_ONE, "out,pidx_out,pval,pidx,nparts"),
        E(SM, apply_temperature, GEO_THREADS, "logits,inv_temp,n"),
        E(SM, reduce_max_partial, GEO_THREADS, "pmax,x,n,nparts"),
        E(SM, reduce_max_final, GEO_ONE, "stats,pmax,nparts"),
        E(SM, softmax_exp_partial, GEO_THREADS, "out,psum,x,stats,n,nparts"),
        E(SM, reduce_sum_partial, GEO_THREADS, "out,in,n,nparts"),
        E(SM, reduce_sum_final, GEO_ONE, "stats,psum,nparts"),
        E(SM, softmax_normalize, GEO_THREADS, "out,stats,n"),
        E(SM, topk_partial, GEO_THREADS, "cval,cidx,x,n,nparts,k"),
        E(SM, topk4_partial, GEO_THREADS, "cval,cidx,x,n,nparts"),
        E(SM, topk_rank_select, GEO_THREADS, "oval,oidx,cval,cidx,ncand,k"),
        E(SM, topk_mask, GEO_THREADS, "logits,topk_val,k,n"),
        E(SM, topp_cutoff, GEO_THREADS, "w,k,p"),
        E(SM, multinomial_sample, GEO_THREADS, "out,idx_out,w,idx,k,u"),
        E(SM, multinomial_strided, GEO_THREADS, "out,idx_out,w,psum,stats,n,nparts,u"),
        // kernels/llm_sampling.cl, prefill shapes
        E(SM, softmax_rows_stats, GEO_WARPS, "stats,x,n_rows,n_cols"),
        E(SM, softmax_rows_apply, GEO_THREADS, "x,stats,n_rows,n_cols"),
        E(SM, attention_scores_prefill, GEO_WARPS,
          "scores,q,kcache,n_heads,kv_heads,head_dim,n_query,seq_len,q_offset,window,scale"),
        E(SM, attention_apply_prefill, GEO_THREADS, "out,probs,vcache,n_heads,kv_heads,head_dim,n_query,seq_len"),
        E(SM, rmsnorm_rows_sumsq, GEO_WARPS, "rowss,in,n_rows,n"),
        E(SM, rmsnorm_rows_apply_gemma, GEO_THREADS, "out,in,w,rowss,n_rows,n,eps"),
        EC(SM, "rmsnorm_heads_rows_gemma", &ops::rmsnorm_heads_rows_gemma, &launch_heads_rows,
           "out,in,w,n_tokens,n_heads,head_dim,eps"),
        E(SM, rope_prefill, GEO_THREADS, "x,n_tokens,n_heads,head_dim,pos0,theta"),
        E(SM, kv_append_rows, GEO_THREADS, "cache,src,n_tokens,row,pos0"),
        E(SM, embed_lookup_rows, GEO_THREADS, "out,table,tokens,n_tokens,n"),
        // kernels/llm_quant.cl
        Entry{QT, "fp16_decode", "out,src,n", Gen<&quant::fp16_decode, GEO_THREADS>::specs(),
              &Gen<&quant::fp16_decode, GEO_THREADS>::launch},
        EC(QT, "dequant_q8_0", &quant::fp16_decode, &launch_dequant<8>, "out,src,n"),
        EC(QT, "dequant_q5_0", &quant::fp16_decode, &launch_dequant<6>, "out,src,n"),
        EC(QT, "dequant_q4_k", &quant::fp16_decode, &launch_dequant<12>, "out,src,n"),
        EC(QT, "dequant_q6_k", &quant::fp16_decode, &launch_dequant<14>, "out,src,n"),
        EC(QT, "matvec_q8_0", &quant::matvec_q32<true>, &launch_mvq<&quant::matvec_q32<true>>, "out,in,w,rows,cols"),
        EC(QT, "matvec_q5_0", &quant::matvec_q32<false>, &launch_mvq<&quant::matvec_q32<false>>, "out,in,w,rows,cols"),
        EC(QT, "matvec_q4_k", &quant::matvec_q4_k, &launch_mvq<&quant::matvec_q4_k>, "out,in,w,rows,cols"),
        EC(QT, "matvec_q6_k", &quant::matvec_q6_k, &launch_mvq<&quant::matvec_q6_k>, "out,in,w,rows,cols"),
        EC(QT, "matvec_rq4_k", &proto_rq4k, (&launch_rqv<quant::RQ4K, false>), "out,in,q,scale,bias,rows,cols"),
        EC(QT, "matvec_rq5_0", &proto_rqhi, (&launch_rqv<quant::RQ50, false>), "out,in,q,hi,scale,rows,cols"),
        EC(QT, "matvec_rq6_k", &proto_rqhi, (&launch_rqv<quant::RQ6K, false>), "out,in,q,hi,scale,rows,cols"),
        EC(QT, "matvec_rq8_0", &proto_rq80, (&launch_rqv<quant::RQ80, false>), "out,in,q,scale,rows,cols"),
        EC(QT, "matvec_rq4_k_split", &proto_rq4k_split, (&launch_rqv<quant::RQ4K, true>),
           "partial,in,q,scale,bias,rows,cols,split"),
        EC(QT, "matvec_rq5_0_split", &proto_rqhi_split, (&launch_rqv<quant::RQ50, true>),
           "partial,in,q,hi,scale,rows,cols,split"),
        EC(QT, "matvec_rq6_k_split", &proto_rqhi_split, (&launch_rqv<quant::RQ6K, true>),
           "partial,in,q,hi,scale,rows,cols,split"),
        EC(QT, "matvec_rq8_0_split", &proto_rq80_split, (&launch_rqv<quant::RQ80, true>),
           "partial,in,q,scale,rows,cols,split"),
        Entry{QT, "mv_reduce", "out,partial,rows,split", Gen<&quant::rq_reduce, GEO_THREADS>::specs(),
              &Gen<&quant::rq_reduce, GEO_THREADS>::launch},
    };
    return t;
}
#undef E
#undef EC

std::string base_name(const std::string& s) {
    const size_t p = s.find_last_of('/');
    return p == std::string::npos ? s : s.substr(p + 1);
}
bool module_match(const char* want, const char* have) {
    if (!want || !*want) return true;
    return base_name(want) == base_name(have);
}
std::string arg_label(const Entry& e, uint32_t i) {
    std::string names(e.arg_names);
    uint32_t k = 0;
    size_t s = 0;
    while (k < i) {
        const size_t c = names.find(',', s);
        if (c == std::string::npos) { s = std::string::npos; break; }
        s = c + 1;
        ++k;
    }
    std::string label = "argument " + std::to_string(i);
    if (s != std::string::npos) {
        const size_t c = names.find(',', s);
        label += " ('" + names.substr(s, c == std::string::npos ? std::string::npos : c - s) + "')";
    }
    return label;
}

// Validation with the reference's error categories and wording
// (src/launch.cpp:21-131).
xp_status validate(const Entry& e, xp_grid g, const xp_arg* args, uint32_t n) {
    if (n != e.args.size())
        return fail(XP_ERR_ARITY, "xp::launch: kernel '%s' expects %zu argument(s) (%s), got %u", e.name,
                    e.args.size(), e.arg_names, n);
    if (n && !args) return fail(XP_ERR_INVALID, "xp::launch('%s'): null argument array", e.name);
    for (uint32_t i = 0; i < n; ++i) {
        const ArgSpec& s = e.args[i];
        if (s.kind == 1) {
            if (args[i].kind != 1)
                return fail(XP_ERR_ARG_KIND, "xp::launch('%s'): %s is a global-memory pointer — pass a buffer, not a POD value",
                            e.name, arg_label(e, i).c_str());
            if (!args[i].ptr)
                return fail(XP_ERR_INVALID, "xp::launch('%s'): %s is an empty (null) buffer", e.name,
                            arg_label(e, i).c_str());
        } else {
            if (args[i].kind != 0)
                return fail(XP_ERR_ARG_KIND, "xp::launch('%s'): %s is a POD value in the kernel — a buffer was passed",
                            e.name, arg_label(e, i).c_str());
            if (args[i].size != s.size)
                return fail(XP_ERR_ARG_SIZE,
                            "xp::launch('%s'): %s is %u byte(s) in the kernel but a %u-byte value was passed (double literal for a float arg? size_t for a uint?)",
                            e.name, arg_label(e, i).c_str(), s.size, args[i].size);
            if (!args[i].ptr) return fail(XP_ERR_INVALID, "xp::launch('%s'): %s has a null value pointer", e.name,
                                          arg_label(e, i).c_str());
        }
    }
    const char axes[3] = {'x', 'y', 'z'};
    const uint32_t v[3] = {g.x, g.y, g.z};
    for (int i = 0; i < 3; ++i)
        if (v[i] == 0)
            return fail(XP_ERR_GRID, "xp::launch('%s'): grid.%c must be nonzero (grid is the global thread count)",
                        e.name, axes[i]);
    return XP_OK;
}

xp_status cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return XP_OK;
    return fail(e == cudaErrorMemoryAllocation ? XP_ERR_OOM : XP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

// ============================================================================
// Context / buffers
// ============================================================================
struct xp_context {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::unordered_map<void*, std::pair<int, void*>> allocs;  // dptr -> (usage, host ptr)
};

extern "C" {

const char* xp_last_error(void) { return xp::g_err.c_str(); }
const char* xp_status_name(int s) {
    switch (s) {
        case XP_OK: return "XP_OK";
        case XP_TIMEOUT: return "XP_TIMEOUT";
        case XP_ERR_INVALID: return "XP_ERR_INVALID";
        case XP_ERR_NO_KERNEL: return "XP_ERR_NO_KERNEL";
        case XP_ERR_ARITY: return "XP_ERR_ARITY";
        case XP_ERR_ARG_KIND: return "XP_ERR_ARG_KIND";
        case XP_ERR_ARG_SIZE: return "XP_ERR_ARG_SIZE";
        case XP_ERR_GRID: return "XP_ERR_GRID";
        case XP_ERR_CUDA: return "XP_ERR_CUDA";
        case XP_ERR_OOM: return "XP_ERR_OOM";
        case XP_ERR_KV_FULL: return "XP_ERR_KV_FULL";
        case XP_ERR_STATE: return "XP_ERR_STATE";
        case XP_ERR_DEVICE: return "XP_ERR_DEVICE";
        case XP_ERR_NO_DEVICE: return "XP_ERR_NO_DEVICE";
        case XP_ERR_UNSUPPORTED: return "XP_ERR_UNSUPPORTED";
        default: return "XP_UNKNOWN";
    }
}
const char* xp_version(void) { return "xpose_b200 0.1 (sm_100a)"; }
int xp_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

xp_status xp_context_create(int device, xp_context** out) {
    if (!out) return fail(XP_ERR_INVALID, "xp_context_create: null out");
    if (xp_device_count() <= device || device < 0)
        return fail(XP_ERR_NO_DEVICE, "xp_context_create: no CUDA device %d", device);
    XP_CUDA_TRY(cudaSetDevice(device));
    auto* c = new xp_context;
    c->device = device;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) { delete c; return cuda_status(e, "cudaStreamCreate"); }
    *out = c;
    return XP_OK;
}
xp_status xp_context_destroy(xp_context* c) {
    if (!c) return XP_OK;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (auto& kv : c->allocs) {
        if (kv.second.first == XP_HOST_VISIBLE) cudaFreeHost(kv.second.second);
        else cudaFree(kv.first);
    }
    cudaStreamDestroy(c->stream);
    delete c;
    return XP_OK;
}
void* xp_context_stream(xp_context* c) { return c ? c->stream : nullptr; }
xp_status xp_context_device_name(xp_context* c, char* buf, size_t n) {
    if (!c || !buf || !n) return fail(XP_ERR_INVALID, "xp_context_device_name: bad args");
    cudaDeviceProp p;
    XP_CUDA_TRY(cudaGetDeviceProperties(&p, c->device));
    std::snprintf(buf, n, "%s", p.name);
    return XP_OK;
}
xp_status xp_context_wait_idle(xp_context* c) {
    if (!c) return fail(XP_ERR_INVALID, "null context");
    XP_CUDA_TRY(cudaStreamSynchronize(c->stream));
    return XP_OK;
}
xp_status xp_alloc(xp_context* c, size_t bytes, xp_usage usage, void** dptr, void** host_ptr) {
    if (!c || !dptr) return fail(XP_ERR_INVALID, "xp_alloc: null argument");
    if (bytes == 0) return fail(XP_ERR_INVALID, "xp_alloc: zero-size buffer");
    cudaSetDevice(c->device);
    if (usage == XP_HOST_VISIBLE) {
        void* h = nullptr;
        XP_CUDA_TRY(cudaHostAlloc(&h, bytes, cudaHostAllocMapped));
        std::memset(h, 0, bytes);
        void* d = nullptr;
        XP_CUDA_TRY(cudaHostGetDevicePointer(&d, h, 0));
        c->allocs[d] = {XP_HOST_VISIBLE, h};
        *dptr = d;
        if (host_ptr) *host_ptr = h;
    } else {
        void* d = nullptr;
        XP_CUDA_TRY(cudaMalloc(&d, bytes));
        // zero-filled on the context's own stream: it is non-blocking, so a
        // fill on the legacy default stream would not be ordered before the
        // uploads and launches that follow and could land after them
        XP_CUDA_TRY(cudaMemsetAsync(d, 0, bytes, c->stream));
        XP_CUDA_TRY(cudaStreamSynchronize(c->stream));
        c->allocs[d] = {XP_DEVICE_LOCAL, nullptr};
        *dptr = d;
        if (host_ptr) *host_ptr = nullptr;
    }
    return XP_OK;
}
xp_status xp_free(xp_context* c, void* d) {
    if (!c) return fail(XP_ERR_INVALID, "xp_free: null context");
    auto it = c->allocs.find(d);
    if (it == c->allocs.end()) return fail(XP_ERR_INVALID, "xp_free: pointer not allocated by this context");
    cudaStreamSynchronize(c->stream);
    if (it->second.first == XP_HOST_VISIBLE) cudaFreeHost(it->second.second);
    else cudaFree(d);
    c->allocs.erase(it);
    return XP_OK;
}
xp_status xp_upload(xp_context* c, void* dst, size_t off, const void* src, size_t bytes) {
    if (!c || !dst || (!src && bytes)) return fail(XP_ERR_INVALID, "xp_upload: null argument");
    XP_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(dst) + off, src, bytes, cudaMemcpyHostToDevice, c->stream));
    XP_CUDA_TRY(cudaStreamSynchronize(c->stream));
    return XP_OK;
}
xp_status xp_download(xp_context* c, void* dst, const void* src, size_t off, size_t bytes) {
    if (!c || !dst || (!src && bytes)) return fail(XP_ERR_INVALID, "xp_download: null argument");
    XP_CUDA_TRY(cudaMemcpyAsync(dst, static_cast<const char*>(src) + off, bytes, cudaMemcpyDeviceToHost, c->stream));
    XP_CUDA_TRY(cudaStreamSynchronize(c->stream));
    return XP_OK;
}

// ---- registry -----------------------------------------------------------------------
int xp_kernel_count(void) { return (int)registry().size(); }
xp_status xp_kernel_lookup(const char* module, const char* name, xp_kernel* out) {
    if (!name || !out) return fail(XP_ERR_INVALID, "xp_kernel_lookup: null argument");
    const auto& t = registry();
    for (size_t i = 0; i < t.size(); ++i)
        if (std::strcmp(t[i].name, name) == 0 && module_match(module, t[i].module)) {
            *out = (xp_kernel)i;
            return XP_OK;
        }
    std::string avail;
    for (const auto& e : t)
        if (module_match(module, e.module)) avail += (avail.empty() ? "" : ", ") + std::string(e.name);
    return fail(XP_ERR_NO_KERNEL, "xp::Program('%s'): no kernel named '%s' (module has: %s)", module ? module : "*",
                name, avail.c_str());
}
xp_status xp_kernel_info(xp_kernel k, const char** module, const char** name, uint32_t* nargs) {
    const auto& t = registry();
    if (k < 0 || (size_t)k >= t.size()) return fail(XP_ERR_INVALID, "xp_kernel_info: empty Kernel handle");
    if (module) *module = t[k].module;
    if (name) *name = t[k].name;
    if (nargs) *nargs = (uint32_t)t[k].args.size();
    return XP_OK;
}
xp_status xp_kernel_arg(xp_kernel k, uint32_t i, int* kind, uint32_t* size, const char** arg_name) {
    const auto& t = registry();
    if (k < 0 || (size_t)k >= t.size() || i >= t[k].args.size())
        return fail(XP_ERR_INVALID, "xp_kernel_arg: bad kernel or index");
    if (kind) *kind = t[k].args[i].kind;
    if (size) *size = t[k].args[i].size;
    if (arg_name) {
        static thread_local std::string nm;
        nm = arg_label(t[k], i);
        *arg_name = nm.c_str();
    }
    return XP_OK;
}
xp_status xp_launch(xp_kernel k, xp_grid g, const xp_arg* args, uint32_t n, void* stream) {
    const auto& t = registry();
    if (k < 0 || (size_t)k >= t.size()) return fail(XP_ERR_INVALID, "xp::launch: empty Kernel handle");
    const Entry& e = t[k];
    xp_status s = validate(e, g, args, n);
    if (s != XP_OK) return s;
    return cuda_status(e.launch(args, g, (cudaStream_t)stream), e.name);
}

}  // extern "C"

// ============================================================================
// Batch / Fence
// ============================================================================
struct xp_fence {
    cudaEvent_t ev = nullptr;
    int device = 0;
};
struct BatchItem {
    xp_kernel k;
    xp_grid g;
    std::vector<xp_arg> args;
    std::vector<std::vector<unsigned char>> pods;
};
struct xp_batch {
    xp_context* ctx = nullptr;
    std::vector<BatchItem> items;
    bool spent = false;
};

namespace {
// One cached executable graph per context; Batch::submit updates it in place
// when the recorded node list has the same shape (same kernels, new params),
// which is how a per-token Batch with a changing `pos` re-submits cheaply.
struct GraphCache {
    cudaGraphExec_t exec = nullptr;
};
std::unordered_map<xp_context*, GraphCache>& graph_cache() {
    static std::unordered_map<xp_context*, GraphCache> m;
    return m;
}
}  // namespace

extern "C" {

xp_status xp_batch_create(xp_context* c, xp_batch** out) {
    if (!c || !out) return fail(XP_ERR_INVALID, "xp_batch_create: null argument");
    *out = new xp_batch;
    (*out)->ctx = c;
    return XP_OK;
}
xp_status xp_batch_add(xp_batch* b, xp_kernel k, xp_grid g, const xp_arg* args, uint32_t n) {
    if (!b) return fail(XP_ERR_INVALID, "xp_batch_add: null batch");
    if (b->spent) return fail(XP_ERR_STATE, "xp::Batch: add() after submit()");
    const auto& t = registry();
    if (k < 0 || (size_t)k >= t.size()) return fail(XP_ERR_INVALID, "xp::launch: empty Kernel handle");
    xp_status s = validate(t[k], g, args, n);
    if (s != XP_OK) return s;
    BatchItem it;
    it.k = k;
    it.g = g;
    it.args.assign(args, args + n);
    it.pods.resize(n);
    for (uint32_t i = 0; i < n; ++i)
        if (args[i].kind == 0) {
            it.pods[i].assign((const unsigned char*)args[i].ptr, (const unsigned char*)args[i].ptr + args[i].size);
        }
    b->items.push_back(std::move(it));
    for (uint32_t i = 0; i < n; ++i)
        if (b->items.back().args[i].kind == 0) b->items.back().args[i].ptr = b->items.back().pods[i].data();
    return XP_OK;
}
xp_status xp_batch_size(xp_batch* b, uint32_t* n) {
    if (!b || !n) return fail(XP_ERR_INVALID, "xp_batch_size: null argument");
    *n = (uint32_t)b->items.size();
    return XP_OK;
}
xp_status xp_batch_submit(xp_batch* b, xp_fence** out) {
    if (!b || !out) return fail(XP_ERR_INVALID, "xp_batch_submit: null argument");
    if (b->spent) return fail(XP_ERR_STATE, "xp::Batch: submit() twice");
    b->spent = true;
    xp_context* c = b->ctx;
    cudaSetDevice(c->device);
    auto* f = new xp_fence;
    f->device = c->device;
    if (cudaEventCreateWithFlags(&f->ev, cudaEventDisableTiming) != cudaSuccess) {
        delete f;
        return fail(XP_ERR_CUDA, "cudaEventCreate failed");
    }
    if (!b->items.empty()) {
        const auto& t = registry();
        cudaGraph_t graph = nullptr;
        XP_CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        cudaError_t le = cudaSuccess;
        for (const auto& it : b->items) {
            le = t[it.k].launch(it.args.data(), it.g, c->stream);
            if (le != cudaSuccess) break;
        }
        cudaError_t ce = cudaStreamEndCapture(c->stream, &graph);
        if (le != cudaSuccess || ce != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            delete f;
            return cuda_status(le != cudaSuccess ? le : ce, "xp::Batch::submit capture");
        }
        GraphCache& gc = graph_cache()[c];
        bool updated = false;
        if (gc.exec) {
            cudaGraphExecUpdateResultInfo info;
            if (cudaGraphExecUpdate(gc.exec, graph, &info) == cudaSuccess) updated = true;
            else {
                cudaGetLastError();
                cudaGraphExecDestroy(gc.exec);
                gc.exec = nullptr;
            }
        }
        if (!updated) {
            cudaError_t ie = cudaGraphInstantiate(&gc.exec, graph, 0);
            if (ie != cudaSuccess) {
                cudaGraphDestroy(graph);
                delete f;
                return cuda_status(ie, "cudaGraphInstantiate");
            }
        }
        cudaGraphDestroy(graph);
        XP_CUDA_TRY(cudaGraphLaunch(gc.exec, c->stream));
    }
    XP_CUDA_TRY(cudaEventRecord(f->ev, c->stream));
    *out = f;
    return XP_OK;
}
xp_status xp_context_fence(xp_context* c, xp_fence** out) {
    if (!c || !out) return fail(XP_ERR_INVALID, "xp_context_fence: null argument");
    cudaSetDevice(c->device);
    auto* f = new xp_fence;
    f->device = c->device;
    if (cudaEventCreateWithFlags(&f->ev, cudaEventDisableTiming) != cudaSuccess) {
        delete f;
        return fail(XP_ERR_CUDA, "cudaEventCreate failed");
    }
    XP_CUDA_TRY(cudaEventRecord(f->ev, c->stream));
    *out = f;
    return XP_OK;
}
xp_status xp_batch_destroy(xp_batch* b) {
    delete b;
    return XP_OK;
}
xp_status xp_fence_wait(xp_fence* f, uint64_t timeout_ns) {
    if (!f) return XP_OK;  // empty fence: wait() is a no-op returning true
    cudaSetDevice(f->device);
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaEventQuery(f->ev);
        if (e == cudaSuccess) return XP_OK;
        if (e != cudaErrorNotReady) return fail(XP_ERR_DEVICE, "xp::Fence::wait: %s", cudaGetErrorString(e));
        const uint64_t el = (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                std::chrono::steady_clock::now() - t0).count();
        if (el >= timeout_ns) return XP_TIMEOUT;
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}
xp_status xp_fence_destroy(xp_fence* f) {
    if (!f) return XP_OK;
    cudaSetDevice(f->device);
    cudaEventSynchronize(f->ev);  // the destructor drains (include/vulkore/sync.hpp)
    cudaEventDestroy(f->ev);
    delete f;
    return XP_OK;
}

// ============================================================================
// Typed entry points
// ============================================================================
#define CHECK_PTR(p) \
    if (!(p)) return fail(XP_ERR_INVALID, "%s: argument '%s' is null", __func__, #p)

xp_status xp_mv_km4_bs(void* stream, float* out, const float* in, const uint32_t* wq, const uint32_t* sc,
                       uint32_t rows, uint32_t cols) {
    CHECK_PTR(out); CHECK_PTR(in); CHECK_PTR(wq); CHECK_PTR(sc);
    if (rows == 0 || rows % 128 || cols == 0 || cols % 64)
        return fail(XP_ERR_INVALID, "xp_mv_km4_bs: rows must be a multiple of 128 and cols of 64 (got %u x %u)",
                    rows, cols);
    MvArgs m = mv_plain_args(out, in, wq, sc, rows, cols);
    return cuda_status(launch_mv(m, (cudaStream_t)stream, false, (uint32_t)sm_count() * 4), "mv_km4_bs");
}
xp_status xp_mv_km4_bs_split(void* stream, float* partial, const float* in, const uint32_t* wq, const uint32_t* sc,
                             uint32_t rows, uint32_t cols, uint32_t split) {
    CHECK_PTR(partial); CHECK_PTR(in); CHECK_PTR(wq); CHECK_PTR(sc);
    if (rows == 0 || rows % 128 || cols == 0 || cols % 64 || split == 0)
        return fail(XP_ERR_INVALID, "xp_mv_km4_bs_split: bad shape %u x %u split %u", rows, cols, split);
    MvArgs m = mv_plain_args(partial, in, wq, sc, rows, cols);
    m.ksplit = split;
    m.quad_split = 1;
    m.epi = EPI_PARTIAL;
    return cuda_status(launch_mv(m, (cudaStream_t)stream, false), "mv_km4_bs_split");
}
xp_status xp_mv_reduce(void* stream, float* out, const float* partial, uint32_t cols, uint32_t split) {
    CHECK_PTR(out); CHECK_PTR(partial);
    ops::mv_reduce<<<(cols + 255) / 256, 256, 0, (cudaStream_t)stream>>>(out, partial, cols, split);
    return cuda_status(cudaGetLastError(), "mv_reduce");
}
// ---- batched matvec on tcgen05 -------------------------------------------------
namespace {
struct BmmPlan {
    uint32_t npad, nblk, tiles, ksplit, cb, nitems;
    size_t off_xs, off_err, off_xb, off_acc, bytes, smem;
};
BmmPlan bmm_plan(uint32_t rows, uint32_t cols, uint32_t n) {
    BmmPlan p{};
    p.npad = bmm_npad(n);
    p.nblk = rows / 32;
    p.tiles = cols / BMM_M;
    const uint32_t G = (uint32_t)sm_count();
    p.ksplit = std::max<uint32_t>(1, std::min<uint32_t>(p.nblk, (G + p.tiles - 1) / p.tiles));
    p.cb = ((p.nblk + p.ksplit - 1) / p.ksplit + 3) & ~3u;  // whole quads
    p.ksplit = (p.nblk + p.cb - 1) / p.cb;
    p.nitems = p.tiles * p.ksplit;
    p.off_xs = 0;      // [64] per-sequence scales
    p.off_err = 256;   // error word of the call
    p.off_xb = 512;
    p.off_acc = p.off_xb + (size_t)p.nblk * 2 * 4 * p.npad * 16;
    p.bytes = p.off_acc + (p.ksplit > 1 ? (size_t)p.npad * cols * 8 : 0);
    p.smem = (size_t)BMM_STAGES * (BMM_SB * (2048 + 2 * 4 * p.npad * 16) + BMM_ABYTES) + 8 * (3 * BMM_STAGES + 2 * BMM_ND) + 16;
    return p;
}
}  // namespace
#ifdef XP_ATT_TRACE
void xp_att_trace_read(unsigned long long* out) {
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(out, g_att_trace, sizeof(g_att_trace));
}
#endif
#ifdef BMM_TRACE
void xp_bmm_trace_read(unsigned long long* out) {
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(out, g_bmm_trace, sizeof(g_bmm_trace));
}
#endif
// K ranges of a launch over `cols` total columns (the raw partial count)
static uint32_t bmm_ksplit(uint32_t rows, uint32_t cols, uint32_t n) { return bmm_plan(rows, cols, n).ksplit; }
size_t xp_mv_km4_bs_batch_scratch_bytes(uint32_t rows, uint32_t cols, uint32_t n) {
    if (rows == 0 || rows % 128 || cols == 0 || cols % 128 || n == 0 || n > BMM_MAXN) return 0;
    return bmm_plan(rows, cols, n).bytes;
}
// One batched matvec launch over up to BMM_MAXPARTS matrices that share the
// input (same rows): activation prep once, then the tensor-core kernel over
// every matrix's column tiles. raw: each matrix's result stays as ksplit fp32
// partial sums in its part buffer ([ksplit][n][cols], bmm_ksplit), which the
// consumer adds in K-range order. Otherwise (one matrix) out gets fp32,
// K-split sums going through the scratch and a finish launch that leaves them
// zero.
struct BmmMat {
    const uint32_t* wq;
    const uint32_t* sc;
    uint32_t cols;
    float* out;
    float* part;
};
// prep: the activation operand already written by its producer (xs, xb of
// bmm_put_seq); then `in` is unused and no prep launch runs.
struct BmmPrep {
    const float* xs;
    const unsigned char* xb;
};
// Operand mode (bmm.cuh): BMM_MODE_SCALED when the caller knows every scale of
// the matrices lies in the fp16-exact range (bmm_scales_exact16), else
// BMM_MODE_INTEGER; BMM_MODE_CHECK scans the scale planes on the stream first
// and lets the kernel pick. XP_BMM_SCALED=0 forces the integer mode.
enum { BMM_MODE_INTEGER = 0, BMM_MODE_SCALED = 1, BMM_MODE_CHECK = 2 };
constexpr size_t BMM_OFF_FLAG = 384;  // scratch word: scale-range violation flag of a checking call
static void bmm_launch_scale_check(cudaStream_t st, const uint32_t* sc, uint32_t rows, uint32_t cols, uint32_t* flag) {
    const size_t nwords = (size_t)(rows / 32) * cols / 8;
    const uint32_t grid = (uint32_t)std::min<size_t>((nwords + 255) / 256, 4 * (size_t)sm_count());
    bmm_scale_check_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const uint4*>(sc), nwords, flag);
}
static bool bmm_scaled_allowed() {
    static const bool on = [] {
        const char* v = std::getenv("XP_BMM_SCALED");
        return !(v && *v && std::atoi(v) == 0);
    }();
    return on;
}
static xp_status bmm_run(cudaStream_t st, const BmmMat* mats, uint32_t nmat, bool raw, const float* in, uint32_t rows,
                         uint32_t n, void* scratch, const BmmPrep* prep = nullptr, bool pdl = false,
                         int mode = BMM_MODE_CHECK) {
    if (nmat == 0 || nmat > (uint32_t)BMM_MAXPARTS || (!raw && nmat != 1))
        return fail(XP_ERR_INVALID, "bmm_run: %u matrices", nmat);
    uint32_t cols = 0;
    for (uint32_t m = 0; m < nmat; ++m) cols += mats[m].cols;
    const BmmPlan p = bmm_plan(rows, cols, n);
    unsigned char* base = static_cast<unsigned char*>(scratch);
    float* xs = reinterpret_cast<float*>(base + p.off_xs);
    unsigned char* xb = base + p.off_xb;
    long long* acc = (!raw && p.ksplit > 1) ? reinterpret_cast<long long*>(base + p.off_acc) : nullptr;
    uint32_t* err = reinterpret_cast<uint32_t*>(base + p.off_err);
    if (acc) {
        // The fixed-point sums are zero between calls of one shape (the
        // finish launch clears them). A scratch last used by another shape
        // may hold that call's activations there.
        static std::mutex mu;
        static std::unordered_map<const void*, uint64_t> last_shape;
        const uint64_t sig = ((uint64_t)rows << 40) ^ ((uint64_t)cols << 8) ^ p.npad;
        bool clear = false;
        {
            std::lock_guard<std::mutex> g(mu);
            auto it = last_shape.find(scratch);
            clear = it != last_shape.end() && it->second != sig;
            last_shape[scratch] = sig;
        }
        if (clear) XP_CUDA_TRY(cudaMemsetAsync(base + p.off_acc, 0, p.bytes - p.off_acc, st));
    }
    if (!prep) {
        bmm_xprep_kernel<<<p.npad, BMM_XP_THREADS, 0, st>>>(in, rows, n, p.npad, xs, xb, err);
        XP_CUDA_TRY(cudaGetLastError());
    }
    if (!bmm_scaled_allowed()) mode = BMM_MODE_INTEGER;
    uint32_t* fbflag = nullptr;
    if (mode == BMM_MODE_CHECK) {
        // the kernel reads the flag at its start: a programmatic launch could
        // read it before the check wrote it
        pdl = false;
        fbflag = reinterpret_cast<uint32_t*>(base + BMM_OFF_FLAG);
        XP_CUDA_TRY(cudaMemsetAsync(fbflag, 0, 4, st));
        for (uint32_t m = 0; m < nmat; ++m) bmm_launch_scale_check(st, mats[m].sc, rows, mats[m].cols, fbflag);
        XP_CUDA_TRY(cudaGetLastError());
    }
    static size_t attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && attr_set[dev] < p.smem) {
        XP_CUDA_TRY(cudaFuncSetAttribute(bmm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
        attr_set[dev] = p.smem;
    }
    BmmArgs a{};
    uint32_t tile0 = 0;
    for (uint32_t m = 0; m < nmat; ++m) {
        BmmPart& P = a.part[m];
        P.wq = reinterpret_cast<const uint4*>(mats[m].wq);
        P.sc = reinterpret_cast<const uint2*>(mats[m].sc);
        P.out = mats[m].out;
        P.acc = acc;
        P.part = mats[m].part;
        P.cols = mats[m].cols;
        P.tile0 = tile0;
        tile0 += mats[m].cols / BMM_M;
    }
    a.nparts = nmat;
    a.xb = prep ? prep->xb : xb;
    a.xs = prep ? prep->xs : xs;
    a.raw = raw ? 1u : 0u;
    a.nblk = p.nblk;
    a.N = p.npad;
    a.nreal = n;
    a.ksplit = p.ksplit;
    a.cb = p.cb;
    a.nitems = p.nitems;
    a.err = err;
    a.scaled = mode == BMM_MODE_SCALED ? 1u : 0u;
    a.fbflag = fbflag;
    const uint32_t grid = std::min<uint32_t>(p.nitems, 2 * (uint32_t)sm_count());
    XP_CUDA_TRY(launch_ex(bmm_kernel, dim3(grid), dim3(BMM_THREADS), p.smem, st, 1, pdl, a));
    if (acc) {
        // rows n >= the real sequence count are padding: convert only [n][cols]
        bmm_finish_kernel<<<(uint32_t)(((size_t)n * cols + 255) / 256), 256, 0, st>>>(acc, mats[0].out, (size_t)n * cols);
        XP_CUDA_TRY(cudaGetLastError());
    }
    return XP_OK;
}
// Set-up time: true when every scale of the plane is in the fp16-exact range
// (the scaled operand mode applies); synchronous on the stream.
static cudaError_t bmm_scales_exact16(cudaStream_t st, const void* sc, uint32_t rows, uint32_t cols, uint32_t* dflag,
                                      bool* ok) {
    cudaError_t e = cudaMemsetAsync(dflag, 0, 4, st);
    if (e != cudaSuccess) return e;
    bmm_launch_scale_check(st, static_cast<const uint32_t*>(sc), rows, cols, dflag);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    uint32_t h = 1;
    if ((e = cudaMemcpyAsync(&h, dflag, 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return e;
    *ok = h == 0;
    return cudaSuccess;
}
xp_status xp_mv_km4_bs_batch(void* stream, float* out, const float* in, const uint32_t* wq, const uint32_t* sc,
                             uint32_t rows, uint32_t cols, uint32_t n, void* scratch) {
    CHECK_PTR(out); CHECK_PTR(in); CHECK_PTR(wq); CHECK_PTR(sc); CHECK_PTR(scratch);
    if (rows == 0 || rows % 128 || cols == 0 || cols % 128)
        return fail(XP_ERR_INVALID, "xp_mv_km4_bs_batch: rows must be a multiple of 128 and cols of 128 (got %u x %u)",
                    rows, cols);
    if (n == 0 || n > BMM_MAXN) return fail(XP_ERR_INVALID, "xp_mv_km4_bs_batch: 1..%d sequences (got %u)", BMM_MAXN, n);
    if (reinterpret_cast<uintptr_t>(scratch) % 256)
        return fail(XP_ERR_INVALID, "xp_mv_km4_bs_batch: scratch must be 256-byte aligned");
    const BmmMat m{wq, sc, cols, out, nullptr};
    return bmm_run((cudaStream_t)stream, &m, 1, false, in, rows, n, scratch);
}

struct xp_mv_plan {
    int device = 0;
    MvsJob* jobs = nullptr;
    MvsSrc* src = nullptr;
    XBlk* xq = nullptr;
    uint32_t* next = nullptr;
    float* part = nullptr;
    uint32_t* arrive = nullptr;
    uint32_t njobs = 0, nstrips = 0, nsrc = 0, nxq = 0, grid = 0;
    bool smem_x = false;
    uint64_t bytes = 0;
};
xp_status xp_mv_plan_create(const xp_mv_job* jobs, uint32_t n, xp_mv_plan** plan) {
    CHECK_PTR(jobs); CHECK_PTR(plan);
    *plan = nullptr;
    if (n == 0 || n > MVS_MAXJOBS) return fail(XP_ERR_INVALID, "xp_mv_plan_create: %u jobs (1..%u)", n, MVS_MAXJOBS);
    std::vector<MvsJob> hj(n);
    std::vector<MvsSrc> hs;
    std::vector<uint32_t> src_of(n);
    uint32_t strips = 0, nxq = 0;
    uint64_t bytes = 0;
    size_t part_floats = 0, arrive_words = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const xp_mv_job& j = jobs[i];
        if (!j.out || !j.in || !j.wq || !j.sc)
            return fail(XP_ERR_INVALID, "xp_mv_plan_create: job %u has a null pointer", i);
        if (j.rows == 0 || j.rows % 128 || j.cols == 0 || j.cols % 64)
            return fail(XP_ERR_INVALID, "xp_mv_plan_create: job %u: rows must be a multiple of 128 and cols of 64 "
                        "(got %u x %u)", i, j.rows, j.cols);
        uint32_t k = 0;
        while (k < hs.size() && !(hs[k].x == j.in && hs[k].nblk == j.rows / 32)) ++k;
        if (k == hs.size()) {
            hs.push_back(MvsSrc{j.in, j.rows / 32, nxq});
            nxq += j.rows / 32;
        }
        src_of[i] = k;
        // tall matrices split K into chunks of about MVS_CHUNK blocks so that
        // every SM has work (down-proj: 18 groups, 216 blocks each)
        const uint32_t nblk = j.rows / 32;
        const uint32_t ks = std::max<uint32_t>(1, nblk / MVS_CHUNK);
        const uint32_t cb = ((nblk + ks - 1) / ks + 3) & ~3u;
        const uint32_t kspl = (nblk + cb - 1) / cb;
        hj[i] = MvsJob{reinterpret_cast<const uint4*>(j.wq), reinterpret_cast<const uint2*>(j.sc), j.out, nullptr,
                       nullptr, nblk, j.cols, strips, hs[k].off, kspl, cb};
        strips += j.cols / 64 * kspl;
        if (kspl > 1) { part_floats += (size_t)j.cols * kspl; arrive_words += j.cols / 64; }
        bytes += (uint64_t)j.rows * j.cols / 2 + (uint64_t)j.rows * j.cols / 16 + 4ull * j.rows + 4ull * j.cols;
    }
    auto* p = new xp_mv_plan();
    cudaGetDevice(&p->device);
    auto cleanup = [&](const char* what, cudaError_t e) {
        xp_mv_plan_destroy(p);
        return fail(XP_ERR_OOM, "xp_mv_plan_create: %s: %s", what, cudaGetErrorString(e));
    };
    cudaError_t e;
    if ((e = cudaMalloc(&p->xq, (size_t)nxq * sizeof(XBlk))) != cudaSuccess) return cleanup("limbs", e);
    if (part_floats) {
        if ((e = cudaMalloc(&p->part, part_floats * 4)) != cudaSuccess) return cleanup("partials", e);
        if ((e = cudaMalloc(&p->arrive, arrive_words * 4)) != cudaSuccess) return cleanup("counters", e);
        if ((e = zero_fill_sync(p->arrive, arrive_words * 4)) != cudaSuccess) return cleanup("counters", e);
        size_t po = 0, ao = 0;
        for (auto& j : hj)
            if (j.ksplit > 1) {
                j.part = p->part + po;
                j.arrive = p->arrive + ao;
                po += (size_t)j.cols * j.ksplit;
                ao += j.cols / 64;
            }
    }
    if ((e = cudaMalloc(&p->jobs, n * sizeof(MvsJob))) != cudaSuccess) return cleanup("jobs", e);
    if ((e = cudaMalloc(&p->src, hs.size() * sizeof(MvsSrc))) != cudaSuccess) return cleanup("sources", e);
    if ((e = cudaMalloc(&p->next, 16)) != cudaSuccess) return cleanup("counter", e);
    if ((e = h2d_sync(p->jobs, hj.data(), n * sizeof(MvsJob))) != cudaSuccess)
        return cleanup("upload", e);
    if ((e = h2d_sync(p->src, hs.data(), hs.size() * sizeof(MvsSrc))) != cudaSuccess)
        return cleanup("upload", e);
    p->njobs = n;
    p->nstrips = strips;
    p->nsrc = (uint32_t)hs.size();
    p->nxq = nxq;
    p->bytes = bytes;
    p->smem_x = (size_t)nxq * sizeof(XBlk) <= MVS_SMEM_X_MAX;
    int per_sm = 0;
    if (p->smem_x) {
        static std::atomic<bool> attr_set[kMaxDevices];
        if ((e = smem_attr_once(attr_set, mv_stream_kernel<true>, (int)MVS_SMEM_X_MAX)) != cudaSuccess)
            return cleanup("shared-memory attribute", e);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mv_stream_kernel<true>, MVS_THREADS,
                                                      (size_t)nxq * sizeof(XBlk));
    } else {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mv_stream_kernel<false>, MVS_THREADS, 0);
    }
    p->grid = (uint32_t)sm_count() * (uint32_t)std::max(per_sm, 1);
    *plan = p;
    return XP_OK;
}
xp_status xp_mv_plan_run(xp_mv_plan* p, void* stream) {
    CHECK_PTR(p);
    const cudaStream_t st = (cudaStream_t)stream;
    mv_stream_prep_kernel<<<(p->nxq * 32 + 255) / 256, 256, 0, st>>>(p->src, p->nsrc, p->nxq, p->xq, p->next);
    XP_CUDA_TRY(cudaGetLastError());
    // the stream kernel launches while the limbs are prepared and waits for
    // them (griddepcontrol.wait) after staging its job table
    MvsArgs a{p->jobs, p->xq, p->njobs, p->nstrips, p->nxq, p->next};
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(p->grid);
    c.blockDim = dim3(MVS_THREADS);
    c.dynamicSmemBytes = p->smem_x ? (size_t)p->nxq * sizeof(XBlk) : 0;
    c.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = at;
    c.numAttrs = 1;
    const cudaError_t e = p->smem_x ? cudaLaunchKernelEx(&c, mv_stream_kernel<true>, a)
                                    : cudaLaunchKernelEx(&c, mv_stream_kernel<false>, a);
    return cuda_status(e, "mv_plan_run");
}
xp_status xp_mv_plan_bytes(const xp_mv_plan* p, uint64_t* bytes) {
    CHECK_PTR(p); CHECK_PTR(bytes);
    *bytes = p->bytes;
    return XP_OK;
}
void xp_mv_plan_destroy(xp_mv_plan* p) {
    if (!p) return;
    cudaFree(p->jobs);
    cudaFree(p->src);
    cudaFree(p->xq);
    cudaFree(p->next);
    cudaFree(p->part);
    cudaFree(p->arrive);
    delete p;
}
xp_status xp_rmsnorm_sumsq(void* stream, float* partial, const float* in, uint32_t n, uint32_t nparts) {
    CHECK_PTR(partial); CHECK_PTR(in);
    ops::rmsnorm_sumsq<<<(nparts + 255) / 256, 256, 0, (cudaStream_t)stream>>>(partial, in, n, nparts);
    return cuda_status(cudaGetLastError(), "rmsnorm_sumsq");
}
xp_status xp_rmsnorm_apply_gemma(void* stream, float* out, const float* in, const float* w, const float* partial,
                                 uint32_t n, uint32_t nparts, float eps) {
    CHECK_PTR(out); CHECK_PTR(in); CHECK_PTR(w); CHECK_PTR(partial);
    ops::rmsnorm_apply_gemma<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(out, in, w, partial, n, nparts, eps);
    return cuda_status(cudaGetLastError(), "rmsnorm_apply_gemma");
}
xp_status xp_rmsnorm_heads_gemma(void* stream, float* out, const float* in, const float* w, uint32_t n_heads,
                                 uint32_t head_dim, float eps) {
    CHECK_PTR(out); CHECK_PTR(in); CHECK_PTR(w);
    ops::rmsnorm_heads_gemma<<<(n_heads + 7) / 8, 256, 0, (cudaStream_t)stream>>>(out, in, w, n_heads, head_dim, eps);
    return cuda_status(cudaGetLastError(), "rmsnorm_heads_gemma");
}
xp_status xp_rope(void* stream, float* x, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float theta) {
    CHECK_PTR(x);
    const uint32_t n = n_heads * (head_dim / 2);
    ops::rope<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(x, n_heads, head_dim, pos, theta);
    return cuda_status(cudaGetLastError(), "rope");
}
xp_status xp_geglu(void* stream, float* out, const float* gate, const float* up, uint32_t n) {
    CHECK_PTR(out); CHECK_PTR(gate); CHECK_PTR(up);
    ops::geglu<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(out, gate, up, n);
    return cuda_status(cudaGetLastError(), "geglu");
}
xp_status xp_add_residual(void* stream, float* x, const float* y, uint32_t n) {
    CHECK_PTR(x); CHECK_PTR(y);
    ops::add_residual<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(x, y, n);
    return cuda_status(cudaGetLastError(), "add_residual");
}
xp_status xp_kv_append(void* stream, float* cache, const float* src, uint32_t n, uint32_t pos) {
    CHECK_PTR(cache); CHECK_PTR(src);
    ops::kv_append<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(cache, src, n, pos);
    return cuda_status(cudaGetLastError(), "kv_append");
}
xp_status xp_attention_scores(void* stream, float* scores, const float* q, const float* kcache, uint32_t n_heads,
                              uint32_t kv_heads, uint32_t head_dim, uint32_t span, float scale, uint32_t kv_start) {
    CHECK_PTR(scores); CHECK_PTR(q); CHECK_PTR(kcache);
    if (kv_heads == 0 || n_heads % kv_heads) return fail(XP_ERR_INVALID, "attention_scores: n_heads %% kv_heads != 0");
    const uint64_t w = (uint64_t)n_heads * span;
    ops::attention_scores<<<(unsigned)((w * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        scores, q, kcache, n_heads, kv_heads, head_dim, span, scale, kv_start);
    return cuda_status(cudaGetLastError(), "attention_scores");
}
xp_status xp_softmax_rows(void* stream, float* x, uint32_t n_rows, uint32_t n_cols) {
    CHECK_PTR(x);
    ops::softmax_rows<<<n_rows, 256, 0, (cudaStream_t)stream>>>(x, n_rows, n_cols);
    return cuda_status(cudaGetLastError(), "softmax_rows");
}
xp_status xp_attention_apply(void* stream, float* out, const float* probs, const float* vcache, uint32_t n_heads,
                             uint32_t kv_heads, uint32_t head_dim, uint32_t span, uint32_t kv_start) {
    CHECK_PTR(out); CHECK_PTR(probs); CHECK_PTR(vcache);
    if (kv_heads == 0 || n_heads % kv_heads) return fail(XP_ERR_INVALID, "attention_apply: n_heads %% kv_heads != 0");
    const uint32_t n = n_heads * head_dim;
    ops::attention_apply<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(out, probs, vcache, n_heads, kv_heads,
                                                                            head_dim, span, kv_start);
    return cuda_status(cudaGetLastError(), "attention_apply");
}
xp_status xp_argmax(void* stream, float* out, uint32_t* idx_out, const float* logits, uint32_t n) {
    CHECK_PTR(out); CHECK_PTR(logits);
    if (n == 0) return fail(XP_ERR_INVALID, "argmax: n must be nonzero");
    ops::argmax<<<1, 1024, 0, (cudaStream_t)stream>>>(out, logits, n);
    if (idx_out) {  // the uint form of the winner, as argmax_final's pidx_out
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_status(e, "argmax");
        ops::argmax_index<<<1, 32, 0, (cudaStream_t)stream>>>(idx_out, out);
    }
    return cuda_status(cudaGetLastError(), "argmax");
}
xp_status xp_topk4_partial(void* stream, float* cval, uint32_t* cidx, const float* x, uint32_t n, uint32_t nparts) {
    CHECK_PTR(cval); CHECK_PTR(cidx); CHECK_PTR(x);
    ops::topk4_partial<<<(nparts + 255) / 256, 256, 0, (cudaStream_t)stream>>>(cval, cidx, x, n, nparts);
    return cuda_status(cudaGetLastError(), "topk4_partial");
}

size_t xp_attention_scratch_bytes(uint32_t nsplit) { return attn_scratch_bytes(nsplit); }
}  // extern "C"
namespace xp {
// Argument checks of xp_attention_decode, shared with the entry point that
// keeps its scratch inside the library (which must refuse a call before it
// touches that shared array).
inline xp_status attn_validate(const float* out, const float* q_raw, const float* k_raw, const float* v_raw,
                               const float* q_norm, const float* k_norm, const uint16_t* kc, const uint16_t* vc,
                               const uint32_t* pos_dev, uint32_t window, uint32_t nsplit, uint32_t max_seq,
                               const void* scratch) {
    const void* ptrs[] = {out, q_raw, k_raw, v_raw, q_norm, k_norm, kc, vc, pos_dev, scratch};
    const char* names[] = {"out", "q_raw", "k_raw", "v_raw", "q_norm", "k_norm", "kcache_f16", "vcache_f16",
                           "pos_dev", "scratch"};
    for (int i = 0; i < 10; ++i)
        if (!ptrs[i]) return fail(XP_ERR_INVALID, "attention_decode: argument '%s' is null", names[i]);
    if (nsplit == 0 || nsplit > 1024) return fail(XP_ERR_INVALID, "attention_decode: nsplit must be 1..1024");
    if (max_seq == 0) return fail(XP_ERR_INVALID, "attention_decode: max_seq must be at least 1");
    if (attn_smem(attn_chunk_max(nsplit, attn_span_max(window, max_seq)), attn_cluster(attn_grid(nsplit))) > ATT_SMEM_MAX)
        return fail(XP_ERR_INVALID, "attention_decode: max_seq/nsplit too large for shared memory");
    if (((uintptr_t)out | (uintptr_t)kc | (uintptr_t)vc | (uintptr_t)scratch) & 15)
        return fail(XP_ERR_INVALID, "attention_decode: out, the caches and scratch must be 16-byte aligned");
    return XP_OK;
}
}  // namespace xp
extern "C" {
xp_status xp_attention_decode(void* stream, float* out, const float* q_raw, const float* k_raw, const float* v_raw,
                              const float* q_norm, const float* k_norm, uint16_t* kc, uint16_t* vc,
                              const uint32_t* pos_dev, uint32_t window, float theta, float eps, float scale,
                              uint32_t nsplit, uint32_t max_seq, void* scratch) {
    if (xp_status s = attn_validate(out, q_raw, k_raw, v_raw, q_norm, k_norm, kc, vc, pos_dev, window, nsplit,
                                    max_seq, scratch);
        s != XP_OK)
        return s;
    AttnArgs a{};
    a.q_raw = q_raw; a.k_raw = k_raw; a.v_raw = v_raw; a.q_norm = q_norm; a.k_norm = k_norm;
    a.kcache = reinterpret_cast<__half*>(kc);
    a.vcache = reinterpret_cast<__half*>(vc);
    a.pos = pos_dev;
    a.cache_rows = max_seq;
    a.window = window; a.theta = theta; a.eps = eps; a.scale = scale;
    a.att = out;
    a.att_xq = nullptr;
    // programmatic dependent launch: the kernel reads nothing before
    // griddepcontrol.wait, so its launch may overlap any predecessor's tail
    return cuda_status(launch_attn(a, scratch, nsplit, attn_span_max(window, max_seq), (cudaStream_t)stream, true),
                       "attention_decode");
}
xp_status xp_selftest_wait_timeout(uint32_t spin_limit, uint32_t* err_word) {
    CHECK_PTR(err_word);
    if (spin_limit == 0 || spin_limit > TK_SPIN_LIMIT)
        return fail(XP_ERR_INVALID, "selftest_wait_timeout: spin_limit 1..%u", TK_SPIN_LIMIT);
    uint32_t* d = nullptr;
    XP_CUDA_TRY(cudaMalloc(&d, 64));
    cudaError_t e = cudaMemset(d, 0, 64);
    if (e == cudaSuccess) {
        selftest_wait_kernel<<<1, 32>>>(reinterpret_cast<uint64_t*>(d + 8), d, spin_limit);
        e = cudaDeviceSynchronize();
    }
    if (e == cudaSuccess) e = cudaMemcpy(err_word, d, 4, cudaMemcpyDeviceToHost);
    cudaFree(d);
    return cuda_status(e, "selftest_wait_timeout");
}
size_t xp_sample_scratch_bytes(uint32_t n) { return sample_scratch_bytes(n); }
xp_status xp_sample_topk(void* stream, uint32_t* token_dev, float* out_vals, uint32_t* out_idx, const float* logits,
                         uint32_t n, uint32_t top_k, float temperature, float top_p, uint64_t seed, uint64_t seq_id,
                         const uint32_t* pos_dev, void* scratch) {
    CHECK_PTR(token_dev); CHECK_PTR(logits); CHECK_PTR(pos_dev); CHECK_PTR(scratch);
    if (n < TOPK_TK) return fail(XP_ERR_INVALID, "sample_topk: n must be >= %u", TOPK_TK);
    if ((n + TOPK_SLICE - 1) / TOPK_SLICE * TOPK_TK > TOPK_MAX_CAND)
        return fail(XP_ERR_INVALID, "sample_topk: n must be <= %u", TOPK_MAX_CAND / TOPK_TK * TOPK_SLICE);
    if (top_k > TOPK_TK) return fail(XP_ERR_INVALID, "sample_topk: top_k must be <= %u", TOPK_TK);
    return cuda_status(launch_sample_topk(token_dev, nullptr, const_cast<uint32_t*>(pos_dev), out_vals, out_idx,
                                          logits, n, top_k, temperature, top_p, seed, seq_id, scratch,
                                          (cudaStream_t)stream, true, false),
                       "sample_topk");
}
xp_status xp_pack_km4bf16(void* stream, const float* w, uint32_t rows, uint32_t cols, uint32_t* words,
                          uint32_t* scales) {
    CHECK_PTR(w); CHECK_PTR(words); CHECK_PTR(scales);
    if (rows == 0 || rows % 128 || cols == 0 || cols % 64)
        return fail(XP_ERR_INVALID, "pack_km4bf16: rows %% 128 and cols %% 64 must be 0 (got %u x %u)", rows, cols);
    const uint64_t total = (uint64_t)cols * (rows / 32);
    const unsigned blocks = (unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 32);
    pack_km4bf16_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(w, rows, cols, reinterpret_cast<uint4*>(words),
                                                                  scales);
    return cuda_status(cudaGetLastError(), "pack_km4bf16");
}
xp_status xp_gen_normal(void* stream, float* out, uint64_t n, uint64_t offset, uint64_t seed, uint64_t stream_id,
                        float sigma) {
    CHECK_PTR(out);
    if (n == 0) return XP_OK;
    const unsigned blocks = (unsigned)std::min<uint64_t>((n + 255) / 256, (uint64_t)sm_count() * 32);
    gen_normal_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(out, n, offset, seed, stream_id, sigma);
    return cuda_status(cudaGetLastError(), "gen_normal");
}
xp_status xp_stream4(void* stream, float* out, const void* src, uint32_t n, uint32_t threads) {
    CHECK_PTR(out); CHECK_PTR(src);
    if (threads == 0) return fail(XP_ERR_GRID, "stream4: threads must be nonzero");
    ops::stream4<<<(threads + 255) / 256, 256, 0, (cudaStream_t)stream>>>(out, (const uint4*)src, n, threads);
    return cuda_status(cudaGetLastError(), "stream4");
}

}  // extern "C"
