// CPU checker: the reference's own OpenCL C kernels (kernels/llm_matvec.cl,
// kernels/llm_transformer.cl, kernels/llm_sampling.cl, kernels/llm.cl,
// kernels/llm_quant.cl)
// compiled VERBATIM as host C++ through cl_shim.hpp, and dispatched over the
// same global grids the reference runtime uses (src/launch.cpp:21-35: grid =
// global thread count, every kernel bound-checks its id).
//
// TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile into oracle/_ref/ from the
// sources where they lie in the reference tree (REF_DIR); never shipped, never
// on the product path. Exposes a C entry point so Python tests and the stub
// vulkore runtime (oracle/refstub) can launch any kernel by (module, name).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>
#include <omp.h>

#include "cl_shim.hpp"

namespace clshim { thread_local uint32_t tl_gid = 0; }

#define XSTR(x) #x
#define STR(x) XSTR(x)

namespace ref_llm {
#include STR(REF_DIR/kernels/llm.cl)
}
#undef BLK
namespace ref_matvec {
#include STR(REF_DIR/kernels/llm_matvec.cl)
}
#undef BLK
#undef GRP
namespace ref_transformer {
#include STR(REF_DIR/kernels/llm_transformer.cl)
}
namespace ref_sampling {
#include STR(REF_DIR/kernels/llm_sampling.cl)
}
namespace ref_quant {
#include STR(REF_DIR/kernels/llm_quant.cl)
}
#undef NIB8
#undef N5_8
#undef N6_8
#undef B4
#undef SPLIT_PROLOGUE
#undef kernel
#undef global
#undef constant
#undef __attribute__

#include "ref_kernels.h"

namespace {

template <class T> T get_arg(const xpref_arg& a) {
    if constexpr (std::is_pointer_v<T>) {
        return (T)(const_cast<void*>(a.ptr));
    } else {
        T v{};
        std::memcpy(&v, a.ptr, sizeof(T));
        return v;
    }
}
template <class T> constexpr int arg_kind() { return std::is_pointer_v<T> ? 1 : 0; }
template <class T> constexpr uint32_t arg_size() {
    if constexpr (std::is_pointer_v<T>) return 0; else return sizeof(T);
}

struct Entry {
    const char* module;
    const char* name;
    uint32_t nargs;
    int kinds[16];
    uint32_t sizes[16];
    void (*invoke)(const xpref_arg*, uint32_t grid, int threads);
};

template <auto F> struct Invoker;
template <class... P, void (*F)(P...)> struct Invoker<F> {
    template <size_t... I>
    static void one(const xpref_arg* a, std::index_sequence<I...>) { F(get_arg<P>(a[I])...); }
    static void run(const xpref_arg* a, uint32_t grid, int threads) {
        if (threads <= 0) threads = omp_get_max_threads();
        // Work items are independent within one dispatch (the reference's own
        // contract: no __local, no barriers), so any interleaving is valid.
        #pragma omp parallel for schedule(static) num_threads(threads)
        for (int64_t i = 0; i < (int64_t)grid; ++i) {
            clshim::tl_gid = (uint32_t)i;
            one(a, std::index_sequence_for<P...>{});
        }
    }
    static Entry make(const char* module, const char* name) {
        Entry e{module, name, sizeof...(P), {arg_kind<P>()...}, {arg_size<P>()...}, &run};
        return e;
    }
};

#define K(mod, ns, fn) Invoker<&ns::fn>::make(mod, #fn)
const char* M_LLM = "kernels/llm.spv";
const char* M_MV = "kernels/llm_matvec.spv";
const char* M_TF = "kernels/llm_transformer.spv";
const char* M_SM = "kernels/llm_sampling.spv";
const char* M_QT = "kernels/llm_quant.spv";

const std::vector<Entry>& table() {
    static const std::vector<Entry> t = {
        K(M_LLM, ref_llm, matvec_f32), K(M_LLM, ref_llm, matvec_q4),
        K(M_LLM, ref_llm, stream_read), K(M_LLM, ref_llm, matvec_q4_split),
        K(M_LLM, ref_llm, matvec_reduce),
        K(M_MV, ref_matvec, mv_ref), K(M_MV, ref_matvec, mv_ref_split),
        K(M_MV, ref_matvec, mv_reduce), K(M_MV, ref_matvec, mv_kmn),
        K(M_MV, ref_matvec, mv_km), K(M_MV, ref_matvec, mv_km4),
        K(M_MV, ref_matvec, mv_km4_c2), K(M_MV, ref_matvec, mv_km4_c4),
        K(M_MV, ref_matvec, mv_km4_wg32), K(M_MV, ref_matvec, mv_km4_wg128),
        K(M_MV, ref_matvec, mv_km4_wg256), K(M_MV, ref_matvec, mv_km4_c2_wg32),
        K(M_MV, ref_matvec, mv_km4_split), K(M_MV, ref_matvec, stream4),
        K(M_MV, ref_matvec, mv_km4_bs), K(M_MV, ref_matvec, mv_km4_bs_split),
        K(M_TF, ref_transformer, rmsnorm), K(M_TF, ref_transformer, rmsnorm_gemma),
        K(M_TF, ref_transformer, rmsnorm_sumsq), K(M_TF, ref_transformer, rmsnorm_apply_gemma),
        K(M_TF, ref_transformer, rmsnorm_heads_gemma), K(M_TF, ref_transformer, rope),
        K(M_TF, ref_transformer, rope_cached), K(M_TF, ref_transformer, geglu),
        K(M_TF, ref_transformer, swiglu), K(M_TF, ref_transformer, geglu_fused),
        K(M_TF, ref_transformer, attention_scores), K(M_TF, ref_transformer, softmax_rows),
        K(M_TF, ref_transformer, softmax_rows_partial), K(M_TF, ref_transformer, softmax_rows_finish),
        K(M_TF, ref_transformer, softmax_rows_scale), K(M_TF, ref_transformer, attention_scores_mq4),
        K(M_TF, ref_transformer, attention_apply), K(M_TF, ref_transformer, attention_apply_mq4),
        K(M_TF, ref_transformer, attention_apply_reduce), K(M_TF, ref_transformer, add_residual),
        K(M_TF, ref_transformer, add_vec), K(M_TF, ref_transformer, mul_scalar),
        K(M_TF, ref_transformer, kv_append), K(M_TF, ref_transformer, embed_lookup),
        K(M_TF, ref_transformer, argmax),
        K(M_SM, ref_sampling, argmax_partial), K(M_SM, ref_sampling, argmax_reduce),
        K(M_SM, ref_sampling, argmax_final), K(M_SM, ref_sampling, apply_temperature),
        K(M_SM, ref_sampling, reduce_max_partial), K(M_SM, ref_sampling, reduce_max_final),
        K(M_SM, ref_sampling, softmax_exp_partial), K(M_SM, ref_sampling, reduce_sum_partial),
        K(M_SM, ref_sampling, reduce_sum_final), K(M_SM, ref_sampling, softmax_normalize),
        K(M_SM, ref_sampling, topk_partial), K(M_SM, ref_sampling, topk4_partial),
        K(M_SM, ref_sampling, topk_rank_select), K(M_SM, ref_sampling, topk_mask),
        K(M_SM, ref_sampling, topp_cutoff), K(M_SM, ref_sampling, multinomial_sample),
        K(M_SM, ref_sampling, multinomial_strided),
        K(M_SM, ref_sampling, softmax_rows_stats), K(M_SM, ref_sampling, softmax_rows_apply),
        K(M_SM, ref_sampling, attention_scores_prefill), K(M_SM, ref_sampling, attention_apply_prefill),
        K(M_SM, ref_sampling, rmsnorm_rows_sumsq), K(M_SM, ref_sampling, rmsnorm_rows_apply_gemma),
        K(M_SM, ref_sampling, rmsnorm_heads_rows_gemma), K(M_SM, ref_sampling, rope_prefill),
        K(M_SM, ref_sampling, kv_append_rows), K(M_SM, ref_sampling, embed_lookup_rows),
        K(M_QT, ref_quant, fp16_decode), K(M_QT, ref_quant, dequant_q8_0), K(M_QT, ref_quant, matvec_q8_0),
        K(M_QT, ref_quant, dequant_q5_0), K(M_QT, ref_quant, matvec_q5_0), K(M_QT, ref_quant, dequant_q4_k),
        K(M_QT, ref_quant, matvec_q4_k), K(M_QT, ref_quant, dequant_q6_k), K(M_QT, ref_quant, matvec_q6_k),
        K(M_QT, ref_quant, matvec_rq4_k), K(M_QT, ref_quant, matvec_rq5_0), K(M_QT, ref_quant, matvec_rq6_k),
        K(M_QT, ref_quant, matvec_rq8_0), K(M_QT, ref_quant, matvec_rq4_k_split),
        K(M_QT, ref_quant, matvec_rq5_0_split), K(M_QT, ref_quant, matvec_rq6_k_split),
        K(M_QT, ref_quant, matvec_rq8_0_split), K(M_QT, ref_quant, mv_reduce),
    };
    return t;
}

bool module_matches(const char* want, const char* have) {
    // Accept the full module path or just its file name.
    std::string w(want), h(have);
    if (w == h) return true;
    auto base = [](const std::string& s) { auto p = s.find_last_of('/'); return p == std::string::npos ? s : s.substr(p + 1); };
    return base(w) == base(h);
}

thread_local std::string g_err;

}  // namespace

extern "C" {

const char* xpref_last_error(void) { return g_err.c_str(); }

int xpref_find(const char* module, const char* name) {
    const auto& t = table();
    for (size_t i = 0; i < t.size(); ++i)
        if (std::strcmp(t[i].name, name) == 0 && (!module || module_matches(module, t[i].module)))
            return (int)i;
    return -1;
}

int xpref_kernel_info(int id, const char** module, const char** name, uint32_t* nargs,
                      int* kinds, uint32_t* sizes) {
    const auto& t = table();
    if (id < 0 || (size_t)id >= t.size()) return -1;
    const Entry& e = t[id];
    if (module) *module = e.module;
    if (name) *name = e.name;
    if (nargs) *nargs = e.nargs;
    for (uint32_t i = 0; i < e.nargs; ++i) {
        if (kinds) kinds[i] = e.kinds[i];
        if (sizes) sizes[i] = e.sizes[i];
    }
    return 0;
}

int xpref_count(void) { return (int)table().size(); }

int xpref_launch(const char* module, const char* name, uint32_t grid, const xpref_arg* args,
                 uint32_t nargs, int threads) {
    int id = xpref_find(module, name);
    if (id < 0) { g_err = std::string("no kernel '") + name + "'"; return -1; }
    const Entry& e = table()[id];
    if (nargs != e.nargs) { g_err = "arity mismatch for " + std::string(name); return -2; }
    for (uint32_t i = 0; i < nargs; ++i) {
        const int want_buf = e.kinds[i];
        if (want_buf && !args[i].is_buffer) { g_err = "arg " + std::to_string(i) + " wants a buffer"; return -3; }
        if (!want_buf && (args[i].is_buffer || args[i].size != e.sizes[i])) {
            g_err = "arg " + std::to_string(i) + " wants a " + std::to_string(e.sizes[i]) + "-byte POD";
            return -3;
        }
    }
    if (grid == 0) { g_err = "grid must be nonzero"; return -4; }
    // The runtime rounds the grid up to whole workgroups of 64 (or the
    // reqd_work_group_size); kernels bound-check, so running the rounded grid
    // and the exact grid are equivalent. The exact grid is used here.
    e.invoke(args, grid, threads);
    return 0;
}

}  // extern "C"
