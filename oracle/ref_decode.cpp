// CPU checker: the reference's host engine (examples/llm/decode.cpp: the int4
// packer, DecodeSession, record_token, draw) compiled VERBATIM against the CPU
// stand-in runtime in oracle/refstub, so its Batch::add calls run the
// reference's own kernels (ref_kernels.cpp). Including the .cpp gives this
// translation unit the anonymous-namespace packer functions, which are
// re-exported below with a C ABI for the parity tests.
//
// TEST INFRASTRUCTURE ONLY, built into oracle/_ref/ by oracle/Makefile.
#define VULKORE_LLM_DECODE_NO_MAIN 1
#define XSTR(x) #x
#define STR(x) XSTR(x)
#include STR(REF_DIR/examples/llm/decode.cpp)

#include <cstring>
#include <memory>

#include "quant_repack.hpp"

using namespace vulkore::llm;

extern "C" {

// fp32 [cols][rows] weights (GGUF order: row j of the source tensor is output
// column j) -> the KM4 nibble plane (uint4 per (group, block, col) = 4 words)
// and the bf16 scale plane (uint2 per (quad, col) = 2 words). cols % 64 == 0,
// rows % 128 == 0. Follows the reference load path: pack_group per 64-column
// group (decode.cpp:177-229) then pack_scales_bf16_cols (decode.cpp:157-169).
int xpref_pack_km4bf16(const float* w_cols_rows, uint32_t rows, uint32_t cols,
                       uint32_t* words, uint32_t* scales_u32, float* scales_f32) {
    if (rows % 128 || cols % 64) return -1;
    const uint32_t nblk = rows / 32;
    std::vector<float> sc((size_t)nblk * cols);
    for (uint32_t g = 0; g < cols / 64; ++g)
        pack_group(w_cols_rows + (size_t)g * 64 * rows, rows, cols, g, MatvecLayout::Km4Bf16,
                   words, sc.data());
    pack_scales_bf16_cols(sc.data(), nblk, cols, 0, cols, scales_u32);
    if (scales_f32) std::memcpy(scales_f32, sc.data(), sc.size() * 4);
    return 0;
}

float xpref_best_bf16_scale(const float* blk32, float s0) { return best_bf16_scale(blk32, s0); }

// examples/llm/model/gguf.cpp GGUFFile::dequantize, for the GGUF-type pins
int xpref_gguf_dequantize(uint32_t type, const void* src, float* dst, uint64_t n) {
    return GGUFFile::dequantize(static_cast<GGMLType>(type), src, dst, (size_t)n) ? 0 : -1;
}
// the .xpack payload hash (decode.cpp:784-834)
uint64_t xpref_xpack_hash(const void* data, uint64_t n) { return xpack_hash(data, (size_t)n); }
uint64_t xpref_xpack_hash_mt(const void* data, uint64_t n, uint32_t threads) {
    return xpack_hash_mt(data, (size_t)n, threads);
}
uint32_t xpref_quantise(float v, float inv) { return quantise(v, inv); }

// examples/llm/quant_repack.cpp repack(): native GGUF blocks -> the planes of
// the matvec_rq* kernels. sizes[4] receives the element counts of quant,
// high, scale and bias; each output pointer may be null (size query).
int xpref_quant_repack(uint32_t type, const void* src, uint32_t rows, uint32_t cols, uint32_t* quant,
                       uint32_t* high, float* scale, float* bias, uint64_t* sizes) {
    RepackedTensor t;
    if (!repack(static_cast<GGMLType>(type), src, rows, cols, t)) return -1;
    sizes[0] = t.quant.size();
    sizes[1] = t.high.size();
    sizes[2] = t.scale.size();
    sizes[3] = t.bias.size();
    if (quant) std::memcpy(quant, t.quant.data(), t.quant.size() * 4);
    if (high) std::memcpy(high, t.high.data(), t.high.size() * 4);
    if (scale) std::memcpy(scale, t.scale.data(), t.scale.size() * 4);
    if (bias) std::memcpy(bias, t.bias.data(), t.bias.size() * 4);
    return 0;
}

uint64_t xpref_plan_weight_bytes(void) {
    return plan_token(DecodeConfig::gemma3_1b(), MatvecConfig{}).weight_bytes;
}
uint32_t xpref_plan_dispatches(void) {
    return plan_token(DecodeConfig::gemma3_1b(), MatvecConfig{}).total;
}

// ---- a whole reference DecodeSession on a GGUF file --------------------------
struct xpref_session { std::unique_ptr<DecodeSession> s; std::string err; };

static thread_local std::string g_sess_err;
const char* xpref_session_error(void) { return g_sess_err.c_str(); }

// examples/llm/model/tokenizer.cpp over a GGUF file, for the tokenizer pins
struct xpref_tok { GGUFFile f; std::unique_ptr<Tokenizer> t; };
void* xpref_tok_create(const char* path) {
    try {
        auto* h = new xpref_tok{GGUFFile::open(path), nullptr};
        h->t = std::make_unique<Tokenizer>(Tokenizer::from_gguf(h->f));
        return h;
    } catch (const std::exception& e) { g_sess_err = e.what(); return nullptr; }
}
void xpref_tok_destroy(void* h) { delete (xpref_tok*)h; }
int xpref_tok_encode(void* h, const char* text, size_t len, int bos, int eos, int32_t* out, uint32_t cap) {
    auto v = ((xpref_tok*)h)->t->encode(std::string_view(text, len), bos != 0, eos != 0);
    for (size_t i = 0; i < v.size() && i < cap; ++i) out[i] = v[i];
    return (int)v.size();
}
long xpref_tok_piece(void* h, int32_t id, char* out, size_t cap) {
    std::string s = ((xpref_tok*)h)->t->decode_one(id);
    if (s.size() + 1 <= cap) std::memcpy(out, s.c_str(), s.size() + 1);
    return (long)s.size();
}
long xpref_tok_decode(void* h, const int32_t* ids, uint32_t n, int skip, char* out, size_t cap) {
    std::string s = ((xpref_tok*)h)->t->decode(std::vector<int32_t>(ids, ids + n), skip != 0);
    if (s.size() + 1 <= cap) std::memcpy(out, s.c_str(), s.size() + 1);
    return (long)s.size();
}

// The .xpack cache the next xpref_session_create uses (empty: none)
static std::string g_pack_cache;
void xpref_set_pack_cache(const char* path) { g_pack_cache = path ? path : ""; }

void* xpref_session_create(const char* gguf_path, const char* kernel_dir, uint32_t max_seq,
                           int greedy, float temperature, uint32_t top_k, float top_p,
                           uint64_t seed, uint32_t global_every) {
    try {
        Paths p;
        std::string kd = kernel_dir ? kernel_dir : "kernels";
        p.matvec.module = kd + "/llm_matvec.spv";
        p.transformer_spv = kd + "/llm_transformer.spv";
        p.sampling_spv = kd + "/llm_sampling.spv";
        p.model_gguf = gguf_path;
        p.use_pack_cache = !g_pack_cache.empty();
        p.pack_cache = g_pack_cache;
        DecodeConfig c;
        c.max_seq = max_seq;
        c.sampling.mode = greedy ? SampleMode::Greedy : SampleMode::Temperature;
        c.sampling.temperature = temperature;
        c.sampling.top_k = top_k;
        c.sampling.top_p = top_p;
        c.sampling.seed = seed;
        c.global_every = global_every;
        auto* h = new xpref_session;
        h->s = std::make_unique<DecodeSession>(p, c);
        return h;
    } catch (const std::exception& e) {
        g_sess_err = e.what();
        return nullptr;
    }
}
void xpref_session_destroy(void* h) { delete (xpref_session*)h; }
int xpref_session_prefill(void* h, const uint32_t* toks, uint32_t n) {
    try { ((xpref_session*)h)->s->prefill(std::span<const uint32_t>(toks, n)); return 0; }
    catch (const std::exception& e) { g_sess_err = e.what(); return -1; }
}
int64_t xpref_session_step(void* h) {
    try { return ((xpref_session*)h)->s->decode_step(); }
    catch (const std::exception& e) { g_sess_err = e.what(); return -1; }
}
int xpref_session_logits(void* h, float* out, uint32_t n) {
    try {
        auto v = ((xpref_session*)h)->s->last_logits();
        if (v.size() != n) { g_sess_err = "logit count mismatch"; return -1; }
        std::memcpy(out, v.data(), n * 4);
        return 0;
    } catch (const std::exception& e) { g_sess_err = e.what(); return -1; }
}
uint32_t xpref_session_position(void* h) { return ((xpref_session*)h)->s->position(); }

}  // extern "C"
