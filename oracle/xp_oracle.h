/* CPU ORACLE -- test infrastructure only.
 *
 * A plain-C restatement of the reference algorithms on the Gemma-3 decode hot
 * path (badnikhil/Xpose, "Vulkore"): the host int4 packer, the matvec and
 * transformer kernels, the sampling chain and the per-token op order. Each
 * function cites the reference file:line it restates.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library, and only as the checker. The product path (the CUDA
 * library under xpose_b200/) never links, loads or falls back to it.
 *
 * Parity is pinned: tests/test_oracle_pin.py checks every function here
 * against the reference's own kernels and packer compiled from source into
 * oracle/_ref/ (see oracle/Makefile), and against tests/golden/ fixtures made
 * by tests/golden/make_golden.py from that build.
 */
#ifndef XP_ORACLE_H
#define XP_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded synthetic inputs ------------------------------------------ */
/* Counter-based generator shared bit-for-bit with the CUDA library:
 * splitmix64 over (seed, stream, index), and an Irwin-Hall(12) approximation
 * of N(0, sigma) built only from exact integer->float conversions and
 * fixed-order fp32 adds, so host and device produce identical values. */
uint64_t xo_splitmix64(uint64_t x);
void xo_gen_normal(uint64_t seed, uint64_t stream, uint64_t offset, uint64_t n, float sigma,
                   float* out);
void xo_gen_tokens(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab, uint32_t* out);
/* uniform in [0, 1) with 24 random bits, the sampler's draw */
float xo_uniform(uint64_t seed, uint64_t stream, uint64_t index);

/* ---- fp16 (KV cache storage) ------------------------------------------ */
uint16_t xo_f32_to_f16(float f); /* round to nearest even */
float xo_f16_to_f32(uint16_t h);

/* ---- int4 KM4 + bf16 packer (examples/llm/decode.cpp:94-229) ----------- */
uint32_t xo_quantise(float v, float inv_scale);
float xo_best_bf16_scale(const float* blk32, float s0);
/* w is [cols][rows] (row j = output column j). rows % 128 == 0, cols % 64 == 0.
 * words: 4 uint32 per (group, block, col); scales: 2 uint32 per (quad, col). */
int xo_pack_km4bf16(const float* w_cols_rows, uint32_t rows, uint32_t cols, uint32_t* words,
                    uint32_t* scales);
/* Dequantised weight W[k][j] exactly as the kernel reconstructs it:
 * (nibble - 8) * bf16(scale). */
float xo_dequant(const uint32_t* words, const uint32_t* scales, uint32_t rows, uint32_t cols,
                 uint32_t k, uint32_t j);

/* ---- kernels (kernels/llm_matvec.cl, llm_transformer.cl, llm_sampling.cl) */
void xo_mv_km4_bs(float* out, const float* in, const uint32_t* wq, const uint32_t* sc,
                  uint32_t rows, uint32_t cols);
void xo_mv_km4_bs_split(float* out, const float* in, const uint32_t* wq, const uint32_t* sc,
                        uint32_t rows, uint32_t cols, uint32_t split);
void xo_rmsnorm_gemma(float* out, const float* in, const float* w, uint32_t n, uint32_t nparts,
                      float eps);
void xo_rmsnorm_heads_gemma(float* out, const float* in, const float* w, uint32_t n_heads,
                            uint32_t head_dim, float eps);
void xo_rope(float* x, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float theta);
void xo_geglu(float* out, const float* gate, const float* up, uint32_t n);
void xo_add_residual(float* x, const float* y, uint32_t n);
/* Single-query attention over cache positions [kv_start, kv_start+span).
 * Cache rows are [t][kv_heads][head_dim]; kv_fp16 selects uint16 storage. */
void xo_attention(float* out, const float* q, const void* kcache, const void* vcache,
                  int kv_fp16, uint32_t n_heads, uint32_t kv_heads, uint32_t head_dim,
                  uint32_t kv_start, uint32_t span, float scale);
uint32_t xo_argmax(const float* logits, uint32_t n, float* best_val);
/* exact top-k, descending, ties -> lower index; returns the count written */
uint32_t xo_topk(const float* x, uint32_t n, uint32_t k, float* vals, uint32_t* idx);
/* decode.cpp:1873-1917 draw() over the exact top-k of the full vocab, with
 * the multinomial's uniform supplied (u in [0,1)) instead of mt19937_64. */
uint32_t xo_sample(const float* logits, uint32_t n, float temperature, uint32_t top_k,
                   float top_p, float u);

/* ---- GGUF tensor types (ggml block formats, examples/llm/model/gguf.cpp:448-634)
 * type: 0 F32, 1 F16, 2 Q4_0, 3 Q4_1, 6 Q5_0, 7 Q5_1, 8 Q8_0, 12 Q4_K, 14 Q6_K,
 * 30 BF16. n elements (a multiple of the block size). Returns 0, or -1 for a
 * type that is not dequantised. */
int xo_gguf_dequantize(uint32_t type, const void* src, float* dst, uint64_t n);
/* the .xpack payload hash (examples/llm/decode.cpp:784-834): FNV-1a over
 * 64-bit words with a final avalanche, folded over 4 MiB chunks */
uint64_t xo_xpack_hash(const void* data, uint64_t nbytes);
uint64_t xo_xpack_hash_chunked(const void* data, uint64_t nbytes);

/* ---- prefill shapes (kernels/llm_sampling.cl:495-736) ------------------ */
void xo_softmax_rows_stats(float* stats, const float* x, uint32_t n_rows, uint32_t n_cols);
void xo_softmax_rows_apply(float* x, const float* stats, uint32_t n_rows, uint32_t n_cols);
void xo_attention_scores_prefill(float* scores, const float* q, const float* kcache, uint32_t n_heads,
                                 uint32_t kv_heads, uint32_t head_dim, uint32_t n_query,
                                 uint32_t seq_len, uint32_t q_offset, uint32_t window, float scale);
void xo_attention_apply_prefill(float* out, const float* probs, const float* vcache, uint32_t n_heads,
                                uint32_t kv_heads, uint32_t head_dim, uint32_t n_query,
                                uint32_t seq_len);
void xo_rmsnorm_rows_sumsq(float* rowss, const float* in, uint32_t n_rows, uint32_t n);
void xo_rmsnorm_rows_apply_gemma(float* out, const float* in, const float* w, const float* rowss,
                                 uint32_t n_rows, uint32_t n, float eps);
void xo_rmsnorm_heads_rows_gemma(float* out, const float* in, const float* w, uint32_t n_tokens,
                                 uint32_t n_heads, uint32_t head_dim, float eps);
void xo_rope_prefill(float* x, uint32_t n_tokens, uint32_t n_heads, uint32_t head_dim,
                     uint32_t pos0, float theta);
void xo_kv_append_rows(float* cache, const float* src, uint32_t n_tokens, uint32_t row,
                       uint32_t pos0);
void xo_embed_lookup_rows(float* out, const float* table, const uint32_t* tokens,
                          uint32_t n_tokens, uint32_t n);

/* ---- one decode token (examples/llm/decode.cpp:1634-1780) -------------- */
typedef struct xo_qweight {
    uint32_t rows, cols; /* K inputs, N outputs */
    const uint32_t* wq;
    const uint32_t* sc;
} xo_qweight;

typedef struct xo_layer {
    xo_qweight wq, wk, wv, wo, gate, up, down;
    const float *attn_norm, *post_attn_norm, *ffn_norm, *post_ffn_norm, *q_norm, *k_norm;
} xo_layer;

typedef struct xo_model {
    uint32_t n_layers, hidden, ffn, n_heads, n_kv_heads, head_dim, vocab, max_seq;
    uint32_t sliding_window, global_every, norm_parts;
    float rms_eps, theta_global, theta_local, embed_scale, attn_scale;
    int kv_fp16;
    const xo_layer* layers;
    xo_qweight lm_head;
    const float* final_norm;
    const float* embed; /* [vocab][hidden] fp32 rows, scaled by embed_scale on lookup */
} xo_model;

/* KV caches: per layer max_seq*kv_dim elements of fp32 or fp16 (kv_fp16). */
typedef struct xo_state {
    void** kcache;
    void** vcache;
} xo_state;

/* Runs one position. logits may be NULL (a prompt token). Returns 0. */
int xo_forward(const xo_model* m, xo_state* st, uint32_t token, uint32_t pos, float* logits);
uint32_t xo_layer_kv_start(const xo_model* m, uint32_t layer, uint32_t seq_len);

#ifdef __cplusplus
}
#endif
#endif
