/* xp_cuda.h -- C ABI of the B200 (sm_100a) Gemma-3 int4 decode path.
 *
 * This is the drop-in boundary for the reference's operator surface
 * (badnikhil/Xpose, "Vulkore"): the kernel entry points of
 * kernels/llm_matvec.cl, kernels/llm_transformer.cl and kernels/llm_sampling.cl
 * that examples/llm/decode.cpp drives, the runtime calls it makes on them
 * (include/vulkore/{context,buffer,program,launch,sync}.hpp), and the engine
 * unit of work, DecodeSession (examples/llm/decode.hpp:605-676).
 *
 * Plain pointers and sizes only. Device pointers are CUDA device addresses;
 * `stream` is a cudaStream_t (NULL = legacy default stream). Every call
 * returns an xp_status; on failure xp_last_error() holds a message naming the
 * kernel and argument, in the form the reference's vulkore::Error uses
 * (src/launch.cpp:21-131). Not thread-safe per context; one context per
 * thread per device (the reference's Context is single-threaded too,
 * agent-docs/vulkore-core.md:76-77).
 */
#ifndef XP_CUDA_H
#define XP_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status --------------------------------------------------------------- */
typedef enum xp_status {
    XP_OK = 0,
    XP_TIMEOUT = 1,           /* Fence::wait timed out (include/vulkore/sync.hpp:25-28) */
    XP_ERR_INVALID = -1,      /* bad argument value (null, size, shape) */
    XP_ERR_NO_KERNEL = -2,    /* Program::kernel: unknown name (include/vulkore/program.hpp:107) */
    XP_ERR_ARITY = -3,        /* launch: wrong argument count (src/launch.cpp:63-74) */
    XP_ERR_ARG_KIND = -4,     /* launch: buffer where a POD is expected or vice versa (:85-111) */
    XP_ERR_ARG_SIZE = -5,     /* launch: POD size mismatch (:112-121) */
    XP_ERR_GRID = -6,         /* launch: zero grid or too many groups (:21-35) */
    XP_ERR_CUDA = -7,         /* a CUDA runtime error */
    XP_ERR_OOM = -8,
    XP_ERR_KV_FULL = -9,      /* decode: KV cache is full (decode.cpp:1823-1826) */
    XP_ERR_STATE = -10,       /* decode_step before prefill (decode.cpp:1821-1822), spent Batch */
    XP_ERR_DEVICE = -11,      /* device lost / kernel fault */
    XP_ERR_NO_DEVICE = -12,
    XP_ERR_UNSUPPORTED = -13  /* shape outside what the kernels implement */
} xp_status;

const char* xp_last_error(void);
const char* xp_status_name(int status);
/* Library / device info. */
const char* xp_version(void);
int xp_device_count(void);

/* ---- context and buffers (include/vulkore/context.hpp, buffer.hpp) -------- */
typedef struct xp_context xp_context;
typedef enum xp_usage { XP_DEVICE_LOCAL = 0, XP_HOST_VISIBLE = 1 } xp_usage;

xp_status xp_context_create(int device, xp_context** out);
xp_status xp_context_destroy(xp_context* ctx);
/* The stream all Batch submissions and typed launches of this context use. */
void* xp_context_stream(xp_context* ctx);
xp_status xp_context_device_name(xp_context* ctx, char* buf, size_t n);
xp_status xp_context_wait_idle(xp_context* ctx);

/* ctx.alloc<T>(n, Usage) (include/vulkore/context.hpp:55-60). HOST_VISIBLE is
 * pinned, mapped host memory; the returned pointer is its device alias and
 * *host_ptr (if non-null) the host view. */
xp_status xp_alloc(xp_context* ctx, size_t bytes, xp_usage usage, void** dptr, void** host_ptr);
xp_status xp_free(xp_context* ctx, void* dptr);
/* Buffer::upload/download (include/vulkore/buffer.hpp:83-92); synchronous. */
xp_status xp_upload(xp_context* ctx, void* dst, size_t dst_offset, const void* src, size_t bytes);
xp_status xp_download(xp_context* ctx, void* dst, const void* src, size_t src_offset, size_t bytes);

/* ---- kernel registry (include/vulkore/program.hpp:96-110) -------------------
 * Kernels are looked up by (module path, entry-point name). Module paths are
 * the reference's: "kernels/llm_matvec.spv", "kernels/llm_transformer.spv",
 * "kernels/llm_sampling.spv" (a bare file name also matches). An unknown name
 * returns XP_ERR_NO_KERNEL and the message lists the module's kernels. */
typedef int32_t xp_kernel;
xp_status xp_kernel_lookup(const char* module, const char* name, xp_kernel* out);
xp_status xp_kernel_info(xp_kernel k, const char** module, const char** name, uint32_t* nargs);
/* argument i: kind 1 = buffer (device pointer), 0 = POD of `size` bytes */
xp_status xp_kernel_arg(xp_kernel k, uint32_t i, int* kind, uint32_t* size, const char** arg_name);
int xp_kernel_count(void);

typedef struct xp_grid { uint32_t x, y, z; } xp_grid; /* GLOBAL thread counts */
typedef struct xp_arg {
    const void* ptr;  /* kind 1: the device pointer VALUE; kind 0: address of the POD */
    uint32_t size;    /* POD byte size (ignored for buffers) */
    int32_t kind;     /* 1 buffer, 0 POD */
} xp_arg;

/* vulkore::launch (include/vulkore/launch.hpp:148-160): validate the arguments
 * against the kernel's signature, then enqueue it on `stream`. */
xp_status xp_launch(xp_kernel k, xp_grid grid, const xp_arg* args, uint32_t nargs, void* stream);

/* ---- Batch / Fence (include/vulkore/launch.hpp:165-213, sync.hpp:15-50) ----
 * A Batch records launches; submit() captures them into one CUDA graph (the
 * counterpart of one vkQueueSubmit), instantiates it, or updates the cached
 * executable graph in place when the node list matches, and launches it. */
typedef struct xp_batch xp_batch;
typedef struct xp_fence xp_fence;
xp_status xp_batch_create(xp_context* ctx, xp_batch** out);
xp_status xp_batch_add(xp_batch* b, xp_kernel k, xp_grid grid, const xp_arg* args, uint32_t nargs);
xp_status xp_batch_size(xp_batch* b, uint32_t* n);
xp_status xp_batch_submit(xp_batch* b, xp_fence** out);  /* the Batch is spent afterwards */
xp_status xp_batch_destroy(xp_batch* b);
/* A fence signaled once everything enqueued on the context's stream so far
 * has completed (vulkore::launch returns one, include/vulkore/launch.hpp:148). */
xp_status xp_context_fence(xp_context* ctx, xp_fence** out);
/* XP_OK when signaled, XP_TIMEOUT on timeout, XP_ERR_DEVICE on a device error */
xp_status xp_fence_wait(xp_fence* f, uint64_t timeout_ns);
xp_status xp_fence_destroy(xp_fence* f);                  /* drains first */

/* ---- typed entry points, reference names and argument order --------------
 * Each replaces the same-named entry point of the cited .cl file; `grid` is
 * chosen by the library. Matvec convention (kernels/llm.cl:11-19): rows = K
 * inputs, cols = N outputs, out[j] = sum_k in[k] * W[k][j]. */
/* kernels/llm_matvec.cl:422-434 */
xp_status xp_mv_km4_bs(void* stream, float* out, const float* in, const uint32_t* wq, const uint32_t* sc,
                       uint32_t rows, uint32_t cols);
/* kernels/llm_matvec.cl:439-456 (partial[p*cols + j], split over quads) */
xp_status xp_mv_km4_bs_split(void* stream, float* partial, const float* in, const uint32_t* wq,
                             const uint32_t* sc, uint32_t rows, uint32_t cols, uint32_t split);
/* kernels/llm_matvec.cl:128-135 */
xp_status xp_mv_reduce(void* stream, float* out, const float* partial, uint32_t cols, uint32_t split);

/* ---- one matrix, many sequences, on the tensor cores ------------------------
 * out[s][j] = sum_k in[s][k] W[k][j] for s < n (<= 64): the skinny GEMM of
 * batched decode, each row the value kernels/llm_matvec.cl:422-434 computes for
 * that sequence (same planes; products of exact operands summed in fp32: when
 * every bf16 scale is 0 or within [2^-14, 8160] the dequantised weight itself
 * is the fp16 operand, otherwise the scale is applied in fp32 per 32-row
 * block; each call scans the scale plane on the stream to choose).
 * in is [n][rows], out [n][cols]; rows % 128 == 0, cols % 128 == 0. `scratch`
 * (256-byte aligned, xp_mv_km4_bs_batch_scratch_bytes) is caller-owned and
 * must be zero-initialised once (every call leaves it reusable; switching a
 * scratch to another shape costs one memset, so keep one per shape); its 32-bit
 * word at byte offset 256 is nonzero after a call whose tensor-core pipeline
 * wait ran out, and the word at byte offset 384 is 1 after a call that took
 * the per-block scale path. No counterpart entry in the reference (which
 * dispatches mv_km4_bs once per sequence). */
size_t xp_mv_km4_bs_batch_scratch_bytes(uint32_t rows, uint32_t cols, uint32_t n);
xp_status xp_mv_km4_bs_batch(void* stream, float* out, const float* in, const uint32_t* wq, const uint32_t* sc,
                             uint32_t rows, uint32_t cols, uint32_t n, void* scratch);

/* ---- many matvecs in one launch ---------------------------------------------
 * The reference submits a token's matvecs as mv_km4_bs dispatches recorded in
 * one Batch (examples/llm/decode.cpp:1634-1780, include/vulkore/launch.hpp:
 * 179-213); each job here computes exactly that kernel's output
 * (kernels/llm_matvec.cl:422-434) from the same planes, and a plan runs all of
 * its jobs in ONE persistent launch that streams the weights at HBM rate.
 * A plan owns device memory (job table, activation limbs); create it once, run
 * it any number of times on any stream of its device, destroy it last. Jobs
 * may share an input vector; outputs must not overlap. rows % 128 == 0,
 * cols % 64 == 0, at most 512 jobs. */
typedef struct xp_mv_job {
    float* out;              /* [cols] */
    const float* in;         /* [rows] */
    const uint32_t* wq;      /* nibble plane (uint4 per 32 rows x column) */
    const uint32_t* sc;      /* bf16 scale plane (uint2 per 128 rows x column) */
    uint32_t rows, cols;
} xp_mv_job;
typedef struct xp_mv_plan xp_mv_plan;
xp_status xp_mv_plan_create(const xp_mv_job* jobs, uint32_t n, xp_mv_plan** plan);
xp_status xp_mv_plan_run(xp_mv_plan* plan, void* stream);
/* algorithmic bytes one run reads and writes (nibbles + scales + in + out) */
xp_status xp_mv_plan_bytes(const xp_mv_plan* plan, uint64_t* bytes);
void xp_mv_plan_destroy(xp_mv_plan* plan);
/* kernels/llm_transformer.cl:96-116 */
xp_status xp_rmsnorm_sumsq(void* stream, float* partial, const float* in, uint32_t n, uint32_t nparts);
xp_status xp_rmsnorm_apply_gemma(void* stream, float* out, const float* in, const float* w,
                                 const float* partial, uint32_t n, uint32_t nparts, float eps);
/* kernels/llm_transformer.cl:122-134 */
xp_status xp_rmsnorm_heads_gemma(void* stream, float* out, const float* in, const float* w, uint32_t n_heads,
                                 uint32_t head_dim, float eps);
/* kernels/llm_transformer.cl:158-179 */
xp_status xp_rope(void* stream, float* x, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float theta);
/* kernels/llm_transformer.cl:223-231 */
xp_status xp_geglu(void* stream, float* out, const float* gate, const float* up, uint32_t n);
/* kernels/llm_transformer.cl:564-568 */
xp_status xp_add_residual(void* stream, float* x, const float* y, uint32_t n);
/* kernels/llm_transformer.cl:590-595 */
xp_status xp_kv_append(void* stream, float* cache, const float* src, uint32_t n, uint32_t pos);
/* kernels/llm_transformer.cl:287-305, :318-335, :478-497 */
xp_status xp_attention_scores(void* stream, float* scores, const float* q, const float* kcache, uint32_t n_heads,
                              uint32_t kv_heads, uint32_t head_dim, uint32_t span, float scale,
                              uint32_t kv_start);
xp_status xp_softmax_rows(void* stream, float* x, uint32_t n_rows, uint32_t n_cols);
xp_status xp_attention_apply(void* stream, float* out, const float* probs, const float* vcache, uint32_t n_heads,
                             uint32_t kv_heads, uint32_t head_dim, uint32_t span, uint32_t kv_start);
/* kernels/llm_sampling.cl:57-123 (three-level argmax; out[0] = index as float,
 * out[1] = value; ties -> lowest index) */
xp_status xp_argmax(void* stream, float* out, uint32_t* idx_out, const float* logits, uint32_t n);
/* kernels/llm_sampling.cl:318-347 */
xp_status xp_topk4_partial(void* stream, float* cval, uint32_t* cidx, const float* x, uint32_t n,
                           uint32_t nparts);

/* ---- fused B200 kernels (no single reference counterpart) -----------------
 * Fused split-K flash-decode attention over an fp16 KV cache for one position
 * (replaces rmsnorm_heads_gemma x2, rope x2, kv_append x2, attention_scores,
 * softmax_rows, attention_apply: examples/llm/decode.cpp:1676-1731). n_heads
 * must be 4, kv_heads 1, head_dim 256 (Gemma-3-1B). `pos` is a DEVICE
 * pointer. `max_seq` is the rows each cache holds (the splits are sized for
 * the window when `window` is non-zero and smaller, else for max_seq).
 * `scratch` needs xp_attention_scratch_bytes(nsplit) bytes and must
 * be zero-initialised once (the kernel leaves it reusable). The uint32 at
 * byte 4 of `scratch` is the call's error word (sticky: bits are only ORed
 * in): 1 = the split count was too small for max_seq (a prefix was attended),
 * 4 = a bulk-copy wait ran out, 128 = *pos_dev >= max_seq (nothing was
 * written: the KV append would have landed past the caches). */
size_t xp_attention_scratch_bytes(uint32_t nsplit);
xp_status xp_attention_decode(void* stream, float* out, const float* q_raw, const float* k_raw,
                              const float* v_raw, const float* q_norm, const float* k_norm, uint16_t* kcache_f16,
                              uint16_t* vcache_f16, const uint32_t* pos_dev, uint32_t window, float theta,
                              float eps, float scale, uint32_t nsplit, uint32_t max_seq, void* scratch);
/* xp_attention_decode for callers that cannot allocate device memory (a host
 * framework's arena they do not own, a memory-capped plugin, a path that must
 * not call cudaMalloc): same arguments minus `scratch`, which lives instead in
 * a fixed array inside the library (XP_ATTN_STATIC_SCRATCH_BYTES, enough for
 * nsplit <= XP_ATTN_STATIC_MAX_NSPLIT, held on every GPU that loads the
 * library until exit). Larger nsplit returns XP_ERR_INVALID. Runs on the
 * current device; the first call on a device looks up the array's address, so
 * make that first call before any stream capture. All calls share the one
 * array: calls that overlap on the GPU race. Allocates nothing. No counterpart
 * in the reference. Every argument check runs before the array is touched.
 * A device reset (cudaDeviceReset) invalidates the cached address: do not use
 * this entry point on a device after resetting it. */
#define XP_ATTN_STATIC_MAX_NSPLIT 64u
#define XP_ATTN_STATIC_SCRATCH_BYTES (512u + 64u * (4u * 256u * 4u + 8u * 4u))
xp_status xp_attention_decode_static(void* stream, float* out, const float* q_raw, const float* k_raw,
                                     const float* v_raw, const float* q_norm, const float* k_norm,
                                     uint16_t* kcache_f16, uint16_t* vcache_f16, const uint32_t* pos_dev,
                                     uint32_t window, float theta, float eps, float scale, uint32_t nsplit,
                                     uint32_t max_seq);
/* The error word of the array xp_attention_decode_static uses (same bits as
 * xp_attention_decode's), copied to host `*word` after the work already on
 * `stream`; cleared afterwards when `clear` is non-zero. Synchronises
 * `stream`. Allocates nothing. No counterpart in the reference. */
xp_status xp_attention_static_error_word(void* stream, uint32_t* word, int clear);
/* Exact top-k (k <= 64) + temperature + top-p + multinomial over n logits
 * (replaces topk4_partial + host draw(), decode.cpp:1873-1917). `u` index for
 * the seeded uniform is *pos_dev. Writes the chosen id to *token_dev and the
 * k survivors (descending) to out_vals/out_idx when non-null. */
size_t xp_sample_scratch_bytes(uint32_t n);
xp_status xp_sample_topk(void* stream, uint32_t* token_dev, float* out_vals, uint32_t* out_idx,
                         const float* logits, uint32_t n, uint32_t top_k, float temperature, float top_p,
                         uint64_t seed, uint64_t seq_id, const uint32_t* pos_dev, void* scratch);

/* ---- load path -------------------------------------------------------------- */
/* Device twin of the reference packer (examples/llm/decode.cpp:101-229): fp32
 * weights [cols][rows] (GGUF order) -> KM4 nibble plane (cols*rows/2 bytes)
 * and bf16 scale plane (cols*rows/16 bytes). Bit-exact with the host packer.
 * rows % 128 == 0, cols % 64 == 0. */
xp_status xp_pack_km4bf16(void* stream, const float* w, uint32_t rows, uint32_t cols, uint32_t* words,
                          uint32_t* scales);
/* Seeded synthetic N(0, sigma) (Irwin-Hall(12)), identical to the test oracle. */
xp_status xp_gen_normal(void* stream, float* out, uint64_t n, uint64_t offset, uint64_t seed, uint64_t stream_id,
                        float sigma);
/* Bandwidth probe with the reference's stream4 contract (llm_matvec.cl:370-378). */
xp_status xp_stream4(void* stream, float* out, const void* src, uint32_t n_uint4, uint32_t threads);

/* ---- decode session (examples/llm/decode.hpp:605-676) ----------------------- */
typedef struct xp_session xp_session;

typedef struct xp_model_config {
    uint32_t n_layers, hidden, ffn, n_heads, n_kv_heads, head_dim, vocab;
    uint32_t max_seq;          /* KV capacity in positions */
    uint32_t sliding_window;   /* 512 for Gemma 3 */
    uint32_t global_every;     /* layer i is global iff (i+1) % global_every == 0 */
    float rms_eps, rope_theta_global, rope_theta_local;
    float embed_scale;         /* 0 -> sqrt(hidden) */
    float attn_scale;          /* 0 -> 1/sqrt(head_dim) */
} xp_model_config;

typedef struct xp_sampling {
    int greedy;               /* 1: argmax (SampleMode::Greedy); 0: temperature/top-k/top-p */
    float temperature;
    uint32_t top_k;           /* <= 64 on the device sampler; 0 -> 64 */
    float top_p;
    uint64_t seed;
    uint64_t seq_id;          /* stream id of this sequence's uniforms */
} xp_sampling;

/* Random-init weights generated and packed on the device: every fp32 master
 * tensor is N(0, 0.02) from the seeded generator with a fixed stream id per
 * tensor (see xp_session_tensor_stream), norm weights N(0, 0.02) offsets, the
 * LM head tied to the embedding. */
xp_status xp_session_create_random(int device, const xp_model_config* cfg, const xp_sampling* sp, uint64_t seed,
                                   xp_session** out);
/* Host-provided weights: every pointer is HOST memory; packed planes in the
 * reference layout, fp32 norm offsets, fp32 embedding [vocab][hidden].
 * Per layer: wq,wk,wv,wo,gate,up,down words then scales. */
typedef struct xp_layer_weights {
    const uint32_t* words[7];
    const uint32_t* scales[7];
    const float* attn_norm;
    const float* post_attn_norm;
    const float* ffn_norm;
    const float* post_ffn_norm;
    const float* q_norm;
    const float* k_norm;
} xp_layer_weights;
xp_status xp_session_create(int device, const xp_model_config* cfg, const xp_sampling* sp,
                            const xp_layer_weights* layers, const uint32_t* lm_words, const uint32_t* lm_scales,
                            const float* final_norm, const float* embed, xp_session** out);
/* A session from a GGUF model file: the reference's real-weight load path
 * (examples/llm/decode.cpp:1418-1535, DecodeSession::DecodeSession). Shapes
 * come from the file's metadata (DecodeConfig::from_model, decode.cpp:258-275);
 * `policy` (may be NULL) supplies max_seq, global_every, sliding_window (if
 * non-zero), rope_theta_local (if > 0), embed_scale and attn_scale. Tensors of
 * ggml types F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K and Q6_K are
 * dequantised on the device and packed to KM4 + bf16 (bit-exact with the
 * reference packer); norm weights are stored as (1 + w) and loaded as w; the
 * output head is token_embd unless the file has output.weight. `pack_cache`:
 * NULL = "<gguf_path>.xpack", "" = no cache, else a path. A valid cache
 * (the reference's .xpack format, decode.cpp:711-1328, same validation rules)
 * is loaded instead of packing; otherwise the planes are packed and the cache
 * is written through "<cache>.tmp" + rename. */
xp_status xp_session_create_gguf(int device, const char* gguf_path, const xp_model_config* policy,
                                 const xp_sampling* sp, const char* pack_cache, xp_session** out);
/* How a GGUF session's weights were loaded: from the cache, whether a cache
 * was written, and a one-line description (truncated to msg_bytes). */
xp_status xp_session_load_info(xp_session* s, int* from_cache, int* cache_written, char* msg, uint32_t msg_bytes);
/* The session's effective model configuration. */
xp_status xp_session_config(xp_session* s, xp_model_config* cfg);
/* Dequantise n elements of a ggml block type on the device (src, dst device
 * pointers): examples/llm/model/gguf.cpp:448-634 GGUFFile::dequantize, bit-exact.
 * Types as for xp_session_create_gguf. */
xp_status xp_gguf_dequantize(void* stream, uint32_t ggml_type, const void* src, float* dst, uint64_t n);
/* Element counts of the planes examples/llm/quant_repack.cpp repack() makes
 * for a rows x cols tensor of ggml type Q8_0 (8), Q5_0 (6), Q4_K (12) or
 * Q6_K (14): sizes[0] quant words, [1] high words, [2] fp32 scales,
 * [3] fp32 biases (0 where the type has no such plane). XP_ERR_INVALID for
 * another type, cols not a multiple of 32 (256 for the K types) or rows 0. */
xp_status xp_quant_repack_sizes(uint32_t ggml_type, uint32_t rows, uint32_t cols, uint64_t* sizes);
/* That repack on the device (every pointer a device pointer): native GGUF
 * blocks -> the interleaved planes the kernels/llm_quant.spv matvec_rq*
 * entries read, bit-identical to the host repack (quant_repack.cpp:130-210),
 * padding rows written as zeros. `quant` 16-byte aligned; `high` and `bias`
 * may be NULL for types without them. */
xp_status xp_quant_repack(void* stream, uint32_t ggml_type, const void* src, uint32_t rows, uint32_t cols,
                          uint32_t* quant, uint32_t* high, float* scale, float* bias);
/* ---- tokenizer (examples/llm/model/tokenizer.{hpp,cpp}) --------------------
 * The SentencePiece vocabulary of a GGUF file (tokenizer.ggml.*): encode with
 * CONTROL/UNKNOWN tokens cut out first, the leading space marker, best-score
 * merges (ties: leftmost) and byte fallback; decode with special tokens
 * optionally skipped and one leading space dropped. Host only (no GPU).
 * Encode/decode/piece: pass a NULL buffer to get the size first. */
typedef struct xp_tokenizer xp_tokenizer;
xp_status xp_tokenizer_create(const char* gguf_path, xp_tokenizer** out);   /* Tokenizer::from_gguf */
void xp_tokenizer_destroy(xp_tokenizer* t);
xp_status xp_tokenizer_info(const xp_tokenizer* t, uint32_t* vocab, int32_t* bos, int32_t* eos, int32_t* unk,
                            int32_t* pad);
xp_status xp_tokenizer_encode(const xp_tokenizer* t, const char* text, size_t len, int add_bos, int add_eos,
                              int32_t* ids, uint32_t cap, uint32_t* n);   /* Tokenizer::encode */
xp_status xp_tokenizer_decode(const xp_tokenizer* t, const int32_t* ids, uint32_t n, int skip_special, char* out,
                              size_t cap, size_t* len);                    /* Tokenizer::decode */
xp_status xp_tokenizer_piece(const xp_tokenizer* t, int32_t id, char* out, size_t cap, size_t* len); /* decode_one */

/* ---- chat front-end (android/app/src/main/cpp/llm_jni.cpp:59-186) ---------
 * create: a GGUF session + its tokenizer; sampling NULL = temperature 0.7,
 * top-k 64, top-p 0.95, seed 1234. prefill: `text` in the Gemma turn template
 * ("<start_of_turn>user\n...<end_of_turn>\n<start_of_turn>model\n", a "\n"
 * before later turns), BOS on the first turn only. step: one token's text, or
 * *done = 1 at <end_of_turn>, EOS or a full KV cache. metrics: {ms, tok/s,
 * kernels, submits, position, record_ms, gpu_ms} of the last step. */
typedef struct xp_chat xp_chat;
xp_status xp_chat_create(int device, const char* gguf_path, uint32_t max_seq, const xp_sampling* sp,
                         const char* pack_cache, xp_chat** out);
xp_status xp_chat_prefill(xp_chat* c, const char* text, uint32_t* n_tokens);
xp_status xp_chat_step(xp_chat* c, char* piece, size_t cap, int* done);
xp_status xp_chat_metrics(const xp_chat* c, double out[7]);
xp_status xp_chat_session(xp_chat* c, xp_session** s);
xp_status xp_chat_reset(xp_chat* c);
void xp_chat_destroy(xp_chat* c);
xp_status xp_session_destroy(xp_session* s);
/* Stream id used for tensor (layer, which) by create_random; which: 0..6 the
 * matrices q,k,v,o,gate,up,down; 7..12 the norms; layer = n_layers: 0 embed,
 * 7 final norm. */
uint64_t xp_session_tensor_stream(uint32_t layer, uint32_t which);
/* DecodeSession::prefill (decode.cpp:1790-1817): logits only for the last
 * token. Tokens are host memory. Prompts of 32 or more tokens (environment
 * XP_PREFILL_CHUNK_MIN) run 64 positions per pass on the batched tensor-core
 * engine over the session's KV caches; shorter ones one pass per token. The
 * first chunked prefill of a session allocates that engine (~80 MB for the
 * Gemma-3-1B shape); if that fails the call falls back to one pass per token. */
xp_status xp_session_prefill(xp_session* s, const uint32_t* tokens, uint32_t n);
/* DecodeSession::decode_step (decode.cpp:1819-1866): sample from the
 * previous pass's logits, run the network on it, return the sampled id. */
xp_status xp_session_decode_step(xp_session* s, uint32_t* token);
/* Device-resident generation: n steps back to back with no host round trip
 * (the sampled token feeds the next step on the device); tokens (host) may be
 * NULL. Returns the device time in *ms if non-null. With greedy sampling on
 * one GPU the token kernel decodes up to 512 positions per launch. */
xp_status xp_session_generate(xp_session* s, uint32_t n, uint32_t* tokens, float* ms);
xp_status xp_session_reset(xp_session* s);            /* DecodeSession::reset */
xp_status xp_session_position(xp_session* s, uint32_t* pos);
xp_status xp_session_logits(xp_session* s, float* host_out, uint32_t n);  /* last_logits() */
/* Current token buffer (the next input) and per-kernel counts. */
xp_status xp_session_stats(xp_session* s, uint32_t* kernels_per_token, uint64_t* weight_bytes);
/* Device pointers of internal buffers, for tests: name in {"x","logits","kcache0",...} */
xp_status xp_session_debug_ptr(xp_session* s, const char* name, void** dptr, size_t* bytes);
/* Roofline probe of the dominant kernel: replays a graph holding only the
 * token's int4 matvecs (same kernels and launch shapes as the decode graph)
 * `iters` times back to back and reports device ms, algorithmic bytes
 * (nibbles + scales + activations) and launches per token. */
xp_status xp_session_profile_matvec(xp_session* s, uint32_t iters, float* ms_per_token, uint64_t* bytes_per_token,
                                    uint32_t* launches_per_token);
/* Phase timeline of the last token (XP_TRACE=1 at session creation):
 * out[0] = barriers; out[1] = start ns; out[2k], out[2k+1] = barrier k
 * arrive / leave ns (CTA 0, %globaltimer); out[2*barriers+2] = end ns. */
xp_status xp_session_trace(xp_session* s, uint64_t* out, uint32_t n);

/* Failure path self-test: launches one thread whose mbarrier wait and
 * grid-barrier wait nothing satisfies, each bounded by `spin_limit` polls (the
 * kernels' own bound is 1 << 22), and returns the error bits they recorded in
 * *err_word (4 = mbarrier wait, 2 = grid barrier) with the context still
 * usable. No counterpart in the reference. */
xp_status xp_selftest_wait_timeout(uint32_t spin_limit, uint32_t* err_word);

/* ---- tensor-parallel LM head ------------------------------------------------
 * `world` processes (one GPU each, same weights, same tokens) split the LM
 * head's 262,144 rows evenly; each token kernel computes its rank's logits and
 * argmax, then writes its (value, index) into every rank's exchange buffer over
 * NVLink (CUDA IPC mappings) and takes the lowest-index maximum (the reference's
 * argmax rule, kernels/llm_sampling.cl:57-123) once all ranks' entries arrived
 * (bounded wait; error bit 32 on timeout). Greedy sampling only. Collective:
 * every rank calls xp_session_tp_handle, the handles (64 bytes each, rank
 * order) are exchanged on the host, then every rank calls
 * xp_session_tp_attach before its next decode. No counterpart in the
 * reference, which runs on one device. */
xp_status xp_session_tp_handle(xp_session* s, void* handle64);
xp_status xp_session_tp_attach(xp_session* s, uint32_t rank, uint32_t world, const void* handles);
/* As xp_session_tp_attach; flags: XP_TP_SHARD_FFN also splits the FFN over
 * the ranks (gate|up columns and the matching down-proj rows; the down-proj
 * sums are exchanged between the ranks inside every launch in int64). Its
 * token kernel fixes each 16-row down-proj unit's partial sum separately, so
 * logits are bit-identical for every world size, including one rank attached
 * with this flag (the single-GPU default kernel groups units per CTA before
 * fixing: the same tokens, logits equal to fp32 rounding). Greedy only. */
#define XP_TP_SHARD_FFN 1u
xp_status xp_session_tp_attach_ex(xp_session* s, uint32_t rank, uint32_t world, const void* handles, uint32_t flags);

/* ---- batched decode ---------------------------------------------------------
 * nseq (<= 64) independent sequences advance one position together over the
 * weights of session `s` (which must outlive the batch): per step every int4
 * matvec is one tensor-core launch for all sequences (xp_mv_km4_bs_batch), the
 * per-sequence norms, RoPE, fp16 KV append and attention run one CTA per
 * sequence, and sampling is the batch-1 sampler per sequence with the uniform
 * keyed (seed, seq0 + sequence, position). Each sequence computes what a
 * DecodeSession (examples/llm/decode.cpp:1790-1866) computes for it alone; the
 * reference has no batched engine. Calls follow its order: prefill feeds
 * tokens [n][nseq] (position-major) one position at a time; step samples the
 * previous pass's logits, returns those tokens and runs the network on them. */
typedef struct xp_bdec xp_bdec;
xp_status xp_bdec_create(xp_session* s, uint32_t nseq, uint32_t max_seq, const xp_sampling* sp, uint64_t seq0,
                         xp_bdec** out);
xp_status xp_bdec_prefill(xp_bdec* b, const uint32_t* tokens, uint32_t n);
xp_status xp_bdec_step(xp_bdec* b, uint32_t* tokens_out);
/* n steps on the device without reading tokens back; device time in ms */
xp_status xp_bdec_generate(xp_bdec* b, uint32_t n, float* ms);
xp_status xp_bdec_logits(xp_bdec* b, float* out, size_t n);
xp_status xp_bdec_position(xp_bdec* b, uint32_t* pos);
void xp_bdec_destroy(xp_bdec* b);
/* CUDA events on the session stream: stop = 0 records the start, 1 the end
 * and returns the elapsed device ms (brackets host-driven decode_step loops). */
xp_status xp_session_timer(xp_session* s, int stop, float* ms);
/* The device error word (bit 0: attention chunk overflow); cleared on read. */
xp_status xp_session_error_word(xp_session* s, uint32_t* word);

#ifdef __cplusplus
}
#endif
#endif
