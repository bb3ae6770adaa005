// Single translation unit of libxp_cuda.so (kernels are defined in headers).
#include "capi.cuh"
#include "engine.cuh"
#include "gguf_model.cuh"
#include "tokenizer.cuh"

// ---------------------------------------------------------------------------
// Attention without caller-provided scratch.
//
// Some callers cannot allocate device memory at all: code that runs under an
// allocator it does not own (a host framework's arena, a memory-capped
// plugin), or a latency path that must not touch cudaMalloc. For them,
// xp_attention_decode_static keeps its scratch (flash-decode partials, the
// combine ticket and the error word) in the file-scope array below instead of
// a `scratch` argument. The array is a fixed XP_ATTN_STATIC_MAX_NSPLIT splits
// in size and lives on every GPU that loads this library until the process
// exits. Every call shares it, so calls that overlap on the GPU race.
//
// Layout (the kernel's scratch layout): byte 0 the combine ticket (each
// launch leaves it at zero), byte 4 the error word (sticky: kernels only OR
// bits into it; xp_attention_static_error_word reads and clears it).
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_attn_static_scratch[XP_ATTN_STATIC_SCRATCH_BYTES];

namespace {
// Device address of the array, per device, looked up once with that device
// current (concurrent first calls store the same value). cudaDeviceReset
// destroys the context that owns the array, so a process that resets a device
// must not use these entry points on it afterwards.
std::atomic<void*> g_attn_static[kMaxDevices];

xp_status attn_static_scratch(const char* who, void** out) {
    int dev = 0;
    XP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(XP_ERR_NO_DEVICE, "%s: device %d", who, dev);
    void* p = g_attn_static[dev].load(std::memory_order_acquire);
    if (!p) {
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
        if (e != cudaSuccess) return fail(XP_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
        g_attn_static[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return XP_OK;
}
}  // namespace

extern "C" xp_status xp_attention_decode_static(void* stream, float* out, const float* q_raw, const float* k_raw,
                                                const float* v_raw, const float* q_norm, const float* k_norm,
                                                uint16_t* kcache_f16, uint16_t* vcache_f16, const uint32_t* pos_dev,
                                                uint32_t window, float theta, float eps, float scale,
                                                uint32_t nsplit, uint32_t max_seq) {
    if (nsplit == 0 || nsplit > XP_ATTN_STATIC_MAX_NSPLIT)
        return fail(XP_ERR_INVALID, "xp_attention_decode_static: nsplit %u is outside 1..%u (the fixed scratch)",
                    nsplit, (unsigned)XP_ATTN_STATIC_MAX_NSPLIT);
    static_assert(XP_ATTN_STATIC_SCRATCH_BYTES >= attn_scratch_bytes(XP_ATTN_STATIC_MAX_NSPLIT),
                  "static scratch smaller than the largest split count needs");
    void* scratch = nullptr;
    if (xp_status s = attn_static_scratch("xp_attention_decode_static", &scratch); s != XP_OK) return s;
    // every check that could refuse the call runs before the shared array is touched
    if (xp_status s = attn_validate(out, q_raw, k_raw, v_raw, q_norm, k_norm, kcache_f16, vcache_f16, pos_dev,
                                    window, nsplit, max_seq, scratch);
        s != XP_OK)
        return s;
    // the combine ticket must start at zero (each launch leaves it so; this
    // covers a launch that never ran to its end). The error word is kept.
    XP_CUDA_TRY(cudaMemsetAsync(scratch, 0, 4, (cudaStream_t)stream));
    return xp_attention_decode(stream, out, q_raw, k_raw, v_raw, q_norm, k_norm, kcache_f16, vcache_f16, pos_dev,
                               window, theta, eps, scale, nsplit, max_seq, scratch);
}

extern "C" xp_status xp_attention_static_error_word(void* stream, uint32_t* word, int clear) {
    if (!word) return fail(XP_ERR_INVALID, "xp_attention_static_error_word: argument 'word' is null");
    void* scratch = nullptr;
    if (xp_status s = attn_static_scratch("xp_attention_static_error_word", &scratch); s != XP_OK) return s;
    uint32_t* err = static_cast<uint32_t*>(scratch) + 1;
    const cudaStream_t st = (cudaStream_t)stream;
    XP_CUDA_TRY(cudaMemcpyAsync(word, err, 4, cudaMemcpyDeviceToHost, st));
    if (clear) XP_CUDA_TRY(cudaMemsetAsync(err, 0, 4, st));
    XP_CUDA_TRY(cudaStreamSynchronize(st));
    return XP_OK;
}
