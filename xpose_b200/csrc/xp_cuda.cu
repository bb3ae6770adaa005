// Single translation unit of libxp_cuda.so (kernels are defined in headers).
#include "capi.cuh"
#include "engine.cuh"

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
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_attn_static_scratch[XP_ATTN_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
void* g_attn_static_ptr[kMaxDevices] = {};  // device address of the array, per device
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
    int dev = 0;
    XP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(XP_ERR_NO_DEVICE, "xp_attention_decode_static: device %d", dev);
    if (!g_attn_static_ptr[dev]) {
        // first call on this device (the device is current): resolve the
        // array's device address once
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
        if (e != cudaSuccess)
            return fail(XP_ERR_CUDA, "xp_attention_decode_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_attn_static_ptr[dev] = p;
    }
    void* scratch = g_attn_static_ptr[dev];
    // the combine tickets and the error word start at zero for every call
    XP_CUDA_TRY(cudaMemsetAsync(scratch, 0, ATT_SCRATCH_HDR, (cudaStream_t)stream));
    return xp_attention_decode(stream, out, q_raw, k_raw, v_raw, q_norm, k_norm, kcache_f16, vcache_f16, pos_dev,
                               window, theta, eps, scale, nsplit, max_seq, scratch);
}
