// Shared device helpers for the sm_100a Gemma-3 decode path.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define XP_DEV __device__ __forceinline__

namespace xp {

// ---- programmatic dependent launch ---------------------------------------
// Every kernel of the decode graph is launched with programmatic stream
// serialization. A kernel may issue loads that do not depend on its producer
// (weights) before pdl_wait(); pdl_wait() returns once the producer grid has
// completed and its writes are visible. Every kernel calls pdl_wait() before
// it exits, so completion is transitive along the chain.
XP_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
XP_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- small numerics -------------------------------------------------------
XP_DEV float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
XP_DEV float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

XP_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
XP_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024). `red` holds 32
// floats of shared scratch. Every thread gets the same total, reduced in a
// fixed order (deterministic).
XP_DEV float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.0f;
    t = warp_sum(t);
    return t;
}

// Ordered float -> uint32 map: a > b (as floats, no NaN) iff key(a) > key(b).
XP_DEV uint32_t float_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
XP_DEV float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// tanh-approximate GELU with the clamped-exp tanh of the reference
// (kernels/llm_transformer.cl:213-231).
XP_DEV float gelu_tanh_ref(float g) {
    const float inner = 0.7978845608028654f * (g + 0.044715f * g * g * g);
    const float z = fminf(fmaxf(inner, -10.0f), 10.0f);
    const float e = expf(-2.0f * z);
    return 0.5f * g * (1.0f + (1.0f - e) / (1.0f + e));
}

}  // namespace xp
