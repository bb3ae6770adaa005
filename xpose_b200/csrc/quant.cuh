// The reference's GGUF quant module (kernels/llm_quant.cl) on B200: fp16
// decode, per-element dequantisation of Q8_0 / Q5_0 / Q4_K / Q6_K blocks, the
// fused matvecs over those native block layouts, and the matvecs over the
// repacked planes of examples/llm/quant_repack.hpp (matvec_rq*, with split-K
// partials and their reduce).
//
// Same entry points, arguments and output contract as the reference; the
// work decomposition is this file's own:
//   * fp16 decode and the dequant kernels are per element and bit-exact (the
//     same products in the same order, no contraction, through the ggml
//     element decoder the GGUF loader uses; fp16_decode through integer bit
//     surgery so every NaN payload and subnormal decodes as the reference
//     does, llm_quant.cl:52-86);
//   * native-layout matvecs (llm_quant.cl:101-341): one warp per output row,
//     lanes over the row's 32-weight (sub-)blocks, warp-reduced;
//   * repacked matvecs (llm_quant.cl:344-606): the planes are interleaved in
//     64-row groups, idx = (g * nkb + kb) * 64 + t, so a CTA takes one group
//     (64 rows) and four K slices (256 threads: a warp pair reads one
//     k-block of 64 consecutive rows, 1 KB contiguous) and adds the slices in
//     slice order through shared memory. Split-K launches add a grid axis per
//     split and write partial[p * rows + r].
// Summation order differs from the reference's one-thread-per-row loop, so
// the matvecs agree within fp32 rounding (the reference's own harness bar is
// max |diff| / max |out| < 1e-5), not bit for bit.
#pragma once
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "runtime.cuh"

namespace xp {

// ---- ggml tensor types (block sizes are the ggml ABI) -------------------------
struct GgmlType {
    uint32_t id, block, bytes;
    const char* name;
};
inline const GgmlType* ggml_type(uint32_t id) {
    static const GgmlType t[] = {{0, 1, 4, "F32"},      {1, 1, 2, "F16"},      {30, 1, 2, "BF16"},
                                 {2, 32, 18, "Q4_0"},   {3, 32, 20, "Q4_1"},   {6, 32, 22, "Q5_0"},
                                 {7, 32, 24, "Q5_1"},   {8, 32, 34, "Q8_0"},   {12, 256, 144, "Q4_K"},
                                 {14, 256, 210, "Q6_K"}};
    for (const auto& e : t)
        if (e.id == id) return &e;
    return nullptr;
}

XP_DEV float gg_f16(const uint8_t* p) { return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8)))); }

// One element of a ggml block tensor (the formats of gguf.cpp:448-634).
// Products and sums are rounded one operation at a time (no contraction), as
// the host formula does, so the values are bit-identical to it.
XP_DEV float gg_elem(uint32_t type, const uint8_t* src, uint64_t i) {
    switch (type) {
        case 1: return gg_f16(src + 2 * i);
        case 30: return __uint_as_float((uint32_t)(src[2 * i] | (src[2 * i + 1] << 8)) << 16);
        case 8: {
            const uint8_t* b = src + (i / 32) * 34;
            return __fmul_rn((float)(int8_t)b[2 + i % 32], gg_f16(b));
        }
        case 2: case 3: {
            const uint32_t bs = type == 2 ? 18 : 20, j = i % 32;
            const uint8_t* b = src + (i / 32) * bs;
            const uint8_t q = b[(type == 2 ? 2 : 4) + (j & 15)];
            const int v = j < 16 ? (q & 0xF) : (q >> 4);
            if (type == 2) return __fmul_rn((float)(v - 8), gg_f16(b));
            return __fadd_rn(__fmul_rn((float)v, gg_f16(b)), gg_f16(b + 2));
        }
        case 6: case 7: {
            const bool one = type == 7;
            const uint32_t j = i % 32, jj = j & 15;
            const uint8_t* b = src + (i / 32) * (one ? 24 : 22);
            const uint8_t* h = b + (one ? 4 : 2);
            const uint32_t qh = h[0] | (h[1] << 8) | (h[2] << 16) | ((uint32_t)h[3] << 24);
            const uint8_t q = b[(one ? 8 : 6) + jj];
            const int v = j < 16 ? ((q & 0xF) | (int)(((qh >> jj) << 4) & 0x10))
                                 : ((q >> 4) | (int)((qh >> (jj + 12)) & 0x10));
            if (!one) return __fmul_rn((float)(v - 16), gg_f16(b));
            return __fadd_rn(__fmul_rn((float)v, gg_f16(b)), gg_f16(b + 2));
        }
        case 12: {
            const uint8_t* b = src + (i / 256) * 144;
            const uint32_t e = i % 256, c = e / 64, w = e % 64, is = 2 * c + (w >= 32), l = w % 32;
            const uint8_t* sc = b + 4;
            uint32_t s, m;  // the 6-bit scale and min of sub-block `is`
            if (is < 4) {
                s = sc[is] & 63;
                m = sc[is + 4] & 63;
            } else {
                s = (sc[is + 4] & 0xF) | ((sc[is - 4] >> 6) << 4);
                m = (sc[is + 4] >> 4) | ((sc[is] >> 6) << 4);
            }
            const uint8_t qb = b[16 + 32 * c + l];
            const float q = (float)(w < 32 ? (qb & 0xF) : (qb >> 4));
            return __fsub_rn(__fmul_rn(__fmul_rn(gg_f16(b), (float)s), q), __fmul_rn(gg_f16(b + 2), (float)m));
        }
        case 14: {
            const uint8_t* b = src + (i / 256) * 210;
            const uint32_t e = i % 256, h = e / 128, r = e % 128, g = r / 32, l = r % 32;
            const uint8_t lo = b[64 * h + l + ((g & 1) ? 32 : 0)];
            const uint32_t nib = g < 2 ? (lo & 0xF) : (lo >> 4);
            const int q = (int)(nib | (((b[128 + 32 * h + l] >> (2 * g)) & 3) << 4)) - 32;
            const int8_t s = (int8_t)b[192 + 8 * h + l / 16 + 2 * g];
            return __fmul_rn(__fmul_rn(gg_f16(b + 208), (float)s), (float)q);
        }
        default: return __int_as_float(((const int*)src)[i]);  // F32
    }
}

__global__ void gguf_dequant_kernel(uint32_t type, const uint8_t* src, float* dst, uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        dst[i] = gg_elem(type, src, i);
}

inline cudaError_t gguf_dequant(cudaStream_t st, uint32_t type, const void* src, float* dst, uint64_t n) {
    const uint64_t blocks = std::min<uint64_t>((n + 255) / 256, (uint64_t)sm_count() * 16);
    gguf_dequant_kernel<<<(unsigned)std::max<uint64_t>(blocks, 1), 256, 0, st>>>(
        type, static_cast<const uint8_t*>(src), dst, n);
    return cudaGetLastError();
}

namespace quant {

// IEEE binary16 bit pattern -> binary32, exact for all 65536 patterns
// (signed zeros, subnormals, infinities, NaN payloads).
XP_DEV float f16_bits(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0u) {
        if (m == 0u) {
            bits = sign;
        } else {
            // m * 2^-24 with its top bit at position p: 1.f * 2^(p - 24)
            const uint32_t p = 31u - (uint32_t)__clz(m);
            bits = sign | ((p + 103u) << 23) | ((m << (23u - p)) & 0x7FFFFFu);
        }
    } else if (e == 31u) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    return __uint_as_float(bits);
}
XP_DEV uint32_t rd_u8(const uint8_t* p) { return __ldg(p); }
XP_DEV uint32_t rd_u16(const uint8_t* p) { return rd_u8(p) | (rd_u8(p + 1) << 8); }
XP_DEV float rd_f16(const uint8_t* p) { return f16_bits(rd_u16(p)); }

__global__ void fp16_decode(float* out, const uint32_t* src, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = rd_f16(reinterpret_cast<const uint8_t*>(src) + 2u * i);
}

XP_DEV float warp_total(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---- native block layouts: one warp per output row ------------------------------
// Q8_0: 34 B blocks (fp16 d, 32 x int8), w = d * q.
// Q5_0: 22 B blocks (fp16 d, u32 of 5th bits, 16 B of nibbles: byte j holds
//       weights j and j + 16), w = d * (q - 16).
template <bool Q8>
__global__ void matvec_q32(float* out, const float* x, const uint32_t* wq, uint32_t rows, uint32_t cols) {
    const uint32_t lane = threadIdx.x & 31, r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (r >= rows) return;
    constexpr uint32_t BS = Q8 ? 34u : 22u;
    const uint32_t nblk = cols >> 5;
    const uint8_t* row = reinterpret_cast<const uint8_t*>(wq) + (size_t)r * nblk * BS;
    float acc = 0.0f;
    for (uint32_t b = lane; b < nblk; b += 32) {
        const uint8_t* blk = row + (size_t)b * BS;
        const float* xb = x + (size_t)b * 32;
        float s = 0.0f;
        if (Q8) {
#pragma unroll 8
            for (uint32_t l = 0; l < 32; ++l) s = fmaf(__ldg(xb + l), (float)(int8_t)rd_u8(blk + 2 + l), s);
        } else {
            const uint32_t qh = rd_u8(blk + 2) | (rd_u8(blk + 3) << 8) | (rd_u8(blk + 4) << 16) | (rd_u8(blk + 5) << 24);
#pragma unroll 4
            for (uint32_t l = 0; l < 16; ++l) {
                const uint32_t byte = rd_u8(blk + 6 + l);
                const int q0 = (int)((byte & 0xFu) | (((qh >> l) & 1u) << 4)) - 16;
                const int q1 = (int)((byte >> 4) | (((qh >> (l + 16)) & 1u) << 4)) - 16;
                s = fmaf(__ldg(xb + l), (float)q0, s);
                s = fmaf(__ldg(xb + l + 16), (float)q1, s);
            }
        }
        acc = fmaf(rd_f16(blk), s, acc);
    }
    acc = warp_total(acc);
    if (lane == 0) out[r] = acc;
}

// Q4_K: 144 B super-blocks of 256 (fp16 d, fp16 dmin, 12 B of six-bit
// scale / min pairs, 128 B of nibbles: sub-block s uses byte (s/2)*32 + l,
// high nibble for odd s), w = d sc q - dmin mn. A lane takes one sub-block.
XP_DEV void q4k_scale_min(const uint8_t* s, uint32_t j, uint32_t& d, uint32_t& m) {
    if (j < 4) {
        d = rd_u8(s + j) & 63u;
        m = rd_u8(s + j + 4) & 63u;
    } else {
        d = (rd_u8(s + j + 4) & 0xFu) | ((rd_u8(s + j - 4) >> 6) << 4);
        m = (rd_u8(s + j + 4) >> 4) | ((rd_u8(s + j) >> 6) << 4);
    }
}
__global__ void matvec_q4_k(float* out, const float* x, const uint32_t* wq, uint32_t rows, uint32_t cols) {
    const uint32_t lane = threadIdx.x & 31, r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const uint32_t nsb = cols >> 8;
    const uint8_t* row = reinterpret_cast<const uint8_t*>(wq) + (size_t)r * nsb * 144;
    float acc = 0.0f;
    for (uint32_t u = lane; u < nsb * 8; u += 32) {
        const uint32_t sb = u >> 3, s = u & 7;
        const uint8_t* blk = row + (size_t)sb * 144;
        uint32_t sc, mn;
        q4k_scale_min(blk + 4, s, sc, mn);
        const uint8_t* qs = blk + 16 + (s >> 1) * 32;
        const uint32_t sh = (s & 1) ? 4u : 0u;
        const float* xb = x + (size_t)sb * 256 + s * 32;
        float sq = 0.0f, sx = 0.0f;
#pragma unroll 8
        for (uint32_t l = 0; l < 32; ++l) {
            const float xv = __ldg(xb + l);
            sq = fmaf(xv, (float)((rd_u8(qs + l) >> sh) & 0xFu), sq);
            sx += xv;
        }
        acc += rd_f16(blk) * (float)sc * sq - rd_f16(blk + 2) * (float)mn * sx;
    }
    acc = warp_total(acc);
    if (lane == 0) out[r] = acc;
}

// Q6_K: 210 B super-blocks of 256 (128 B low nibbles, 64 B of 2-bit highs,
// 16 int8 group scales, fp16 d), w = d sc (q - 32). Element 128 h + 32 g + l
// takes the low (g < 2) or high nibble of ql[64 h + l + 32 (g & 1)], bits
// 2g..2g+1 of qh[32 h + l] and scale sc[8 h + l / 16 + 2 g]. A lane takes one
// (h, g) quarter of 32.
__global__ void matvec_q6_k(float* out, const float* x, const uint32_t* wq, uint32_t rows, uint32_t cols) {
    const uint32_t lane = threadIdx.x & 31, r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const uint32_t nsb = cols >> 8;
    const uint8_t* row = reinterpret_cast<const uint8_t*>(wq) + (size_t)r * nsb * 210;
    float acc = 0.0f;
    for (uint32_t u = lane; u < nsb * 8; u += 32) {
        const uint32_t sb = u >> 3, h = (u >> 2) & 1, g = u & 3;
        const uint8_t* blk = row + (size_t)sb * 210;
        const uint8_t* ql = blk + h * 64 + (g & 1) * 32;
        const uint8_t* qh = blk + 128 + h * 32;
        const uint32_t lsh = g < 2 ? 0u : 4u;
        const float* xb = x + (size_t)sb * 256 + h * 128 + g * 32;
        float s16[2] = {0.0f, 0.0f};
#pragma unroll
        for (uint32_t half = 0; half < 2; ++half) {
            float s = 0.0f;
#pragma unroll 8
            for (uint32_t l = half * 16; l < half * 16 + 16; ++l) {
                const int q = (int)(((rd_u8(ql + l) >> lsh) & 0xFu) | (((rd_u8(qh + l) >> (2 * g)) & 3u) << 4)) - 32;
                s = fmaf(__ldg(xb + l), (float)q, s);
            }
            s16[half] = s * (float)(int8_t)rd_u8(blk + 192 + h * 8 + half + 2 * g);
        }
        acc = fmaf(rd_f16(blk + 208), s16[0] + s16[1], acc);
    }
    acc = warp_total(acc);
    if (lane == 0) out[r] = acc;
}

// ---- repacked planes (examples/llm/quant_repack.hpp) ---------------------------
// quant: uint4 per idx, component c holds k 8c..8c+7 at shift 4 (k % 8)
//        (Q8_0: two uint4, byte k at shift 8 (k % 4) of word k / 4);
// high:  Q5_0 one uint per idx (bit k), Q6_K two (field k at shift 2 (k % 16)
//        of word k / 16); scale: fp32 per idx (Q6_K two, per 16); bias: Q4_K.
constexpr int RQ4K = 0, RQ50 = 1, RQ6K = 2, RQ80 = 3;
struct RqArgs {
    float* out;            // [rows] or partial [split][rows]
    const float4* x;       // [cols / 4]
    const uint4* q;
    const uint32_t* hi;
    const float* scale;
    const float* bias;
    uint32_t rows, cols, split;
};

XP_DEV float nib(uint32_t w, uint32_t i) { return (float)((w >> (4 * i)) & 0xFu); }

template <int F>
XP_DEV float rq_block(const RqArgs& a, size_t idx, uint32_t kb) {
    const float4* xb = a.x + (size_t)kb * 8;
    if (F == RQ80) {
        const uint4 w0 = __ldg(a.q + 2 * idx), w1 = __ldg(a.q + 2 * idx + 1);
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float sq = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float4 v = __ldg(xb + c);
            sq = fmaf((float)(int8_t)(w[c] & 0xFFu), v.x, sq);
            sq = fmaf((float)(int8_t)((w[c] >> 8) & 0xFFu), v.y, sq);
            sq = fmaf((float)(int8_t)((w[c] >> 16) & 0xFFu), v.z, sq);
            sq = fmaf((float)(int8_t)(w[c] >> 24), v.w, sq);
        }
        return __ldg(a.scale + idx) * sq;
    }
    const uint4 w4 = __ldg(a.q + idx);
    const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
    uint32_t h0 = 0, h1 = 0;
    if (F == RQ50) h0 = __ldg(a.hi + idx);
    if (F == RQ6K) { h0 = __ldg(a.hi + 2 * idx); h1 = __ldg(a.hi + 2 * idx + 1); }
    float sq[2] = {0.0f, 0.0f}, sx = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float4 va = __ldg(xb + 2 * c), vb = __ldg(xb + 2 * c + 1);
        const float xv[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t k = 8 * c + i;
            float q;
            if (F == RQ4K) q = nib(w[c], i);
            else if (F == RQ50) q = (float)((int)(((w[c] >> (4 * i)) & 0xFu) | (((h0 >> k) & 1u) << 4)) - 16);
            else {
                const uint32_t hh = k < 16 ? h0 : h1;
                q = (float)((int)(((w[c] >> (4 * i)) & 0xFu) | (((hh >> (2 * (k & 15))) & 3u) << 4)) - 32);
            }
            sq[F == RQ6K ? (c >> 1) : 0] = fmaf(q, xv[i], sq[F == RQ6K ? (c >> 1) : 0]);
            if (F == RQ4K) sx += xv[i];
        }
    }
    if (F == RQ4K) return __ldg(a.scale + idx) * sq[0] - __ldg(a.bias + idx) * sx;
    if (F == RQ6K) return __ldg(a.scale + 2 * idx) * sq[0] + __ldg(a.scale + 2 * idx + 1) * sq[1];
    return __ldg(a.scale + idx) * sq[0];
}

constexpr int RQ_THREADS = 256;  // 64 rows x 4 K slices
template <int F>
__global__ void __launch_bounds__(RQ_THREADS) rq_kernel(const __grid_constant__ RqArgs a) {
    __shared__ float part[4][64];
    const uint32_t t = threadIdx.x & 63, s = threadIdx.x >> 6, g = blockIdx.x, p = blockIdx.y;
    const uint32_t nkb = a.cols >> 5;
    const uint32_t per = (nkb + a.split - 1) / a.split;
    const uint32_t kb0 = p * per, kb1 = min(kb0 + per, nkb);
    float acc = 0.0f;
    for (uint32_t kb = kb0 + s; kb < kb1; kb += 4) acc += rq_block<F>(a, ((size_t)g * nkb + kb) * 64 + t, kb);
    part[s][t] = acc;
    __syncthreads();
    const uint32_t r = g * 64 + t;
    if (s == 0 && r < a.rows) {
        const float v = (part[0][t] + part[1][t]) + (part[2][t] + part[3][t]);
        a.out[(size_t)p * a.rows + r] = kb0 < nkb ? v : 0.0f;
    }
}

// partial[p * rows + r] summed over p in order (llm_quant.cl:608-615)
__global__ void rq_reduce(float* out, const float* partial, uint32_t rows, uint32_t split) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float acc = 0.0f;
    for (uint32_t p = 0; p < split; ++p) acc += partial[(size_t)p * rows + r];
    out[r] = acc;
}

// ---- repack on the device: native blocks -> the rq planes -----------------------
// examples/llm/quant_repack.cpp repack(), one thread per plane slot
// idx = (g * nkb + kb) * 64 + t (row r = 64 g + t, k-block kb): it reads the
// 32 weights of block kb of row r from the native layout and writes every
// plane of that slot (zeros for the padding rows r >= rows). The stored
// scales are the same fp32 products of the fp16 fields and the integer
// sub-scales as the host repack forms, so the planes are identical bit for bit.
struct RepackArgs {
    const uint8_t* src;
    uint4* quant;          // 1 uint4 per slot (Q8_0: 2)
    uint32_t* high;        // Q5_0: 1 per slot, Q6_K: 2
    float* scale;          // 1 per slot (Q6_K: 2)
    float* bias;           // Q4_K
    uint32_t type, rows, cols, nkb, slots;
};
XP_DEV uint32_t nib_word(const uint32_t* q8) {  // 8 values < 16 -> one word, value i at shift 4 i
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w |= (q8[i] & 0xFu) << (4 * i);
    return w;
}
__global__ void repack_kernel(const __grid_constant__ RepackArgs a) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= a.slots) return;
    const uint32_t t = idx & 63, kb = (idx >> 6) % a.nkb, g = (idx >> 6) / a.nkb, r = g * 64 + t;
    uint32_t q[32];
    uint32_t hi0 = 0, hi1 = 0;
    float s0 = 0.0f, s1 = 0.0f, b0 = 0.0f;
    if (r < a.rows) {
        if (a.type == 8) {  // Q8_0: 34 B blocks
            const uint8_t* blk = a.src + ((size_t)r * a.nkb + kb) * 34;
            s0 = rd_f16(blk);
#pragma unroll
            for (int j = 0; j < 32; ++j) q[j] = rd_u8(blk + 2 + j);
        } else if (a.type == 6) {  // Q5_0: 22 B blocks; the 5th bits are qh itself
            const uint8_t* blk = a.src + ((size_t)r * a.nkb + kb) * 22;
            s0 = rd_f16(blk);
            hi0 = rd_u8(blk + 2) | (rd_u8(blk + 3) << 8) | (rd_u8(blk + 4) << 16) | (rd_u8(blk + 5) << 24);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t byte = rd_u8(blk + 6 + j);
                q[j] = byte & 0xFu;
                q[j + 16] = byte >> 4;
            }
        } else if (a.type == 12) {  // Q4_K: sub-block kb % 8 of super-block kb / 8
            const uint32_t s = kb & 7;
            const uint8_t* blk = a.src + ((size_t)r * (a.nkb / 8) + kb / 8) * 144;
            uint32_t sc, mn;
            q4k_scale_min(blk + 4, s, sc, mn);
            s0 = __fmul_rn(rd_f16(blk), (float)sc);
            b0 = __fmul_rn(rd_f16(blk + 2), (float)mn);
            const uint8_t* qs = blk + 16 + (s >> 1) * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) q[j] = (s & 1) ? (rd_u8(qs + j) >> 4) : (rd_u8(qs + j) & 0xFu);
        } else {  // Q6_K: quarter (h, g) = (kb % 8) / 4, (kb % 8) % 4 of super-block kb / 8
            const uint32_t hg = kb & 7, h = hg >> 2, gq = hg & 3;
            const uint8_t* blk = a.src + ((size_t)r * (a.nkb / 8) + kb / 8) * 210;
            const float dd = rd_f16(blk + 208);
            s0 = __fmul_rn(dd, (float)(int8_t)rd_u8(blk + 192 + h * 8 + 2 * gq));
            s1 = __fmul_rn(dd, (float)(int8_t)rd_u8(blk + 192 + h * 8 + 1 + 2 * gq));
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t byte = rd_u8(blk + h * 64 + j + (gq & 1) * 32);
                const uint32_t lo = gq < 2 ? (byte & 0xFu) : (byte >> 4);
                const uint32_t hb = (rd_u8(blk + 128 + h * 32 + j) >> (2 * gq)) & 3u;
                q[j] = lo;
                if (j < 16) hi0 |= hb << (2 * j);
                else hi1 |= hb << (2 * (j - 16));
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) q[j] = 0;
    }
    if (a.type == 8) {
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = q[4 * i] | (q[4 * i + 1] << 8) | (q[4 * i + 2] << 16) | (q[4 * i + 3] << 24);
        a.quant[2 * (size_t)idx] = make_uint4(w[0], w[1], w[2], w[3]);
        a.quant[2 * (size_t)idx + 1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
        a.quant[idx] = make_uint4(nib_word(q), nib_word(q + 8), nib_word(q + 16), nib_word(q + 24));
    }
    if (a.type == 6) a.high[idx] = hi0;
    if (a.type == 14) {
        a.high[2 * (size_t)idx] = hi0;
        a.high[2 * (size_t)idx + 1] = hi1;
        a.scale[2 * (size_t)idx] = s0;
        a.scale[2 * (size_t)idx + 1] = s1;
    } else {
        a.scale[idx] = s0;
    }
    if (a.type == 12) a.bias[idx] = b0;
}

// Element counts of the planes: quant words, high words, scales, biases
// (examples/llm/quant_repack.cpp repack(); 0 for an unsupported shape).
inline bool repack_sizes(uint32_t type, uint32_t rows, uint32_t cols, uint64_t sizes[4]) {
    if (rows == 0 || cols == 0 || cols % 32) return false;
    if ((type == 12 || type == 14) && cols % 256) return false;
    if (type != 8 && type != 6 && type != 12 && type != 14) return false;
    const uint64_t slots = (uint64_t)((rows + 63) / 64) * (cols / 32) * 64;
    sizes[0] = slots * (type == 8 ? 8 : 4);
    sizes[1] = type == 6 ? slots : type == 14 ? 2 * slots : 0;
    sizes[2] = slots * (type == 14 ? 2 : 1);
    sizes[3] = type == 12 ? slots : 0;
    return true;
}

inline cudaError_t launch_rq(int f, const RqArgs& a, cudaStream_t st) {
    const dim3 grid((a.rows + 63) / 64, a.split);
    switch (f) {
        case RQ4K: rq_kernel<RQ4K><<<grid, RQ_THREADS, 0, st>>>(a); break;
        case RQ50: rq_kernel<RQ50><<<grid, RQ_THREADS, 0, st>>>(a); break;
        case RQ6K: rq_kernel<RQ6K><<<grid, RQ_THREADS, 0, st>>>(a); break;
        default: rq_kernel<RQ80><<<grid, RQ_THREADS, 0, st>>>(a); break;
    }
    return cudaGetLastError();
}

}  // namespace quant
}  // namespace xp
