// Activation "limb" format consumed by the int4 matvec.
//
// The reference matvec (kernels/llm_matvec.cl:422-434) computes, per output
// column j, sum_k x[k] * (nibble(k,j) - 8) * scale(k/32, j) in fp32. On B200
// that dequantise-and-FMA form costs ~3 issue slots per weight, which at
// 6.4 TB/s is more than the SM array can issue. This build instead splits
// every 32-element block of x into three int8 limbs against a power-of-two
// block scale s:
//
//     x = s * (d0 + d1/128 + d2/16384) + r,   |d_L| <= 64,  |r| <= s * 2^-15
//
// so each weight nibble multiplies an int8 with dp4a in exact integer
// arithmetic, the -8 bias becomes one precomputed integer per block, and a
// block costs one int->float conversion and one FMA per column. Relative to
// the block's largest |x| the representation error is <= 2^-20, the same
// order as fp32 accumulation over 1152 terms.
//
// One XBlk (128 B) per 32-element block. Word order matches the nibble split
// the matvec uses: for uint32 word i of a KM4 uint4, (w & 0x0F0F0F0F) holds
// the nibbles of k = 8i+{0,2,4,6} in bytes 0..3 and ((w >> 4) & 0x0F0F0F0F)
// holds k = 8i+{1,3,5,7}. So limb L word i carries d_L[8i+0,2,4,6] and word
// 4+i carries d_L[8i+1,3,5,7].
#pragma once
#include "common.cuh"

namespace xp {

struct __align__(16) XBlk {
    int w[3][8];   // limb words (int8 x4)
    int bias;      // -8 * (S0*16384 + S1*128 + S2), S_L = sum of limb L
    float f;       // s / 16384
    int pad[6];
};
static_assert(sizeof(XBlk) == 128, "XBlk is 128 bytes");

// One warp converts one block: lane k holds x[k] of the block.
XP_DEV void xq_prep_block(float v, XBlk* dst) {
    const int lane = threadIdx.x & 31;
    // |v| as bits orders like |v|, so one integer max reduction finds the
    // exponent of the block's largest magnitude
    const uint32_t amax = __reduce_max_sync(0xffffffffu, __float_as_uint(v) & 0x7FFFFFFFu);
    const int eb = (int)((amax >> 23) & 0xFFu);
    int d0 = 0, d1 = 0, d2 = 0;
    float f = 0.0f;
    if (eb >= 8) {
        // amax = m * 2^(eb-126), m in [0.5,1); s = 2^(eb-132) puts |x/s| < 64.
        const float inv_s = __uint_as_float((uint32_t)(132 + 127 - eb) << 23);
        const float s = __uint_as_float((uint32_t)(eb - 132 + 127) << 23);
        const float y = v * inv_s;            // exact (power of two)
        const float r0f = rintf(y);
        const float r0 = y - r0f;             // exact, |r0| <= 0.5
        const float y1 = r0 * 128.0f;         // exact
        const float r1f = rintf(y1);
        const float r1 = y1 - r1f;            // exact
        const float r2f = rintf(r1 * 128.0f);
        d0 = (int)r0f;
        d1 = (int)r1f;
        d2 = (int)r2f;
        f = s * (1.0f / 16384.0f);
    }
    const int slot = (lane & 1) ? 4 + (lane >> 3) : (lane >> 3);
    const int byte = (lane & 7) >> 1;
    reinterpret_cast<int8_t*>(&dst->w[0][slot])[byte] = (int8_t)d0;
    reinterpret_cast<int8_t*>(&dst->w[1][slot])[byte] = (int8_t)d1;
    reinterpret_cast<int8_t*>(&dst->w[2][slot])[byte] = (int8_t)d2;
    // one reduction of the combined limb value (|d0 16384 + d1 128 + d2| <
    // 2^21 per lane, < 2^26 over the block): the same integer as summing
    // each limb and combining afterwards
    const int sc = __reduce_add_sync(0xffffffffu, (d0 * 16384 + d1 * 128) + d2);
    if (lane == 0) {
        dst->bias = -8 * sc;
        dst->f = f;
    }
}

// dot of one KM4 uint4 (32 nibbles of one column) against a block's limbs,
// returning the exact integer sum_k (n_k - 8) * (d0 16384 + d1 128 + d2)_k.
XP_DEV int xq_dot(const uint4 w, const int4* X /* 6 int4 = w[3][8] */, int bias) {
    const int4 l0a = X[0], l0b = X[1], l1a = X[2], l1b = X[3], l2a = X[4], l2b = X[5];
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    const int x0[8] = {l0a.x, l0a.y, l0a.z, l0a.w, l0b.x, l0b.y, l0b.z, l0b.w};
    const int x1[8] = {l1a.x, l1a.y, l1a.z, l1a.w, l1b.x, l1b.y, l1b.z, l1b.w};
    const int x2[8] = {l2a.x, l2a.y, l2a.z, l2a.w, l2b.x, l2b.y, l2b.z, l2b.w};
    int a0 = 0, a1 = 0, a2 = bias;  // the bias rides in the last limb's sum (integer: exact)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int lo = (int)(ws[i] & 0x0F0F0F0Fu);
        const int hi = (int)((ws[i] >> 4) & 0x0F0F0F0Fu);
        a0 = __dp4a(lo, x0[i], a0);
        a0 = __dp4a(hi, x0[4 + i], a0);
        a1 = __dp4a(lo, x1[i], a1);
        a1 = __dp4a(hi, x1[4 + i], a1);
        a2 = __dp4a(lo, x2[i], a2);
        a2 = __dp4a(hi, x2[4 + i], a2);
    }
    return (a0 * 128 + a1) * 128 + a2;
}

}  // namespace xp
