// Load-path, norm and sampling kernels of the decode engine (sm_100a).
#pragma once
#include "common.cuh"
#include "xq.cuh"

namespace xp {

// ---- seeded synthetic inputs ---------------------------------------------------
// splitmix64 counter generator and an Irwin-Hall(12) approximation of
// N(0, sigma): integer sum, one correctly rounded int->float conversion, one
// fp32 multiply. Bit-identical to the host generator used by the tests.
XP_DEV uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
XP_DEV uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ splitmix64(stream + 0x632BE59BD9B4E019ull));
}
XP_DEV float uniform01(uint64_t seed, uint64_t stream, uint64_t index) {
    const uint64_t h = splitmix64(stream_key(seed, stream) + index * 0x9E3779B97F4A7C15ull);
    return __fmul_rn((float)(h >> 40), 1.0f / 16777216.0f);
}

__global__ void gen_normal_kernel(float* out, uint64_t n, uint64_t offset, uint64_t seed, uint64_t stream,
                                  float sigma) {
    const uint64_t key = stream_key(seed, stream);
    const float mul = __fmul_rn(sigma, 1.0f / 16777216.0f);
    for (uint64_t ii = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; ii < n;
         ii += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = ii + offset;
        int64_t s = 0;
#pragma unroll
        for (uint64_t j = 0; j < 6; ++j) {
            const uint64_t h = splitmix64(key + (i * 6 + j) * 0x9E3779B97F4A7C15ull);
            s += (int64_t)(h >> 40) + (int64_t)((h >> 8) & 0xFFFFFFull);
        }
        s -= 6ll * 16777216ll;
        out[ii] = __fmul_rn((float)s, mul);
    }
}

// ---- int4 KM4 + bf16 packer (examples/llm/decode.cpp:101-229) --------------------
// One thread per (column, 32-row block). Bit-exact with the host packer:
// divisions and the lround are correctly rounded, and the double-precision
// error sums are written with explicit _rn intrinsics so no FMA contraction
// changes which bf16 neighbour wins.
XP_DEV uint32_t quantise_dev(float v, float inv) {
    long long r = llroundf(__fmul_rn(v, inv));
    long long q = r + 8;
    q = q < 0 ? 0 : (q > 15 ? 15 : q);
    return (uint32_t)q;
}
XP_DEV double block_err_dev(const float* blk, float s) {
    if (!(s > 0.0f)) return __longlong_as_double(0x7FF0000000000000ll);
    const float inv = __fdiv_rn(1.0f, s);
    double e = 0.0;
    for (int t = 0; t < 32; ++t) {
        const double d = __dsub_rn(__dmul_rn((double)((int)quantise_dev(blk[t], inv) - 8), (double)s), (double)blk[t]);
        e = __dadd_rn(e, __dmul_rn(d, d));
    }
    return e;
}
__global__ void pack_km4bf16_kernel(const float* __restrict__ w, uint32_t rows, uint32_t cols, uint4* words,
                                    uint32_t* scales) {
    const uint32_t nblk = rows / 32;
    const uint64_t total = (uint64_t)cols * nblk;
    for (uint64_t id = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; id < total;
         id += (uint64_t)gridDim.x * blockDim.x) {
        // id -> (block, column) with the column fastest so writes coalesce
        const uint32_t j = (uint32_t)(id % cols), b = (uint32_t)(id / cols);
        float r[32];
        const float4* src = reinterpret_cast<const float4*>(w + (size_t)j * rows + (size_t)b * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = src[i];
            r[4 * i] = v.x; r[4 * i + 1] = v.y; r[4 * i + 2] = v.z; r[4 * i + 3] = v.w;
        }
        float amax = 0.0f;
#pragma unroll
        for (int t = 0; t < 32; ++t) { const float a = fabsf(r[t]); if (amax < a) amax = a; }
        const float s0 = __fdiv_rn(amax, 7.0f);
        float s = 0.0f;
        if (s0 > 0.0f) {
            const uint32_t ulo = __float_as_uint(s0) & 0xFFFF0000u;
            const float lo = __uint_as_float(ulo), hi = __uint_as_float(ulo + 0x10000u);
            s = block_err_dev(r, lo) <= block_err_dev(r, hi) ? lo : hi;
        }
        const float inv = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
        uint32_t wd[4] = {0, 0, 0, 0};
#pragma unroll
        for (int t = 0; t < 32; ++t) wd[(t >> 3) & 3] |= quantise_dev(r[t], inv) << ((t & 7) * 4);
        const uint32_t g = j / 64, c = j % 64;
        words[((size_t)g * nblk + b) * 64 + c] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        // uint2 sc[(b/4)*cols + j]: blocks 4q..4q+3 in lo/hi of .x then .y
        const size_t sw = ((size_t)(b / 4) * cols + j) * 2 + ((b % 4) >> 1);
        const uint16_t bits = (uint16_t)(__float_as_uint(s) >> 16);
        reinterpret_cast<uint16_t*>(scales)[sw * 2 + (b & 1)] = bits;
    }
}

// ---- final norm: residual + post-FFN norm, then the output norm -> limbs -------------
// decode.cpp:1756 (final rmsnorm) preceded by the last layer's post-FFN norm
// and residual add (:1750-1753). One CTA, any hidden size multiple of 32.
__global__ void final_norm_xq_kernel(const float* x, const float* y, const float* w_post, const float* w_final,
                                     uint32_t n, float eps, float* x_out, XBlk* xq) {
    extern __shared__ float buf[];
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float ss = 0.0f;
    for (uint32_t i = tid; i < n; i += blockDim.x) { const float v = y[i]; buf[i] = v; ss += v * v; }
    ss = block_sum(ss, red);
    float sc = rsqrtf(ss / (float)n + eps);
    __syncthreads();
    float ss2 = 0.0f;
    for (uint32_t i = tid; i < n; i += blockDim.x) {
        const float r = x[i] + buf[i] * sc * (1.0f + w_post[i]);
        buf[i] = r;
        if (x_out) x_out[i] = r;
        ss2 += r * r;
    }
    ss2 = block_sum(ss2, red);
    sc = rsqrtf(ss2 / (float)n + eps);
    __syncthreads();
    for (uint32_t i = tid; i < n; i += blockDim.x) buf[i] = buf[i] * sc * (1.0f + w_final[i]);
    __syncthreads();
    for (uint32_t b = warp; b < n / 32; b += blockDim.x / 32) xq_prep_block(buf[b * 32 + lane], &xq[b]);
}

// ---- greedy: reduce per-tile (max, lowest index) partials -----------------------------
// Semantics of argmax_partial/_reduce/_final (llm_sampling.cl:57-123): the
// maximum logit, ties to the lowest index. Writes the token, the (index,
// value) pair in the reference's out[2] layout, and advances the position.
__global__ void greedy_final_kernel(const float* pval, const uint32_t* pidx, uint32_t nparts, uint32_t* token,
                                    float* sample_out, uint32_t* pos, uint32_t* hist) {
    __shared__ float sv[32];
    __shared__ uint32_t si[32];
    pdl_wait();
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t p = threadIdx.x; p < nparts; p += blockDim.x) {
        const float v = pval[p];
        const uint32_t i = pidx[p];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        bv = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
        bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0xFFFFFFFFu;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            if (bi == 0xFFFFFFFFu) bi = 0;
            *token = bi;
            if (sample_out) { sample_out[0] = (float)bi; sample_out[1] = bv; }
            if (pos) {
                const uint32_t np = *pos + 1;
                *pos = np;
                if (hist) hist[np] = bi;
            }
        }
    }
}

// Advance the position after a prompt token (no logits).
__global__ void advance_kernel(uint32_t* pos) {
    pdl_wait();
    if (threadIdx.x == 0) *pos = *pos + 1;
}

// ---- exact top-k sampling -----------------------------------------------------------
// Keys order candidates by (value desc, index asc): key = ord(value) << 32 |
// ~index, unique per element, so "the k largest keys" is exactly the
// reference's top-k with ties to the lower index (llm_sampling.cl:249-286).
XP_DEV uint64_t topk_key(float v, uint32_t i) { return ((uint64_t)float_key(v) << 32) | (uint64_t)(~i); }

// In-place bitonic sort of n (power of two) keys in shared memory, descending.
XP_DEV void bitonic_desc(uint64_t* k, uint32_t n) {
    for (uint32_t size = 2; size <= n; size <<= 1)
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (uint32_t i = threadIdx.x; i < n / 2; i += blockDim.x) {
                const uint32_t lo = 2 * stride * (i / stride) + (i % stride);
                const uint32_t hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const uint64_t a = k[lo], b = k[hi];
                if ((a < b) == desc) { k[lo] = b; k[hi] = a; }
            }
        }
    __syncthreads();
}

// Phase 1: CTA b sorts its slice of `slice` logits (power of two) and emits
// its best TK keys. Any global top-TK element is in its slice's top-TK.
XP_DEV void topk_slice_body(const float* logits, uint32_t n, uint32_t slice, uint32_t tk, uint64_t* cand,
                            uint64_t* keys) {
    const uint32_t base = blockIdx.x * slice;
    for (uint32_t i = threadIdx.x; i < slice; i += blockDim.x) {
        const uint32_t g = base + i;
        keys[i] = g < n ? topk_key(logits[g], g) : 0ull;
    }
    bitonic_desc(keys, slice);
    for (uint32_t i = threadIdx.x; i < tk; i += blockDim.x) cand[(size_t)blockIdx.x * tk + i] = keys[i];
}
__global__ void topk_slice_kernel(const float* logits, uint32_t n, uint32_t slice, uint32_t tk, uint64_t* cand) {
    extern __shared__ uint64_t keys[];
    pdl_wait();
    topk_slice_body(logits, n, slice, tk, cand, keys);
}
// Batched decode: sequence blockIdx.y, logits [seq][n], candidates [seq][gridDim.x * tk].
__global__ void topk_slice_batch_kernel(const float* logits, uint32_t n, uint32_t slice, uint32_t tk, uint64_t* cand) {
    extern __shared__ uint64_t keys[];
    topk_slice_body(logits + (size_t)blockIdx.y * n, n, slice, tk, cand + (size_t)blockIdx.y * gridDim.x * tk, keys);
}

// Phase 2 (one CTA): exact top-k of the candidates, then decode.cpp:1873-1917's
// draw(): weights exp((l - max)/T) in fp32, sums in double, top-p keeps the
// crossing token, multinomial walk with r = u * sum, u from the seeded
// counter generator keyed (seed, sequence, position).
XP_DEV void topk_sample_body(const uint64_t* cand, uint32_t ncand_pow2, uint32_t ncand, uint32_t top_k,
                             float temperature, float top_p, uint64_t seed, uint64_t seq_id, uint32_t* token,
                             float* sample_out, uint32_t* pos, float* out_vals, uint32_t* out_idx,
                             const uint32_t* pos_read, uint32_t* hist, uint64_t* keys, float* w) {
    for (uint32_t i = threadIdx.x; i < ncand_pow2; i += blockDim.x) keys[i] = i < ncand ? cand[i] : 0ull;
    bitonic_desc(keys, ncand_pow2);
    uint32_t k = top_k ? min(top_k, ncand) : ncand;
    if (k > 256) k = 256;
    if (threadIdx.x == 0) {
        const float t = temperature > 0.0f ? temperature : 1.0f;
        const float maxl = key_float((uint32_t)(keys[0] >> 32));
        double sum = 0.0;
        for (uint32_t i = 0; i < k; ++i) {
            const float l = key_float((uint32_t)(keys[i] >> 32));
            w[i] = expf(__fdiv_rn(__fsub_rn(l, maxl), t));
            sum += (double)w[i];
            if (out_vals) { out_vals[i] = l; out_idx[i] = ~(uint32_t)keys[i]; }
        }
        if (top_p > 0.0f && top_p < 1.0f && sum > 0.0) {
            double acc = 0.0;
            const double cut = (double)top_p * sum;
            uint32_t keep = 0;
            for (; keep < k; ++keep) { acc += (double)w[keep]; if (acc >= cut) break; }
            k = keep + 1 < k ? keep + 1 : k;
            sum = 0.0;
            for (uint32_t i = 0; i < k; ++i) sum += (double)w[i];
        }
        const uint32_t p = pos ? *pos : (pos_read ? *pos_read : 0u);
        const float u = uniform01(seed, seq_id, p);
        double r = (double)u * sum;
        uint32_t chosen = ~(uint32_t)keys[k - 1];
        for (uint32_t i = 0; i < k; ++i) {
            r -= (double)w[i];
            if (r <= 0.0) { chosen = ~(uint32_t)keys[i]; break; }
        }
        *token = chosen;
        if (sample_out) { sample_out[0] = (float)chosen; sample_out[1] = 0.0f; }
        if (pos) {
            *pos = p + 1;
            if (hist) hist[p + 1] = chosen;
        }
    }
}
__global__ void topk_sample_kernel(const uint64_t* cand, uint32_t ncand_pow2, uint32_t ncand, uint32_t top_k,
                                   float temperature, float top_p, uint64_t seed, uint64_t seq_id,
                                   uint32_t* token, float* sample_out, uint32_t* pos, float* out_vals,
                                   uint32_t* out_idx, const uint32_t* pos_read, uint32_t* hist) {
    extern __shared__ uint64_t keys[];
    __shared__ float w[256];
    pdl_wait();
    topk_sample_body(cand, ncand_pow2, ncand, top_k, temperature, top_p, seed, seq_id, token, sample_out, pos,
                     out_vals, out_idx, pos_read, hist, keys, w);
}
// Batched decode: sequence blockIdx.x draws from its candidates with the
// uniform keyed (seed, seq0 + sequence, pos[sequence]); positions are read,
// not advanced.
__global__ void topk_sample_batch_kernel(const uint64_t* cand, uint32_t ncand_pow2, uint32_t ncand, uint32_t top_k,
                                         float temperature, float top_p, uint64_t seed, uint64_t seq0, uint32_t* tokens,
                                         const uint32_t* pos) {
    extern __shared__ uint64_t keys[];
    __shared__ float w[256];
    const uint32_t b = blockIdx.x;
    topk_sample_body(cand + (size_t)b * ncand, ncand_pow2, ncand, top_k, temperature, top_p, seed, seq0 + b,
                     tokens + b, nullptr, nullptr, nullptr, nullptr, pos + b, nullptr, keys, w);
}

}  // namespace xp
