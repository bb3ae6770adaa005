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
    if (!pidx && nparts % 4 == 0) {
        // pval is the logits themselves: float4 loads, eight in flight
        const float4* p4 = reinterpret_cast<const float4*>(pval);
        const uint32_t n4 = nparts / 4;
#pragma unroll 8
        for (uint32_t q = threadIdx.x; q < n4; q += blockDim.x) {
            const float4 v = p4[q];
            const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint32_t i = 4 * q + r;
                if (vv[r] > bv || (vv[r] == bv && i < bi)) { bv = vv[r]; bi = i; }
            }
        }
    } else {
        for (uint32_t p = threadIdx.x; p < nparts; p += blockDim.x) {
            const float v = pval[p];
            const uint32_t i = pidx ? pidx[p] : p;  // no index array: pval is the logits themselves
            if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
        }
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

constexpr int TOPK_THREADS = 512;

struct SelShared {
    uint32_t hist[256];
    uint32_t digit, remaining, done, count;
};

// Block-wide radix select over keys[0, n) in shared memory (n >= k, blockDim a
// multiple of 32): eight-bit
// digits from the top, one histogram per digit over the keys that still share
// the selected prefix, until the bin holding the k-th largest key is taken
// whole. Afterwards key is among the k largest iff (key & mask) >= prefix.
XP_DEV void block_select(const uint64_t* keys, uint32_t n, uint32_t k, SelShared& s, uint64_t& prefix,
                         uint64_t& mask) {
    const uint32_t tid = threadIdx.x, lane = tid & 31;
    prefix = 0;
    mask = 0;
    uint32_t rem = k;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (uint32_t i = tid; i < 256; i += blockDim.x) s.hist[i] = 0;
        __syncthreads();
        // logits crowd a few bins: one atomic per distinct bin per warp
        for (uint32_t i0 = 0; i0 < n; i0 += blockDim.x) {
            const uint32_t i = i0 + tid;
            uint32_t bin = 256;
            if (i < n) {
                const uint64_t key = keys[i];
                if ((key & mask) == prefix) bin = (uint32_t)(key >> shift) & 255u;
            }
            const uint32_t peers = __match_any_sync(0xffffffffu, bin);
            if (bin < 256 && lane == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&s.hist[bin], (uint32_t)__popc(peers));
        }
        __syncthreads();
        if (tid < 32) {
            // lane L owns bins 255 - 8L down to 248 - 8L
            uint32_t c[8], tot = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = s.hist[255 - 8 * lane - j];
                tot += c[j];
            }
            uint32_t incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= (uint32_t)o) incl += t;
            }
            uint32_t acc = incl - tot;
            if (acc < rem && rem <= incl) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (acc + c[j] >= rem) {
                        s.digit = 255 - 8 * lane - j;
                        s.remaining = rem - acc;
                        s.done = c[j] == rem - acc;
                        break;
                    }
                    acc += c[j];
                }
            }
        }
        __syncthreads();
        prefix |= (uint64_t)s.digit << shift;
        mask |= 255ull << shift;
        rem = s.remaining;
        const bool done = s.done;
        __syncthreads();
        if (done) break;
    }
}

// Writes the k selected keys (any order) to out[0, k).
XP_DEV void block_collect(const uint64_t* keys, uint32_t n, uint32_t k, uint64_t prefix, uint64_t mask, SelShared& s,
                          uint64_t* out) {
    if (threadIdx.x == 0) s.count = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const uint64_t key = keys[i];
        if ((key & mask) >= prefix) {
            const uint32_t slot = atomicAdd(&s.count, 1u);
            if (slot < k) out[slot] = key;
        }
    }
    __syncthreads();
}

// ---- fast path: an exact lower bound on the k-th largest key, then ranks ------------
// Candidates ranked by all-pairs counting; more than this takes the radix path.
constexpr uint32_t TOPK_FAST_MAX = 512;

XP_DEV uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t t = __shfl_xor_sync(0xffffffffu, v, o);
        v = t > v ? t : v;
    }
    return v;
}

// out[rank] = key for the keys of c[0, m) whose rank (descending, ties by
// position) is below k. G consecutive lanes share one key's count (G the
// largest power of two <= 32 with m * G <= blockDim.x).
template <class T>
XP_DEV void rank_place(const T* c, uint32_t m, uint32_t k, T* out) {
    uint32_t G = 1;
    while (G < 32 && m * G * 2 <= blockDim.x) G <<= 1;
    const uint32_t part = threadIdx.x & (G - 1);
    for (uint32_t t0 = 0; t0 < m * G; t0 += blockDim.x) {
        const uint32_t i = (t0 + threadIdx.x) / G;
        uint32_t r = 0;
        T me = 0;
        if (i < m) {
            me = c[i];
            for (uint32_t j = part; j < m; j += G) r += (c[j] > me) || (c[j] == me && j < i);
        }
        for (uint32_t o = 1; o < G; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
        if (i < m && part == 0 && r < k) out[r] = me;
    }
}

// Warp-aggregated append of `key` (when take) to list[*count] (capacity cap;
// *count keeps counting past it).
XP_DEV void append_key(bool take, uint64_t key, uint64_t* list, uint32_t* count, uint32_t cap) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t bal = __ballot_sync(0xffffffffu, take);
    if (!bal) return;
    const uint32_t leader = __ffs(bal) - 1;
    uint32_t off = 0;
    if (lane == leader) off = atomicAdd(count, (uint32_t)__popc(bal));
    off = __shfl_sync(0xffffffffu, off, leader);
    if (take) {
        const uint32_t idx = off + __popc(bal & ((1u << lane) - 1u));
        if (idx < cap) list[idx] = key;
    }
}

// Phase 1: CTA (slice, sequence) writes the TOPK_TK largest keys of its slice
// of TOPK_THREADS * 8 logits, in descending order. Any global top-k element
// (k <= TOPK_TK) survives in its slice's list. Only keys >= a lower bound L on
// the slice's 64th largest key are ranked (L from a sample of warp maxima).
// cand: [sequence][slices][TOPK_TK]. The launch covers slices
// [s0, s0 + gridDim.x) of ns slices (all of them unless the logits are
// sharded: then only this rank's slices are valid).
__global__ void __launch_bounds__(TOPK_THREADS) topk_cand_kernel(const float* logits, uint32_t n, uint64_t* cand,
                                                                 uint32_t s0, uint32_t ns) {
    constexpr uint32_t SL = TOPK_THREADS * 8, TK = 64, NW = TOPK_THREADS / 32;
    static_assert(NW * 8 >= TK, "the sample holds at least 64 keys");
    __shared__ uint64_t keys[SL];  // radix fallback only
    __shared__ uint64_t fc[TOPK_FAST_MAX];
    __shared__ uint32_t samp[NW * 8], sel[TK];
    __shared__ uint32_t fcount;
    __shared__ SelShared s;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_launch_dependents();
    pdl_wait();
    const float* lg = logits + (size_t)blockIdx.y * n;
    const uint32_t base = (blockIdx.x + s0) * SL;
    uint64_t k[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t g = base + j * TOPK_THREADS + tid;
        k[j] = g < n ? topk_key(lg[g], g) : 0ull;
    }
    // each warp's 8 largest values (8 rounds of a one-instruction warp max
    // over the 32-bit value keys) sample the slice; every sample stands for a
    // distinct key at or above it, so the 64th largest of the 128 samples
    // bounds the slice's 64th largest value from below
    uint32_t hv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) hv[j] = (uint32_t)(k[j] >> 32);
#pragma unroll 1
    for (int r = 0; r < 8; ++r) {
        uint32_t lb = hv[0];
#pragma unroll
        for (int j = 1; j < 8; ++j) lb = max(lb, hv[j]);
        const uint32_t wm = __reduce_max_sync(0xffffffffu, lb);
        if (lane == 0) samp[warp * 8 + r] = wm;
        if (lb == wm) {
            bool gone = false;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (!gone && hv[j] == wm) { hv[j] = 0; gone = true; }
        }
    }
    if (tid == 0) fcount = 0;
    __syncthreads();
    rank_place(samp, NW * 8, TK, sel);
    __syncthreads();
    const uint64_t L = (uint64_t)sel[TK - 1] << 32;
#pragma unroll
    for (int j = 0; j < 8; ++j) append_key(k[j] >= L, k[j], fc, &fcount, TOPK_FAST_MAX);
    __syncthreads();
    const uint32_t m = fcount;
    uint64_t* out = cand + ((size_t)blockIdx.y * ns + blockIdx.x + s0) * TK;
    if (m <= TOPK_FAST_MAX) {
        rank_place(fc, m, TK, out);
        return;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) keys[j * TOPK_THREADS + tid] = k[j];
    __syncthreads();
    uint64_t prefix, mask;
    block_select(keys, SL, TK, s, prefix, mask);
    block_collect(keys, SL, TK, prefix, mask, s, fc);
    rank_place(fc, TK, TK, out);
}

// Tensor-parallel sampling: every rank copies its slices' candidate lists
// [s0, s1) (TOPK_TK keys each) into every rank's candidate area (peer
// mappings; its own too), publishes `flag` to every rank and waits, bounded,
// for every rank's flag; then copies the whole vocabulary's lists back into
// `cand`, from which it draws the same token as every other rank. Areas and
// flags have two banks, chosen by the flag's parity: a rank can be at most
// one exchange ahead of another (the next needs everyone's flag). One CTA.
struct TpCandArgs {
    uint64_t* cand;               // this rank's lists, [ns][TOPK_TK]; receives all of them
    uint32_t s0, s1, ns;          // this rank's slices of ns
    uint32_t rank, world;
    uint64_t* area[8];            // every rank's candidate area: 2 banks of ns * TOPK_TK keys
    uint32_t* flags[8];           // every rank's flag words: 2 banks of 8
    uint32_t* count;              // exchanges so far (this rank); advanced here
    uint32_t* err;
};
__global__ void tp_cand_exchange_kernel(TpCandArgs a) {
    pdl_wait();
    const uint32_t flag = *a.count + 1, bank = flag & 1u;
    const size_t W = (size_t)a.ns * 64, lo = (size_t)a.s0 * 64, hi = (size_t)a.s1 * 64;
    for (uint32_t r = 0; r < a.world; ++r)
        for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x)
            asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(a.area[r] + bank * W + i), "l"(a.cand[i]) : "memory");
    __syncthreads();
    if (threadIdx.x < a.world) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flags[threadIdx.x] + bank * 8 + a.rank), "r"(flag)
                     : "memory");
        uint32_t f = 0, it = 0;
        do {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(a.flags[a.rank] + bank * 8 + threadIdx.x)
                         : "memory");
            if (++it > (1u << 22)) { atomicOr(a.err, 32u); break; }
        } while (f != flag);
    }
    __syncthreads();
    const uint64_t* mine = a.area[a.rank] + bank * W;
    for (size_t i = threadIdx.x; i < W; i += blockDim.x) a.cand[i] = mine[i];
    if (threadIdx.x == 0) *a.count = flag;
}

// Phase 2 (one CTA per sequence): exact top-k of the candidates, then
// decode.cpp:1873-1917's draw(): weights exp((l - max)/T) in fp32, sums in
// double in rank order, top-p keeps the crossing token, multinomial walk with
// r = u * sum, u from the seeded counter generator keyed (seed, sequence,
// position). The slice lists are sorted: the k-th largest of their leading keys
// bounds the global k-th largest from below; only candidates >= it are ranked.
struct TopkDrawArgs {
    const uint64_t* cand;  // [sequence][ncand], TOPK_TK-key lists sorted descending
    uint32_t ncand, top_k;
    float temperature, top_p;
    uint64_t seed, seq0;        // sequence b draws with stream seq0 + b
    uint32_t* token;            // [sequence]
    float* sample_out;          // optional (id, 0) of sequence 0
    uint32_t* pos_adv;          // single sequence: read and advanced (hist[p + 1] = token)
    const uint32_t* pos_read;   // [sequence], read only
    float* out_vals;            // optional [k] survivors of sequence 0
    uint32_t* out_idx;
    uint32_t* hist;
};
__global__ void __launch_bounds__(TOPK_THREADS) topk_draw_kernel(const TopkDrawArgs a) {
    extern __shared__ uint64_t ckeys[];  // radix fallback only
    __shared__ SelShared s;
    __shared__ uint64_t fc[TOPK_FAST_MAX];
    __shared__ uint64_t sorted[64];
    __shared__ float w[64];
    __shared__ double cum[64];
    __shared__ uint32_t fcount, s_keep;
    pdl_wait();
    const uint32_t b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t* cand = a.cand + (size_t)b * a.ncand;
    const uint32_t k = a.top_k, nsl = a.ncand / 64;
    // lower bound T0 on the global k-th largest key: the k-th largest of the J
    // leading keys of every (sorted) slice list
    const uint32_t J = min(64u, max(1u, 128u / nsl)), S = nsl * J;
    for (uint32_t i = tid; i < S; i += TOPK_THREADS) fc[i] = cand[(i / J) * 64 + i % J];
    if (tid == 0) fcount = 0;
    __syncthreads();
    rank_place(fc, S, k, sorted);
    __syncthreads();
    const uint64_t T0 = sorted[k - 1];
    __syncthreads();
    for (uint32_t i0 = 0; i0 < a.ncand; i0 += TOPK_THREADS) {
        const uint32_t i = i0 + tid;
        const uint64_t key = i < a.ncand ? cand[i] : 0ull;
        append_key(i < a.ncand && key >= T0, key, fc, &fcount, TOPK_FAST_MAX);
    }
    __syncthreads();
    const uint32_t m = fcount;
    if (m <= TOPK_FAST_MAX) {
        rank_place(fc, m, k, sorted);
    } else {
        for (uint32_t i = tid; i < a.ncand; i += TOPK_THREADS) ckeys[i] = cand[i];
        __syncthreads();
        uint64_t prefix, mask;
        block_select(ckeys, a.ncand, k, s, prefix, mask);
        block_collect(ckeys, a.ncand, k, prefix, mask, s, fc);
        rank_place(fc, k, k, sorted);
    }
    __syncthreads();
    const float tt = a.temperature > 0.0f ? a.temperature : 1.0f;
    const float maxl = key_float((uint32_t)(sorted[0] >> 32));
    if (tid < 64) {
        float wv = 0.0f;
        if (tid < k) {
            const float l = key_float((uint32_t)(sorted[tid] >> 32));
            wv = expf(__fdiv_rn(__fsub_rn(l, maxl), tt));
            if (a.out_vals && b == 0) { a.out_vals[tid] = l; a.out_idx[tid] = ~(uint32_t)sorted[tid]; }
        }
        w[tid] = wv;  // zero past k: adding +0.0 leaves a double sum unchanged
    }
    __syncthreads();
    if (tid == 0) {
        // running sums in rank order (the reference's sequential double sum)
        double acc = 0.0;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            acc += (double)w[i];
            cum[i] = acc;
        }
    }
    __syncthreads();
    bool use_p = a.top_p > 0.0f && a.top_p < 1.0f && cum[63] > 0.0;
    if (use_p && warp == 0) {
        // first rank whose running sum reaches top_p * sum
        const double cut = (double)a.top_p * cum[63];
        const bool h0 = lane < k && cum[lane] >= cut, h1 = lane + 32 < k && cum[lane + 32] >= cut;
        const uint32_t b0 = __ballot_sync(0xffffffffu, h0), b1 = __ballot_sync(0xffffffffu, h1);
        if (lane == 0) s_keep = b0 ? __ffs(b0) - 1 : (b1 ? 32 + __ffs(b1) - 1 : 64);
    }
    __syncthreads();
    if (tid == 0) {
        uint32_t kk = k;
        if (use_p && s_keep + 1 < kk) kk = s_keep + 1;
        const double sum = cum[kk - 1];
        const uint32_t p = a.pos_adv ? *a.pos_adv : (a.pos_read ? a.pos_read[b] : 0u);
        const float u = uniform01(a.seed, a.seq0 + b, p);
        double r = (double)u * sum;
        uint32_t chosen = kk - 1;
        bool found = false;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            r -= (double)((uint32_t)i < kk ? w[i] : 0.0f);
            if (!found && r <= 0.0 && (uint32_t)i < kk) { chosen = i; found = true; }
        }
        const uint32_t id = ~(uint32_t)sorted[chosen];
        a.token[b] = id;
        if (a.sample_out && b == 0) { a.sample_out[0] = (float)id; a.sample_out[1] = 0.0f; }
        if (a.pos_adv) {
            *a.pos_adv = p + 1;
            if (a.hist) a.hist[p + 1] = id;
        }
    }
}

}  // namespace xp
