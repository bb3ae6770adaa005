// Batched int4 matvec on the 5th-generation tensor cores (tcgen05): N
// activation vectors (sequences) times one KM4 + bf16-scale weight matrix,
// out[n][j] = sum_k x[n][k] * W[k][j], the reference's mv_km4_bs
// (kernels/llm_matvec.cl:422-434) for every sequence at once. This is the
// skinny GEMM (M = weight columns, N = sequences, K = rows) of batched decode.
//
// Exactness. The reference dequantises (nibble - 8) * bf16(scale) in fp32.
// The activation enters as x / 2^e = hi + lo, two fp16 halves (about 22
// significant bits), with one power-of-two e per sequence applied at the end.
// Two operand modes, chosen per launch:
//   scaled  (every scale s of the launch's matrices is 0 or 2^-14 <= |s| <=
//            8160): (nibble - 8) * s has at most 8 + 3 significant bits and
//            stays a normal fp16 below 65504, so the dequant warps write the
//            exact dequantised weight as the fp16 A operand, one TMEM
//            accumulator runs over the item's whole K range, and the epilogue
//            runs once per item. hi and lo are the two halves of one MMA's N
//            (N' = 2N columns: hi sums, then lo sums).
//   integer (any other scale): A holds the exact integers (nibble - 8), one
//            K = 32 block per accumulator, and the epilogue adds
//            scale(j, b) * D_b to a register sum per block; hi and lo are two
//            MMAs into the same accumulator.
// Both give fp32 products of exact operands; they differ only in the fp32
// summation order.
//
// CTA (448 threads) per work item = 128 output columns x one K range:
//   warp 0   producer: bulk copies of the nibbles (2 x 1 KB per block, the
//            reference plane read in place) and the prepared activations
//   warp 1   MMA issuer (one thread) + TMEM owner (alloc/dealloc, 4N columns)
//   warps 2-5  dequant: thread = column j, 32 nibbles -> fp16 A tile
//   warps 6-13 epilogue: thread = column j x half of the sequences,
//            tcgen05.ld of the sums (per item, or per block and scaled); the
//            item's result goes to out (one K range), to int64 fixed-point
//            sums (K split across CTAs), or, for the batched-decode engine, to
//            its K range's fp32 partial that the consuming kernel adds
// A pipeline stage is two 32-row blocks (one bulk copy per KM4 group and one
// for the activations); three stages, each with its own A tile, and four
// accumulator slots (two of 2N columns in scaled mode) keep the MMA ahead of
// the epilogue; two CTAs share an SM. Waiting warps poll with one lane.
// Shared-memory operands use the K-major, no-swizzle canonical layout: 8 rows x
// 16 bytes per core matrix. Within each 8-element K chunk the order is the
// nibble extraction order (k0 k4 k1 k5 k2 k6 k3 k7) on both operands.
//
// Every wait is bounded and reports through an error word; no multicast.
#pragma once
#include "common.cuh"
#include "tk_primitives.cuh"

namespace xp {

constexpr int BMM_THREADS = 448;     // producer, MMA, 4 dequant, 8 epilogue warps
constexpr int BMM_M = 128;           // output columns per tile
constexpr int BMM_SB = 2;            // 32-row blocks per pipeline stage
constexpr int BMM_STAGES = 3;        // copy ring depth (stages), one A tile each
constexpr int BMM_ABYTES = BMM_SB * 8192;  // dequantised A tile of a stage: 128 columns x 64 rows fp16
constexpr int BMM_ND = 4;            // TMEM accumulator slots (integer mode; two of 2N columns when scaled)
constexpr int BMM_MAXN = 64;
// sequences padded to the MMA's N (32 or 64)
inline uint32_t bmm_npad(uint32_t n) { return n <= 32 ? 32u : 64u; }
// bytes of a prepared activation operand of `rows` for n sequences
inline size_t bmm_xb_bytes(uint32_t rows, uint32_t n) { return (size_t)(rows / 32) * 2 * 4 * bmm_npad(n) * 16; }         // sequences per launch (N is 32 or 64)
constexpr uint32_t BMM_ERR_WAIT = 64u;

// One weight matrix of a launch; a launch covers up to BMM_MAXPARTS matrices
// with the same rows (K), their 128-column tiles numbered consecutively.
struct BmmPart {
    const uint4* wq;          // nibble plane of the matrix (reference layout)
    const uint2* sc;          // bf16 scale plane
    float* out;               // [N][cols] (ksplit == 1 and not raw)
    long long* acc;           // [N][cols] fixed-point sums (ksplit > 1, not raw), zero at launch
    float* part;              // raw: [ksplit][nreal][cols] fp32 sums of each K range (plain stores)
    uint32_t cols;            // columns of this matrix
    uint32_t tile0;           // first tile of this matrix in the launch
};
constexpr int BMM_MAXPARTS = 3;
struct BmmArgs {
    BmmPart part[BMM_MAXPARTS];
    uint32_t nparts;
    const unsigned char* xb;  // prepared activations: [nblk][chunk 4][hi, lo][N][16 B]
    const float* xs;          // [N] per-sequence power-of-two scale 2^e
    uint32_t nblk, N;         // N = padded sequence count (32 or 64)
    uint32_t nreal;           // sequences actually present (rows of out)
    uint32_t ksplit, cb;      // K ranges per tile, blocks per range
    uint32_t nitems;          // tiles * ksplit
    uint32_t raw;             // 1: leave the result as per-K-range partial sums in part (the consumer adds them)
    uint32_t scaled;          // 1: scaled-operand mode (every scale in the fp16-exact range)
    const uint32_t* fbflag;   // if set, the mode is read here instead: 0 scaled, else integer
    uint32_t* err;
};
// The matrix holding launch tile `tile`, and the tile's index within it.
XP_DEV const BmmPart& bmm_part(const BmmArgs& a, uint32_t tile, uint32_t& lt) {
    const uint32_t p = (a.nparts > 2 && tile >= a.part[2].tile0) ? 2u : (a.nparts > 1 && tile >= a.part[1].tile0) ? 1u : 0u;
    lt = tile - a.part[p].tile0;
    return a.part[p];
}


// ---- tcgen05 helpers (PTX of the sm_100a tensor-core and TMEM instructions) ----
XP_DEV uint64_t bmm_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // K-major, SWIZZLE_NONE: start >> 4, leading (K) byte offset >> 4, stride
    // (8-row group) byte offset >> 4, descriptor version 1 (bit 46)
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
XP_DEV uint32_t bmm_idesc(uint32_t n) {
    // kind::f16: D f32 (bit 4), A = B = f16, both K-major, N >> 3 at bit 17, M >> 4 at bit 24
    return (1u << 4) | ((n >> 3) << 17) | ((uint32_t)(BMM_M >> 4) << 24);
}
XP_DEV void bmm_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
XP_DEV void bmm_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
XP_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
XP_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 16 columns of the warp's 32 TMEM lanes into v[0..15]
XP_DEV void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// bounded wait that records the failure and returns
XP_DEV void bmm_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
    uint32_t it = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (++it > TK_SPIN_LIMIT) {
            atomicOr(err, BMM_ERR_WAIT);
            return;
        }
    }
}

// Warp-wide wait: lane 0 polls, the other lanes park at the warp barrier
// (which also orders their later reads after lane 0's acquire).
XP_DEV void bmm_wait_warp(uint64_t* bar, uint32_t parity, uint32_t* err) {
    if ((threadIdx.x & 31) == 0) bmm_wait(bar, parity, err);
    __syncwarp();
}

// 8 nibbles (one word: k = 8c .. 8c+7) -> 8 fp16 (nibble - 8) in the order
// k0 k4 k1 k5 k2 k6 k3 k7, exact (1024 + n - 1032 in fp16).
XP_DEV uint4 bmm_unpack8(uint32_t w) {
    const uint32_t magic = 0x64006400u;  // fp16 1024.0 in both halves
    const __half2 bias = __halves2half2(__float2half_rn(1032.0f), __float2half_rn(1032.0f));
    uint4 r;
    uint32_t h;
    h = (w & 0x000F000Fu) | magic;
    *reinterpret_cast<__half2*>(&r.x) = __hsub2(*reinterpret_cast<__half2*>(&h), bias);
    h = ((w >> 4) & 0x000F000Fu) | magic;
    *reinterpret_cast<__half2*>(&r.y) = __hsub2(*reinterpret_cast<__half2*>(&h), bias);
    h = ((w >> 8) & 0x000F000Fu) | magic;
    *reinterpret_cast<__half2*>(&r.z) = __hsub2(*reinterpret_cast<__half2*>(&h), bias);
    h = ((w >> 12) & 0x000F000Fu) | magic;
    *reinterpret_cast<__half2*>(&r.w) = __hsub2(*reinterpret_cast<__half2*>(&h), bias);
    return r;
}

// bf16 scale magnitudes for which (nibble - 8) * s is an exact normal fp16:
// 0, or 2^-14 (0x3880) <= |s| <= 8160 (0x45FF; 8 * 8160 <= 65504)
XP_DEV bool bmm_scale_exact16(uint32_t bits16) {
    const uint32_t m = bits16 & 0x7FFFu;
    return m == 0 || (m >= 0x3880u && m <= 0x45FFu);
}
// Any scale of the plane (nwords uint4 = 8 bf16 each) outside that range ->
// *flag |= 1 (the flag is cleared before the launch).
__global__ void bmm_scale_check_kernel(const uint4* sc, size_t nwords, uint32_t* flag) {
    bool bad = false;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nwords; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 w = __ldg(sc + i);
        const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) bad = bad || !bmm_scale_exact16(v[k] & 0xFFFFu) || !bmm_scale_exact16(v[k] >> 16);
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1u);
}
// 8 nibbles -> 8 fp16 (nibble - 8) * s, exact for s in the range above
XP_DEV uint4 bmm_unpack8s(uint32_t w, __half2 s2) {
    uint4 r = bmm_unpack8(w);
    *reinterpret_cast<__half2*>(&r.x) = __hmul2(*reinterpret_cast<__half2*>(&r.x), s2);
    *reinterpret_cast<__half2*>(&r.y) = __hmul2(*reinterpret_cast<__half2*>(&r.y), s2);
    *reinterpret_cast<__half2*>(&r.z) = __hmul2(*reinterpret_cast<__half2*>(&r.z), s2);
    *reinterpret_cast<__half2*>(&r.w) = __hmul2(*reinterpret_cast<__half2*>(&r.w), s2);
    return r;
}

// Activation prep, pass 1: per sequence the power-of-two 2^e >= max |x| (one
// warp per sequence); also zeroes the fixed-point sums of this call.
// Activations of one call, one CTA per (padded) sequence: the power-of-two
// scale 2^e > max |x| of the sequence, then x / 2^e as hi + lo fp16 in the
// B-operand layout [nblk][chunk 4][hi, lo][N][8 halves]. Padded sequences get
// zeros. CTA 0 also clears the call's error word. Rows up to 8 x 1024 are
// loaded once into registers (every load in flight together).
constexpr int BMM_XP_THREADS = 1024, BMM_XP_PER = 8;
XP_DEV void bmm_xput(unsigned char* xb, uint32_t Npad, uint32_t n, uint32_t i, float y) {
    // element k = i % 32 of block b = i / 32: chunk c = k / 8, position of k in
    // the extraction order k0 k4 k1 k5 k2 k6 k3 k7
    const uint32_t b = i >> 5, k = i & 31, c = k >> 3, e = k & 7, pos = (e & 3) * 2 + (e >> 2);
    const __half hi = __float2half_rn(y);
    const __half lo = __float2half_rn(y - __half2float(hi));
    __half* base = reinterpret_cast<__half*>(xb + (size_t)b * 2 * 4 * Npad * 16);
    base[((c * 2 + 0) * Npad + n) * 8 + pos] = hi;
    base[((c * 2 + 1) * Npad + n) * 8 + pos] = lo;
}
// The same operand written by the kernel that produces the activations: the
// calling CTA holds sequence n, element i = threadIdx.x + j * blockDim.x in
// v[j] (rows <= J * blockDim.x, blockDim.x a multiple of 32). Every thread of
// the CTA must call it.
template <int J>
XP_DEV void bmm_put_seq(const float (&v)[J], uint32_t rows, uint32_t n, uint32_t Npad, float* xs, unsigned char* xb) {
    __shared__ float bmm_red[32];
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float am = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) am = fmaxf(am, fabsf(v[j]));
    am = warp_max(am);
    __syncthreads();  // bmm_red free
    if (lane == 0) bmm_red[warp] = am;
    __syncthreads();
    am = warp_max(lane < nw ? bmm_red[lane] : 0.0f);
    const int eb = (int)((__float_as_uint(am) >> 23) & 0xFFu);
    const float sc = eb > 0 && eb < 253 ? __uint_as_float((uint32_t)(eb + 1) << 23) : 1.0f;
    if (tid == 0) xs[n] = sc;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const uint32_t i = tid + j * blockDim.x;
        if (i < rows) bmm_xput(xb, Npad, n, i, v[j] / sc);  // exact: power of two
    }
}

__global__ void __launch_bounds__(BMM_XP_THREADS) bmm_xprep_kernel(const float* x, uint32_t rows, uint32_t N,
                                                                  uint32_t Npad, float* xs, unsigned char* xb,
                                                                  uint32_t* err) {
    __shared__ float red[BMM_XP_THREADS / 32];
    const uint32_t n = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (n == 0 && tid == 0) *err = 0;
    const float* xr = x + (size_t)n * rows;
    const bool inreg = rows <= BMM_XP_THREADS * BMM_XP_PER;
    float v[BMM_XP_PER];
    float am = 0.0f;
    if (inreg) {
#pragma unroll
        for (int r = 0; r < BMM_XP_PER; ++r) {
            const uint32_t i = tid + r * BMM_XP_THREADS;
            v[r] = (n < N && i < rows) ? xr[i] : 0.0f;
            am = fmaxf(am, fabsf(v[r]));
        }
    } else if (n < N) {
        for (uint32_t i = tid; i < rows; i += BMM_XP_THREADS) am = fmaxf(am, fabsf(xr[i]));
    }
    am = warp_max(am);
    if (lane == 0) red[warp] = am;
    __syncthreads();
    am = warp_max(red[lane]);
    // am = m 2^(eb-127), m in [1,2): 2^(eb-126) > am
    const int eb = (int)((__float_as_uint(am) >> 23) & 0xFFu);
    const float sc = eb > 0 && eb < 253 ? __uint_as_float((uint32_t)(eb + 1) << 23) : 1.0f;
    if (tid == 0) xs[n] = sc;
    if (inreg) {
#pragma unroll
        for (int r = 0; r < BMM_XP_PER; ++r) {
            const uint32_t i = tid + r * BMM_XP_THREADS;
            if (i < rows) bmm_xput(xb, Npad, n, i, v[r] / sc);  // exact: power of two
        }
    } else {
        for (uint32_t i = tid; i < rows; i += BMM_XP_THREADS) bmm_xput(xb, Npad, n, i, n < N ? xr[i] / sc : 0.0f);
    }
}

// Per-role timeline of the first CTAs (a build with BMM_TRACE only):
// [cta][role][stage] %globaltimer ns; roles: 0 producer issued, 1 MMA inputs
// ready, 2 MMA issued, 3 dequant input ready, 4 dequant done.
#ifdef BMM_TRACE
__device__ unsigned long long g_bmm_trace[4][6][64];
#define BMM_TR(role, t) \
    if (blockIdx.x < 4 && (t) < 64) g_bmm_trace[blockIdx.x][role][t] = globaltimer_ns();
#else
#define BMM_TR(role, t)
#endif

XP_DEV void bmm_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// fixed-point sums -> fp32, leaving the sums zero for the next call
__global__ void bmm_finish_kernel(long long* acc, float* out, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        out[i] = __ll2float_rn(acc[i]) * 2.3283064365386963e-10f;
        acc[i] = 0;
    }
}

__global__ void __launch_bounds__(BMM_THREADS, 2) bmm_kernel(const __grid_constant__ BmmArgs a) {
    extern __shared__ __align__(1024) unsigned char bsm[];
    __shared__ float s_xs[BMM_MAXN];  // per-sequence scales 2^e (epilogue)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) { BMM_TR(5, 0) }
    const uint32_t N = a.N;
    const uint32_t xbytes = 2 * 4 * N * 16;              // activations per block
    const uint32_t sbytes = BMM_SB * 2048 + BMM_SB * xbytes;  // one stage: nibbles + activations of two blocks
    // layout: [stages][nibbles: group 0 blocks b, b+1 | group 1 blocks b, b+1 | activations b, b+1]
    //         [A tiles, one per stage] [mbarriers] [tmem addr]
    unsigned char* stage0 = bsm;
    unsigned char* atile = bsm + BMM_STAGES * sbytes;
    uint64_t* mb = reinterpret_cast<uint64_t*>(atile + BMM_STAGES * BMM_ABYTES);
    uint64_t* full = mb;                         // [STAGES] producer -> dequant, MMA
    uint64_t* empty = mb + BMM_STAGES;           // [STAGES] dequant + MMA commit -> producer, dequant (stage and A tile free)
    uint64_t* afull = mb + 2 * BMM_STAGES;       // [STAGES] dequant -> MMA
    uint64_t* dfull = afull + BMM_STAGES;        // [ND] MMA commit -> epilogue
    uint64_t* dempty = dfull + BMM_ND;           // [ND] epilogue -> MMA
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dempty + BMM_ND);

    if (tid == 0) {
        for (int i = 0; i < BMM_STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 2);
            mbar_init(&afull[i], 1);
        }
        for (int i = 0; i < BMM_ND; ++i) {
            mbar_init(&dfull[i], 1);
            mbar_init(&dempty[i], 1);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        const uint32_t ncols = BMM_ND * N;  // accumulator slots of N columns (128 or 256)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t G = gridDim.x;
    // operand mode of the launch (uniform over the CTA)
    const bool S = a.fbflag ? (*reinterpret_cast<const volatile uint32_t*>(a.fbflag) == 0u) : (a.scaled != 0u);
    // launch scalars in registers: `a` has its address taken (bmm_part), and a
    // load through that generic pointer after a store or an asm memory
    // clobber would be issued again each time
    const uint32_t nitems = a.nitems, ksplit = a.ksplit, cbk = a.cb, nblk = a.nblk, nreal = a.nreal;
    const bool raw = a.raw != 0u;
    uint32_t* const err = a.err;
    const unsigned char* const xb = a.xb;

    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            // The weights do not depend on the kernel before this one, the
            // activations do: the first stages' nibbles are requested before
            // griddepcontrol.wait (under the previous kernel's tail when this
            // launch is programmatic), their activations after it.
            uint32_t t = 0;  // stage counter of this CTA (two blocks each)
            uint32_t deferred[BMM_STAGES];
            uint32_t ndef = 0;
            bool waited = false;
            auto release = [&]() {
                pdl_wait();
                waited = true;
                for (uint32_t i = 0; i < ndef; ++i)
                    bulk_g2s(stage0 + i * sbytes + BMM_SB * 2048, xb + (size_t)deferred[i] * xbytes, BMM_SB * xbytes,
                             &full[i]);
            };
            for (uint32_t item = blockIdx.x; item < nitems; item += G) {
                const uint32_t tile = item / ksplit, kc = item % ksplit;
                const uint32_t b0 = kc * cbk, b1 = min(b0 + cbk, nblk);
                uint32_t lt;
                const uint4* wq = bmm_part(a, tile, lt).wq;
                for (uint32_t b = b0; b < b1; b += BMM_SB, ++t) {
                    const uint32_t s = t % BMM_STAGES;
                    if (t >= BMM_STAGES) {
                        if (!waited) release();
                        bmm_wait(&empty[s], ((t / BMM_STAGES) - 1) & 1, err);
                    }
                    unsigned char* st = stage0 + s * sbytes;
                    fence_proxy_async();
                    mbar_expect_tx(&full[s], sbytes);
                    // columns 128 tile .. +63 and +64 .. +127 are two KM4 groups;
                    // a group's consecutive blocks are contiguous (1 KB each)
                    bulk_g2s(st, wq + ((size_t)(2 * lt) * nblk + b) * 64, BMM_SB * 1024, &full[s]);
                    bulk_g2s(st + BMM_SB * 1024, wq + ((size_t)(2 * lt + 1) * nblk + b) * 64, BMM_SB * 1024, &full[s]);
                    if (waited) bulk_g2s(st + BMM_SB * 2048, xb + (size_t)b * xbytes, BMM_SB * xbytes, &full[s]);
                    else deferred[ndef++] = b;  // stage s == ndef while t < BMM_STAGES
                    BMM_TR(0, t)
                }
            }
            if (!waited) release();
        }
        __syncwarp();  // the whole warp reaches the closing CTA barrier together
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            uint32_t t = 0, tb = 0, it = 0;  // stages, blocks, items of this CTA
            const uint32_t idesc = bmm_idesc(S ? 2 * N : N);
            for (uint32_t item = blockIdx.x; item < nitems; item += G, ++it) {
                const uint32_t kc = item % ksplit;
                const uint32_t b0 = kc * cbk, b1 = min(b0 + cbk, nblk);
                // scaled: one accumulator of 2N columns (hi sums | lo sums) per
                // item over its whole K range; two slots alternate
                const uint32_t qi = it & 1;
                if (S && it >= 2) bmm_wait(&dempty[qi], ((it >> 1) - 1) & 1, err);  // slot drained
                for (uint32_t b = b0; b < b1; b += BMM_SB, ++t) {
                    const uint32_t s = t % BMM_STAGES;
                    bmm_wait(&afull[s], (t / BMM_STAGES) & 1, err);  // A tile of the stage dequantised
                    bmm_wait(&full[s], (t / BMM_STAGES) & 1, err);   // activations landed
                    BMM_TR(1, t)
                    tc_fence_after();
                    const uint32_t ab = smem_u32(atile + s * BMM_ABYTES);
                    const uint32_t xbase = smem_u32(stage0 + s * sbytes + BMM_SB * 2048);
                    if (S) {
                        const uint32_t d = tmem + qi * 2 * N;
#pragma unroll
                        for (int kk = 0; kk < 2 * BMM_SB; ++kk) {
                            // A: K chunks 2kk, 2kk+1 of 128 columns (chunk stride 2 KB, 8-row groups 128 B)
                            const uint64_t ad = bmm_desc(ab + kk * 4096, 2048, 128);
                            // B: the same K chunks, rows hi 0..N-1 then lo N..2N-1
                            // (chunk stride 32N B, 8-row groups 128 B; blocks follow each other)
                            const uint64_t bd = bmm_desc(xbase + kk * 4 * N * 16, 2 * N * 16, 128);
                            bmm_mma(d, ad, bd, idesc, (b != b0 || kk != 0) ? 1u : 0u);
                        }
                    } else {
                        for (uint32_t h = 0; h < BMM_SB; ++h, ++tb) {
                            const uint32_t q = tb % BMM_ND;
                            if (tb >= BMM_ND) bmm_wait(&dempty[q], ((tb / BMM_ND) - 1) & 1, err);  // slot q read
                            tc_fence_after();
                            const uint32_t d = tmem + q * N;
                            uint32_t acc = 0;
#pragma unroll
                            for (int kk = 0; kk < 2; ++kk)
#pragma unroll
                                for (int hl = 0; hl < 2; ++hl) {
                                    const uint64_t ad = bmm_desc(ab + (2 * h + kk) * 4096, 2048, 128);
                                    // B: chunks 2kk, 2kk+1 of block h, half hl, N sequences
                                    const uint64_t bd = bmm_desc(xbase + h * xbytes + (2 * kk * 2 + hl) * N * 16, 2 * N * 16, 128);
                                    bmm_mma(d, ad, bd, idesc, acc);
                                    acc = 1;
                                }
                            bmm_commit(&dfull[q]);  // accumulator of block tb ready
                        }
                    }
                    bmm_commit(&empty[s]);  // stage s and its A tile no longer read
                    BMM_TR(2, t)
                }
                if (S) bmm_commit(&dfull[qi]);  // the item's sums are complete
            }
        }
        __syncwarp();
    } else if (warp < 6) {
        // ------------------------------ dequant ------------------------------
        const uint32_t j = tid - 64;  // column within the tile, 0..127
        uint32_t t = 0;
        for (uint32_t item = blockIdx.x; item < nitems; item += G) {
            const uint32_t tile = item / ksplit, kc = item % ksplit;
            const uint32_t b0 = kc * cbk, b1 = min(b0 + cbk, nblk);
            uint2 sw{}, sw_next{};
            const uint2* scp = nullptr;
            uint32_t cols = 0;
            if (S) {
                // this column's scales (one uint2 = four blocks)
                uint32_t lt;
                const BmmPart& P = bmm_part(a, tile, lt);
                cols = P.cols;
                scp = P.sc + lt * BMM_M + j;
                sw = __ldg(scp + (size_t)(b0 >> 2) * cols);
            }
            for (uint32_t b = b0; b < b1; b += BMM_SB, ++t) {
                const uint32_t s = t % BMM_STAGES;
                __half2 s2[BMM_SB];
                if (S) {
                    // the next quad's scales load while this stage is dequantised
                    if ((b & 3) == 0 && b + 4 < b1) sw_next = __ldg(scp + (size_t)((b >> 2) + 1) * cols);
#pragma unroll
                    for (int h = 0; h < BMM_SB; ++h) {
                        const uint32_t bb = b + h;
                        const uint32_t word = (bb & 2) ? sw.y : sw.x;
                        const __half v = __float2half_rn((bb & 1) ? bf16_hi(word) : bf16_lo(word));  // exact in range
                        s2[h] = __halves2half2(v, v);
                    }
                }
                bmm_wait_warp(&full[s], (t / BMM_STAGES) & 1, err);
                if (j == 0) { BMM_TR(3, t) }
                const unsigned char* nb = stage0 + s * sbytes + (j >> 6) * (BMM_SB * 1024) + (j & 63) * 16;
                uint4 w[BMM_SB];
#pragma unroll
                for (int h = 0; h < BMM_SB; ++h) w[h] = *reinterpret_cast<const uint4*>(nb + h * 1024);
                if (t >= BMM_STAGES) bmm_wait_warp(&empty[s], ((t / BMM_STAGES) - 1) & 1, err);  // A tile free
                unsigned char* at = atile + s * BMM_ABYTES + j * 16;
#pragma unroll
                for (int h = 0; h < BMM_SB; ++h) {
                    unsigned char* ah = at + h * 4 * 2048;
                    if (S) {
                        *reinterpret_cast<uint4*>(ah + 0 * 2048) = bmm_unpack8s(w[h].x, s2[h]);
                        *reinterpret_cast<uint4*>(ah + 1 * 2048) = bmm_unpack8s(w[h].y, s2[h]);
                        *reinterpret_cast<uint4*>(ah + 2 * 2048) = bmm_unpack8s(w[h].z, s2[h]);
                        *reinterpret_cast<uint4*>(ah + 3 * 2048) = bmm_unpack8s(w[h].w, s2[h]);
                    } else {
                        *reinterpret_cast<uint4*>(ah + 0 * 2048) = bmm_unpack8(w[h].x);
                        *reinterpret_cast<uint4*>(ah + 1 * 2048) = bmm_unpack8(w[h].y);
                        *reinterpret_cast<uint4*>(ah + 2 * 2048) = bmm_unpack8(w[h].z);
                        *reinterpret_cast<uint4*>(ah + 3 * 2048) = bmm_unpack8(w[h].w);
                    }
                }
                if (S && ((b + BMM_SB) & 3) == 0) sw = sw_next;
                fence_proxy_async();  // generic smem writes -> async-proxy MMA reads
                asm volatile("bar.sync 2, 128;" ::: "memory");
                if (j == 0) {
                    bmm_arrive(&afull[s]);
                    bmm_arrive(&empty[s]);
                    BMM_TR(4, t)
                }
            }
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        pdl_wait();  // the sequence scales and the sums it adds into follow the previous kernel
        // the sequences' scales in shared memory: a global load after the
        // output stores (which may alias it) would wait for each of them
        if (tid - 192 < BMM_MAXN) s_xs[tid - 192] = tid - 192 < (int)N ? a.xs[tid - 192] : 0.0f;
        asm volatile("bar.sync 3, 256;" ::: "memory");
        const uint32_t e = warp - 6;
        const uint32_t q4 = warp & 3;                // TMEM lane quadrant of this warp
        const uint32_t j = q4 * 32 + lane;           // column within the tile
        const uint32_t half = e >> 2;                // sequences [half * N/2, +N/2)
        const uint32_t nh = N / 2;                   // 16 or 32
        uint32_t t = 0, it = 0;
        for (uint32_t item = blockIdx.x; item < nitems; item += G) {
            const uint32_t tile = item / ksplit, kc = item % ksplit;
            const uint32_t b0 = kc * cbk, b1 = min(b0 + cbk, nblk);
            uint32_t lt;
            const BmmPart& P = bmm_part(a, tile, lt);
            const uint32_t col = lt * BMM_M + j;
            // output addresses in registers: P lives in parameter space behind a
            // generic pointer, and a load through it after a store would wait
            // for that store
            const size_t cstride = P.cols;
            float* dst = raw ? P.part + (size_t)kc * nreal * cstride + col : P.out + col;
            long long* accp = P.acc + col;
            // sequences n0 .. n0 + 15 of this thread's column: x 2^e, then out
            // (raw: this K range's partial, which the consumer adds in order;
            // one K range: the result) or the fixed-point sums
            auto emit16 = [&](uint32_t n0, const float* val) {
                if (raw || ksplit == 1) {
                    // 4 x 4 transposes within groups of four lanes (two
                    // butterfly stages of shuffles), so each lane stores a
                    // float4: 4 columns of one sequence. A warp store is then
                    // 512 B of 4 rows instead of 128 B of one, a quarter of
                    // the store instructions.
                    const bool b0 = lane & 1, b1 = (lane & 2) != 0;
                    const uint32_t row = (b1 ? 2u : 0u) + (b0 ? 1u : 0u);
                    float* colbase = dst - lane + (lane & ~3u);  // this lane's 4 columns, sequence 0
#pragma unroll
                    for (int r = 0; r < 16; r += 4) {
                        const float v0 = val[r] * s_xs[n0 + r], v1 = val[r + 1] * s_xs[n0 + r + 1];
                        const float v2 = val[r + 2] * s_xs[n0 + r + 2], v3 = val[r + 3] * s_xs[n0 + r + 3];
                        const float a0 = __shfl_xor_sync(0xffffffffu, b0 ? v0 : v1, 1);
                        const float a1 = __shfl_xor_sync(0xffffffffu, b0 ? v2 : v3, 1);
                        const float2 p0 = b0 ? make_float2(a0, v1) : make_float2(v0, a0);  // sequence r + b0
                        const float2 p1 = b0 ? make_float2(a1, v3) : make_float2(v2, a1);  // sequence r + 2 + b0
                        const float2 sd = b1 ? p0 : p1;
                        const float rx = __shfl_xor_sync(0xffffffffu, sd.x, 2), ry = __shfl_xor_sync(0xffffffffu, sd.y, 2);
                        const float4 o4 = b1 ? make_float4(rx, ry, p1.x, p1.y) : make_float4(p0.x, p0.y, rx, ry);
                        const uint32_t n = n0 + r + row;
                        if (n < nreal) *reinterpret_cast<float4*>(colbase + (size_t)n * cstride) = o4;
                    }
                    return;
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t n = n0 + i;
                    if (n < nreal) {
                        const float f = val[i] * s_xs[n] * 4294967296.0f;
                        long long fx = 0;
                        if (fabsf(f) < 9.2e18f) fx = __float2ll_rn(f);
                        else atomicOr(err, TK_ERR_RANGE);
                        asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(accp + (size_t)n * cstride),
                                     "l"(fx) : "memory");
                    }
                }
            };
            if (S) {
                // one read of the item's accumulator, 16 sequences at a time:
                // hi sums + lo sums, out; the slot is released after the last
                const uint32_t q = it & 1;
                bmm_wait_warp(&dfull[q], (it >> 1) & 1, err);
                tc_fence_after();
                const uint32_t taddr = tmem + ((q4 * 32) << 16) + q * 2 * N + half * nh;
                for (uint32_t c = 0; c < nh; c += 16) {
                    float hi[16], lo[16];
                    tmem_ld16(taddr + c, hi);
                    tmem_ld16(taddr + N + c, lo);
#pragma unroll
                    for (int i = 0; i < 16; ++i) hi[i] += lo[i];
                    emit16(half * nh + c, hi);
                }
                tc_fence_before();
                asm volatile("bar.sync 3, 256;" ::: "memory");
                if (tid == 192) bmm_arrive(&dempty[q]);
                ++it;
            } else {
                float sum[BMM_MAXN / 2];
#pragma unroll
                for (int n = 0; n < BMM_MAXN / 2; ++n) sum[n] = 0.0f;
                // scales one quad ahead: the scale plane is read from HBM
                const uint2* scp = P.sc + col;
                const size_t scs = P.cols;
                uint2 sw = __ldg(scp + (size_t)(b0 >> 2) * scs);
                uint2 sw_next = b0 + 4 < b1 ? __ldg(scp + (size_t)((b0 >> 2) + 1) * scs) : sw;
                for (uint32_t b = b0; b < b1; ++b, ++t) {
                    const uint32_t q = t % BMM_ND;
                    if ((b & 3) == 0 && b != b0) {
                        sw = sw_next;
                        if (b + 4 < b1) sw_next = __ldg(scp + (size_t)((b >> 2) + 1) * scs);
                    }
                    const uint32_t word = (b & 2) ? sw.y : sw.x;
                    const float scale = (b & 1) ? bf16_hi(word) : bf16_lo(word);
                    bmm_wait_warp(&dfull[q], (t / BMM_ND) & 1, err);
                    tc_fence_after();
                    const uint32_t taddr = tmem + ((q4 * 32) << 16) + q * N + half * nh;
                    float v[16];
                    tmem_ld16(taddr, v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) sum[i] = fmaf(scale, v[i], sum[i]);
                    if (nh == 32) {
                        tmem_ld16(taddr + 16, v);
#pragma unroll
                        for (int i = 0; i < 16; ++i) sum[16 + i] = fmaf(scale, v[i], sum[16 + i]);
                    }
                    tc_fence_before();
                    asm volatile("bar.sync 3, 256;" ::: "memory");
                    if (tid == 192) bmm_arrive(&dempty[q]);
                }
                emit16(half * nh, sum);
                if (nh == 32) emit16(half * nh + 16, sum + 16);
            }
        }
    }
    if (tid == 64 + 128) { BMM_TR(5, 1) }
    pdl_launch_dependents();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) { BMM_TR(5, 2) }
    if (warp == 1) {
        tc_fence_after();
        const uint32_t ncols = BMM_ND * N;
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
    }
}


}  // namespace xp
