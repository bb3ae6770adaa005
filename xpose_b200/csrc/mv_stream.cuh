// Streaming int4 matvec: many independent matvecs (same arithmetic as
// kernels/llm_matvec.cl:422-434, one output per column) in ONE persistent
// launch, for the per-token matvec sweep and repeated single matvecs.
//
// The weight planes are the reference's, read in place (decode.cpp:157-229):
// nibbles uint4[(g*nblk + b)*64 + t] for column j = 64g + t, bf16 scales
// uint2[(b/4)*cols + j]. A work item is one 64-column GROUP of one matrix over
// its full K: one warp, lane = columns t and t + 32, so every block of the
// group is one contiguous 1 KB load and every quad of blocks two 256-byte
// scale loads. Each lane keeps two quads (sixteen 16-byte loads) in flight and
// accumulates its columns in registers: no shared-memory reduction, no
// synchronisation. Warps take groups from a global counter, so groups of
// different K (1152 and 6912) balance across the SMs. The activation arrives
// as limbs (xq.cuh), prepared once per distinct vector; each block's limbs
// serve two columns.
#pragma once
#include "common.cuh"
#include "xq.cuh"

namespace xp {

struct MvsJob {
    const uint4* wq;
    const uint2* sc;
    float* out;
    float* part;        // ksplit > 1: [groups][ksplit][64] chunk partials
    uint32_t* arrive;   // ksplit > 1: [groups] chunks done (reset by the last)
    uint32_t nblk;      // rows / 32 (a multiple of 4)
    uint32_t cols;      // a multiple of 64
    uint32_t strip0;    // first work item of this job in the plan
    uint32_t xoff;      // first block of this job's activation limbs
    uint32_t ksplit;    // K chunks per group
    uint32_t cb;        // blocks per chunk (a multiple of 4)
};

struct MvsArgs {
    const MvsJob* jobs;
    const XBlk* xq;     // limbs of every distinct activation
    uint32_t njobs;
    uint32_t nstrips;   // work items (group x K chunk) over all jobs
    uint32_t nxq;       // blocks in xq
    uint32_t* next;     // group counter, zero at launch
};
constexpr uint32_t MVS_SMEM_X_MAX = 64 * 1024;  // limbs staged in shared memory up to this size

constexpr int MVS_THREADS = 256;
constexpr uint32_t MVS_MAXJOBS = 512;
constexpr uint32_t MVS_CHUNK = 36;  // target K blocks per work item

// One quad (four blocks) of a lane's two columns (t and t + 32 of a group):
// nibbles and the scale words.
struct MvsQuad {
    uint4 w0[4], w1[4];
    uint2 s0, s1;
};
XP_DEV void mvs_load(MvsQuad& q, const uint4* wp, const uint2* sp, uint32_t quad, uint32_t cols) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        q.w0[i] = __ldg(wp + (size_t)(4 * quad + i) * 64);
        q.w1[i] = __ldg(wp + (size_t)(4 * quad + i) * 64 + 32);
    }
    q.s0 = __ldg(sp + (size_t)quad * cols);
    q.s1 = __ldg(sp + (size_t)quad * cols + 32);
}
XP_DEV void mvs_quad(const MvsQuad& q, const XBlk* xq, uint32_t quad, float& acc0, float& acc1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const XBlk& X = xq[4 * quad + i];
        const int4* xw = reinterpret_cast<const int4*>(X.w);
        int4 l[6];
#pragma unroll
        for (int r = 0; r < 6; ++r) l[r] = xw[r];
        const int2 bf = *reinterpret_cast<const int2*>(&X.bias);
        const int d0 = xq_dot(q.w0[i], l, bf.x);
        const int d1 = xq_dot(q.w1[i], l, bf.x);
        const uint32_t sw0 = i < 2 ? q.s0.x : q.s0.y, sw1 = i < 2 ? q.s1.x : q.s1.y;
        const float f = __int_as_float(bf.y);
        acc0 = fmaf((float)d0, f * ((i & 1) ? bf16_hi(sw0) : bf16_lo(sw0)), acc0);
        acc1 = fmaf((float)d1, f * ((i & 1) ? bf16_hi(sw1) : bf16_lo(sw1)), acc1);
    }
}

// Work item: one 64-column group of one matrix over its full K (a warp; lane
// owns columns t and t + 32, so a block is one contiguous 1 KB load).
// Activation limbs live in shared memory (copied once per CTA) when they fit,
// else they are read through L1.
template <bool SMEM_X>
__global__ void __launch_bounds__(MVS_THREADS, 2) mv_stream_kernel(const MvsArgs a) {
    __shared__ MvsJob sj[MVS_MAXJOBS];
    extern __shared__ __align__(16) unsigned char mvs_dyn[];
    for (uint32_t i = threadIdx.x; i < a.njobs; i += MVS_THREADS) sj[i] = a.jobs[i];
    // the limb kernel (launched just before, programmatic serialization) has
    // written the limbs and zeroed the counter once this returns
    pdl_wait();
    const XBlk* xbase = a.xq;
    if (SMEM_X) {
        int4* dst = reinterpret_cast<int4*>(mvs_dyn);
        const int4* src = reinterpret_cast<const int4*>(a.xq);
        for (uint32_t i = threadIdx.x; i < a.nxq * 8; i += MVS_THREADS) dst[i] = src[i];
        xbase = reinterpret_cast<const XBlk*>(mvs_dyn);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    uint32_t s = 0;
    if (lane == 0) s = atomicAdd(a.next, 1u);
    s = __shfl_sync(0xffffffffu, s, 0);
    while (s < a.nstrips) {
        uint32_t sn = 0;
        if (lane == 0) sn = atomicAdd(a.next, 1u);  // next group, fetched while this one streams
        uint32_t lo = 0, hi = a.njobs - 1;
        while (lo < hi) {
            const uint32_t mid = (lo + hi + 1) >> 1;
            if (sj[mid].strip0 <= s) lo = mid;
            else hi = mid - 1;
        }
        const MvsJob& J = sj[lo];
        const uint32_t item = s - J.strip0;
        const uint32_t g = J.ksplit > 1 ? item / J.ksplit : item;
        const uint32_t kc = item - g * J.ksplit;
        const uint32_t b0 = kc * J.cb;
        const uint32_t nb = min(J.cb, J.nblk - b0);
        const XBlk* xq = xbase + J.xoff + b0;
        const uint4* wp = J.wq + ((size_t)g * J.nblk + b0) * 64 + lane;
        const uint2* sp = J.sc + (size_t)(b0 >> 2) * J.cols + (size_t)g * 64 + lane;
        const uint32_t nq = nb >> 2;
        float acc0 = 0.0f, acc1 = 0.0f;
        MvsQuad qa, qb;
        mvs_load(qa, wp, sp, 0, J.cols);
        if (nq > 1) mvs_load(qb, wp, sp, 1, J.cols);
#pragma unroll 1
        for (uint32_t q = 0; q < nq; q += 2) {
            mvs_quad(qa, xq, q, acc0, acc1);
            if (q + 2 < nq) mvs_load(qa, wp, sp, q + 2, J.cols);
            if (q + 1 < nq) {
                mvs_quad(qb, xq, q + 1, acc0, acc1);
                if (q + 3 < nq) mvs_load(qb, wp, sp, q + 3, J.cols);
            }
        }
        if (J.ksplit == 1) {
            J.out[(size_t)g * 64 + lane] = acc0;
            J.out[(size_t)g * 64 + lane + 32] = acc1;
        } else {
            // chunk partials; the last chunk of the group to finish adds them
            // in chunk order (deterministic) and resets the group's counter
            float* pp = J.part + ((size_t)g * J.ksplit + kc) * 64;
            pp[lane] = acc0;
            pp[lane + 32] = acc1;
            __threadfence();
            uint32_t old = 0;
            if (lane == 0) old = atomicAdd(&J.arrive[g], 1u);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == J.ksplit - 1) {
                __threadfence();
                const float* gp = J.part + (size_t)g * J.ksplit * 64;
                float t0 = 0.0f, t1 = 0.0f;
                for (uint32_t k = 0; k < J.ksplit; ++k) {
                    t0 += __ldcg(gp + k * 64 + lane);
                    t1 += __ldcg(gp + k * 64 + lane + 32);
                }
                J.out[(size_t)g * 64 + lane] = t0;
                J.out[(size_t)g * 64 + lane + 32] = t1;
                if (lane == 0) J.arrive[g] = 0;
            }
        }
        s = __shfl_sync(0xffffffffu, sn, 0);
    }
}

// Limbs of several activations: source i has nblk[i] blocks at x[i], written
// to xq + off[i]; one warp per block. Also resets the group counter.
struct MvsSrc {
    const float* x;
    uint32_t nblk;
    uint32_t off;
};
__global__ void mv_stream_prep_kernel(const MvsSrc* src, uint32_t nsrc, uint32_t total, XBlk* xq, uint32_t* next) {
    pdl_launch_dependents();
    const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw == 0 && lane == 0) *next = 0;
    if (gw >= total) return;
    uint32_t i = 0;
    while (i + 1 < nsrc && src[i + 1].off <= gw) ++i;
    const uint32_t b = gw - src[i].off;
    xq_prep_block(src[i].x[(size_t)b * 32 + lane], &xq[gw]);
}

}  // namespace xp
