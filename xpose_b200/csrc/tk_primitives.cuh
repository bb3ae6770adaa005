// Primitives of the persistent token kernel: mbarriers, 1-D bulk async
// copies (cp.async.bulk, no tensor map, no multicast), a bounded grid
// barrier, and bounded waits that report through an error word instead of
// hanging.
#pragma once
#include "common.cuh"

namespace xp {

constexpr uint32_t TK_ERR_ATTN_CHUNK = 1u;   // attention chunk larger than staged
constexpr uint32_t TK_ERR_GRID_BAR = 2u;     // grid barrier wait ran out
constexpr uint32_t TK_ERR_MBAR = 4u;         // bulk-copy wait ran out
constexpr uint32_t TK_ERR_PLAN = 8u;         // a unit did not fit its slot
constexpr uint32_t TK_ERR_RANGE = 16u;       // a K-split sum outside the fixed-point range
constexpr uint32_t TK_ERR_TP_WAIT = 32u;     // a tensor-parallel peer's entry never arrived
constexpr uint32_t TK_ERR_LL_WAIT = 64u;     // a flagged attention partial never arrived
constexpr uint32_t TK_ERR_POS = 128u;        // a device-resident position at or past the KV caches' rows

// A wait of ~1 s on these loops is far beyond any phase (a token is < 1 ms).
constexpr uint32_t TK_SPIN_LIMIT = 1u << 22;

XP_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

XP_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
XP_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
XP_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

XP_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global to this CTA's shared memory, completing on `bar`.
XP_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 prefetch of a global range (16-byte aligned, size a multiple of 16): a
// hint with no effect on what later loads read.
XP_DEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

XP_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with `parity` to complete. On timeout sets the
// error bit and returns (the data is then unspecified, the kernel finishes).
XP_DEV void mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
    uint32_t it = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (++it > TK_SPIN_LIMIT) {
            atomicOr(err, TK_ERR_MBAR);
            return;
        }
    }
}

// Flagged 8-byte words: value in the low half, the writer's flag in the high
// half, stored and loaded as one 64-bit access (single-copy atomic), so a
// reader that sees the expected flag has the value that came with it.
XP_DEV void st_flagged(unsigned long long* p, float v, uint32_t flag) {
    const unsigned long long w = ((unsigned long long)flag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
XP_DEV ulonglong2 ld_flagged2(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
XP_DEV unsigned long long ld_flagged(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
XP_DEV bool flag_is(unsigned long long w, uint32_t flag) { return (uint32_t)(w >> 32) == flag; }
XP_DEV float flag_val(unsigned long long w) { return __uint_as_float((uint32_t)w); }

XP_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Release-add: orders every prior write of the CTA (made visible to this
// thread by the preceding bar.sync) before the increment, at GPU scope.
XP_DEV void red_release_add_u64(uint64_t* p, uint64_t v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

XP_DEV uint64_t ld_acquire_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier over a monotonically increasing arrival counter: the
// caller's k-th barrier of a launch waits for base + k * gridDim.x arrivals.
// One CTA-wide bar.sync orders every thread's writes before thread 0's
// release fence; thread 0's acquire load plus the closing bar.sync orders
// every thread's later reads after the other CTAs' writes.
XP_DEV void grid_barrier(uint64_t* counter, uint64_t target, uint32_t* err) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(reinterpret_cast<unsigned long long*>(counter), 1ull);
        uint32_t it = 0;
        while (ld_acquire_u64(counter) < target) {
            if (++it > TK_SPIN_LIMIT) {
                atomicOr(err, TK_ERR_GRID_BAR);
                break;
            }
        }
        __threadfence();
    }
    __syncthreads();
}

// Failure-path self-test: one thread waits on an mbarrier nothing arrives on
// and on a grid-barrier counter nothing increments, each with `limit` polls;
// both waits give up, record their bits in *err and return, leaving the
// context usable.
__global__ void selftest_wait_kernel(uint64_t* counter, uint32_t* err, uint32_t limit) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_mbar_init();
    uint32_t it = 0;
    while (!mbar_try_wait(&bar, 0)) {
        if (++it > limit) {
            atomicOr(err, TK_ERR_MBAR);
            break;
        }
    }
    it = 0;
    while (ld_acquire_u64(counter) < 1ull) {
        if (++it > limit) {
            atomicOr(err, TK_ERR_GRID_BAR);
            break;
        }
    }
}

}  // namespace xp
