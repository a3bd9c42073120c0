// sm100.cuh -- thin inline-PTX wrappers for the sm_100a features the
// kernels use: mbarriers, TMA tile loads (no multicast), programmatic
// dependent launch, and bounded waits that report instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kllm {

// Status bits a kernel leaves in the context's device status word.
enum : int {
    ST_WAIT_TIMEOUT = 1,   // an mbarrier wait gave up
    ST_BAD_TOKEN = 2,      // a token id outside the vocabulary
};

// Upper bound for any single wait (ns of %globaltimer).  A TMA tile lands
// in microseconds; this only ends a wait that can never complete.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// 16-byte asynchronous global -> shared copy (no register staging) and its
// completion, for small descriptors a warp prefetches.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// `count` arrivals at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar`; false (and ST_WAIT_TIMEOUT in *status)
// when it did not complete within `limit` ns.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *status,
                                          unsigned long long limit = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > limit) {
            if (status) atomicOr(status, ST_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

// 2-D TMA tile load into shared memory, completion counted on `bar`.
// c0 is the innermost (column) coordinate; c0 * element size must be a
// multiple of 16 bytes (the callers only pass multiples of 8 uint16).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// 1-D bulk copy global -> shared (no multicast); dst, src 16-byte aligned,
// bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk copy with an L2 eviction hint (policy from l2_evict_first()).
__device__ __forceinline__ void bulk_load_hint(void *dst, const void *src, uint32_t bytes,
                                               uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Bring a line into L2 ahead of its use, kept there in preference to
// streamed data.
__device__ __forceinline__ void prefetch_l2_keep(const void *p) {
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}

// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes a
// multiple of 16); no completion to wait for.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Bring the line holding p into L2 (normal eviction priority).
__device__ __forceinline__ void prefetch_l2_line(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// L2 policy for data read once (streamed weights): evict first.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Ordered sum of T <= 8 chunk partials p[0], p[stride], ... written by
// other CTAs: all loads are issued before the adds (a loop bounded by a
// runtime T would wait one memory round trip per partial), then added in
// chunk order -- the reference's reduction (_tape_runner.c:646-662).
__device__ __forceinline__ float sum_parts(const float *p, size_t stride, int T) {
    float v[8];
#pragma unroll
    for (int t = 0; t < 8; t++) v[t] = t < T ? __ldcg(p + t * stride) : 0.f;
    float a = v[0];
#pragma unroll
    for (int t = 1; t < 8; t++)
        if (t < T) a = __fadd_rn(a, v[t]);
    return a;
}

// Programmatic dependent launch: let the next kernel in the stream start
// its independent prologue, and wait for the previous kernel's results.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

}  // namespace kllm
