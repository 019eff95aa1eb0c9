// Device-side building blocks for sm_100a: warp/CTA reductions, the mbarrier
// and bulk-copy (TMA engine) primitives the weight streamer uses, and the
// tagged 64-bit exchange words through which CTAs of the persistent frame
// kernel hand activations to each other without grid barriers.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace navi::dev {

// ---- warp / CTA reductions --------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Named barrier over the first `nthreads` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads: every
// thread gets the same answer, so decisions taken on it never diverge.
__device__ __forceinline__ bool named_sync_or(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(pred ? 1u : 0u), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier + bulk copies ----------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Global -> shared bulk copy on the TMA engine; completion is counted on `bar`.
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void * src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---- tagged exchange words --------------------------------------------------------------------
// A value travels as one 64-bit word {f32 bits, u32 tag}; a 64-bit aligned store is
// single-copy atomic, so a reader that sees the expected tag also sees the value it
// was written with. Producers store with relaxed gpu-scope stores; consumers poll with
// relaxed gpu-scope loads (served by L2, never a stale L1 line).

__device__ __forceinline__ void ll_store(uint64_t * p, float v, uint32_t tag) {
    const uint64_t w = (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ll_load(const uint64_t * p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const unsigned * p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u32(unsigned * p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---- f16 helpers ---------------------------------------------------------------------------------

__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }

// 4 f16 (8 bytes) dotted with 4 f32.
__device__ __forceinline__ float dot4h(uint2 w, float4 x) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
    return a.x * x.x + a.y * x.y + b.x * x.z + b.y * x.w;
}

} // namespace navi::dev
