// Device-side building blocks for sm_100a: warp/CTA reductions, the mbarrier
// and bulk-copy (TMA engine) primitives the weight streamer uses, and the
// tagged 64-bit exchange words through which CTAs of the persistent frame
// kernel hand activations to each other without grid barriers.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>
#include <utility>
#include <cuda_runtime.h>

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

// sum_{k < slices} p[k * stride] added in k order (so the result does not depend on how the
// loads are batched), with up to eight L2 loads in flight: the split-K reductions.
__device__ __forceinline__ float sum_slices(const float * p, int slices, std::size_t stride) {
    float acc = 0.f;
    int k = 0;
    for (; k + 8 <= slices; k += 8) {
        float q[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) q[u] = __ldcg(p + static_cast<std::size_t>(k + u) * stride);
#pragma unroll
        for (int u = 0; u < 8; ++u) acc += q[u];
    }
    if (k + 4 <= slices) {
        float q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) q[u] = __ldcg(p + static_cast<std::size_t>(k + u) * stride);
#pragma unroll
        for (int u = 0; u < 4; ++u) acc += q[u];
        k += 4;
    }
    if (k + 2 <= slices) {
        const float q0 = __ldcg(p + static_cast<std::size_t>(k) * stride), q1 = __ldcg(p + static_cast<std::size_t>(k + 1) * stride);
        acc += q0;
        acc += q1;
        k += 2;
    }
    if (k < slices) acc += __ldcg(p + static_cast<std::size_t>(k) * stride);
    return acc;
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

// ---- programmatic dependent launch (sm_90 and later) -------------------------------------------
// A kernel launched with launch_pdl() may start while the kernel before it in the stream is
// still running. griddep_wait() returns once that kernel has completed and its writes are
// visible (at once when there is no such dependency), so every such kernel calls it before
// its first read of another kernel's output; griddep_launch_dependents() lets the next
// kernel start launching (its own wait still holds it until this one completes).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launches kernel<<<grid, block, smem, stream>>>(args...) with programmatic stream
// serialisation allowed, so its launch overlaps the tail of the previous kernel.
template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args &&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
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
__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
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
// The same copy with an L2 eviction policy (from l2_policy) for the lines it reads.
__device__ __forceinline__ void bulk_g2s_hint(void * dst, const void * src, uint32_t bytes, uint64_t * bar, uint64_t policy) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
                 : "memory");
}
// 2-D tiled TMA load of one box of the tensor map at `tmap` (device memory) at element
// coordinates (x inner, y outer); completion counted on `bar`. No multicast. x * element size
// must be a multiple of 16 bytes. The map must have been acquired by this thread
// (tensormap_acquire) after it was last written.
__device__ __forceinline__ void tma_box_2d(void * dst, const void * tmap, int x, int y, uint64_t * bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                     smem_addr(dst)),
                 "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
                 : "memory");
}
// Orders this thread's later tensor-map reads after generic-proxy writes of the map (the host's
// copy before the launch), so a map rewritten at the same address is not read stale.
__device__ __forceinline__ void tensormap_acquire(const void * tmap) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(tmap) : "memory");
}
// L2 policies: keep (evict_last) for data read again soon, stream (evict_first) for data
// read once per frame, so the streamed bytes do not push out the kept ones.
__device__ __forceinline__ uint64_t l2_policy_keep() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_stream() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
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
__device__ __forceinline__ uint64_t ll_load1(const uint64_t * p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Two adjacent exchange words (16-byte aligned) in one load; each 64-bit element is
// single-copy atomic on its own.
__device__ __forceinline__ void ll_load2(const uint64_t * p, uint64_t & a, uint64_t & b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const unsigned * p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u32(unsigned * p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---- cp.async (16-byte, L2-only) ----------------------------------------------------------------

__device__ __forceinline__ void cp_async16(void * smem_dst, const void * gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---- f16 helpers ---------------------------------------------------------------------------------

__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }

// 8 f16 (16 bytes) dotted with 8 f32 as a depth-3 tree (short dependency chain).
__device__ __forceinline__ float dot8h(uint4 w, float4 a, float4 b) {
    const float2 w0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
    const float2 w1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
    const float2 w2 = __half22float2(*reinterpret_cast<const __half2 *>(&w.z));
    const float2 w3 = __half22float2(*reinterpret_cast<const __half2 *>(&w.w));
    const float p0 = fmaf(w0.y, a.y, w0.x * a.x), p1 = fmaf(w1.y, a.w, w1.x * a.z);
    const float p2 = fmaf(w2.y, b.y, w2.x * b.x), p3 = fmaf(w3.y, b.w, w3.x * b.z);
    return (p0 + p1) + (p2 + p3);
}

// 8 f16 (16 bytes) times 8 f32 accumulated on the packed fp32 pipe (FFMA2, sm_100): acc.x takes
// the even products, acc.y the odd ones, each as a chain of fused multiply-adds.
__device__ __forceinline__ float2 dot8h2(uint4 w, float4 a, float4 b, float2 acc) {
    acc = __ffma2_rn(__half22float2(*reinterpret_cast<const __half2 *>(&w.x)), make_float2(a.x, a.y), acc);
    acc = __ffma2_rn(__half22float2(*reinterpret_cast<const __half2 *>(&w.y)), make_float2(a.z, a.w), acc);
    acc = __ffma2_rn(__half22float2(*reinterpret_cast<const __half2 *>(&w.z)), make_float2(b.x, b.y), acc);
    acc = __ffma2_rn(__half22float2(*reinterpret_cast<const __half2 *>(&w.w)), make_float2(b.z, b.w), acc);
    return acc;
}

} // namespace navi::dev
