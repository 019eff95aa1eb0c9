// 5th-generation tensor-core (tcgen05) building blocks for sm_100a: tensor-memory
// allocation, shared-memory matrix descriptors, the f16 MMA with an f32 accumulator in
// tensor memory, its completion commit to an mbarrier, and the tensor-memory loads of
// the epilogue.  One CTA (cta_group::1) throughout.
//
// Operand layout used by every caller: K-major, no swizzle.  A "core matrix" is 8 rows
// of 16 bytes (8 f16) stored as 128 contiguous bytes.  Rows follow one another at a
// 16-byte pitch for the whole tile (stride-dimension offset 128 bytes between groups of
// 8 rows), and the tile's 8-element column groups ("k chunks") are planes `lbo` bytes
// apart (leading-dimension offset).  Because rows are contiguous at a 16-byte pitch, a
// descriptor whose start address is moved by r * 16 bytes describes the same tile
// shifted down by r rows -- the implicit-GEMM convolution uses that for its taps.
#pragma once

#include <cstdint>

namespace navi::umma {

// Matrix descriptor (tcgen05 shared-memory descriptor): start address, leading- and
// stride-dimension byte offsets (all >> 4), descriptor version 1 (bits 46-47), base
// offset 0, legacy LBO mode, layout type 0 = no swizzle (bits 61-63).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t smem_byte_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    return d;
}

// The same for a K-major tile in the 128-byte swizzled layout a TMA load with
// CU_TENSOR_MAP_SWIZZLE_128B writes (rows of 64 f16 = 128 B, 8-row atoms of 1024 B, the
// start 1024-byte aligned): leading offset unused (1), stride offset 1024 B, layout type 2.
// A 16-wide K step inside the atom advances the start address by 32 bytes.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_byte_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor for kind::f16 with f16 A and B (both K-major), f32 accumulate:
// D format f32 (bits 4-5 = 1), A/B format f16 (0), N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---- tensor memory -----------------------------------------------------------------------------
// Whole-warp operations. ncols: a power of two, 32..512.
__device__ __forceinline__ void tmem_alloc(uint32_t * smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- MMA ------------------------------------------------------------------------------------------
// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}
// Arrives once on `bar` when every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
                 : "memory");
}

// ---- TMA --------------------------------------------------------------------------------------
// 2-D tiled load of one box of `tmap` at element coordinates (x inner, y outer) into shared
// memory, completion counted on `bar`. No multicast. x * element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void * dst, const void * tmap, int x, int y, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
        "l"(tmap), "r"(x), "r"(y), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
        : "memory");
}

// ---- epilogue loads -----------------------------------------------------------------------------
// Warp-wide: lane i of warp w (w % 4 = q) receives row 32 q + i, columns col..col+15 of
// the accumulator at taddr (taddr's lane field must be 32 q).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    // the load and its wait in one statement, so no use of r[] can be scheduled between them
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

} // namespace navi::umma
