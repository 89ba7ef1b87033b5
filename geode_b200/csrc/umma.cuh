// umma.cuh - the fifth-generation tensor core (tcgen05) from inline PTX: shared-memory matrix descriptors, the
// instruction descriptor of the int8 MMA, tensor-memory allocation, the MMA, its commit to an mbarrier, loads from
// tensor memory, the fences between the thread and async proxies, and mbarrier arrivals and bounded waits.
//
// Operand layout used here (the "no swizzle" K-major canonical layout): a core matrix is 8 rows x 16 bytes stored as
// 128 contiguous bytes (row i at +16 i); core matrices next to each other along K are `lbo` bytes apart, along M (or
// N) `sbo` bytes apart. For an int8 MMA of K = 32 a row's 32 bytes are two core-matrix columns.
//
// The descriptor bit layouts (checked on the host against CuTe's own builders by tests/test_umma_desc.py):
//   smem descriptor: start address >> 4 in bits [0, 14), leading byte offset >> 4 in [16, 30), stride byte offset
//   >> 4 in [32, 46), version 1 in [46, 48), base offset 0, lbo mode 0, layout type in [61, 64) (0: no swizzle);
//   instruction descriptor (kind::i8): D format in [4, 6) (2: s32), A format in [7, 10) and B format in [10, 13)
//   (0: u8, 1: s8), A and B K-major (bits 15, 16 zero), N >> 3 in [17, 23), M >> 4 in [24, 29).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace gcu {

__host__ __device__ constexpr uint64_t umma_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu)) | (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1) << 46);
}

// The same for the K-major layout with the 128-byte swizzle (layout type 2): an atom of 8 rows x 128 bytes, the 16-byte
// chunk c of row r stored at chunk c ^ (r % 8); atoms along M (or N) `sbo` bytes apart; the leading byte offset is
// fixed at 16 bytes (one K-atom per operand here). A K step inside the atom advances the start address by its bytes.
__host__ __device__ constexpr uint64_t umma_smem_desc_sw128(uint32_t smem_addr, uint32_t sbo_bytes) {
    return umma_smem_desc(smem_addr, 16, sbo_bytes) | (static_cast<uint64_t>(2) << 61);
}

// int8 x int8 -> s32, both operands K-major; a_signed / b_signed: s8 (else u8)
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N, bool a_signed, bool b_signed) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
           ((static_cast<uint32_t>(N) >> 3) << 17) | ((static_cast<uint32_t>(M) >> 4) << 24);
}

#if defined(__CUDA_ARCH__)

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return smem_addr(p); }

// ---- mbarriers (mbar_init, mbar_expect_tx, mbar_try_wait and the 1-D bulk copy bulk_g2s are common.cuh's; every
// wait here is bounded: after `limit` polls it gives up and returns false)
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// ---- fences
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- tensor memory (one warp allocates for the CTA; the address lands in shared memory)
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D (tensor memory) = A (smem) x B (smem), or D += when accumulate; issued by one thread
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, bool accumulate) {
    // (every output lane enabled: the disable-output-lane mask all zero)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// the mbarrier arrives once every MMA this thread issued before has completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 8 columns of 32 bits: lane i of the warp gets row (taddr's lane + i), columns taddr's column .. + 7
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
// 32 lanes x X columns (X = 4, 8, 16 or 32)
template <int X>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t *v);
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, uint32_t *v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t *v) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t *v) {
    tmem_ld<8>(taddr, v);
    tmem_ld<8>(taddr + 8, v + 8);
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, uint32_t *v) {
    tmem_ld<16>(taddr, v);
    tmem_ld<16>(taddr + 16, v + 16);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

#endif  // __CUDA_ARCH__

}  // namespace gcu
