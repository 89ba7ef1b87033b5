// common.cuh - device helpers shared by the verify-step kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gcu {

constexpr int kBlock = 16;          // values per E4M3 block scale (the engine's q4 block)
constexpr int kMaxTok = 8;          // token columns of one GEMV pass (mma n = 8); the verify step uses up to 5
constexpr uint32_t kBiasBits = 0x4B400000u;   // 1.5 * 2^23: an int32 added here reads back as a float exactly
constexpr float kBiasF = 12582912.0f;

// Error flags a kernel raises in the handle's device status word (never a trap).
enum : uint32_t { kErrWaitTimeout = 1u, kErrBadShape = 2u, kErrBadToken = 4u, kErrUnion = 8u };

// ---------------------------------------------------------------------------------------------- conversions ----
// Two E4M3 bytes (lo, hi halves of a 16-bit value) to two floats: the hardware e4m3x2 -> f16x2 conversion (every
// E4M3 value is exact in f16), then f16 -> f32 (exact).
__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two_bytes) {
    uint32_t h2;
    const uint16_t in = static_cast<uint16_t>(two_bytes);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(in));
    __half2 h = *reinterpret_cast<__half2 *>(&h2);
    return __half22float2(h);
}

// int32 block sum that was accumulated onto kBiasBits -> its exact float value
__device__ __forceinline__ float unbias(int32_t d) { return __fsub_rn(__int_as_float(d), kBiasF); }

// ---------------------------------------------------------------------------------------------- tensor core ----
// D (16x8 s32) = A (16x16 s8, row) * B (16x8 s8, col) + C: the int8 block products of one 16-value block
__device__ __forceinline__ void mma_s8_16816(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t b, const int32_t (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}

// the same with unsigned A (the weight codes as 16 c, 0..240)
__device__ __forceinline__ void mma_u8s8_16816(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t b, const int32_t (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}

// D (16x8 f32) = A (16x16 f16, row) * B (16x8 f16, col) + C
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// ---------------------------------------------------------------------------------------------- mbarrier + bulk copy ----
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// 1-D bulk copy global -> shared, completion counted on bar (16-byte aligned addresses, size a multiple of 16)
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// A bounded wait: false (and the status flag raised) when the copy never lands; the kernel then stops using it.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase, uint32_t *status) {
    for (uint32_t i = 0; i < (1u << 22); ++i)
        if (mbar_try_wait(bar, phase)) return true;
    if (status) atomicOr(status, kErrWaitTimeout);
    return false;
}

// ---------------------------------------------------------------------------------------------- loads ----
__device__ __forceinline__ uint4 ld_shared_v4(const void *p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_addr(p)));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Cephes expf as the engine's fast_exp (engine/src/kernels.hpp:146-163), every operation rounded on its own (no
// contraction), so it gives the CPU's bits.
__device__ __forceinline__ float fast_exp_exact(float x) {
    x = fminf(fmaxf(x, -87.0f), 88.0f);
    const float n = floorf(__fadd_rn(__fmul_rn(x, 1.44269504088896341f), 0.5f));
    float r = __fsub_rn(x, __fmul_rn(n, 0.693359375f));
    r = __fadd_rn(r, __fmul_rn(n, 2.12194440e-4f));
    float p = 1.9875691500e-4f;
    p = __fadd_rn(__fmul_rn(p, r), 1.3981999507e-3f);
    p = __fadd_rn(__fmul_rn(p, r), 8.3334519073e-3f);
    p = __fadd_rn(__fmul_rn(p, r), 4.1665795894e-2f);
    p = __fadd_rn(__fmul_rn(p, r), 1.6666665459e-1f);
    p = __fadd_rn(__fmul_rn(p, r), 5.0000001201e-1f);
    p = __fadd_rn(__fadd_rn(__fmul_rn(__fmul_rn(p, r), r), r), 1.0f);
    uint32_t bits = __float_as_uint(p);
    bits += static_cast<uint32_t>(static_cast<int32_t>(n)) << 23;
    return __uint_as_float(bits);
}
__device__ __forceinline__ float silu_fast_exact(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, fast_exp_exact(-x))); }
// expf rounded once from a double exp: the correctly rounded value in all but vanishingly rare cases (glibc's expf
// is too)
__device__ __forceinline__ float expf_cr(float x) { return static_cast<float>(exp(static_cast<double>(x))); }
__device__ __forceinline__ float sigmoid_cr(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cr(-x))); }
__device__ __forceinline__ float silu_cr(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf_cr(-x))); }

}  // namespace gcu
