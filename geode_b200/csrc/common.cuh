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
// The reference's float exp is glibc's expf (std::exp on a float, in route_topk's softmax, the Sampler's weights, the
// Gated DeltaNet's gates, silu and sigmoid). glibc's expf is not correctly rounded: a double exp rounded to float
// differs from it on 170 648 of the 2^32 inputs. expf_ref restates glibc's algorithm instead (the ARM
// optimized-routines expf by Szabolcs Nagy, in glibc since 2.27): x * 32/ln2 = k + r with k the nearest integer,
// 2^(k/32) from a 32-entry table of 2^(i/32) (each entry the double nearest 2^(i/32), its exponent field less i << 47,
// computed to 80 digits for this file), 2^(r/32) by a cubic in double precision, the product rounded once to float;
// the multiply-adds fused, as in glibc's FMA build. It equals glibc's expf on all 2^32 inputs (checked on the host and
// on the device against the host's glibc by the tests).
// (global memory read through L1, not __constant__: the lanes of a warp index it with different k, which the constant
// cache would serve one address at a time)
__device__ const uint64_t kExp2Table[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};
__device__ __forceinline__ float expf_ref(float x) {
    const uint32_t ux = __float_as_uint(x);
    if (((ux >> 20) & 0x7ffu) >= 0x42bu) {   // |x| >= 88: the ends of the range
        if (ux == 0xff800000u) return 0.0f;                  // -inf
        if (((ux >> 20) & 0x7ffu) >= 0x7f8u) return __fadd_rn(x, x);   // +inf, NaN
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);       // overflows
        if (x < -0x1.9fe368p6f) return 0.0f;                             // underflows to zero
    }
    constexpr double kInvLn2x32 = 0x1.71547652b82fep+0 * 32.0;
    constexpr double kShift = 0x1.8p+52;   // (adding it rounds to an integer in the low mantissa bits)
    constexpr double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0, c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0,
                     c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = static_cast<double>(x);
    double kd = __fma_rn(kInvLn2x32, xd, kShift);
    const uint64_t ki = static_cast<uint64_t>(__double_as_longlong(kd));
    kd = __dsub_rn(kd, kShift);
    const double r = __fma_rn(kInvLn2x32, xd, -kd);
    const double s = __longlong_as_double(static_cast<long long>(__ldg(&kExp2Table[ki & 31u]) + (ki << 47)));
    const double z = __fma_rn(c0, r, c1);
    const double r2 = __dmul_rn(r, r);
    const double y = __fma_rn(z, r2, __fma_rn(c2, r, 1.0));
    return __double2float_rn(__dmul_rn(y, s));
}
__device__ __forceinline__ float sigmoid_ref(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_ref(-x))); }
__device__ __forceinline__ float silu_ref(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf_ref(-x))); }

}  // namespace gcu
