// small_kernels.cuh - the verify step's small exact pieces: the bf16 GEMV (router, Gated DeltaNet a/b) and the
// router's softmax top-k.
#pragma once

#include "common.cuh"

namespace gcu {

// matvec_rows_bf16_multi (engine/src/kernels.cpp:1449-1518): per (row, token) eight partial sums a[j] over the
// columns j, j+8, ... in order (a separate multiply and add), then ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7)).
// Eight lanes per (row, token); the combine by shuffles (float addition commutes, so the bits are the reference's).
// x [n][cols], y [n][ystride] (y + t * ystride + r). cols % 8 == 0.
__device__ __forceinline__ void bf16_dot8(const uint16_t *__restrict__ w, const float *__restrict__ x, int cols, int j,
                                          float &out) {
    float a = 0.0f;
#pragma unroll 8
    for (int c = j; c < cols; c += 8) {
        const float wf = __uint_as_float(static_cast<uint32_t>(w[c]) << 16);
        a = __fadd_rn(a, __fmul_rn(wf, x[c]));
    }
    a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));   // j < 4: a_j + a_{j+4}
    a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));   // (a0+a4)+(a1+a5), (a2+a6)+(a3+a7)
    a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
    out = a;
}

// kBf16Rows rows per CTA, one warp per row: lane (j = lane & 7, tg = lane >> 3) carries partial sum j of tokens tg and
// tg + 4. The CTA's rows (contiguous) arrive by one bulk copy issued before the wait for the previous kernel (weights do
// not depend on it); x is staged after it, token rows padded by 8 floats (the four tg lanes hit different banks).
// Bits as bf16_dot8's. w 16-byte aligned, cols % 8 == 0. Dynamic smem: bf16_gemv_smem(cols, n).
constexpr int kBf16Rows = 8;
__host__ __device__ inline size_t bf16_gemv_smem(int cols, int n) {
    return 16 + static_cast<size_t>(kBf16Rows) * cols * 2 + static_cast<size_t>(n) * (cols + 8) * 4;
}

__global__ void __launch_bounds__(kBf16Rows * 32) k_bf16_gemv(const uint16_t *__restrict__ w, int rows, int cols,
                                                               const float *__restrict__ x, int xstride, int n,
                                                               float *__restrict__ y, int ystride, uint32_t *status) {
    extern __shared__ __align__(16) uint8_t sm[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm);
    uint16_t *ws = reinterpret_cast<uint16_t *>(sm + 16);
    float *xs = reinterpret_cast<float *>(sm + 16 + static_cast<size_t>(kBf16Rows) * cols * 2);
    const int r0 = blockIdx.x * kBf16Rows, nr = min(kBf16Rows, rows - r0);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
        const uint32_t bytes = static_cast<uint32_t>(nr) * cols * 2;
        mbar_expect_tx(bar, bytes);
        bulk_g2s(ws, w + static_cast<size_t>(r0) * cols, bytes, bar);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int xs_stride = cols + 8;
    {   // (loads issued in batches before their stores: one round trip per batch, not per load)
        constexpr int kB = 8;
        const int items = n * (cols / 4);
        for (int base = threadIdx.x; base < items; base += blockDim.x * kB) {
            float4 v[kB];
#pragma unroll
            for (int u = 0; u < kB; ++u) {
                const int i = base + u * blockDim.x;
                if (i < items)
                    v[u] = *reinterpret_cast<const float4 *>(x + static_cast<size_t>(i / (cols / 4)) * xstride + 4 * (i % (cols / 4)));
            }
#pragma unroll
            for (int u = 0; u < kB; ++u) {
                const int i = base + u * blockDim.x;
                if (i < items) *reinterpret_cast<float4 *>(xs + (i / (cols / 4)) * xs_stride + 4 * (i % (cols / 4))) = v[u];
            }
        }
    }
    __syncthreads();
    const bool landed = mbar_wait_bounded(bar, 0, status);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 7, tg = lane >> 3;
    if (landed && warp < nr) {
        const uint16_t *wr = ws + static_cast<size_t>(warp) * cols;
        const float *x0 = xs + tg * xs_stride, *x1 = xs + (tg + 4) * xs_stride;
        float a0 = 0.0f, a1 = 0.0f;
        if (tg + 4 < n) {
#pragma unroll 8
            for (int c = j; c < cols; c += 8) {
                const float wf = __uint_as_float(static_cast<uint32_t>(wr[c]) << 16);
                a0 = __fadd_rn(a0, __fmul_rn(wf, x0[c]));
                a1 = __fadd_rn(a1, __fmul_rn(wf, x1[c]));
            }
        } else if (tg < n) {
#pragma unroll 8
            for (int c = j; c < cols; c += 8) {
                const float wf = __uint_as_float(static_cast<uint32_t>(wr[c]) << 16);
                a0 = __fadd_rn(a0, __fmul_rn(wf, x0[c]));
            }
        }
        // (a lane group of 8 shares tg: the shuffles below stay inside it)
        a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 4));   // j < 4: a_j + a_{j+4}
        a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 1));   // (a0+a4)+(a1+a5), (a2+a6)+(a3+a7)
        a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
        a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 4));
        a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
        a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
        if (j == 0) {
            if (tg < n) y[static_cast<size_t>(tg) * ystride + r0 + warp] = a0;
            if (tg + 4 < n) y[static_cast<size_t>(tg + 4) * ystride + r0 + warp] = a1;
        }
    }
    if (!landed) mbar_wait_bounded(bar, 0, nullptr);   // (the copy may still land: not before the CTA ends)
}

// route_topk (engine/src/model.cpp:4021-4065) for one token row, by one warp: softmax (max, exp, a float sum in
// expert order, division), the K largest probabilities (ties: the lower index), weights p / (their sum in pick
// order). exp: correctly rounded (glibc's expf is, but for vanishingly rare cases). p: scratch of E floats.
__device__ inline void route_row(const float *__restrict__ logits, int E, int K, float *p, int *ids, float *weights) {
    const int lane = threadIdx.x & 31;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, logits[e]);
    mx = warp_max(mx);
    for (int e = lane; e < E; e += 32) p[e] = expf_cr(__fsub_rn(logits[e], mx));
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) {   // in expert order; the loads four at a time, issued ahead of the adds
        int e = 0;
        if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
            const float4 *p4 = reinterpret_cast<const float4 *>(p);
#pragma unroll 4
            for (; e + 4 <= E; e += 4) {
                const float4 v = p4[e >> 2];
                sum = __fadd_rn(sum, v.x);
                sum = __fadd_rn(sum, v.y);
                sum = __fadd_rn(sum, v.z);
                sum = __fadd_rn(sum, v.w);
            }
        }
        for (; e < E; ++e) sum = __fadd_rn(sum, p[e]);
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
    __syncwarp();
    for (int e = lane; e < E; e += 32) p[e] = __fdiv_rn(p[e], sum);
    __syncwarp();
    float top = 0.0f;
    uint32_t taken = 0;       // bit s: expert lane + 32 s taken
    for (int k = 0; k < K; ++k) {
        float best = -1.0f;
        int bi = 0x7fffffff;
        for (int s = 0, e = lane; e < E; ++s, e += 32)
            if (!((taken >> s) & 1) && (p[e] > best || (p[e] == best && e < bi))) best = p[e], bi = e;
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) best = ob, bi = oi;
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        if (lane == 0) {
            ids[k] = bi;
            top = __fadd_rn(top, best);
        }
    }
    __syncwarp();
    if (lane == 0 && weights)
        for (int k = 0; k < K; ++k) weights[k] = __fdiv_rn(p[ids[k]], top);
}

// one warp per token row; p scratch in shared memory (E floats per warp)
__global__ void k_route_topk(const float *__restrict__ logits, int n, int E, int K, int *__restrict__ ids,
                             float *__restrict__ weights) {
    extern __shared__ float psm[];
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int t = blockIdx.x * nw + warp; t < n; t += gridDim.x * nw)
        route_row(logits + static_cast<size_t>(t) * E, E, K, psm + warp * E, ids + static_cast<size_t>(t) * K,
                  weights + static_cast<size_t>(t) * K);
}

}  // namespace gcu
