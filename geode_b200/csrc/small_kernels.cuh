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

// 32 rows per CTA, 8 lanes (j) per row; every lane carries all n tokens' partial sums (the row's bf16 is read once
// for them), x staged in shared memory. Bits as bf16_dot8's. Dynamic smem: n * cols floats.
__global__ void __launch_bounds__(256) k_bf16_gemv(const uint16_t *__restrict__ w, int rows, int cols,
                                                   const float *__restrict__ x, int xstride, int n, float *__restrict__ y,
                                                   int ystride) {
    extern __shared__ float xs[];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int i = threadIdx.x; i < n * cols; i += blockDim.x) xs[i] = x[static_cast<size_t>(i / cols) * xstride + i % cols];
    __syncthreads();
    const int j = threadIdx.x & 7, r = blockIdx.x * 32 + (threadIdx.x >> 3);
    const bool live = r < rows;
    const uint16_t *wr = w + static_cast<size_t>(live ? r : 0) * cols;
    float a[kMaxTok];
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) a[t] = 0.0f;
#pragma unroll 4
    for (int c = j; c < cols; c += 8) {
        const float wf = __uint_as_float(static_cast<uint32_t>(wr[c]) << 16);
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t)
            if (t < n) a[t] = __fadd_rn(a[t], __fmul_rn(wf, xs[t * cols + c]));
    }
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) {
        if (t >= n) break;
        float v = a[t];
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));   // j < 4: a_j + a_{j+4}
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));   // (a0+a4)+(a1+a5), (a2+a6)+(a3+a7)
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
        if (live && j == 0) y[static_cast<size_t>(t) * ystride + r] = v;
    }
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
    if (lane == 0)
        for (int e = 0; e < E; ++e) sum = __fadd_rn(sum, p[e]);
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
