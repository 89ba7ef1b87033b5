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

// A CTA per (kBf16Rows rows, group of kBf16Tokens token columns), a warp per row: lane (j = lane & 7, t = lane >> 3)
// carries partial sum j of token 4 * group + t, a chain over the columns j, j + 8, ... (cols / 8 long, the reference's
// order). Small CTAs, so the rows' chains spread over the SMs. The rows (contiguous) arrive by one bulk copy issued
// before the wait for the previous kernel (weights do not depend on it); the group's activations are staged after it
// transposed - xs[t][j][i] = x[t][8 i + j], each (t, j) run padded by 4 floats - so a lane reads four of its columns
// in one load and the 32 lanes' loads hit distinct banks. Bits as bf16_dot8's. w 16-byte aligned, cols % 32 == 0.
// Dynamic smem: bf16_gemv_smem(cols).
constexpr int kBf16Rows = 4;     // rows (warps) per CTA
constexpr int kBf16Tokens = 4;   // token columns per CTA
__host__ __device__ inline int bf16_run(int cols) { return cols / 8 + 4; }
__host__ __device__ inline size_t bf16_gemv_smem(int cols) {
    return 16 + static_cast<size_t>(kBf16Rows) * cols * 2 + static_cast<size_t>(kBf16Tokens) * 8 * bf16_run(cols) * 4;
}

__global__ void __launch_bounds__(kBf16Rows * 32) k_bf16_gemv(const uint16_t *__restrict__ w, int rows, int cols,
                                                               const float *__restrict__ x, int xstride, int n,
                                                               float *__restrict__ y, int ystride, uint32_t *status) {
    extern __shared__ __align__(16) uint8_t sm[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm);
    uint16_t *ws = reinterpret_cast<uint16_t *>(sm + 16);
    float *xs = reinterpret_cast<float *>(sm + 16 + static_cast<size_t>(kBf16Rows) * cols * 2);
    const int groups = (n + kBf16Tokens - 1) / kBf16Tokens;
    const int r0 = (blockIdx.x / groups) * kBf16Rows, t0 = (blockIdx.x % groups) * kBf16Tokens;
    const int nr = min(kBf16Rows, rows - r0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 7, t = lane >> 3;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
        const uint32_t bytes = static_cast<uint32_t>(nr) * cols * 2;
        mbar_expect_tx(bar, bytes);
        bulk_g2s(ws, w + static_cast<size_t>(r0) * cols, bytes, bar);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int run = bf16_run(cols);
    {   // the group's tokens, transposed (zeros past n): thread i takes float4 column c4 = i, i + blockDim, ... of every
        // token (no division), every load of a batch issued before its stores
        const int c4n = cols / 4;
        for (int c4b = threadIdx.x; c4b < c4n; c4b += blockDim.x * 4) {
            float4 v[kBf16Tokens][4];
#pragma unroll
            for (int tt = 0; tt < kBf16Tokens; ++tt)
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int c4 = c4b + u * blockDim.x;
                    v[tt][u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (c4 < c4n && t0 + tt < n)
                        v[tt][u] = *reinterpret_cast<const float4 *>(x + static_cast<size_t>(t0 + tt) * xstride + 4 * c4);
                }
#pragma unroll
            for (int tt = 0; tt < kBf16Tokens; ++tt)
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int c4 = c4b + u * blockDim.x;
                    if (c4 < c4n) {
                        const int c = 4 * c4;
                        float *d = xs + (tt * 8 + (c & 7)) * run + (c >> 3);   // columns c .. c+3: j = c % 8 .., i = c / 8
                        d[0] = v[tt][u].x;
                        d[run] = v[tt][u].y;
                        d[2 * run] = v[tt][u].z;
                        d[3 * run] = v[tt][u].w;
                    }
                }
        }
    }
    __syncthreads();
    const bool landed = mbar_wait_bounded(bar, 0, status);
    if (landed && warp < nr) {
        const float *xr = xs + (t * 8 + j) * run;
        const uint16_t *wr = ws + static_cast<size_t>(warp) * cols + j;
        float a = 0.0f;
#pragma unroll 8
        for (int i = 0; i < cols / 8; i += 4) {
            const float4 xv = *reinterpret_cast<const float4 *>(xr + i);
            const float w0 = __uint_as_float(static_cast<uint32_t>(wr[8 * i]) << 16);
            const float w1 = __uint_as_float(static_cast<uint32_t>(wr[8 * i + 8]) << 16);
            const float w2 = __uint_as_float(static_cast<uint32_t>(wr[8 * i + 16]) << 16);
            const float w3 = __uint_as_float(static_cast<uint32_t>(wr[8 * i + 24]) << 16);
            a = __fadd_rn(a, __fmul_rn(w0, xv.x));
            a = __fadd_rn(a, __fmul_rn(w1, xv.y));
            a = __fadd_rn(a, __fmul_rn(w2, xv.z));
            a = __fadd_rn(a, __fmul_rn(w3, xv.w));
        }
        // (a lane group of 8 shares t: the shuffles below stay inside it)
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));   // j < 4: a_j + a_{j+4}
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));   // (a0+a4)+(a1+a5), (a2+a6)+(a3+a7)
        a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
        if (j == 0 && t0 + t < n) y[static_cast<size_t>(t0 + t) * ystride + r0 + warp] = a;
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
    for (int e = lane; e < E; e += 32) p[e] = expf_ref(__fsub_rn(logits[e], mx));
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
