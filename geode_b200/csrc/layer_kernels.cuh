// layer_kernels.cuh - the verify step's per-layer kernels besides the weight GEMVs: the embedding, the residual
// norms with their int8 quantization, the Gated DeltaNet recurrence, gated attention over the int8 KV cache, the
// router's top-k with the union of the picked experts, and the MoE combine.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "q4_gemv.cuh"
#include "small_kernels.cuh"

namespace gcu {

namespace cg = cooperative_groups;

// ------------------------------------------------------------------------------------------- embedding ----
// x[t] = dequant_row(embed, toks[t]) (engine/src/pack.cpp:353-363, engine/src/kernels.cpp:1214-1228) from the
// pack-layout table; a token out of range raises kErrBadToken and leaves zeros.
__global__ void k_embed(const uint8_t *__restrict__ table, int64_t vocab, int H, float global, const int *__restrict__ toks,
                        int n, float *__restrict__ x, uint32_t *status) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const size_t rb = static_cast<size_t>(H / 16) * 9;
    const int t = blockIdx.y;
    if (t >= n) return;
    const int tok = toks[t];
    const bool ok = tok >= 0 && tok < vocab;
    if (!ok && threadIdx.x == 0 && blockIdx.x == 0) atomicOr(status, kErrBadToken);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) {
        float v = 0.0f;
        if (ok) {
            const uint8_t *row = table + static_cast<size_t>(tok) * rb;
            const uint8_t byte = row[i / 2];
            const int c = (i & 1) ? (byte >> 4) : (byte & 15);
            const int level = c < 8 ? 2 * c + 1 : -(2 * (c - 8) + 1);
            const float e4 = e4m3x2_to_float2(row[H / 2 + i / 16]).x;
            v = __fmul_rn(__fmul_rn(static_cast<float>(level), 1.0f), __fmul_rn(e4, global));
        }
        x[static_cast<size_t>(t) * H + i] = v;
    }
}

// ------------------------------------------------------------------------------------------- norm + quantize ----
// Per token (one CTA each, kNormThreads): h = x * (1 / sqrt(ss / H + eps)) * (1 + w), ss the sum of squares in double
// (engine/src/kernels.cpp:1520-1529); then h quantized per 16 values (quantize_activation). hf may be NULL.
// Optionally first x += gs * shared + sum_k w_k * y_k (the MoE combine). A thread holds the values
// tid + k * kNormThreads (k < kNormPer) in registers from load to store; the norm weights are read before the wait
// for the previous kernel (they do not depend on it). H <= kNormThreads * kNormPer.
constexpr int kNormThreads = 512, kNormPer = 8;

struct NormArgs {
    float *x;                 // [n][H] residual
    const float *w;           // norm weight [H]
    float eps;
    int H, n;
    float *hf;                // [n][H] or NULL
    int8_t *q;                // [n][ostride]: row t's H values at q + t * ostride
    float *scale;             // [n][ostride / 16]
    int32_t *bsum;
    int ostride;              // the output rows' width (H, or wider: one part of a wider row); 0 = H
    // the MoE combine, when sh != NULL: x += gs[t] * sh[t] + sum_k w[t][k] * eout[t*K + k] (rank order)
    const float *sh, *gs, *eout, *wk;
    int K;
    float *trace_moe;         // [n][H] or NULL: the MoE output (tests)
};

__global__ void __launch_bounds__(kNormThreads) k_norm_quant(NormArgs a) {
    __shared__ double red[kNormThreads / 32];
    const int tid = threadIdx.x, H = a.H;
    float wv[kNormPer];
#pragma unroll
    for (int k = 0; k < kNormPer; ++k) {
        const int i = tid + k * kNormThreads;
        wv[k] = i < H ? __fadd_rn(1.0f, a.w[i]) : 0.0f;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int t = blockIdx.x;
    if (t >= a.n) return;
    float *xr = a.x + static_cast<size_t>(t) * H;
    float xv[kNormPer];
#pragma unroll
    for (int k = 0; k < kNormPer; ++k) {
        const int i = tid + k * kNormThreads;
        xv[k] = i < H ? xr[i] : 0.0f;
    }
    if (a.sh) {
        // engine/src/model.cpp:4554-4585 then 5363-5365: out = gs * shared; out += w_k * y_k (k in order, w == 0
        // skipped); x += out. Every pick's value loaded before the sum (K <= 8, checked at set-up).
        const float gs = a.gs[t];
        float wk[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) wk[kk] = kk < a.K ? a.wk[t * a.K + kk] : 0.0f;
        // every value of the thread's columns loaded before any store (x, the output, might alias them for all the
        // compiler knows: loads after a store would wait a round trip each)
        float yk[kNormPer][8], shv[kNormPer];
#pragma unroll
        for (int k = 0; k < kNormPer; ++k) {
            const int i = tid + k * kNormThreads;
            shv[k] = i < H ? a.sh[static_cast<size_t>(t) * H + i] : 0.0f;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                yk[k][kk] = kk < a.K && i < H ? a.eout[(static_cast<size_t>(t) * a.K + kk) * H + i] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < kNormPer; ++k) {
            const int i = tid + k * kNormThreads;
            if (i >= H) break;
            float o = __fmul_rn(gs, shv[k]);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                if (kk >= a.K) break;
                if (wk[kk] == 0.0f) continue;
                o = __fadd_rn(o, __fmul_rn(wk[kk], yk[k][kk]));
            }
            if (a.trace_moe) a.trace_moe[static_cast<size_t>(t) * H + i] = o;
            xv[k] = __fadd_rn(xv[k], o);
            xr[i] = xv[k];
        }
    }
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < kNormPer; ++k) ss += static_cast<double>(xv[k]) * xv[k];
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(tot / H), a.eps)));
    float *hf = a.hf ? a.hf + static_cast<size_t>(t) * H : nullptr;
    const int os = a.ostride ? a.ostride : H;
    int8_t *q = a.q + static_cast<size_t>(t) * os;
    float *scale = a.scale + static_cast<size_t>(t) * (os / 16);
    int32_t *bsum = a.bsum + static_cast<size_t>(t) * (os / 16);
    // 16 consecutive values per half-warp
#pragma unroll
    for (int k = 0; k < kNormPer; ++k) {
        const int i = tid + k * kNormThreads;
        if (k * kNormThreads >= H) break;   // (uniform)
        const float h = i < H ? __fmul_rn(__fmul_rn(xv[k], inv), wv[k]) : 0.0f;
        if (hf && i < H) hf[i] = h;
        float amax = fabsf(h);
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float iv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        const int qv = max(-127, min(127, __float2int_rn(__fmul_rn(h, iv))));
        int sq = qv;
        for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (i < H) {
            q[i] = static_cast<int8_t>(qv);
            if ((i & 15) == 0) {
                scale[i / 16] = __fdiv_rn(amax, 127.0f);
                bsum[i / 16] = sq;
            }
        }
    }
}

// ------------------------------------------------------------------------------------------- Gated DeltaNet ----
// Model::gdn (engine/src/model.cpp:3527-3688) after its products, for the n tokens of the batch, as one kernel.
// Grid: nv value heads x S = dv/16 strips, one cluster (S CTAs) per value head; 128 threads per CTA. Thread
// (j = tid / 8, rg = tid % 8) holds column j of the strip's recurrent state, rows 32 m + 4 rg .. 32 m + 4 rg + 3 for
// m < dk / 32 (four float4 per thread at dk = 128), in registers for the whole batch: the eight rg lanes of a column
// cover 128 contiguous bytes per m, so every state and backup store is whole lines. The column sums over rows reduce
// across the rg lanes by shuffles. The state layout: [layer][vh][dv column j][dk row i] (a column contiguous). The
// gated RMSNorm's sum over the head's dv outputs crosses the cluster: every CTA pushes its partial sums into every
// peer's shared memory, and all add them in rank order (identical on every CTA).
// Rollback: after each token t < n-1 the conv and recurrent states are written to backup slot t.
struct GdnArgs {
    const float *proj;    // [n][conv_dim] (qkv product, before the convolution)
    const float *z;       // [n][vd]
    const float *ab;      // [n][2 nv]: a then b
    const float *convw;   // [conv_dim][K]
    const float *A_log, *dt_bias, *gnorm;
    float *conv_st;       // [conv_dim][K-1] (this layer)
    float *state;         // [nv][dv][dk] (this layer)
    float *conv_bk;       // backups: slot t at conv_bk + t * bk_conv_stride (this layer's part)
    float *state_bk;
    size_t bk_conv_stride, bk_state_stride;
    int n, nk, nv, dk, dv, K;
    float eps;
    int8_t *q;            // the core ActSet [n][vd]
    float *scale;
    int32_t *bsum;
    float *core_f;        // [n][vd] or NULL (tests)
};

// The causal depthwise convolution over [state (K-1 earlier inputs) | the n tokens] and silu_fast, for every channel
// (engine/src/model.cpp:3555-3583), one thread per channel: conv outputs [n][conv_dim]; the state after each token
// t < n-1 to backup slot t, the last to the state. (Its own kernel: the q and k channels are read by several value
// heads, so the state may change only after every reader has read it.)
__global__ void k_gdn_conv(GdnArgs a, int conv_dim, float *__restrict__ out) {
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    const int K = a.K;
    // the weights and the state before the wait: written long before the previous kernel (the state by this layer's
    // last step, which every launch since has waited for)
    float w[8], st[8];
    if (ch < conv_dim) {
        for (int k = 0; k < K; ++k) w[k] = a.convw[static_cast<size_t>(ch) * K + k];
        for (int k = 0; k < K - 1; ++k) st[k] = a.conv_st[static_cast<size_t>(ch) * (K - 1) + k];
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    if (ch >= conv_dim) return;
    float ins[kMaxTok];
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t)
        if (t < a.n) ins[t] = a.proj[static_cast<size_t>(t) * conv_dim + ch];
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) {
        if (t >= a.n) break;
        const float in = ins[t];
        float acc = 0.0f;
        for (int k = 0; k < K - 1; ++k) acc = __fadd_rn(acc, __fmul_rn(w[k], st[k]));
        acc = __fadd_rn(acc, __fmul_rn(w[K - 1], in));
        for (int k = 0; k + 1 < K - 1; ++k) st[k] = st[k + 1];
        if (K > 1) st[K - 2] = in;
        out[static_cast<size_t>(t) * conv_dim + ch] = silu_fast_exact(acc);
        if (t + 1 < a.n)
            for (int k = 0; k < K - 1; ++k) a.conv_bk[t * a.bk_conv_stride + static_cast<size_t>(ch) * (K - 1) + k] = st[k];
    }
    for (int k = 0; k < K - 1; ++k) a.conv_st[static_cast<size_t>(ch) * (K - 1) + k] = st[k];
}

template <int DK>
__global__ void __launch_bounds__(128) k_gdn(GdnArgs a) {
    constexpr int M = DK / 32;   // float4 row chunks per thread
    __shared__ __align__(16) float s_q[kMaxTok][DK], s_k[kMaxTok][DK], s_v[kMaxTok][16], s_o[kMaxTok][16];
    __shared__ float s_beta[kMaxTok], s_decay[kMaxTok];
    __shared__ float s_ss[8][kMaxTok];   // [source rank][token]: the cluster's partial sums of squares (S <= 8)
    cg::cluster_group cluster = cg::this_cluster();
    const int S = a.dv / 16;
    const int vh = blockIdx.x / S, s = blockIdx.x % S;
    const int rep = a.nv / a.nk, kh = vh / rep;
    const int kd = a.nk * a.dk, vd = a.nv * a.dv;
    const int tid = threadIdx.x, n = a.n, warp = tid >> 5, lane = tid & 31;
    // (every CTA of the cluster has started before any writes a peer's shared memory: this arrival, waited for below)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    // before the wait, what the previous kernels cannot change: the recurrent state (written by this layer's last
    // step, which every launch since has waited for), the gates' and the norm's weights
    const int j = tid >> 3, rg = tid & 7;
    const int col = s * 16 + j;
    float *Sg = a.state + (static_cast<size_t>(vh) * a.dv + col) * DK + 4 * rg;
    float4 Sr[M];
#pragma unroll
    for (int m = 0; m < M; ++m) Sr[m] = *reinterpret_cast<const float4 *>(Sg + 32 * m);
    const int gt = tid - 96;   // warp 3's lanes t < n: token t's gates
    const bool gate = gt >= 0 && gt < n;
    float nAe = 0.0f, dtb = 0.0f;
    if (gate) {
        nAe = -expf_ref(a.A_log[vh]);
        dtb = a.dt_bias[vh];
    }
    const int jj = lane & 15;
    const float gw = a.gnorm[s * 16 + jj];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    // 1. every load of the previous kernels' outputs at once: this CTA's conv outputs (q and k of key head kh, the
    // strip's v columns; k_gdn_conv, in a.proj) as float4 pieces, the gate inputs, z of the tokens this warp outputs
    const int cd = 2 * kd + vd;
    constexpr int P = 2 * (DK / 4) + 4;   // pieces per token
    constexpr int kB = (kMaxTok * P + 127) / 128;
    float4 v[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
        const int c = tid + u * 128;
        if (c < n * P) {
            const int t = c / P, cc = c % P;
            const float *row = a.proj + static_cast<size_t>(t) * cd;
            const float *src = cc < DK / 4 ? row + kh * DK + 4 * cc
                             : cc < DK / 2 ? row + kd + kh * DK + 4 * (cc - DK / 4)
                                           : row + 2 * kd + vh * a.dv + s * 16 + 4 * (cc - DK / 2);
            v[u] = *reinterpret_cast<const float4 *>(src);
        }
    }
    float av = 0.0f, bv = 0.0f;
    if (gate) {
        av = a.ab[static_cast<size_t>(gt) * 2 * a.nv + vh];
        bv = a.ab[static_cast<size_t>(gt) * 2 * a.nv + a.nv + vh];
    }
    const int zc = vh * a.dv + s * 16 + jj;
    float zv[2] = {0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < 2; ++i)
        if (warp + 4 * i < n) zv[i] = a.z[static_cast<size_t>(warp + 4 * i) * vd + zc];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
        const int c = tid + u * 128;
        if (c < n * P) {
            const int t = c / P, cc = c % P;
            float *dst = cc < DK / 4 ? &s_q[t][4 * cc] : cc < DK / 2 ? &s_k[t][4 * (cc - DK / 4)] : &s_v[t][4 * (cc - DK / 2)];
            *reinterpret_cast<float4 *>(dst) = v[u];
        }
    }
    __syncthreads();
    if (warp == 3) {
        // gates (engine/src/model.cpp:3604-3611): beta = sigmoid(b), decay = exp(-exp(A_log) * softplus(a + dt_bias))
        if (gate) {
            s_beta[gt] = sigmoid_ref(bv);
            const float x = __fadd_rn(av, dtb);
            const float sp = x > 20.0f ? x : static_cast<float>(log1p(static_cast<double>(expf_ref(x))));
            s_decay[gt] = expf_ref(__fmul_rn(nAe, sp));
        }
    } else {
        // 2. q, k L2-normalised over dk (eps 1e-6), q times 1/sqrt(dk): warp w < 3 takes tokens w, w + 3 (q and k
        // together)
        const float qscale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(DK)));
        for (int t = warp; t < n; t += 3) {
            float sq = 0.0f, sk = 0.0f;
            for (int i = lane; i < DK; i += 32) {
                sq = __fadd_rn(sq, __fmul_rn(s_q[t][i], s_q[t][i]));
                sk = __fadd_rn(sk, __fmul_rn(s_k[t][i], s_k[t][i]));
            }
            sq = warp_sum(sq);
            sk = warp_sum(sk);
            const float iq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sq, 1e-6f)));
            const float ik = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sk, 1e-6f)));
            for (int i = lane; i < DK; i += 32) {
                s_q[t][i] = __fmul_rn(__fmul_rn(s_q[t][i], iq), qscale);
                s_k[t][i] = __fmul_rn(s_k[t][i], ik);
            }
        }
    }
    __syncthreads();
    // 3. the delta rule, token by token (engine/src/model.cpp:3501-3524); the row sums as M chains, then the shuffles
    for (int t = 0; t < n; ++t) {
        const float decay = s_decay[t], beta = s_beta[t];
        float4 kv[M], qv[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            kv[m] = *reinterpret_cast<const float4 *>(&s_k[t][32 * m + 4 * rg]);
            qv[m] = *reinterpret_cast<const float4 *>(&s_q[t][32 * m + 4 * rg]);
        }
        float pm[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            Sr[m].x = __fmul_rn(Sr[m].x, decay);
            Sr[m].y = __fmul_rn(Sr[m].y, decay);
            Sr[m].z = __fmul_rn(Sr[m].z, decay);
            Sr[m].w = __fmul_rn(Sr[m].w, decay);
            pm[m] = __fmaf_rn(Sr[m].w, kv[m].w, __fmaf_rn(Sr[m].z, kv[m].z, __fmaf_rn(Sr[m].y, kv[m].y, __fmul_rn(Sr[m].x, kv[m].x))));
        }
        float mem = pm[0];
#pragma unroll
        for (int m = 1; m < M; ++m) mem = __fadd_rn(mem, pm[m]);
        mem += __shfl_xor_sync(0xffffffffu, mem, 1);
        mem += __shfl_xor_sync(0xffffffffu, mem, 2);
        mem += __shfl_xor_sync(0xffffffffu, mem, 4);
        const float delta = __fmul_rn(__fsub_rn(s_v[t][j], mem), beta);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            Sr[m].x = __fmaf_rn(kv[m].x, delta, Sr[m].x);
            Sr[m].y = __fmaf_rn(kv[m].y, delta, Sr[m].y);
            Sr[m].z = __fmaf_rn(kv[m].z, delta, Sr[m].z);
            Sr[m].w = __fmaf_rn(kv[m].w, delta, Sr[m].w);
            pm[m] = __fmaf_rn(Sr[m].w, qv[m].w, __fmaf_rn(Sr[m].z, qv[m].z, __fmaf_rn(Sr[m].y, qv[m].y, __fmul_rn(Sr[m].x, qv[m].x))));
        }
        float o = pm[0];
#pragma unroll
        for (int m = 1; m < M; ++m) o = __fadd_rn(o, pm[m]);
        o += __shfl_xor_sync(0xffffffffu, o, 1);
        o += __shfl_xor_sync(0xffffffffu, o, 2);
        o += __shfl_xor_sync(0xffffffffu, o, 4);
        if (rg == 0) s_o[t][j] = o;
        if (t + 1 < n) {
            float *bk = a.state_bk + t * a.bk_state_stride + (static_cast<size_t>(vh) * a.dv + col) * DK + 4 * rg;
#pragma unroll
            for (int m = 0; m < M; ++m) *reinterpret_cast<float4 *>(bk + 32 * m) = Sr[m];
        }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) *reinterpret_cast<float4 *>(Sg + 32 * m) = Sr[m];
    __syncthreads();
    // 4. gated RMSNorm over the head's dv outputs: o / rms(o) * w * silu_fast(z) (engine/src/model.cpp:3670-3682).
    // This CTA's sums of squares into slot s of every peer (the peers have started: the arrival above), then one
    // cluster barrier (release / acquire) before the sums are read.
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    if (tid < n) {
        float ss = 0.0f;
        for (int c = 0; c < 16; ++c) ss = __fmaf_rn(s_o[tid][c], s_o[tid][c], ss);
        for (int r = 0; r < S; ++r) cluster.map_shared_rank(&s_ss[0][0], r)[s * kMaxTok + tid] = ss;
    }
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    // one warp per token: 16 values = lanes 0..15 (lanes 16..31 idle copies), quantized as one block
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int t = warp + 4 * i;
        if (t >= n) break;
        float tot = 0.0f;
        for (int r = 0; r < S; ++r) tot = __fadd_rn(tot, s_ss[r][t]);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(a.dv)), a.eps)));
        const float h = __fmul_rn(__fmul_rn(__fmul_rn(s_o[t][jj], inv), gw), silu_fast_exact(zv[i]));
        if (a.core_f && lane < 16) a.core_f[static_cast<size_t>(t) * vd + zc] = h;
        float amax = fabsf(h);
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float iv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        const int qv = max(-127, min(127, __float2int_rn(__fmul_rn(h, iv))));
        int sm = qv;
        for (int o = 8; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
        if (lane < 16) a.q[static_cast<size_t>(t) * vd + zc] = static_cast<int8_t>(qv);
        if (lane == 0) {
            a.scale[static_cast<size_t>(t) * (vd / 16) + zc / 16] = __fdiv_rn(amax, 127.0f);
            a.bsum[static_cast<size_t>(t) * (vd / 16) + zc / 16] = sm;
        }
    }
}

}  // namespace gcu

namespace gcu {

// ------------------------------------------------------------------------------------------- attention ----
// Model::attention's per-head steps (engine/src/model.cpp:3705-3733) and the KV store (3782-3797): queries and keys
// through the zero-centred head RMSNorm and partial rotary (rotate-half over the first rope_dim dims, angle
// pos * inv_freq[i]); keys and values to int8 rows (amax / 127, round half even, engine/src/model.cpp:3767-3774)
// at positions pos .. pos + n - 1. One warp per (token, vector); q rows -> qn [n][nh][hd] f32.
struct AttnPrepArgs {
    const float *qg;     // [n][nh][2 hd] (query | gate)
    const float *kb, *vb;   // [n][nkv * hd]
    const float *q_norm, *k_norm, *inv_freq;
    const int *pos;
    int n, nh, nkv, hd, half;
    float eps;
    float *qn;           // [n][nh][hd]
    int8_t *kc, *vc;     // this layer's cache [ctx][nkv][hd]
    float *ks, *vs;      // [ctx][nkv]
    int ctx;
    uint32_t *status;
};

__global__ void k_attn_prep(AttnPrepArgs a) {
    extern __shared__ float sv[];   // per warp hd floats
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int per = a.nh + 2 * a.nkv;
    const int p0 = *a.pos;
    float *v = sv + warp * a.hd;
    for (int item = blockIdx.x * nw + warp; item < a.n * per; item += gridDim.x * nw) {
        const int t = item / per, w = item % per;
        const int p = p0 + t;
        if (p >= a.ctx) {
            if (lane == 0) atomicOr(a.status, kErrBadShape);
            continue;
        }
        const float *src;
        const float *nw8 = nullptr;
        if (w < a.nh) src = a.qg + (static_cast<size_t>(t) * a.nh + w) * 2 * a.hd, nw8 = a.q_norm;
        else if (w < a.nh + a.nkv) src = a.kb + static_cast<size_t>(t) * a.nkv * a.hd + (w - a.nh) * a.hd, nw8 = a.k_norm;
        else src = a.vb + static_cast<size_t>(t) * a.nkv * a.hd + (w - a.nh - a.nkv) * a.hd;
        for (int i = lane; i < a.hd; i += 32) v[i] = src[i];
        __syncwarp();
        if (nw8) {
            double ss = 0.0;
            for (int i = lane; i < a.hd; i += 32) ss += static_cast<double>(v[i]) * v[i];
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ss / a.hd), a.eps)));
            for (int i = lane; i < a.hd; i += 32) v[i] = __fmul_rn(__fmul_rn(v[i], inv), __fadd_rn(1.0f, nw8[i]));
            __syncwarp();
            for (int i = lane; i < a.half; i += 32) {
                const float f = __fmul_rn(static_cast<float>(p), a.inv_freq[i]);
                float sn, cs;
                sincosf(f, &sn, &cs);
                const float x1 = v[i], x2 = v[i + a.half];
                v[i] = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
                v[i + a.half] = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
            }
            __syncwarp();
        }
        if (w < a.nh) {
            float *dst = a.qn + (static_cast<size_t>(t) * a.nh + w) * a.hd;
            for (int i = lane; i < a.hd; i += 32) dst[i] = v[i];
        } else {
            const bool isk = w < a.nh + a.nkv;
            const int kh = isk ? w - a.nh : w - a.nh - a.nkv;
            float amax = 0.0f;
            for (int i = lane; i < a.hd; i += 32) amax = fmaxf(amax, fabsf(v[i]));
            amax = warp_max(amax);
            const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            int8_t *dst = (isk ? a.kc : a.vc) + (static_cast<size_t>(p) * a.nkv + kh) * a.hd;
            for (int i = lane; i < a.hd; i += 32)
                dst[i] = static_cast<int8_t>(max(-127, min(127, __float2int_rn(__fmul_rn(v[i], inv)))));
            if (lane == 0) (isk ? a.ks : a.vs)[static_cast<size_t>(p) * a.nkv + kh] = __fdiv_rn(amax, 127.0f);
        }
        __syncwarp();
    }
}

// Flash-decoding over the int8 cache (the arithmetic of attend / attend_heads, engine/src/model.cpp:3815-4019,
// regrouped): one CTA (kAttnThreads) per (KV head, chunk of kAttnChunk positions); its rows are the n tokens x G query
// heads sharing the KV head (<= 32 rows, two m16 tiles). The chunk's raw int8 K and V rows arrive kAttnSub positions at
// a time by 16-byte cp.async copies into two stages (the next sub-chunk in flight while the current one is used), are
// widened to f16 in shared memory (int8 is exact in f16: byte | 0x6400 - 1152 with the sign bit flipped), and then:
// scores Q.K^T on the tensor cores (mma.sync f16, f32 accumulate) times (1/sqrt(hd) * k_scale[p]), causal mask
// p <= pos + t, an online softmax, P (times v_scale[p], as the reference folds it into the weights) in f16, O += P.V.
// Partial (O, max, sum) per (token, head, chunk) for k_attn_merge.
constexpr int kAttnSub = 64;
constexpr int kAttnChunk = 256;
constexpr int kAttnThreads = 256;   // 8 warps

struct AttnArgs {
    const float *qn;       // [n][nh][hd]
    const int8_t *kc, *vc; // [ctx][nkv][hd]
    const float *ks, *vs;  // [ctx][nkv]
    const int *pos;
    int n, nh, nkv, ctx;
    float scale;           // 1 / sqrt(hd)
    float *part;           // [n][nh][nchunks][hd + 2]
    int nchunks;
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_addr(p)));
}

// four int8 (a word) -> two f16 pairs, exactly: (b ^ 0x80) placed under the f16 exponent of 1024 gives 1024 + b + 128
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t x = w ^ 0x80808080u;
    lo = __byte_perm(x, 0x64646464u, 0x5140);
    hi = __byte_perm(x, 0x64646464u, 0x7362);
    const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));   // 1152
    const __half2 l = __hsub2(*reinterpret_cast<__half2 *>(&lo), off), h = __hsub2(*reinterpret_cast<__half2 *>(&hi), off);
    lo = *reinterpret_cast<const uint32_t *>(&l);
    hi = *reinterpret_cast<const uint32_t *>(&h);
}

template <int HD>
struct AttnSmem {
    static constexpr int QS = HD + 8;   // f16 row stride (elements) of Q, K, V tiles
    static constexpr int PS = kAttnSub + 8;
    static constexpr size_t q = 0;
    static constexpr size_t k = q + 32 * QS * 2;
    static constexpr size_t v = k + kAttnSub * QS * 2;
    static constexpr size_t pm = v + kAttnSub * QS * 2;
    static constexpr size_t sc = pm + 32 * PS * 2;                 // scores [32][kAttnSub] f32
    static constexpr size_t raw = sc + 32 * kAttnSub * 4;          // [2 stages][K, V][kAttnSub][HD] int8
    static constexpr size_t scl = raw + 2 * 2 * kAttnSub * HD;     // [2 stages][K, V][kAttnSub] f32
    static constexpr size_t rows = scl + 2 * 2 * kAttnSub * 4;     // row_m, row_l, row_f [32] each
    static constexpr size_t total = rows + 3 * 32 * 4;
};
template <int HD>
constexpr size_t attn_smem_bytes() { return AttnSmem<HD>::total; }

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(AttnArgs a) {
    using L = AttnSmem<HD>;
    constexpr int QS = L::QS, PS = L::PS;
    constexpr int NT_O = HD / 64;         // O n-tiles (8 dims) per warp: 8 warps x HD/8 dims
    extern __shared__ __align__(16) uint8_t sm[];
    __half *Qs = reinterpret_cast<__half *>(sm + L::q);
    __half *Ks = reinterpret_cast<__half *>(sm + L::k);
    __half *Vs = reinterpret_cast<__half *>(sm + L::v);
    __half *Ps = reinterpret_cast<__half *>(sm + L::pm);
    float *Ss = reinterpret_cast<float *>(sm + L::sc);
    int8_t *raw = reinterpret_cast<int8_t *>(sm + L::raw);
    float *scl = reinterpret_cast<float *>(sm + L::scl);
    float *row_m = reinterpret_cast<float *>(sm + L::rows);
    float *row_l = row_m + 32;
    float *row_f = row_l + 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
    const int kh = blockIdx.y, chunk = blockIdx.x;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int G = a.nh / a.nkv, rows = a.n * G;
    const int pos = *a.pos, plim = pos + a.n;   // positions < plim exist
    const int c0 = chunk * kAttnChunk;
    if (c0 >= plim) return;
    const int c1 = min(c0 + kAttnChunk, plim);
    // sub-chunk s0's raw rows and scales into stage st (positions >= plim: not copied; widened as zeros below)
    auto fetch = [&](int s0, int st) {
        constexpr int pieces = HD / 16;   // 16-byte pieces of a row
        int8_t *rk = raw + (st * 2 + 0) * kAttnSub * HD, *rv = raw + (st * 2 + 1) * kAttnSub * HD;
        for (int i = tid; i < kAttnSub * pieces; i += kAttnThreads) {
            const int p = i / pieces, c = i % pieces, gp = s0 + p;
            if (gp < plim) {
                const size_t off = (static_cast<size_t>(gp) * a.nkv + kh) * HD + 16 * c;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(rk + p * HD + 16 * c)), "l"(a.kc + off) : "memory");
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(rv + p * HD + 16 * c)), "l"(a.vc + off) : "memory");
            }
        }
        if (tid < 2 * kAttnSub) {
            const int which = tid / kAttnSub, p = tid % kAttnSub, gp = s0 + p;
            if (gp < plim)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(scl + (st * 2 + which) * kAttnSub + p)),
                             "l"((which ? a.vs : a.ks) + static_cast<size_t>(gp) * a.nkv + kh) : "memory");
            else
                scl[(st * 2 + which) * kAttnSub + p] = 0.0f;   // (masked positions: finite scales)
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch(c0, 0);
    // Q rows r = t * G + g -> f16 (rows past n * G zero): thread tid takes dim tid % HD of rows tid / HD + kRp * k,
    // every load issued before the stores; (t, g) stepped along, no index divides by G
    {
        constexpr int kRp = kAttnThreads / HD;   // rows per pass
        constexpr int kQ = 32 / kRp;
        const int d = tid % HD, r0 = tid / HD;
        int t = 0, g = r0;
        while (g >= G) g -= G, ++t;
        float qv[kQ];
#pragma unroll
        for (int k = 0; k < kQ; ++k) {
            const int r = r0 + kRp * k;
            qv[k] = r < rows ? a.qn[(static_cast<size_t>(t) * a.nh + kh * G + g) * HD + d] : 0.0f;
            g += kRp;
            while (g >= G) g -= G, ++t;
        }
#pragma unroll
        for (int k = 0; k < kQ; ++k) Qs[(r0 + kRp * k) * QS + d] = __float2half_rn(qv[k]);
    }
    // the token of each score row this lane holds (rows gid + 8 h + 16 m): its causal limit pos + t
    int lim[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int r = gid + 8 * k;
        int tt = 0;
        while ((tt + 1) * G <= r) ++tt;
        lim[k] = pos + tt;
    }
    if (tid < 32) {
        row_m[tid] = -INFINITY;
        row_l[tid] = 0.0f;
    }
    float o[2][NT_O][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int j = 0; j < NT_O; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[m][j][e] = 0.0f;
    int st = 0;
    for (int s0 = c0; s0 < c1; s0 += kAttnSub, st ^= 1) {
        const bool more = s0 + kAttnSub < c1;
        if (more) fetch(s0 + kAttnSub, st ^ 1);
        if (more) asm volatile("cp.async.wait_group 1;" ::: "memory");
        else asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();   // every thread's copies of this sub-chunk landed; the previous sub-chunk's tiles are free
        {   // widen: 16 int8 of a row per item
            const int8_t *rk = raw + (st * 2 + 0) * kAttnSub * HD, *rv = raw + (st * 2 + 1) * kAttnSub * HD;
            for (int i = tid; i < kAttnSub * HD / 16; i += kAttnThreads) {
                const int p = i / (HD / 16), c = (i % (HD / 16)) * 16;
                uint4 kw = make_uint4(0, 0, 0, 0), vw = kw;
                if (s0 + p < plim) {
                    kw = *reinterpret_cast<const uint4 *>(rk + p * HD + c);
                    vw = *reinterpret_cast<const uint4 *>(rv + p * HD + c);
                }
                uint4 k0, k1, v0, v1;
                i8x4_to_h2x2(kw.x, k0.x, k0.y);
                i8x4_to_h2x2(kw.y, k0.z, k0.w);
                i8x4_to_h2x2(kw.z, k1.x, k1.y);
                i8x4_to_h2x2(kw.w, k1.z, k1.w);
                i8x4_to_h2x2(vw.x, v0.x, v0.y);
                i8x4_to_h2x2(vw.y, v0.z, v0.w);
                i8x4_to_h2x2(vw.z, v1.x, v1.y);
                i8x4_to_h2x2(vw.w, v1.z, v1.w);
                *reinterpret_cast<uint4 *>(Ks + p * QS + c) = k0;
                *reinterpret_cast<uint4 *>(Ks + p * QS + c + 8) = k1;
                *reinterpret_cast<uint4 *>(Vs + p * QS + c) = v0;
                *reinterpret_cast<uint4 *>(Vs + p * QS + c + 8) = v1;
            }
        }
        const float *ksc = scl + (st * 2 + 0) * kAttnSub, *vsc = scl + (st * 2 + 1) * kAttnSub;
        __syncthreads();
        // S = Q K^T: warp w -> positions 8 w .. 8 w + 7 (one n8 tile), both m tiles
        {
            float sacc[2][4] = {};
#pragma unroll
            for (int kk = 0; kk < HD / 32; ++kk) {
                // B: rows = positions (n), k contiguous: matrices (n 0-7, k 0-7), (n 0-7, k 8-15) for two k-steps
                uint32_t bq[4];
                {
                    const int mi = lane >> 3, rr = lane & 7;
                    ldsm_x4(bq, Ks + (8 * warp + rr) * QS + 32 * kk + 8 * mi);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        uint32_t aq[4];
                        const int mi = lane >> 3, rr = lane & 7;
                        const int r = 16 * m + rr + 8 * (mi & 1), k = 32 * kk + 16 * h + 8 * (mi >> 1);
                        ldsm_x4(aq, Qs + r * QS + k);
                        const uint32_t b[2] = {bq[2 * h], bq[2 * h + 1]};
                        mma_f16_16816(sacc[m], aq, b);
                    }
            }
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int r = 16 * m + gid + 8 * (e >> 1), c = 8 * warp + 2 * tig + (e & 1);
                    const int gp = s0 + c;
                    float v = __fmul_rn(sacc[m][e], __fmul_rn(a.scale, ksc[c]));
                    if (r >= rows || gp > lim[2 * m + (e >> 1)] || gp >= plim) v = -INFINITY;
                    Ss[r * kAttnSub + c] = v;
                }
        }
        __syncthreads();
        // online softmax: warp w -> rows 4 w .. 4 w + 3, lanes over 64 columns (2 each)
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int r = 4 * warp + rr;
            const float s_a = Ss[r * kAttnSub + lane], s_b = Ss[r * kAttnSub + lane + 32];
            const float mx = warp_max(fmaxf(s_a, s_b));
            const float m_old = row_m[r], m_new = fmaxf(m_old, mx);
            // (the attention's softmax is not bit-exact across the regrouped blocks anyway: the fast exp)
            const float ea = s_a == -INFINITY ? 0.0f : __expf(s_a - m_new);
            const float eb = s_b == -INFINITY ? 0.0f : __expf(s_b - m_new);
            const float sum = warp_sum(ea + eb);
            const float f = m_old == -INFINITY ? 0.0f : __expf(m_old - m_new);
            Ps[r * PS + lane] = __float2half_rn(__fmul_rn(ea, vsc[lane]));
            Ps[r * PS + lane + 32] = __float2half_rn(__fmul_rn(eb, vsc[lane + 32]));
            if (lane == 0) {
                row_l[r] = __fadd_rn(__fmul_rn(row_l[r], f), sum);
                row_m[r] = m_new;
                row_f[r] = f;
            }
        }
        __syncthreads();
        // O = O * f + P V: warp w -> dims [w * HD/8, (w+1) * HD/8)
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const float f0 = row_f[16 * m + gid], f1 = row_f[16 * m + gid + 8];
#pragma unroll
            for (int j = 0; j < NT_O; ++j) {
                o[m][j][0] *= f0;
                o[m][j][1] *= f0;
                o[m][j][2] *= f1;
                o[m][j][3] *= f1;
            }
        }
#pragma unroll
        for (int kk = 0; kk < kAttnSub / 16; ++kk) {
            uint32_t ap[2][4];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int mi = lane >> 3, rr = lane & 7;
                const int r = 16 * m + rr + 8 * (mi & 1), k = 16 * kk + 8 * (mi >> 1);
                ldsm_x4(ap[m], Ps + r * PS + k);
            }
            if constexpr (NT_O == 1) {
                // one n tile per warp: matrices (k 0-7, the tile), (k 8-15, the tile)
                uint32_t bv[2];
                const int mi = (lane >> 3) & 1, rr = lane & 7;
                ldsm_x2_t(bv, Vs + (16 * kk + rr + 8 * mi) * QS + warp * (HD / 8));
#pragma unroll
                for (int m = 0; m < 2; ++m) mma_f16_16816(o[m][0], ap[m], bv);
            } else {
#pragma unroll
                for (int j = 0; j < NT_O; j += 2) {
                    // V rows = k (positions), dims = n: .trans gives the col-major fragments; matrices (k 0-7, n tile j),
                    // (k 8-15, tile j), (k 0-7, tile j+1), (k 8-15, tile j+1)
                    uint32_t bv[4];
                    const int mi = lane >> 3, rr = lane & 7;
                    const int k = 16 * kk + rr + 8 * (mi & 1), n = warp * (HD / 8) + 8 * (j + (mi >> 1));
                    ldsm_x4_t(bv, Vs + k * QS + n);
                    const uint32_t b0[2] = {bv[0], bv[1]}, b1[2] = {bv[2], bv[3]};
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        mma_f16_16816(o[m][j], ap[m], b0);
                        mma_f16_16816(o[m][j + 1], ap[m], b1);
                    }
                }
            }
        }
    }
    __syncthreads();
    // partial results: rows < rows
    const size_t pstride = HD + 2;
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int j = 0; j < NT_O; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = 16 * m + gid + 8 * (e >> 1);
                if (r >= rows) continue;
                const int d = warp * (HD / 8) + 8 * j + 2 * tig + (e & 1);
                const int t = r / G, h = kh * G + r % G;
                a.part[((static_cast<size_t>(t) * a.nh + h) * a.nchunks + chunk) * pstride + d] = o[m][j][e];
            }
    if (tid < rows) {
        const int t = tid / G, h = kh * G + tid % G;
        float *pp = a.part + ((static_cast<size_t>(t) * a.nh + h) * a.nchunks + chunk) * pstride;
        pp[HD] = row_m[tid];
        pp[HD + 1] = row_l[tid];
    }
}

// The chunks joined (engine/src/model.cpp:3832-3853): M = max m_c, O = sum O_c exp(m_c - M), L = sum l_c exp(m_c - M),
// o = O * (1 / L) * sigmoid(gate); quantized per 16 into the core ActSet.
struct MergeArgs {
    const float *part;
    const float *qg;     // gates: [n][nh][2 hd] second half
    const int *pos;
    int n, nh, hd, nchunks;
    int8_t *q;
    float *scale;
    int32_t *bsum;
    float *core_f;       // [n][nh * hd] or NULL
};

// One CTA per (token, head), one thread per dim (blockDim = hd, a multiple of 32).
__global__ void k_attn_merge(MergeArgs a) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int tid = threadIdx.x, lane = tid & 31;
    const int pos = *a.pos;
    const int W = a.nh * a.hd;
    const size_t cs = a.hd + 2;
    const int t = blockIdx.x / a.nh, h = blockIdx.x % a.nh;
    const int nc = min(a.nchunks, (pos + t) / kAttnChunk + 1);
    const float *pp = a.part + (static_cast<size_t>(t) * a.nh + h) * a.nchunks * cs;
    // every thread on its own (no reductions, no barriers): the chunks' (m, l) - the same addresses for the whole CTA -
    // and its dim's partials, kMergeBatch chunks' loads in flight at once, folded in with the online rescaling
    // (M the running max, L and acc rescaled by exp(M_old - M_new) when it grows)
    constexpr int kMergeBatch = 40;
    const int d = tid;
    float M = -INFINITY, L = 0.0f, acc = 0.0f;
    for (int c0 = 0; c0 < nc; c0 += kMergeBatch) {
        float mv[kMergeBatch], lv[kMergeBatch], vv[kMergeBatch];
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
            const bool in = c0 + u < nc;
            const float *q = pp + static_cast<size_t>(c0 + u) * cs;
            mv[u] = in ? q[a.hd] : -INFINITY;
            lv[u] = in ? q[a.hd + 1] : 0.0f;
            vv[u] = in ? q[d] : 0.0f;
        }
        float mb = M;
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) mb = fmaxf(mb, mv[u]);
        if (mb > M) {
            const float r = M == -INFINITY ? 0.0f : __expf(M - mb);
            L *= r;
            acc *= r;
            M = mb;
        }
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
            const float f = mv[u] == -INFINITY ? 0.0f : __expf(mv[u] - M);
            L = fmaf(lv[u], f, L);
            acc = fmaf(vv[u], f, acc);
        }
    }
    const float *gate = a.qg + (static_cast<size_t>(t) * a.nh + h) * 2 * a.hd + a.hd;
    const float v = __fmul_rn(__fmul_rn(acc, 1.0f / L), sigmoid_ref(gate[d]));
    const int col = h * a.hd + d;
    if (a.core_f) a.core_f[static_cast<size_t>(t) * W + col] = v;
    float amax = fabsf(v);
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float iv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    const int qv = max(-127, min(127, __float2int_rn(__fmul_rn(v, iv))));
    int sm = qv;
    for (int o = 8; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    a.q[static_cast<size_t>(t) * W + col] = static_cast<int8_t>(qv);
    if ((lane & 15) == 0) {
        a.scale[static_cast<size_t>(t) * (W / 16) + col / 16] = __fdiv_rn(amax, 127.0f);
        a.bsum[static_cast<size_t>(t) * (W / 16) + col / 16] = sm;
    }
}

// ------------------------------------------------------------------------------------------- routing ----
// route_topk per token (engine/src/model.cpp:4021-4065), the shared expert's gate sigmoid(w . h)
// (engine/src/model.cpp:4564-4567; its dot product is the router's last row here), and the union of the picked
// experts (engine/src/model.cpp:4183-4196): ascending expert ids, each with the tokens that picked it and the
// pick's slot t * K + k. One CTA of kRouteWarpsPerTok warps per token slot:
//   1. every warp of token t finds the row's max (each on its own: no barrier), then exps its quarter of the row;
//   2. warp (t, 0): the sum in expert order (one lane: the float sum is sequential), p = e / sum, then K rounds of
//      the warp's max p (redux on the bit patterns: p >= 0) and, among lanes holding it, the lowest expert id - the
//      reference's selection with its tie rule; only the winning lane rescans its experts; warp (t, 1) the gate;
//   3. every pick's union slot from popcounts of the union's bit set.
constexpr int kMaxUnion = 64;
constexpr int kRouteWarpsPerTok = 4;
constexpr int kRouteThreads = 32 * kRouteWarpsPerTok * kMaxTok;
struct RouteOut {
    int n_union;
    int ex[kMaxUnion];
    int mask[kMaxUnion];
    int slot[kMaxUnion][kMaxTok];
    int ids[kMaxTok * 8];
    float w[kMaxTok * 8];
    float gs[kMaxTok];
    // expert parallelism: the union members this rank computes (expert e on rank e % world), as union indices in
    // ascending order; n_own == n_union and own[u] == u on one GPU
    int n_own;
    int own[kMaxUnion];
    int own_ex[kMaxUnion];   // ex[own[m]]: the expert of this rank's m-th member (one load for the expert kernels)
};

__global__ void __launch_bounds__(kRouteThreads) k_route(const float *__restrict__ logits, int n, int E, int K,
                                                          RouteOut *out, int *union_acc, int ep_rank, int ep_world) {
    extern __shared__ __align__(16) float ps[];   // [kMaxTok][E]
    __shared__ int s_ids[kMaxTok * 8];
    __shared__ uint32_t s_bits[32];   // the union as a bit set over the experts (E <= 1024)
    __shared__ int s_mask[kMaxUnion];
    __shared__ int s_ex[kMaxUnion];   // the union's expert ids (for the expert-parallel ownership below)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // warp w: token w / 4, quarter (w - t) % 4: a token's four warps on the four SM sub-partitions (w % 4), token t's
    // lead warp (q = 0) on sub-partition t % 4
    static_assert(kRouteWarpsPerTok == 4, "one warp per sub-partition");
    const int t = warp >> 2, q = (warp - t) & 3;
    if (threadIdx.x < 32) s_bits[threadIdx.x] = 0;
    if (threadIdx.x < kMaxUnion) s_mask[threadIdx.x] = 0;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const bool live = t < n;
    const float *row = logits + static_cast<size_t>(t) * (E + 1);
    float *p = ps + static_cast<size_t>(t) * E;
    if (live) {
        float mx = -INFINITY;
        for (int e = lane; e < E; e += 32) mx = fmaxf(mx, row[e]);
        mx = warp_max(mx);
        for (int e = lane + 32 * q; e < E; e += 32 * kRouteWarpsPerTok) p[e] = expf_ref(__fsub_rn(row[e], mx));
        if (q == 1 && lane == 0) out->gs[t] = sigmoid_ref(row[E]);
    }
    __syncthreads();
    if (live && q == 0) {
        float sum = 0.0f;
        if (lane == 0) {   // in expert order, 32 values' loads ahead of their adds
            int e = 0;
            for (; e + 32 <= E; e += 32) {
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = p[e + i];
#pragma unroll
                for (int i = 0; i < 32; ++i) sum = __fadd_rn(sum, v[i]);
            }
            for (; e < E; ++e) sum = __fadd_rn(sum, p[e]);
        }
        sum = __shfl_sync(0xffffffffu, sum, 0);
        // K rounds: the warp's largest p (the bit patterns order as the values: p >= 0), the lowest id among the lanes
        // holding it; only the winning lane recomputes its best untaken expert
        float top = 0.0f, mine = 0.0f;
        uint32_t lb = 0;
        int li = 0x7fffffff;
        if (E <= 256) {
            float v[8];   // expert lane + 32 s
            uint32_t taken = 0;
#pragma unroll
            for (int s2 = 0; s2 < 8; ++s2) {
                const int e = lane + 32 * s2;
                v[s2] = e < E ? __fdiv_rn(p[e], sum) : 0.0f;
                if (e >= E) taken |= 1u << s2;
            }
            auto local_best = [&]() {
                lb = 0;
                li = 0x7fffffff;
#pragma unroll
                for (int s2 = 0; s2 < 8; ++s2) {
                    const uint32_t b2 = __float_as_uint(v[s2]);
                    if (!((taken >> s2) & 1) && (li == 0x7fffffff || b2 > lb)) lb = b2, li = lane + 32 * s2;
                }
            };
            local_best();
            for (int k = 0; k < K; ++k) {
                const uint32_t best = __reduce_max_sync(0xffffffffu, li == 0x7fffffff ? 0u : lb);
                const int bi = static_cast<int>(
                    __reduce_min_sync(0xffffffffu, li != 0x7fffffff && lb == best ? static_cast<uint32_t>(li) : 0x7fffffffu));
                const float bv = __uint_as_float(best);
                top = __fadd_rn(top, bv);
                if (lane == k) mine = bv;
                if (lane == 0) s_ids[t * K + k] = bi;
                if (bi == li) {
                    taken |= 1u << (bi >> 5);
                    local_best();
                }
            }
        } else {   // (wider routers: the probabilities stay in shared memory)
            for (int e = lane; e < E; e += 32) p[e] = __fdiv_rn(p[e], sum);
            __syncwarp();
            uint32_t taken = 0;   // bit s: expert lane + 32 s taken
            auto local_best = [&]() {
                lb = 0;
                li = 0x7fffffff;
                for (int s2 = 0, e = lane; e < E; ++s2, e += 32) {
                    const uint32_t b2 = __float_as_uint(p[e]);
                    if (!((taken >> s2) & 1) && (li == 0x7fffffff || b2 > lb)) lb = b2, li = e;
                }
            };
            local_best();
            for (int k = 0; k < K; ++k) {
                const uint32_t best = __reduce_max_sync(0xffffffffu, li == 0x7fffffff ? 0u : lb);
                const int bi = static_cast<int>(
                    __reduce_min_sync(0xffffffffu, li != 0x7fffffff && lb == best ? static_cast<uint32_t>(li) : 0x7fffffffu));
                const float bv = __uint_as_float(best);
                top = __fadd_rn(top, bv);
                if (lane == k) mine = bv;
                if (lane == 0) s_ids[t * K + k] = bi;
                if (bi == li) {
                    taken |= 1u << (bi >> 5);
                    local_best();
                }
            }
        }
        if (lane < K) {
            const int pk = t * K + lane;
            out->w[pk] = __fdiv_rn(mine, top);
        }
        __syncwarp();
        if (lane < K) {
            const int e = s_ids[t * K + lane];
            out->ids[t * K + lane] = e;
            atomicOr(&s_bits[e >> 5], 1u << (e & 31));
        }
    }
    __syncthreads();
    // each pick's union slot: the members below its expert (popcounts of the bit set)
    const int P = n * K, pk = threadIdx.x;
    if (pk < P) {
        const int e = s_ids[pk], w = e >> 5, tk = pk / K;
        int u = __popc(s_bits[w] & ((1u << (e & 31)) - 1u));
        for (int i = 0; i < w; ++i) u += __popc(s_bits[i]);
        out->ex[u] = e;   // (every pick of the expert writes the same id)
        s_ex[u] = e;
        out->slot[u][tk] = pk;
        atomicOr(&s_mask[u], 1 << tk);
    }
    __syncthreads();
    int nu = 0;
    for (int i = 0; i < (E + 31) / 32; ++i) nu += __popc(s_bits[i]);
    if (static_cast<int>(threadIdx.x) < nu) out->mask[threadIdx.x] = s_mask[threadIdx.x];
    if (threadIdx.x == 0) out->n_union = nu;
    // this rank's members of the union (expert e on rank e % world), ascending, by ballots over the union in 32s
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int base = 0;
        for (int u0 = 0; u0 < nu; u0 += 32) {
            const int u = u0 + lane;
            const bool mine = u < nu && s_ex[u] % ep_world == ep_rank;
            const uint32_t bal = __ballot_sync(0xffffffffu, mine);
            if (mine) {
                out->own[base + __popc(bal & ((1u << lane) - 1u))] = u;
                out->own_ex[base + __popc(bal & ((1u << lane) - 1u))] = s_ex[u];
            }
            base += __popc(bal);
        }
        if (lane == 0) {
            out->n_own = base;
            if (union_acc) atomicAdd(union_acc, base);   // (the experts this rank reads: the whole union on one GPU)
        }
    }
}

}  // namespace gcu

namespace gcu {

// ------------------------------------------------------------------------------------------- synthetic weights ----
// Seeded random bytes for measuring runs whose values do not matter (the self-test weights of
// engine/src/gpu_check.cpp:51-63: random codes, E4M3 scales in 0x30..0x48), written straight into device memory.
__device__ __forceinline__ uint64_t mix64(uint64_t x) {   // splitmix64's finalizer
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
__device__ __forceinline__ float unit_f(uint64_t h) { return static_cast<float>(h >> 40) * (1.0f / 16777216.0f); }
__device__ __forceinline__ float normal_f(uint64_t h) {   // Box-Muller
    const float u1 = fmaxf(unit_f(h), 1e-7f), u2 = unit_f(mix64(h));
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// tiled q4 bytes: codes random, the scale bytes (offsets 512..575 of every 576-byte group) in 0x30..0x48
__global__ void k_synth_tiled(uint8_t *p, size_t bytes, uint64_t seed) {
    for (size_t i = (blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x) * 8; i < bytes;
         i += static_cast<size_t>(gridDim.x) * blockDim.x * 8) {
        const uint64_t h = mix64(seed ^ (i * 0x100000001B3ull));
        uint8_t b[8];
        for (int k = 0; k < 8; ++k) {
            const size_t at = i + k;
            const uint8_t r = static_cast<uint8_t>(h >> (8 * k));
            b[k] = (at % kGroupBytes) >= 512 ? static_cast<uint8_t>(0x30 + r % 25) : r;
        }
        if (i + 8 <= bytes) *reinterpret_cast<uint2 *>(p + i) = *reinterpret_cast<uint2 *>(b);
        else
            for (int k = 0; i + k < bytes; ++k) p[i + k] = b[k];
    }
}

// pack-layout q4 rows (the embedding table): codes random, each row's last cols/16 bytes scales
__global__ void k_synth_rows(uint8_t *p, int64_t rows, int cols, uint64_t seed) {
    const size_t rb = static_cast<size_t>(cols / 16) * 9, total = static_cast<size_t>(rows) * rb;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total; i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint8_t r = static_cast<uint8_t>(mix64(seed ^ i));
        p[i] = (i % rb) >= static_cast<size_t>(cols / 2) ? static_cast<uint8_t>(0x30 + r % 25) : r;
    }
}

// f32 (dtype 0) or bf16 (1) values mean + std * N(0, 1)
__global__ void k_synth_values(void *p, size_t count, int dtype, float mean, float stdv, uint64_t seed) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count; i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float v = mean + stdv * normal_f(mix64(seed ^ (i * 0x9E3779B97F4A7C15ull)));
        if (dtype == 0) static_cast<float *>(p)[i] = v;
        else static_cast<uint16_t *>(p)[i] = static_cast<uint16_t>((__float_as_uint(v) + 0x7FFFu + ((__float_as_uint(v) >> 16) & 1u)) >> 16);
    }
}

// int8 KV rows with their scales, for a synthetic context: values uniform in +-127, scales std * |N(0,1)| / 127
__global__ void k_synth_kv(int8_t *kv, size_t n, float *sc, size_t ns, float stdv, uint64_t seed) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x)
        kv[i] = static_cast<int8_t>(static_cast<int>(mix64(seed ^ i) % 255) - 127);
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < ns; i += static_cast<size_t>(gridDim.x) * blockDim.x)
        sc[i] = stdv * fabsf(normal_f(mix64(~seed ^ i))) / 127.0f + 1e-4f;
}

// ------------------------------------------------------------------------------------------- device-side step ----
// The acceptance decision on the device (engine/src/geode.cpp:327-350) for a chained device-resident loop: from the
// rows' samples and the batch's tokens, kept and next; the next batch starts with `next` (its drafts: the caller's);
// the position moves on by kept; the Gated DeltaNet states roll back to backup kept-1 when kept < n (k_rollback).
struct StepState {
    int kept, next, n_union_sum, steps;
};
__global__ void k_decide(const int *samples, int *toks, int n, int *pos, StepState *ss) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    int k = 1, nx = samples[n - 1];
    for (int i = 0; i < n; ++i) {
        if (i + 1 < n && samples[i] == toks[i + 1]) {
            ++k;
            continue;
        }
        nx = samples[i];
        break;
    }
    ss->kept = k;
    ss->next = nx;
    ss->steps += 1;
    *pos += k;
    toks[0] = nx;
}

// The same decision from a rejection-sampling result (k_spec_reject on one sequence: accepted drafts, next token)
__global__ void k_decide_reject(const int *accepted, const int *next, int *toks, int *pos, StepState *ss) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int k = accepted[0] + 1, nx = next[0];
    ss->kept = k;
    ss->next = nx;
    ss->steps += 1;
    *pos += k;
    toks[0] = nx;
}

// state = backup[kept - 1] when kept < n (a grid-stride copy of the conv and recurrent states)
__global__ void k_rollback(float *conv, const float *conv_bk, size_t conv_n, float *gdn, const float *gdn_bk, size_t gdn_n,
                           int n, const StepState *ss) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int kept = ss->kept;
    if (kept >= n) return;
    const size_t b = static_cast<size_t>(kept - 1);
    const float4 *cs = reinterpret_cast<const float4 *>(conv_bk + b * conv_n);
    const float4 *gs = reinterpret_cast<const float4 *>(gdn_bk + b * gdn_n);
    float4 *cd = reinterpret_cast<float4 *>(conv), *gd = reinterpret_cast<float4 *>(gdn);
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < conv_n / 4; i += static_cast<size_t>(gridDim.x) * blockDim.x)
        cd[i] = cs[i];
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < gdn_n / 4; i += static_cast<size_t>(gridDim.x) * blockDim.x)
        gd[i] = gs[i];
}

}  // namespace gcu
