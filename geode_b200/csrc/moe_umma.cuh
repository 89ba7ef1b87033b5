// moe_umma.cuh - the routed experts of many token rows at once on the tensor core (the batched configuration: 64
// sequences x 5 rows, top-8 picks over 256 experts), bit for bit the reference's per-pick products
// (engine/src/model.cpp:4496-4543): for every pick p = t * K + k of expert e = ids[p],
//   gu = W_gu[e] (2 ff x H) . quant(h_t);  a = silu(gu[i]) * gu[ff + i];  y_p = W_dn[e] (H x ff) . quant(a).
// Three steps on the stream: the plan (k_moe_plan: the picks grouped by expert, the two products' unit tables on the
// device), the grouped tcgen05 products (k_umma_gemm over the unit tables), and between them the SwiGLU with the
// activation quantizer (k_swiglu_quant). The combine (the picks' weights, the shared expert) is the caller's.
#pragma once

#include "umma_gemm.cuh"

namespace gcu {

constexpr int kMoeNT = 16;            // token entries per unit of the grouped products
constexpr int kMoeMaxExperts = 1024;
constexpr int kMoePlanThreads = 1024;

// The work buffer of gcuda_op_moe_umma, in order (each piece 256-byte aligned): the counts (2 int), the pick list
// [P] int (grouped by expert, ascending picks inside a group), the gate_up and down unit tables, the gate_up outputs
// [P][2 ff] f32, the SwiGLU activations quantized: q [P][ff] int8, scale and bsum [P][ff / 16].
struct MoeWork {
    int *counts;
    int *toklist;
    UmmaUnit *units_gu, *units_dn;
    float *gu;
    int8_t *aq;
    float *as;
    int32_t *ab;
    int cap_gu, cap_dn;
};
__host__ __device__ inline size_t moe_align(size_t x) { return (x + 255) / 256 * 256; }
// units at most: every expert with picks takes tiles x ceil(picks / kMoeNT) of them
inline int moe_unit_cap(int P, int E, int tiles) { return tiles * (P / kMoeNT + (P < E ? P : E)); }
inline size_t moe_work_layout(int n, int K, int E, int H, int ff, uint8_t *base, MoeWork *w) {
    const int P = n * K;
    const int cap_gu = moe_unit_cap(P, E, 2 * ff / kUmmaRows), cap_dn = moe_unit_cap(P, E, H / kUmmaRows);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t *p = base ? base + off : nullptr;
        off += moe_align(bytes);
        return p;
    };
    uint8_t *counts = take(2 * sizeof(int));
    uint8_t *toklist = take(static_cast<size_t>(P) * sizeof(int));
    uint8_t *ugu = take(static_cast<size_t>(cap_gu) * sizeof(UmmaUnit));
    uint8_t *udn = take(static_cast<size_t>(cap_dn) * sizeof(UmmaUnit));
    uint8_t *gu = take(static_cast<size_t>(P) * 2 * ff * sizeof(float));
    uint8_t *aq = take(static_cast<size_t>(P) * ff);
    uint8_t *as = take(static_cast<size_t>(P) * (ff / 16) * sizeof(float));
    uint8_t *ab = take(static_cast<size_t>(P) * (ff / 16) * sizeof(int32_t));
    if (w) {
        w->counts = reinterpret_cast<int *>(counts);
        w->toklist = reinterpret_cast<int *>(toklist);
        w->units_gu = reinterpret_cast<UmmaUnit *>(ugu);
        w->units_dn = reinterpret_cast<UmmaUnit *>(udn);
        w->gu = reinterpret_cast<float *>(gu);
        w->aq = reinterpret_cast<int8_t *>(aq);
        w->as = reinterpret_cast<float *>(as);
        w->ab = reinterpret_cast<int32_t *>(ab);
        w->cap_gu = cap_gu;
        w->cap_dn = cap_dn;
    }
    return off;
}

struct MoePlanArgs {
    const int *ids;           // [P] expert of pick p
    int P, E;
    const uint8_t *experts;   // expert e's block at experts + e * stride: gate_up (U layout), then down (U layout)
    size_t stride, gu_bytes;
    const float *globals;     // [E][2]
    int tiles_gu, tiles_dn;
    MoeWork w;
    uint32_t *status;
};

// One CTA: the picks counted per expert, each expert's picks listed in ascending order (a thread per expert walks the
// picks - deterministic), then each expert's units (its tiles x its blocks of kMoeNT picks) at an offset from a
// prefix sum over the experts. An expert id out of range raises kErrBadShape and its pick is left out.
__global__ void __launch_bounds__(kMoePlanThreads) k_moe_plan(MoePlanArgs a) {
    __shared__ int cnt[kMoeMaxExperts], start[kMoeMaxExperts], ustart[kMoeMaxExperts];
    __shared__ int totals[2];
    const int tid = threadIdx.x;
    for (int e = tid; e < a.E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = tid; p < a.P; p += blockDim.x) {
        const int e = a.ids[p];
        if (e >= 0 && e < a.E) atomicAdd(&cnt[e], 1);
        else if (a.status) atomicOr(a.status, kErrBadShape);
    }
    __syncthreads();
    if (tid == 0) {
        int s = 0, us = 0;
        for (int e = 0; e < a.E; ++e) {
            start[e] = s;
            ustart[e] = us;
            s += cnt[e];
            us += (cnt[e] + kMoeNT - 1) / kMoeNT;
        }
        totals[0] = us;
        totals[1] = s;
        a.w.counts[0] = us * a.tiles_gu;
        a.w.counts[1] = us * a.tiles_dn;
    }
    __syncthreads();
    const int ublocks = totals[0];
    for (int e = tid; e < a.E; e += blockDim.x) {
        if (!cnt[e]) continue;
        int at = start[e];
        for (int p = 0; p < a.P; ++p)
            if (a.ids[p] == e) a.w.toklist[at++] = p;
        const uint8_t *blk = a.experts + static_cast<size_t>(e) * a.stride;
        const float g0 = a.globals[2 * e], g1 = a.globals[2 * e + 1];
        const int nb = (cnt[e] + kMoeNT - 1) / kMoeNT;
        // unit index = tile * (all experts' blocks) + the expert's block: a tile's units of every expert together, so
        // that consecutive CTAs read different matrices and a matrix's token blocks sit side by side
        for (int b = 0; b < nb; ++b) {
            const int nt = min(kMoeNT, cnt[e] - b * kMoeNT), tok0 = start[e] + b * kMoeNT;
            for (int T = 0; T < a.tiles_gu; ++T)
                a.w.units_gu[T * ublocks + ustart[e] + b] = UmmaUnit{blk, g0, T, nt, tok0};
            for (int T = 0; T < a.tiles_dn; ++T)
                a.w.units_dn[T * ublocks + ustart[e] + b] = UmmaUnit{blk + a.gu_bytes, g1, T, nt, tok0};
        }
    }
}

// a = silu(gate) * up (engine/src/model.cpp:4522-4524, silu on glibc's expf) per pick, quantized per block of 16 as
// quantize_activation (engine/src/kernels.cpp:1254-1295); a half-warp per block
__global__ void k_swiglu_quant(const float *__restrict__ gu, int P, int ff, int8_t *__restrict__ q,
                               float *__restrict__ scale, int32_t *__restrict__ bsum) {
    const int nb = ff / 16;
    const int64_t total = static_cast<int64_t>(P) * ff;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(i / ff), j = static_cast<int>(i % ff);
        const float *g = gu + static_cast<size_t>(p) * 2 * ff;
        const float v = __fmul_rn(silu_ref(g[j]), g[ff + j]);
        float amax = fabsf(v);
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        const int qv = max(-127, min(127, __float2int_rn(__fmul_rn(v, inv))));
        int s = qv;
        for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        q[static_cast<size_t>(p) * ff + j] = static_cast<int8_t>(qv);
        if ((j & 15) == 0) {
            scale[static_cast<size_t>(p) * nb + j / 16] = __fdiv_rn(amax, 127.0f);
            bsum[static_cast<size_t>(p) * nb + j / 16] = s;
        }
    }
}

}  // namespace gcu
