// accept.cuh - the acceptance of a verified batch: every row's sample, as Sampler::sample draws it
// (engine/src/sampler.cpp:16-50), all rows at once (row i's uniform is the i-th draw of the caller's stream), and the
// speculative (rejection) sampling rule for draft models (not in the reference; Leviathan et al. 2023).
#pragma once

#include "common.cuh"

namespace gcu {

// order-preserving key of a float (larger float, larger key; no NaN)
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kSampleThreads = 1024;
constexpr int kMaxCand = 1024;

// The k largest (value desc, index asc) of a row into cv/ci (k <= kMaxCand), sorted. Block-wide (1024 threads).
__device__ void row_topk(const float *__restrict__ row, int V, int k, float *cv, int *ci, uint32_t *hist, int *misc) {
    const int tid = threadIdx.x;
    uint32_t prefix = 0, mask = 0;
    int need = k;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < V; i += blockDim.x) {
            const uint32_t key = fkey(row[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int acc = 0, d = 255;
            for (; d > 0; --d) {
                if (acc + static_cast<int>(hist[d]) >= need) break;
                acc += hist[d];
            }
            misc[0] = d;
            misc[1] = need - acc;
        }
        __syncthreads();
        prefix |= static_cast<uint32_t>(misc[0]) << shift;
        mask |= 255u << shift;
        need = misc[1];
        __syncthreads();
    }
    // prefix = the k-th largest key; `need` of the elements equal to it are taken, the lowest indices first
    const uint32_t tau = prefix;
    const int per = (V + blockDim.x - 1) / blockDim.x, lo = tid * per, hi = min(V, lo + per);
    int eq = 0;
    for (int i = lo; i < hi; ++i) eq += fkey(row[i]) == tau;
    // exclusive scan of eq over threads (in index order)
    __shared__ int scan[kSampleThreads];
    scan[tid] = eq;
    __syncthreads();
    for (int off = 1; off < blockDim.x; off <<= 1) {
        const int v = tid >= off ? scan[tid - off] : 0;
        __syncthreads();
        scan[tid] += v;
        __syncthreads();
    }
    int rank = scan[tid] - eq;
    if (tid == 0) misc[2] = 0;
    __syncthreads();
    for (int i = lo; i < hi; ++i) {
        const uint32_t key = fkey(row[i]);
        if (key > tau || (key == tau && rank++ < need)) {
            const int at = atomicAdd(&misc[2], 1);
            if (at < kMaxCand) {
                cv[at] = row[i];
                ci[at] = i;
            }
        }
    }
    __syncthreads();
    // bitonic sort of kMaxCand slots by (value desc, index asc); empty slots last
    for (int i = tid; i < kMaxCand; i += blockDim.x)
        if (i >= k) {
            cv[i] = -INFINITY;
            ci[i] = 0x7fffffff;
        }
    __syncthreads();
    for (int size = 2; size <= kMaxCand; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < kMaxCand; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    // "before": larger value, or equal value and smaller index
                    const bool ij = cv[i] > cv[j] || (cv[i] == cv[j] && ci[i] < ci[j]);
                    if (ij != up) {
                        const float tv = cv[i];
                        cv[i] = cv[j];
                        cv[j] = tv;
                        const int ti = ci[i];
                        ci[i] = ci[j];
                        ci[j] = ti;
                    }
                }
            }
            __syncthreads();
        }
}

// Greedy rows split over many CTAs: each reduces its slice to the first maximum and merges it into best[r], a 64-bit
// key (order-preserving value bits, then the complement of the index: the largest value, the lowest index first).
__global__ void k_argmax_partial(const float *__restrict__ logits, int V, unsigned long long *best) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int r = blockIdx.y;
    const float *row = logits + static_cast<size_t>(r) * V;
    const int per = (V + gridDim.x - 1) / gridDim.x, lo = blockIdx.x * per, hi = min(V, lo + per);
    unsigned long long k = 0;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = row[i];
        if (v != v) continue;   // (NaN: never the maximum)
        const unsigned long long key = (static_cast<unsigned long long>(fkey(v)) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
        k = key > k ? key : k;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
        k = ok > k ? ok : k;
    }
    if ((threadIdx.x & 31) == 0 && k) atomicMax(&best[r], k);
}
// best -> the rows' samples; best reset for the next use
__global__ void k_argmax_finish(unsigned long long *best, int n, int *out) {
    const int r = threadIdx.x;
    if (r >= n) return;
    const unsigned long long k = best[r];
    out[r] = k ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFu)) : 0;
    best[r] = 0;
}

struct SampleArgs {
    const float *logits;   // [n][V]
    int V, n;
    float temperature, top_p;
    int top_k;
    const double *u;       // [n] uniforms in [0,1)
    int *out;              // [n] samples
};

// One CTA per row.
__global__ void __launch_bounds__(kSampleThreads) k_sample_rows(SampleArgs a) {
    __shared__ float cv[kMaxCand];
    __shared__ int ci[kMaxCand];
    __shared__ uint32_t hist[256];
    __shared__ int misc[4];
    __shared__ double ev[kMaxCand];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int r = blockIdx.x;
    const float *row = a.logits + static_cast<size_t>(r) * a.V;
    const int tid = threadIdx.x;
    if (a.temperature <= 0.0f) {
        // std::max_element: the first maximum
        float best = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = tid; i < a.V; i += blockDim.x)
            if (row[i] > best || (row[i] == best && i < bi)) best = row[i], bi = i;
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) best = ob, bi = oi;
        }
        if ((tid & 31) == 0) {
            cv[tid >> 5] = best;
            ci[tid >> 5] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float b = cv[0];
            int i0 = ci[0];
            for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
                if (cv[w] > b || (cv[w] == b && ci[w] < i0)) b = cv[w], i0 = ci[w];
            // a row of NaN only: index 0, as max_element
            a.out[r] = i0 == 0x7fffffff ? 0 : i0;
        }
        return;
    }
    const int k = min(a.V, a.top_k > 0 ? a.top_k : kMaxCand);
    row_topk(row, a.V, k, cv, ci, hist, misc);
    const float mx = cv[0];
    for (int i = tid; i < k; i += blockDim.x) ev[i] = static_cast<double>(expf_cr(__fdiv_rn(__fsub_rn(cv[i], mx), a.temperature)));
    __syncthreads();
    if (tid == 0) {
        double sum = 0.0;
        for (int i = 0; i < k; ++i) sum += ev[i];
        int keep = k;
        if (a.top_p < 1.0f) {
            double acc = 0.0;
            for (int i = 0; i < k; ++i) {
                acc += ev[i] / sum;
                if (acc >= static_cast<double>(a.top_p)) {
                    keep = i + 1;
                    break;
                }
            }
        }
        double kept = 0.0;
        for (int i = 0; i < keep; ++i) kept += ev[i];
        double rr = a.u[r] * (kept - 0.0) + 0.0;
        int pick = ci[keep - 1];
        for (int i = 0; i < keep; ++i) {
            rr -= ev[i];
            if (rr <= 0.0) {
                pick = ci[i];
                break;
            }
        }
        a.out[r] = pick;
    }
}

}  // namespace gcu
