// accept.cuh - the acceptance of a verified batch: every row's sample, as Sampler::sample draws it
// (engine/src/sampler.cpp:16-50), all rows at once (row i's uniform is the i-th draw of the caller's stream), and the
// speculative (rejection) sampling rule for draft models (not in the reference; Leviathan et al. 2023).
#pragma once

#include <algorithm>

#include "common.cuh"

namespace gcu {

// order-preserving key of a float (larger float, larger key; no NaN)
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kSampleThreads = 1024;
constexpr int kMaxCand = 1024;

constexpr int kFastTopK = 256;   // the candidate pass serves k up to this
constexpr int kFastCap = 1024;   // candidates it holds (more qualify: the radix path)

__device__ __forceinline__ float key_float(uint32_t key) {   // (fkey's inverse)
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// The k largest keys of a row by two reads of it (k <= kFastTopK, blockDim.x == kSampleThreads): every thread's
// largest key, then tau = the k-th largest of those - k distinct elements reach it, so every one of the row's k
// largest does too - then every element with key >= tau into cand (one ballot per warp and element position, one
// shared atomic per warp that has any), sorted by (key desc, index asc); its first k into cv/ci. Returns false, with
// nothing written to cv/ci, when more than kFastCap elements reach tau (ties or a flat row): the radix path then.
__device__ bool row_topk_fast(const float *__restrict__ row, int V, int k, float *cv, int *ci, uint32_t *tk,
                              unsigned long long *cand, int *misc) {
    const int tid = threadIdx.x, lane = tid & 31;
    constexpr int nt = kSampleThreads;
    const bool vec = (V & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0;
    const float4 *r4 = reinterpret_cast<const float4 *>(row);
    const int nv = V >> 2;
    uint32_t m = 0;
    auto mx4 = [](uint32_t a, const float4 &v) {
        return max(max(a, max(fkey(v.x), fkey(v.y))), max(fkey(v.z), fkey(v.w)));
    };
    if (vec) {
        int i = tid;
        for (; i + 3 * nt < nv; i += 4 * nt) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldg(r4 + i + u * nt);
#pragma unroll
            for (int u = 0; u < 4; ++u) m = mx4(m, v[u]);
        }
        for (; i < nv; i += nt) m = mx4(m, __ldg(r4 + i));
    } else {
        for (int i = tid; i < V; i += nt) m = max(m, fkey(__ldg(row + i)));
    }
    tk[tid] = m;   // (0 for a thread without elements: below every key but the all-ones NaN's, which then takes all)
    if (tid == 0) misc[2] = 0;
    __syncthreads();
    for (int size = 2; size <= nt; size <<= 1)   // bitonic, descending
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const int j = tid ^ stride;
            if (j > tid) {
                const bool desc = (tid & size) == 0;
                const uint32_t a = tk[tid], b = tk[j];
                if ((a < b) == desc) {
                    tk[tid] = b;
                    tk[j] = a;
                }
            }
            __syncthreads();
        }
    const uint32_t tau = tk[k - 1];
    auto put = [&](bool p, uint32_t key, int idx) {   // (called by whole warps: every trip count is block-uniform)
        const unsigned bal = __ballot_sync(0xffffffffu, p);
        if (!bal) return;
        const int lead = __ffs(bal) - 1;
        int base = 0;
        if (lane == lead) base = atomicAdd(&misc[2], __popc(bal));
        base = __shfl_sync(0xffffffffu, base, lead);
        const int at = base + __popc(bal & ((1u << lane) - 1u));
        if (p && at < kFastCap)
            cand[at] = (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(idx));
    };
    if (vec) {
        for (int i0 = 0; i0 < nv; i0 += 4 * nt) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * nt + tid;
                v[u] = i < nv ? __ldg(r4 + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * nt + tid;
                const bool in = i < nv;
                const uint32_t kx = fkey(v[u].x), ky = fkey(v[u].y), kz = fkey(v[u].z), kw = fkey(v[u].w);
                put(in && kx >= tau, kx, 4 * i);
                put(in && ky >= tau, ky, 4 * i + 1);
                put(in && kz >= tau, kz, 4 * i + 2);
                put(in && kw >= tau, kw, 4 * i + 3);
            }
        }
    } else {
        for (int i0 = 0; i0 < V; i0 += nt) {
            const int i = i0 + tid;
            const uint32_t kx = i < V ? fkey(__ldg(row + i)) : 0u;
            put(i < V && kx >= tau, kx, i);
        }
    }
    __syncthreads();
    const int n = misc[2];
    if (n > kFastCap) return false;   // (block-uniform)
    int P = 1;
    while (P < n) P <<= 1;
    for (int i = n + tid; i < P; i += nt) cand[i] = 0ull;   // (below every candidate: they sort last)
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < P; i += nt) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = cand[i], b = cand[j];
                    if ((a < b) == desc) {
                        cand[i] = b;
                        cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    for (int i = tid; i < k; i += nt) {
        const unsigned long long c = cand[i];
        cv[i] = key_float(static_cast<uint32_t>(c >> 32));
        ci[i] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(c & 0xFFFFFFFFu));
    }
    return true;
}

// The k largest (value desc, index asc) of a row into cv/ci (k <= kMaxCand), sorted. Block-wide (1024 threads).
// Selection by key (fkey, then the lower index) - the candidate pass when k is small, else a radix select - and the
// selected k ordered by (value desc, index asc) in one bitonic network, so both selections give the same arrays.
__device__ void row_topk(const float *__restrict__ row, int V, int k, float *cv, int *ci, uint32_t *hist, int *misc) {
    const int tid = threadIdx.x;
    __shared__ int scan[kSampleThreads];
    __shared__ unsigned long long cand[kFastCap];
    const bool fast = k <= kFastTopK && blockDim.x == kSampleThreads &&
                      row_topk_fast(row, V, k, cv, ci, reinterpret_cast<uint32_t *>(scan), cand, misc);
    if (!fast) {
        __syncthreads();   // (the candidate pass's last reads of scan and misc)
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
    }   // (the radix path)
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

// The first maximum as std::max_element finds it (`if (*largest < *it) largest = it`), with whole float4 loads, four
// in flight per thread, and one merge per CTA: the CTA's key reduced through shared memory, then a single 64-bit
// atomicMax into best[r] (a row split over gridDim.x CTAs). Under < , -0.0 and +0.0 are equal (the first one stays:
// -0.0 is taken as +0.0), a NaN after the first element never replaces the maximum, and a NaN first element is never
// replaced (index 0: the all-ones key, above every value's). Rows of any
// length; the vector loop when V is a multiple of 4 and the rows' base is 16-byte aligned (every row then is).
constexpr int kArgmaxThreads = 256;
__global__ void __launch_bounds__(kArgmaxThreads) k_argmax_rows(const float *__restrict__ logits, int V,
                                                                unsigned long long *best) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ unsigned long long s_k[kArgmaxThreads / 32];
    const int r = blockIdx.y, tid = threadIdx.x;
    const float *row = logits + static_cast<size_t>(r) * V;
    unsigned long long k = 0;
    auto take = [&](float v, int i) {
        v = __fadd_rn(v, 0.0f);   // (-0 -> +0)
        if (v != v) return;
        const unsigned long long key = (static_cast<unsigned long long>(fkey(v)) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
        k = key > k ? key : k;
    };
    if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0) {
        const int nv = V >> 2, per = (nv + gridDim.x - 1) / gridDim.x, lo = blockIdx.x * per, hi = min(nv, lo + per);
        const float4 *row4 = reinterpret_cast<const float4 *>(row);
        int i = lo + tid;
        for (; i + 3 * kArgmaxThreads < hi; i += 4 * kArgmaxThreads) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldg(row4 + i + u * kArgmaxThreads);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = 4 * (i + u * kArgmaxThreads);
                take(v[u].x, e), take(v[u].y, e + 1), take(v[u].z, e + 2), take(v[u].w, e + 3);
            }
        }
        for (; i < hi; i += kArgmaxThreads) {
            const float4 v = __ldg(row4 + i);
            take(v.x, 4 * i), take(v.y, 4 * i + 1), take(v.z, 4 * i + 2), take(v.w, 4 * i + 3);
        }
    } else {
        const int per = (V + gridDim.x - 1) / gridDim.x, lo = blockIdx.x * per, hi = min(V, lo + per);
        for (int i = lo + tid; i < hi; i += kArgmaxThreads) take(__ldg(row + i), i);
    }
    if (blockIdx.x == 0 && tid == 0 && row[0] != row[0]) k = ~0ull;
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
        k = ok > k ? ok : k;
    }
    if ((tid & 31) == 0) s_k[tid >> 5] = k;
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; ++w) k = s_k[w] > k ? s_k[w] : k;
        if (k) atomicMax(&best[r], k);
    }
}
// CTAs per row for k_argmax_rows: about two waves of the GPU over all rows, at most 64 a row
inline int argmax_slices(int rows, int sms) { return rows >= 2 * sms * 8 ? 1 : std::min(64, std::max(1, 2 * sms * 8 / rows)); }

// softmax_at (engine/src/model.cpp:1287-1292): the probability of the row's entry `*best` under the softmax, the float
// of 1 / sum_i exp(double(lg[i] - lg[best])) - the difference in float, the exp and the sum in double. Each CTA sums
// a strided slice, the last CTA to arrive adds the slices in CTA order: the double sum is grouped unlike the
// reference's one loop, so its last bits may differ; rounded to float the result is the same but where it falls on a
// rounding boundary of the float.
constexpr int kSoftmaxCtas = 64, kSoftmaxThreads = 256;
__global__ void __launch_bounds__(kSoftmaxThreads) k_softmax_at(const float *__restrict__ lg, int V,
                                                                 const int *__restrict__ best, double *part,
                                                                 unsigned int *count, float *prob) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ double red[kSoftmaxThreads / 32];
    __shared__ bool last;
    const float m = lg[*best];
    double acc = 0.0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x)
        acc += exp(static_cast<double>(__fsub_rn(lg[i], m)));
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < kSoftmaxThreads / 32; ++w) t += red[w];
        part[blockIdx.x] = t;
        __threadfence();
        last = atomicAdd(count, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    double sum = 0.0;
    for (int b = 0; b < static_cast<int>(gridDim.x); ++b) sum += *reinterpret_cast<volatile double *>(part + b);
    *prob = static_cast<float>(1.0 / sum);
    *count = 0;
}

// Greedy speculative acceptance of S sequences from their rows' first maxima (best: [S][k+1] keys of k_argmax_rows):
// draft i stands while row i's argmax equals it (geode_generate's rule at temperature 0, engine/src/geode.cpp:327-350,
// without stop tokens); next = the argmax of the first row whose draft fell, or of row k when all stood. One thread
// a sequence; the keys are reset to zero for the next use.
__global__ void k_greedy_decide(unsigned long long *best, const int *__restrict__ drafts, int S, int k, int *accepted,
                                int *next) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= S) return;
    unsigned long long *b = best + static_cast<size_t>(s) * (k + 1);
    auto arg = [&](int i) {
        const unsigned long long key = b[i];
        return key ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFu)) : 0;
    };
    int a = 0;
    while (a < k && arg(a) == drafts[static_cast<size_t>(s) * k + a]) ++a;
    accepted[s] = a;
    next[s] = arg(a);
    for (int i = 0; i <= k; ++i) b[i] = 0;
}

// best -> the rows' samples; best reset for the next use
__global__ void k_argmax_finish(unsigned long long *best, int n, int *out) {
    asm volatile("griddepcontrol.wait;" ::: "memory");   // (the partial maxima are complete and visible)
    asm volatile("griddepcontrol.launch_dependents;");
    const int r = threadIdx.x;
    if (r >= n) return;
    const unsigned long long k = best[r];
    out[r] = k ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFu)) : 0;
    best[r] = 0;
}

// The presence penalty of geode_generate (engine/src/geode.cpp:234-255) on the rows of one verified batch, in place:
// row i loses `penalty` (one f32 subtraction, as the engine's lg[t] -= penalty) at every token the answer sampled
// before row i - the caller's list (distinct ids) and, for i >= 1, the drafts toks[1..i] that are new to it (bit j of
// fresh: toks[j] is neither in the list nor an earlier draft). Those drafts are rows 0..i-1's samples whenever row
// i's sample is used (each of those rows' draft stood), so every row is penalised independently and in parallel.
// Each id is written by one thread. Grid: (slices of the list, rows).
struct PresenceArgs {
    float *logits;   // [n][V]
    int V, n;
    float penalty;
    const int *seen;   // [n_seen] distinct ids in [0, V)
    int n_seen;
    int toks[kMaxTok];
    unsigned fresh;
};
__global__ void k_presence(PresenceArgs a) {
    float *row = a.logits + static_cast<size_t>(blockIdx.y) * a.V;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n_seen; i += gridDim.x * blockDim.x) {
        const int t = a.seen[i];
        row[t] = __fsub_rn(row[t], a.penalty);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0)
        for (int j = 1; j <= static_cast<int>(blockIdx.y); ++j)
            if ((a.fresh >> j) & 1u) row[a.toks[j]] = __fsub_rn(row[a.toks[j]], a.penalty);
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
    for (int i = tid; i < k; i += blockDim.x) ev[i] = static_cast<double>(expf_ref(__fdiv_rn(__fsub_rn(cv[i], mx), a.temperature)));
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

// ------------------------------------------------------------------------------------------- rejection sampling ----
// Speculative sampling (Leviathan et al. 2023, Algorithm 1; Chen et al. 2023) for the draft-model configurations
// (not in the reference, which only has the greedy/sampled acceptance rule above): draft d_i stands when
// u_i * q(d_i) < p(d_i); the first rejection resamples from norm(max(0, p - q)); with every draft standing, a bonus
// token from the last target row. p and q are the rows' filtered distributions (top-k, 1024 when off, by logit with
// ties to the lower id; weights fast_exp((l - max) * (1/T)) summed in double in logit order; the top-p prefix;
// probabilities w / kept). Uniforms: Philox4x32-10 (Salmon et al. 2011), key = seed, counter = (sequence, row);
// words 0-1 the acceptance draw, 2-3 the resample draw, each 53 bits. Resampling walks the support in ascending
// token id. One CTA (kSampleThreads) per sequence; the sums run on one thread in their fixed order.
__device__ inline void philox4x32(uint64_t key, uint64_t hi, uint64_t lo, uint32_t (&out)[4]) {
    uint32_t c0 = static_cast<uint32_t>(lo), c1 = static_cast<uint32_t>(lo >> 32), c2 = static_cast<uint32_t>(hi),
             c3 = static_cast<uint32_t>(hi >> 32);
    uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = 0xD2511F53ull * c0, p1 = 0xCD9E8D57ull * c2;
        const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ c1 ^ k0, n2 = static_cast<uint32_t>(p0 >> 32) ^ c3 ^ k1;
        c1 = static_cast<uint32_t>(p1);
        c3 = static_cast<uint32_t>(p0);
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0, out[1] = c1, out[2] = c2, out[3] = c3;
}
__device__ __forceinline__ double u53(uint32_t a, uint32_t b) {
    return static_cast<double>((static_cast<uint64_t>(a) << 21) ^ (static_cast<uint64_t>(b) >> 11)) * (1.0 / 9007199254740992.0);
}

// (id, value) pairs of n <= kMaxCand by ascending id, in place (bitonic; the padding after n sorts last)
__device__ void sort_by_id(int *ids, double *vals, int n) {
    const int tid = threadIdx.x;
    for (int i = tid; i < kMaxCand; i += blockDim.x)
        if (i >= n) {
            ids[i] = 0x7fffffff;
            vals[i] = 0.0;
        }
    __syncthreads();
    for (int size = 2; size <= kMaxCand; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < kMaxCand; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i && ((ids[i] > ids[j]) == ((i & size) == 0))) {
                    const int ti = ids[i];
                    ids[i] = ids[j];
                    ids[j] = ti;
                    const double tv = vals[i];
                    vals[i] = vals[j];
                    vals[j] = tv;
                }
            }
            __syncthreads();
        }
}

struct RejectArgs {
    const float *target;   // [S][k+1][V]
    const float *draft;    // [S][k][V]
    const int *drafts;     // [S][k]
    int k, V;
    float temperature, top_p;
    int top_k;
    uint64_t seed;
    int *accepted, *next;  // [S]
};

__global__ void __launch_bounds__(kSampleThreads) k_spec_reject(RejectArgs a) {
    __shared__ float cv[kMaxCand];
    __shared__ int ci[kMaxCand];
    __shared__ uint32_t hist[256];
    __shared__ int misc[4];
    __shared__ int pid[kMaxCand], qid[kMaxCand];
    __shared__ double pp[kMaxCand], qp[kMaxCand];
    __shared__ int s_acc, s_best;
    __shared__ double s_pd, s_qd, s_ua, s_ur, s_kept;
    const int tid = threadIdx.x, seq = blockIdx.x;
    const int kk = min(a.V, a.top_k > 0 ? a.top_k : kMaxCand);
    const float it = __fdiv_rn(1.0f, a.temperature);
    // the filtered distribution of one row into (ids, probs) in logit order; returns the kept count
    auto filtered = [&](const float *row, int *ids, double *probs) -> int {
        row_topk(row, a.V, kk, cv, ci, hist, misc);
        const float mx = cv[0];
        for (int i = tid; i < kk; i += blockDim.x) probs[i] = static_cast<double>(fast_exp_exact(__fmul_rn(__fsub_rn(cv[i], mx), it)));
        __syncthreads();
        if (tid == 0) {
            double sum = 0.0;
            for (int i = 0; i < kk; ++i) sum += probs[i];
            int keep = kk;
            if (a.top_p < 1.0f) {
                double acc = 0.0;
                for (int i = 0; i < kk; ++i) {
                    acc += probs[i] / sum;
                    if (acc >= static_cast<double>(a.top_p)) {
                        keep = i + 1;
                        break;
                    }
                }
            }
            double kept = 0.0;
            for (int i = 0; i < keep; ++i) kept += probs[i];
            misc[3] = keep;
            s_kept = kept;
        }
        __syncthreads();
        const int keep = misc[3];
        const double kept = s_kept;
        for (int i = tid; i < keep; i += blockDim.x) {
            ids[i] = ci[i];
            probs[i] = probs[i] / kept;
        }
        __syncthreads();
        return keep;
    };
    // the probability of token tok in a support sorted by id (0 when absent)
    auto lookup = [&](const int *ids, const double *probs, int n, int tok) -> double {
        int lo = 0, hi = n - 1;
        while (lo <= hi) {
            const int mid = (lo + hi) >> 1;
            if (ids[mid] == tok) return probs[mid];
            if (ids[mid] < tok) lo = mid + 1;
            else hi = mid - 1;
        }
        return 0.0;
    };
    int accepted = 0, best = -1;
    for (int i = 0; i <= a.k; ++i) {
        if (tid == 0) {
            uint32_t r[4];
            philox4x32(a.seed, static_cast<uint64_t>(seq), static_cast<uint64_t>(i), r);
            s_ua = u53(r[0], r[1]);
            s_ur = u53(r[2], r[3]);
        }
        __syncthreads();
        const double ua = s_ua, ur = s_ur;
        __syncthreads();
        const int np = filtered(a.target + (static_cast<size_t>(seq) * (a.k + 1) + i) * a.V, pid, pp);
        if (i == a.k) {   // every draft stood: the bonus token from the target row
            if (tid == 0) {
                double total = 0.0;
                for (int j = 0; j < np; ++j) total += pp[j];
                s_qd = total;
            }
            sort_by_id(pid, pp, np);
            if (tid == 0) {
                const double lim = ur * s_qd;
                double acc = 0.0;
                int b = -1;
                for (int j = 0; j < np; ++j) {
                    if (pp[j] <= 0.0) continue;
                    acc += pp[j];
                    b = pid[j];
                    if (acc > lim) break;
                }
                s_best = b;
            }
            __syncthreads();
            best = s_best;
            break;
        }
        const int nq = filtered(a.draft + (static_cast<size_t>(seq) * a.k + i) * a.V, qid, qp);
        const int d = a.drafts[static_cast<size_t>(seq) * a.k + i];
        if (tid == 0) s_pd = s_qd = 0.0;
        __syncthreads();
        for (int j = tid; j < np; j += blockDim.x)
            if (pid[j] == d) s_pd = pp[j];
        for (int j = tid; j < nq; j += blockDim.x)
            if (qid[j] == d) s_qd = qp[j];
        __syncthreads();
        if (tid == 0) s_acc = s_qd > 0.0 && ua * s_qd < s_pd;
        __syncthreads();
        if (s_acc) {
            ++accepted;
            continue;
        }
        // the residual max(0, p - q) over p's support: its total in p's (logit) order, then the walk by id. pp is
        // overwritten with rv = p - q (p itself is read again only when the residual is empty)
        sort_by_id(qid, qp, nq);
        for (int j = tid; j < np; j += blockDim.x) pp[j] = pp[j] - lookup(qid, qp, nq, pid[j]);
        __syncthreads();
        if (tid == 0) {
            double total = 0.0;
            for (int j = 0; j < np; ++j)
                if (pp[j] > 0.0) total += pp[j];
            s_pd = total;
        }
        __syncthreads();
        const double total = s_pd;
        sort_by_id(pid, pp, np);   // (rv by ascending id)
        if (tid == 0) {
            int b = -1;
            double acc = 0.0;
            if (total > 0.0) {
                const double lim = ur * total;
                for (int j = 0; j < np; ++j) {
                    if (pp[j] <= 0.0) continue;
                    acc += pp[j];
                    b = pid[j];
                    if (acc > lim) break;
                }
            }
            s_best = b;
        }
        __syncthreads();
        best = s_best;
        if (total <= 0.0) {   // p == q on the support: sample from p itself, by id
            const int np2 = filtered(a.target + (static_cast<size_t>(seq) * (a.k + 1) + i) * a.V, pid, pp);
            sort_by_id(pid, pp, np2);
            if (tid == 0) {
                double acc = 0.0;
                int b = -1;
                for (int j = 0; j < np2; ++j) {
                    if (pp[j] <= 0.0) continue;
                    acc += pp[j];
                    b = pid[j];
                    if (acc > ur) break;
                }
                s_best = b;
            }
            __syncthreads();
            best = s_best;
        }
        break;
    }
    if (tid == 0) {
        a.accepted[seq] = accepted;
        a.next[seq] = best;
    }
}

}  // namespace gcu
