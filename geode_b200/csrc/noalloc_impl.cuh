// noalloc_impl.cuh - gcuda_op_spec_reject_static: the rejection-sampling operator for callers that must not allocate
// device memory when they call it (a serving loop that holds a fixed device-memory budget, or one that cannot take
// the implicit device synchronisation of cudaMalloc / cudaFree in its step). It runs the same kernel as
// gcuda_spec_reject (k_spec_reject), but its scratch - the drafts copied in and the per-sequence results - is the
// file-scope device array below instead of a handle's lazily allocated buffer. No counterpart in the reference.
// (Included once, by backend.cu, after the kernels it launches.)
#pragma once
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/geode_cuda.h"
#include "accept.cuh"
#include "launch.hpp"

namespace gcu {

// The scratch: drafts [S][k], then accepted [S], then next [S] (int32). Nothing in it needs to start at zero: every
// call writes the drafts and all S results before they are read.
constexpr int kStaticRejectMaxSeqs = 1024;
constexpr int kStaticRejectMaxDrafts = 16;
constexpr size_t kStaticRejectInts = static_cast<size_t>(kStaticRejectMaxSeqs) * (kStaticRejectMaxDrafts + 2);
static __device__ __align__(256) int g_reject_scratch[kStaticRejectInts];

// The array's device address on each device, looked up once (with that device current) by the first call there.
constexpr int kStaticMaxDevices = 64;
struct StaticScratchTable {
    std::mutex mu;
    int *addr[kStaticMaxDevices] = {};
};
inline StaticScratchTable &static_scratch_table() {
    static StaticScratchTable t;
    return t;
}

}  // namespace gcu

extern "C" {

int gcuda_op_spec_reject_static(const float *d_target, const float *d_draft, const int *drafts, int S, int k, int V,
                                const gcuda_sampling *sp, uint64_t seed, int *accepted, int *next, void *stream) {
    using namespace gcu;
    if (!d_target || !d_draft || !drafts || !sp || !accepted || !next || S < 1 || k < 1 || V < 1 ||
        sp->temperature <= 0.0f || sp->top_k > kMaxCand || !(sp->top_p > 0.0f && sp->top_p <= 1.0f))
        return GCUDA_E_ARG;
    if (S > kStaticRejectMaxSeqs || k > kStaticRejectMaxDrafts) return GCUDA_E_ARG;   // beyond the static scratch
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kStaticMaxDevices) return GCUDA_E_DEVICE;
    StaticScratchTable &tab = static_scratch_table();
    int *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(tab.mu);
        if (!tab.addr[dev]) {
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_reject_scratch) != cudaSuccess || !p) return GCUDA_E_CUDA;
            tab.addr[dev] = static_cast<int *>(p);
        }
        scratch = tab.addr[dev];
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int *d_drafts = scratch, *d_acc = scratch + static_cast<size_t>(S) * k, *d_next = d_acc + S;
    if (cudaMemcpyAsync(d_drafts, drafts, sizeof(int) * S * k, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return GCUDA_E_CUDA;
    RejectArgs a{};
    a.target = d_target;
    a.draft = d_draft;
    a.drafts = d_drafts;
    a.k = k;
    a.V = V;
    a.temperature = sp->temperature;
    a.top_p = sp->top_p;
    a.top_k = sp->top_k;
    a.seed = seed;
    a.accepted = d_acc;
    a.next = d_next;
    if (launch_ex(k_spec_reject, dim3(S), dim3(kSampleThreads), 0, st, false, a) != cudaSuccess) return GCUDA_E_CUDA;
    if (cudaMemcpyAsync(accepted, d_acc, sizeof(int) * S, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyAsync(next, d_next, sizeof(int) * S, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return GCUDA_E_CUDA;
    return GCUDA_OK;
}

}  // extern "C"
