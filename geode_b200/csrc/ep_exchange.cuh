// ep_exchange.cuh - expert parallelism's exchange of the routed experts' outputs over NVLink, without a collective
// library in the step: every rank's MoE layer computes the picks whose experts it owns (expert e on rank e % world),
// then k_ep_exchange stores those rows straight into every peer's slot for the layer (peer memory mapped through
// CUDA IPC at set-up), raises this layer's flag in every peer (the step's epoch, a release store at system scope)
// and waits, bounded, until every peer's flag for the layer holds the same epoch. The combine that follows reads
// all the picks' rows from local memory in rank order, as on one GPU, so the step's results equal the one-GPU
// step's bit for bit.
//
// Plain loads and stores on peer memory only: no TMA, no bulk copy, no multicast, no library kernel on peer memory.
#pragma once

#include "common.cuh"
#include "layer_kernels.cuh"

namespace gcu {

constexpr int kMaxEpWorld = 8;
constexpr int kExchangeThreads = 256;
constexpr int kExchangeCtas = 32;
constexpr uint32_t kExchangeWaitLimit = 1u << 24;   // polls of a peer's flag before the wait gives up

struct ExchangeArgs {
    float *eout;                          // this layer's rows [n * K][H] (its own picks computed, the rest to come)
    float *peer_eout[kMaxEpWorld];        // the peers' slots for this layer (this rank's entry: unused)
    uint32_t *peer_flags[kMaxEpWorld];    // the peers' flags [n_layers + 2][world]
    uint32_t *flags;                      // this rank's flags, written by the peers
    const RouteOut *route;
    const int *epoch;
    unsigned int *count;                  // the CTAs' arrival counter (zero between launches)
    uint32_t *status;
    int n, K, H, rank, world, layer;
};

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct TickArgs {
    int *epoch;
    uint32_t *flags;                      // this rank's flags; row `row` is the step-start row
    uint32_t *peer_flags[kMaxEpWorld];
    uint32_t *status;
    int rank, world, row;
};

// The step's start under expert parallelism: the epoch advanced, then a handshake with every peer (the epoch stored
// into the peer's step-start flag, a bounded wait for the peer's). A peer that has started this step has finished
// the last one (its stream's order), so no rank stores a layer's rows into a peer still combining that layer's rows
// of the step before, nor raises a layer's flag there before the peer has read the previous step's - whatever the
// number of MoE layers.
__global__ void k_ep_tick(TickArgs a) {
    __shared__ uint32_t ep;
    if (threadIdx.x == 0) {
        ep = static_cast<uint32_t>(*a.epoch + 1);
        *a.epoch = static_cast<int>(ep);
    }
    __syncthreads();
    const int s = threadIdx.x;
    if (s < a.world && s != a.rank) {
        st_release_sys(a.peer_flags[s] + a.row * a.world + a.rank, ep);
        const uint32_t *f = a.flags + a.row * a.world + s;
        bool ok = false;
        for (uint32_t it = 0; it < kExchangeWaitLimit && !ok; ++it) ok = ld_acquire_sys(f) == ep;
        if (!ok && a.status) atomicOr(a.status, kErrWaitTimeout);
    }
}

__global__ void __launch_bounds__(kExchangeThreads) k_ep_exchange(ExchangeArgs a) {
    const int P = a.n * a.K, row4 = a.H / 4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P * row4; i += gridDim.x * blockDim.x) {
        const int p = i / row4, c = i - p * row4;
        if (a.route->ids[p] % a.world != a.rank) continue;   // (a peer's pick: the peer sends it)
        const float4 v = reinterpret_cast<const float4 *>(a.eout + static_cast<size_t>(p) * a.H)[c];
#pragma unroll
        for (int s = 0; s < kMaxEpWorld; ++s)
            if (s < a.world && s != a.rank) reinterpret_cast<float4 *>(a.peer_eout[s] + static_cast<size_t>(p) * a.H)[c] = v;
    }
    __threadfence_system();   // (this thread's peer stores, before the arrival below)
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) last = atomicAdd(a.count, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    // the last CTA to arrive: every CTA's rows are out; tell the peers, then wait for theirs
    const uint32_t epoch = static_cast<uint32_t>(*reinterpret_cast<const volatile int *>(a.epoch));
    if (threadIdx.x == 0) *a.count = 0;
    const int s = threadIdx.x;
    if (s < a.world && s != a.rank) st_release_sys(a.peer_flags[s] + a.layer * a.world + a.rank, epoch);
    if (s < a.world && s != a.rank) {
        const uint32_t *f = a.flags + a.layer * a.world + s;
        bool ok = false;
        for (uint32_t it = 0; it < kExchangeWaitLimit && !ok; ++it) ok = ld_acquire_sys(f) == epoch;
        if (!ok && a.status) atomicOr(a.status, kErrWaitTimeout);
    }
}

}  // namespace gcu
