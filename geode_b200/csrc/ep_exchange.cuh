// ep_exchange.cuh - expert parallelism's meeting points over NVLink, without a collective library in the step: every
// rank's MoE layer computes the picks whose experts it owns (expert e on rank e % world), and the down kernel
// (k_experts_lane) stores those rows straight into every peer's slot for the layer (peer memory mapped through CUDA
// IPC at set-up), then raises the layer's flag in every peer (the step's epoch, a release store at system scope) and
// waits, bounded, until every peer's flag for the layer holds the same epoch. The combine that follows reads all the
// picks' rows from local memory in rank order, as on one GPU, so the step's results equal the one-GPU step's bit for
// bit. Here: the flags' loads and stores, and the step's start (k_ep_tick).
//
// Plain loads and stores on peer memory only: no TMA, no bulk copy, no multicast, no library kernel on peer memory.
#pragma once

#include "common.cuh"
#include "layer_kernels.cuh"

namespace gcu {

constexpr int kMaxEpWorld = 8;
constexpr uint32_t kExchangeWaitLimit = 1u << 24;   // polls of a peer's flag before the wait gives up

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

}  // namespace gcu
