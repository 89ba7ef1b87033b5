// launch.hpp - host-side launch helpers: the static GEMV's launch (shared-memory opt-in, grid sized to the SMs,
// optionally as a programmatic dependent launch), a process-wide launch counter and the operators' status word.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "../../include/geode_cuda.h"
#include "gemv_kernels.cuh"

namespace gcu {

inline std::atomic<uint64_t> &launch_counter() {
    static std::atomic<uint64_t> n{0};
    return n;
}
inline void count_launch(uint64_t k = 1) { launch_counter().fetch_add(k, std::memory_order_relaxed); }

inline int sm_count() {
    static int n = [] {
        int dev = 0, c = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
        return c;
    }();
    return n;
}

// The operators' status word (device memory, zeroed once): kernels OR error flags into it.
inline uint32_t *device_status() {
    static uint32_t *p = [] {
        void *q = nullptr;
        if (cudaMalloc(&q, 4) != cudaSuccess) return static_cast<uint32_t *>(nullptr);
        cudaMemset(q, 0, 4);
        return static_cast<uint32_t *>(q);
    }();
    return p;
}

// Launch with the programmatic-stream-serialization attribute when pdl: the kernel may begin (its prologue, the
// weight stream) before the previous kernel on the stream ends; it waits for it at griddepcontrol.wait.
template <typename Kern, typename... Args>
inline cudaError_t launch_ex(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    int na = 0;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        na = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    count_launch();
    return e;
}

// The GEMV kernels' shared-memory opt-in: the largest any launch shape takes (plan_relay caps it there).
inline int gemv_opt_in() {
    static const int rc = [] {
        if (cudaFuncSetAttribute(k_gemv_static, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_experts, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem) != cudaSuccess)
            return static_cast<int>(GCUDA_E_CUDA);
        return static_cast<int>(GCUDA_OK);
    }();
    return rc;
}

// p.wpu / p.nslots are set here (plan_static); the grid is one CTA per SM at most
inline int launch_static_gemv(StaticGemv p, cudaStream_t st, bool pdl) {
    RelayShape r;
    if (!plan_static(p.act.cols, p.n_units, sm_count(), r)) return GCUDA_E_ARG;
    if (gemv_opt_in() != GCUDA_OK) return GCUDA_E_CUDA;
    p.wpu = r.wpu;
    p.nslots = r.nslots;
    const int grid = std::max(1, std::min(sm_count(), (p.n_units + r.nslots - 1) / r.nslots));
    return launch_ex(k_gemv_static, dim3(grid), dim3(kGemvWarps * 32), r.smem, st, pdl, p) == cudaSuccess ? GCUDA_OK
                                                                                                            : GCUDA_E_CUDA;
}

}  // namespace gcu
