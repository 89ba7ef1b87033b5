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

inline int launch_static_gemv(const StaticGemv &p, cudaStream_t st, bool pdl) {
    const size_t smem = gemv_smem_bytes(p.act.cols);
    static size_t opted = 0;
    if (smem > opted) {
        if (cudaFuncSetAttribute(k_gemv_static, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess)
            return GCUDA_E_CUDA;
        opted = smem;
    }
    const int units_per_cta = gemv_slots(p.act.cols);
    const int grid = std::max(1, std::min(sm_count(), (p.n_units + units_per_cta - 1) / units_per_cta));
    return launch_ex(k_gemv_static, dim3(grid), dim3(kGemvWarps * 32), smem, st, pdl, p) == cudaSuccess ? GCUDA_OK
                                                                                                          : GCUDA_E_CUDA;
}

}  // namespace gcu
