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

// The GEMV kernels' shared-memory opt-in: the largest any launch shape takes (plan_gemv caps it there).
inline int gemv_opt_in() {
    static const int rc = [] {
        const cudaFuncAttribute a = cudaFuncAttributeMaxDynamicSharedMemorySize;
        if (cudaFuncSetAttribute(k_gemv_static<0>, a, kMaxDynSmem) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_static<kWideStages>, a, kMaxDynSmem) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_static<kDeepStages>, a, kMaxDynSmem) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_static<kSplitStages>, a, kMaxDynSmem) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_experts<0>, a, kMaxDynSmem) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_experts<kWideStages>, a, kMaxDynSmem) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_experts<kDeepStages>, a, kMaxDynSmem) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_experts<kPairStages>, a, kMaxDynSmem) != cudaSuccess)
            return static_cast<int>(GCUDA_E_CUDA);
        return static_cast<int>(GCUDA_OK);
    }();
    return rc;
}

// p.wpu / p.nslots are set here (plan_static); the grid is one CTA per SM at most
// (p.allow_half: a launch with fewer units than SMs runs one-tile units on the fan-in path, twice the CTAs)
inline int launch_static_gemv(StaticGemv p, cudaStream_t st, bool pdl) {
    GemvShape r;
    const bool split = p.allow_split && plan_split(p.act.cols, p.n_units, sm_count(), r);
    if (!split && !plan_static(p.act.cols, p.n_units, sm_count(), r)) return GCUDA_E_ARG;
    if (gemv_opt_in() != GCUDA_OK) return GCUDA_E_CUDA;
    p.wpu = r.wpu;
    p.nslots = r.nslots;
    p.half = r.stages == 0 && p.allow_half && p.n_units < sm_count();
    const int units = p.half ? 2 * p.n_units : p.n_units;
    const int grid = std::max(1, std::min(sm_count(), (units + r.nslots - 1) / r.nslots));
    cudaError_t e;
    if (split)
        e = launch_ex(k_gemv_static<kSplitStages>, dim3(grid), dim3(r.wpu * r.nslots * 32), r.smem, st, pdl, p);
    else if (r.stages == kWideStages)
        e = launch_ex(k_gemv_static<kWideStages>, dim3(grid), dim3(kStreamWarps * 32), r.smem, st, pdl, p);
    else if (r.stages == kDeepStages)
        e = launch_ex(k_gemv_static<kDeepStages>, dim3(grid), dim3(kDeepWarps * 32), r.smem, st, pdl, p);
    else
        e = launch_ex(k_gemv_static<0>, dim3(grid), dim3(kFanThreads), r.smem, st, pdl, p);
    return e == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

// The bf16 GEMV (router, Gated DeltaNet a/b): a CTA per (kBf16Rows rows, group of kBf16Tokens tokens). w and x 16-byte
// aligned, cols a multiple of 32, xstride of 4, n <= kMaxTok.
inline int launch_bf16_gemv(const uint16_t *w, int rows, int cols, const float *x, int xstride, int n, float *y,
                            int ystride, uint32_t *status, cudaStream_t st, bool pdl) {
    if (!w || !x || !y || rows <= 0 || cols <= 0 || cols % 32 || xstride % 4 || n < 1 || n > kMaxTok ||
        (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
        return GCUDA_E_ARG;
    const size_t smem = bf16_gemv_smem(cols);
    if (smem > static_cast<size_t>(kMaxDynSmem)) return GCUDA_E_ARG;
    static const bool opted =
        cudaFuncSetAttribute(k_bf16_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem) == cudaSuccess;
    if (!opted) return GCUDA_E_CUDA;
    const int groups = (n + kBf16Tokens - 1) / kBf16Tokens;
    const int rblocks = (rows + kBf16Rows - 1) / kBf16Rows;
    return launch_ex(k_bf16_gemv, dim3(rblocks * groups), dim3(kBf16Rows * 32), smem, st, pdl, w, rows, cols, x, xstride, n,
                     y, ystride, status) == cudaSuccess
               ? GCUDA_OK
               : GCUDA_E_CUDA;
}

}  // namespace gcu
