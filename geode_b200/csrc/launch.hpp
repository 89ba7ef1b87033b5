// launch.hpp - host-side launch helpers: the static GEMV's launch (shared-memory opt-in, grid sized to the SMs,
// optionally as a programmatic dependent launch), a process-wide launch counter and the operators' status word.
// What depends on the GPU (its SM count, the kernels' shared-memory opt-in, the status word) is kept per device and
// set up the first time a launch on that device (the current one) needs it, so handles on several GPUs of one
// process each get their own.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>

#include "../../include/geode_cuda.h"
#include "gemv_kernels.cuh"

namespace gcu {

inline std::atomic<uint64_t> &launch_counter() {
    static std::atomic<uint64_t> n{0};
    return n;
}
inline void count_launch(uint64_t k = 1) { launch_counter().fetch_add(k, std::memory_order_relaxed); }

// Per-device set-up state, filled lazily under one mutex. gemv_rc / bf16_rc: 0 = not tried yet, else the outcome
// (GCUDA_OK or GCUDA_E_CUDA) of the shared-memory opt-in on that device.
constexpr int kMaxDevices = 64;
struct DeviceState {
    std::mutex mu;
    int sms[kMaxDevices] = {};
    int gemv_rc[kMaxDevices] = {};
    int bf16_rc[kMaxDevices] = {};
    int umma_rc[kMaxDevices] = {};
    int lane_rc[kMaxDevices] = {};
    size_t lane_avail[kMaxDevices] = {};   // the expert lane kernels' dynamic shared memory limit
    uint32_t *status[kMaxDevices] = {};
};
inline DeviceState &device_state() {
    static DeviceState d;
    return d;
}
inline int current_device() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    return dev;
}

inline int sm_count() {
    const int dev = current_device();
    if (dev < 0) return 148;
    DeviceState &d = device_state();
    std::lock_guard<std::mutex> lock(d.mu);
    if (!d.sms[dev]) {
        int c = 0;
        if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
        d.sms[dev] = c;
    }
    return d.sms[dev];
}

// The operators' status word on the current device (device memory, zeroed once): kernels OR error flags into it.
inline uint32_t *device_status() {
    const int dev = current_device();
    if (dev < 0) return nullptr;
    DeviceState &d = device_state();
    std::lock_guard<std::mutex> lock(d.mu);
    if (!d.status[dev]) {
        void *q = nullptr;
        if (cudaMalloc(&q, 4) != cudaSuccess) return nullptr;
        if (cudaMemset(q, 0, 4) != cudaSuccess) {
            cudaFree(q);
            return nullptr;
        }
        d.status[dev] = static_cast<uint32_t *>(q);
    }
    return d.status[dev];
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
// (cudaFuncSetAttribute acts on the current device's context, so each device opts in once.)
inline int gemv_opt_in() {
    const int dev = current_device();
    if (dev < 0) return GCUDA_E_CUDA;
    DeviceState &d = device_state();
    std::lock_guard<std::mutex> lock(d.mu);
    if (!d.gemv_rc[dev]) {
        const cudaFuncAttribute a = cudaFuncAttributeMaxDynamicSharedMemorySize;
        const bool ok = cudaFuncSetAttribute(k_gemv_static<0>, a, kMaxDynSmem) == cudaSuccess &&
                        cudaFuncSetAttribute(k_gemv_static<kWideStages>, a, kMaxDynSmem) == cudaSuccess &&
                        cudaFuncSetAttribute(k_gemv_static<kDeepStages>, a, kMaxDynSmem) == cudaSuccess &&
                        cudaFuncSetAttribute(k_gemv_static<kSplitStages>, a, kMaxDynSmem) == cudaSuccess;
        d.gemv_rc[dev] = ok ? static_cast<int>(GCUDA_OK) : static_cast<int>(GCUDA_E_CUDA);
    }
    return d.gemv_rc[dev];
}

inline int bf16_opt_in() {
    const int dev = current_device();
    if (dev < 0) return GCUDA_E_CUDA;
    DeviceState &d = device_state();
    std::lock_guard<std::mutex> lock(d.mu);
    if (!d.bf16_rc[dev])
        d.bf16_rc[dev] = cudaFuncSetAttribute(k_bf16_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem) ==
                                 cudaSuccess
                             ? static_cast<int>(GCUDA_OK)
                             : static_cast<int>(GCUDA_E_CUDA);
    return d.bf16_rc[dev];
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
    if (bf16_opt_in() != GCUDA_OK) return GCUDA_E_CUDA;
    const int groups = (n + kBf16Tokens - 1) / kBf16Tokens;
    const int rblocks = (rows + kBf16Rows - 1) / kBf16Rows;
    return launch_ex(k_bf16_gemv, dim3(rblocks * groups), dim3(kBf16Rows * 32), smem, st, pdl, w, rows, cols, x, xstride, n,
                     y, ystride, status) == cudaSuccess
               ? GCUDA_OK
               : GCUDA_E_CUDA;
}

}  // namespace gcu
