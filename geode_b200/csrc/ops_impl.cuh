// ops_impl.cuh - the operator layer of geode_cuda.h (gcuda_op_*): single kernels on caller-owned device buffers.
// (Included once, by backend.cu: the kernels live in one translation unit.)
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <functional>

#include "../../include/geode_cuda.h"
#include "accept.cuh"
#include "gemv_kernels.cuh"
#include "small_kernels.cuh"
#include "launch.hpp"
#include "umma_gemm.cuh"
#include "moe_umma.cuh"
#include "experts_lane.cuh"

using namespace gcu;

#define RC_GRID(call)                       \
    do {                                    \
        const int r_ = (call);              \
        if (r_ != GCUDA_OK) return r_;      \
    } while (0)

namespace gcu {
// out[i] = expf_ref of the float whose bits are first + i (the test hook gcuda_debug_expf_table)
__global__ void k_expf_table(uint32_t first, int64_t count, float *out) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = expf_ref(__uint_as_float(first + static_cast<uint32_t>(i)));
}
// Dynamic shared memory of the tensor-core product's launches: its rings, padded to more than half an SM's shared
// memory so that one CTA holds an SM (each allocates all 512 tensor-memory columns).
constexpr int kUmmaSmemFloor = 120 * 1024;
template <int NT>
constexpr int umma_launch_smem() {
    return static_cast<int>(umma_smem_bytes<NT>()) > kUmmaSmemFloor ? static_cast<int>(umma_smem_bytes<NT>()) : kUmmaSmemFloor;
}
// The expert lane kernels' shared-memory opt-in on the current device (the whole limit but their static part), and
// what it leaves them
inline int lane_opt_in(size_t *avail) {
    const int dev = current_device();
    if (dev < 0) return GCUDA_E_CUDA;
    DeviceState &d = device_state();
    std::lock_guard<std::mutex> lock(d.mu);
    if (!d.lane_rc[dev]) {
        bool ok = true;
        size_t least = 0;
        for (const void *fn : {reinterpret_cast<const void *>(k_experts_lane<true, kLaneStageGroups>),
                               reinterpret_cast<const void *>(k_experts_lane<false, kLaneStageGroups>),
                               reinterpret_cast<const void *>(k_experts_lane<true, 1>),
                               reinterpret_cast<const void *>(k_experts_lane<false, 1>)}) {
            cudaFuncAttributes fa{};
            ok = ok && cudaFuncGetAttributes(&fa, fn) == cudaSuccess;
            const int av = kMaxDynSmem - static_cast<int>(fa.sharedSizeBytes);
            ok = ok && cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, av) == cudaSuccess;
            least = least == 0 ? static_cast<size_t>(av) : std::min(least, static_cast<size_t>(av));
        }
        d.lane_avail[dev] = least;
        d.lane_rc[dev] = ok ? static_cast<int>(GCUDA_OK) : static_cast<int>(GCUDA_E_CUDA);
    }
    if (avail) *avail = d.lane_avail[dev];
    return d.lane_rc[dev];
}

// Both expert lane launches of a layer (gate_up, then down) for the route and buffers in `la`
inline int launch_lane_pair(LaneArgs la, int n, int K, int H, int ff, bool pdl, cudaStream_t st,
                            const std::function<bool(int, bool)> &mark = nullptr) {
    size_t avail = 0;
    if (lane_opt_in(&avail) != GCUDA_OK) return GCUDA_E_CUDA;
    const dim3 grid(sm_count()), block(kLaneWarps * 32);
    const int su = lane_stages(true, n, K, H, avail), sd = lane_stages(false, n, K, ff, avail);
    if (su < 2 || sd < 2) return GCUDA_E_ARG;
    if (mark && !mark(0, true)) return GCUDA_E_CUDA;
    la.stages = su;
    const size_t smu = lane_smem_bytes(true, n, K, H, su), smd = lane_smem_bytes(false, n, K, ff, sd);
    cudaError_t e = (H / 64) % kLaneStageGroups == 0
                        ? launch_ex(k_experts_lane<true, kLaneStageGroups>, grid, block, smu, st, pdl, la)
                        : launch_ex(k_experts_lane<true, 1>, grid, block, smu, st, pdl, la);
    if (e != cudaSuccess) return GCUDA_E_CUDA;
    if (mark && (!mark(0, false) || !mark(1, true))) return GCUDA_E_CUDA;
    la.stages = sd;
    e = (ff / 64) % kLaneStageGroups == 0 ? launch_ex(k_experts_lane<false, kLaneStageGroups>, grid, block, smd, st, pdl, la)
                                          : launch_ex(k_experts_lane<false, 1>, grid, block, smd, st, pdl, la);
    if (e != cudaSuccess) return GCUDA_E_CUDA;
    if (mark && !mark(1, false)) return GCUDA_E_CUDA;
    return GCUDA_OK;
}

inline int umma_opt_in() {
    const int dev = current_device();
    if (dev < 0) return GCUDA_E_CUDA;
    DeviceState &d = device_state();
    std::lock_guard<std::mutex> lock(d.mu);
    if (!d.umma_rc[dev]) {
        const cudaFuncAttribute at = cudaFuncAttributeMaxDynamicSharedMemorySize;
        const bool ok = cudaFuncSetAttribute(k_umma_gemm<4>, at, umma_launch_smem<4>()) == cudaSuccess &&
                        cudaFuncSetAttribute(k_umma_gemm<8>, at, umma_launch_smem<8>()) == cudaSuccess &&
                        cudaFuncSetAttribute(k_umma_gemm<16>, at, umma_launch_smem<16>()) == cudaSuccess;
        d.umma_rc[dev] = ok ? static_cast<int>(GCUDA_OK) : static_cast<int>(GCUDA_E_CUDA);
    }
    return d.umma_rc[dev];
}

// The tensor-core q4 product on a U-layout matrix for n token rows of act (the token block NT chosen from n); one
// persistent CTA an SM at most.
inline int launch_umma_gemm(UmmaGemmArgs a, cudaStream_t st) {
    if (umma_opt_in() != GCUDA_OK) return GCUDA_E_CUDA;
    const int nt = a.act.n <= 4 ? 4 : a.act.n <= 8 ? 8 : 16;
    const int units = (a.rows / kUmmaRows) * ((a.act.n + nt - 1) / nt);
    const dim3 grid(std::max(1, std::min(units, sm_count())));
    cudaError_t e;
    if (nt == 4) e = launch_ex(k_umma_gemm<4>, grid, dim3(kUmmaThreads), umma_launch_smem<4>(), st, false, a);
    else if (nt == 8) e = launch_ex(k_umma_gemm<8>, grid, dim3(kUmmaThreads), umma_launch_smem<8>(), st, false, a);
    else e = launch_ex(k_umma_gemm<16>, grid, dim3(kUmmaThreads), umma_launch_smem<16>(), st, false, a);
    return e == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

// the grouped form: the unit count lives on the device, so every SM gets a CTA (up to the table's capacity)
inline int launch_umma_grouped(UmmaGemmArgs a, int cap, cudaStream_t st) {
    if (umma_opt_in() != GCUDA_OK) return GCUDA_E_CUDA;
    const dim3 grid(std::max(1, std::min(cap, sm_count())));
    return launch_ex(k_umma_gemm<kMoeNT>, grid, dim3(kUmmaThreads), umma_launch_smem<kMoeNT>(), st, false, a) == cudaSuccess
               ? GCUDA_OK
               : GCUDA_E_CUDA;
}

}  // namespace gcu

extern "C" {

int gcuda_op_status(int clear) {
    uint32_t *st = device_status();
    if (!st) return GCUDA_E_CUDA;
    uint32_t v = 0;
    if (cudaMemcpy(&v, st, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return GCUDA_E_CUDA;
    if (clear && v && cudaMemset(st, 0, 4) != cudaSuccess) return GCUDA_E_CUDA;
    return static_cast<int>(v & 0x7FFFFFFFu);
}

size_t gcuda_op_q4_umma_bytes(int64_t rows, int64_t cols) {
    if (rows <= 0 || rows % kUmmaRows || cols <= 0 || cols % 256) return 0;
    return static_cast<size_t>(rows) * static_cast<size_t>(cols) / 16 * 9;
}

size_t gcuda_op_moe_umma_expert_bytes(int H, int ff) {
    const size_t gu = gcuda_op_q4_umma_bytes(2 * static_cast<int64_t>(ff), H), dn = gcuda_op_q4_umma_bytes(H, ff);
    return gu && dn ? gu + dn : 0;
}

size_t gcuda_op_moe_umma_work_bytes(int n, int K, int E, int H, int ff) {
    if (n < 1 || K < 1 || E < 1 || E > kMoeMaxExperts || gcuda_op_moe_umma_expert_bytes(H, ff) == 0) return 0;
    return moe_work_layout(n, K, E, H, ff, nullptr, nullptr);
}

int gcuda_op_moe_umma_relayout(const uint8_t *d_pack, size_t pack_stride, int E, int H, int ff, uint8_t *d_u,
                               void *stream) {
    const size_t eb = gcuda_op_moe_umma_expert_bytes(H, ff);
    const size_t gu = gcuda_op_q4_umma_bytes(2 * static_cast<int64_t>(ff), H);
    if (!d_pack || !d_u || eb == 0 || E < 1 || pack_stride < eb || (reinterpret_cast<uintptr_t>(d_u) & 15)) return GCUDA_E_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int e = 0; e < E; ++e) {   // (each expert's pack block: gate_up rows, then down rows - the same bytes, relaid)
        const uint8_t *src = d_pack + static_cast<size_t>(e) * pack_stride;
        uint8_t *dst = d_u + static_cast<size_t>(e) * eb;
        k_umma_relayout<<<148 * 4, 256, 0, st>>>(src, 2 * static_cast<int64_t>(ff), H, dst);
        k_umma_relayout<<<148 * 4, 256, 0, st>>>(src + gu, H, ff, dst + gu);
        count_launch(2);
    }
    return cudaGetLastError() == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

// ---- the verify step's expert kernels (a lane a weight row) as operators ----
namespace {
size_t lane_expert_bytes(int H, int ff) {
    return static_cast<size_t>(2 * ff) * (H / 16) * 9 + static_cast<size_t>(H) * (ff / 16) * 9;
}
struct LaneWork {
    RouteOut *route;
    int8_t *aq, *sq;
    float *as, *ss, *shout;
    int32_t *ab, *sb;
};
size_t lane_work_layout(int n, int K, int H, int ff, uint8_t *base, LaneWork *w) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t *p = base ? base + off : nullptr;
        off += (bytes + 255) / 256 * 256;
        return p;
    };
    const size_t P = static_cast<size_t>(n) * K, nb = static_cast<size_t>(ff / 16);
    uint8_t *r = take(sizeof(RouteOut)), *aq = take(P * ff), *as = take(P * nb * 4), *ab = take(P * nb * 4);
    uint8_t *sq = take(static_cast<size_t>(n) * ff), *ss = take(n * nb * 4), *sb = take(n * nb * 4);
    uint8_t *sh = take(static_cast<size_t>(n) * H * 4);
    if (w) {
        w->route = reinterpret_cast<RouteOut *>(r);
        w->aq = reinterpret_cast<int8_t *>(aq);
        w->as = reinterpret_cast<float *>(as);
        w->ab = reinterpret_cast<int32_t *>(ab);
        w->sq = reinterpret_cast<int8_t *>(sq);
        w->ss = reinterpret_cast<float *>(ss);
        w->sb = reinterpret_cast<int32_t *>(sb);
        w->shout = reinterpret_cast<float *>(sh);
    }
    return off;
}
}  // namespace

size_t gcuda_op_moe_lane_expert_bytes(int H, int ff) {
    return H > 0 && ff > 0 && H % 64 == 0 && ff % 64 == 0 ? lane_expert_bytes(H, ff) : 0;
}

size_t gcuda_op_moe_lane_work_bytes(int n, int K, int H, int ff) {
    if (n < 1 || n > kMaxTok || K < 1 || K > 8 || H % 64 || ff % 64 || H <= 0 || ff <= 0) return 0;
    return lane_work_layout(n, K, H, ff, nullptr, nullptr);
}

int gcuda_op_moe_lane_relayout(const uint8_t *d_pack, size_t pack_stride, int E, int H, int ff, uint8_t *d_out,
                               void *stream) {
    const size_t eb = gcuda_op_moe_lane_expert_bytes(H, ff);
    if (!d_pack || !d_out || eb == 0 || E < 1 || pack_stride < eb || (reinterpret_cast<uintptr_t>(d_out) & 15))
        return GCUDA_E_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the pack's rows -> tiles (into a temporary), then tiles -> R16 for every block at once
    uint8_t *tmp = nullptr;
    if (cudaMalloc(&tmp, static_cast<size_t>(E) * eb) != cudaSuccess) return GCUDA_E_MEMORY;
    const size_t gu = static_cast<size_t>(2 * ff) * (H / 16) * 9;
    int rc = GCUDA_OK;
    for (int e = 0; e < E && rc == GCUDA_OK; ++e) {
        const uint8_t *src = d_pack + static_cast<size_t>(e) * pack_stride;
        uint8_t *dst = tmp + static_cast<size_t>(e) * eb;
        rc = gcuda_op_q4_relayout(src, 2 * static_cast<int64_t>(ff), H, dst, stream);
        if (rc == GCUDA_OK) rc = gcuda_op_q4_relayout(src + gu, H, ff, dst + gu, stream);
    }
    if (rc == GCUDA_OK) {
        const int64_t gt = 2 * ff / 16, dt = H / 16;
        k_relayout_r16<<<relayout_grid(gt * (H / 64) * 16 * E), 256, 0, st>>>(tmp, gt, H, d_out, E, eb);
        k_relayout_r16<<<relayout_grid(dt * (ff / 64) * 16 * E), 256, 0, st>>>(tmp + gu, dt, ff, d_out + gu, E, eb);
        count_launch(2);
        if (cudaStreamSynchronize(st) != cudaSuccess) rc = GCUDA_E_CUDA;
    }
    cudaFree(tmp);
    return rc;
}

int gcuda_op_moe_lane(const uint8_t *d_r16, const float *d_globals, int E, int H, int ff, const int8_t *d_q,
                      const float *d_scale, const int32_t *d_bsum, int n, const int *d_ids, int K, float *d_out,
                      void *d_work, size_t work_bytes, void *stream) {
    const size_t need = gcuda_op_moe_lane_work_bytes(n, K, H, ff);
    if (!d_r16 || !d_globals || !d_q || !d_scale || !d_bsum || !d_ids || !d_out || !d_work || need == 0 ||
        work_bytes < need || E < 1 || E > 1024 || (reinterpret_cast<uintptr_t>(d_work) & 255) ||
        (reinterpret_cast<uintptr_t>(d_r16) & 15) || (reinterpret_cast<uintptr_t>(d_q) & 15))
        return GCUDA_E_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t *status = device_status();
    if (!status) return GCUDA_E_CUDA;
    LaneWork w{};
    lane_work_layout(n, K, H, ff, static_cast<uint8_t *>(d_work), &w);
    if (launch_ex(k_route_from_ids, dim3(1), dim3(256), 0, st, false, d_ids, n, K, E, w.route, status) != cudaSuccess)
        return GCUDA_E_CUDA;
    const size_t eb = lane_expert_bytes(H, ff), tb = static_cast<size_t>(H / 64) * kLaneTileGroup;
    LaneArgs la{};
    la.route = w.route;
    la.experts = d_r16;
    la.stride = eb;
    la.down_off = static_cast<size_t>(2 * ff / 16) * tb;
    la.globals = d_globals;
    // (the kernels always run the layer's shared expert too: expert 0's matrices stand in, into a scratch output)
    la.sh_gate = d_r16;
    la.sh_up = d_r16 + static_cast<size_t>(ff / 16) * tb;
    la.sh_down = d_r16 + la.down_off;
    la.sh_g0 = la.sh_g1 = la.sh_g2 = 1.0f;
    la.H = H;
    la.ff = ff;
    la.K = K;
    la.n = n;
    la.hq = ActSet{d_q, d_scale, d_bsum, H, n, H, H / 16};
    la.amid = ActSet{w.aq, w.as, w.ab, ff, n * K, ff, ff / 16};
    la.shact = ActSet{w.sq, w.ss, w.sb, ff, n, ff, ff / 16};
    la.eout = d_out;
    la.shout = w.shout;
    la.status = status;
    la.world = 1;
    return launch_lane_pair(la, n, K, H, ff, false, st);
}

int gcuda_op_moe_umma(const uint8_t *d_u, const float *d_globals, int E, int H, int ff, const int8_t *d_q,
                      const float *d_scale, const int32_t *d_bsum, int n, const int *d_ids, int K, float *d_out,
                      void *d_work, size_t work_bytes, void *stream) {
    const size_t need = gcuda_op_moe_umma_work_bytes(n, K, E, H, ff);
    if (!d_u || !d_globals || !d_q || !d_scale || !d_bsum || !d_ids || !d_out || !d_work || need == 0 ||
        work_bytes < need || H > kUmmaMaxCols || ff > kUmmaMaxCols || (reinterpret_cast<uintptr_t>(d_work) & 255) ||
        (reinterpret_cast<uintptr_t>(d_u) & 15) || (reinterpret_cast<uintptr_t>(d_q) & 15) ||
        static_cast<int64_t>(n) * K > (1 << 24))
        return GCUDA_E_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t *status = device_status();
    if (!status) return GCUDA_E_CUDA;
    MoeWork w{};
    moe_work_layout(n, K, E, H, ff, static_cast<uint8_t *>(d_work), &w);
    const int P = n * K;
    MoePlanArgs pa{};
    pa.ids = d_ids;
    pa.P = P;
    pa.E = E;
    pa.experts = d_u;
    pa.stride = gcuda_op_moe_umma_expert_bytes(H, ff);
    pa.gu_bytes = gcuda_op_q4_umma_bytes(2 * static_cast<int64_t>(ff), H);
    pa.globals = d_globals;
    pa.tiles_gu = 2 * ff / kUmmaRows;
    pa.tiles_dn = H / kUmmaRows;
    pa.w = w;
    pa.status = status;
    if (launch_ex(k_moe_plan, dim3(1), dim3(kMoePlanThreads), 0, st, false, pa) != cudaSuccess) return GCUDA_E_CUDA;
    UmmaGemmArgs a{};
    a.rows = 2 * ff;
    a.cols = H;
    a.act = ActSet{d_q, d_scale, d_bsum, H, n, H, H / 16};
    a.y = w.gu;
    a.ystride = 2 * ff;
    a.status = status;
    a.units = w.units_gu;
    a.n_units = w.counts;
    a.toklist = w.toklist;
    a.act_div = K;
    RC_GRID(launch_umma_grouped(a, w.cap_gu, st));
    const int64_t work = static_cast<int64_t>(P) * ff;
    if (launch_ex(k_swiglu_quant, dim3(static_cast<int>(std::min<int64_t>((work + 255) / 256, 148 * 16))), dim3(256), 0, st,
                  false, static_cast<const float *>(w.gu), P, ff, w.aq, w.as, w.ab) != cudaSuccess)
        return GCUDA_E_CUDA;
    a.rows = H;
    a.cols = ff;
    a.act = ActSet{w.aq, w.as, w.ab, ff, P, ff, ff / 16};
    a.y = d_out;
    a.ystride = H;
    a.units = w.units_dn;
    a.n_units = w.counts + 1;
    a.act_div = 1;
    RC_GRID(launch_umma_grouped(a, w.cap_dn, st));
    return GCUDA_OK;
}

int gcuda_op_q4_umma_relayout(const uint8_t *d_pack, int64_t rows, int64_t cols, uint8_t *d_u, void *stream) {
    if (!d_pack || !d_u || gcuda_op_q4_umma_bytes(rows, cols) == 0 || (reinterpret_cast<uintptr_t>(d_u) & 15))
        return GCUDA_E_ARG;
    k_umma_relayout<<<148 * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_pack, rows, cols, d_u);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

int gcuda_op_q4_gemm_umma(const uint8_t *d_u, int64_t rows, int64_t cols, float global, const int8_t *d_q,
                          const float *d_scale, const int32_t *d_bsum, int n, float *d_y, void *stream) {
    if (!d_u || !d_q || !d_scale || !d_bsum || !d_y || gcuda_op_q4_umma_bytes(rows, cols) == 0 || n < 1 ||
        rows > (1 << 24) || cols > kUmmaMaxCols || (reinterpret_cast<uintptr_t>(d_u) & 15) ||
        (reinterpret_cast<uintptr_t>(d_q) & 15))
        return GCUDA_E_ARG;
    UmmaGemmArgs a{};
    a.w = d_u;
    a.rows = static_cast<int>(rows);
    a.cols = static_cast<int>(cols);
    a.global = global;
    a.act = ActSet{d_q, d_scale, d_bsum, static_cast<int>(cols), n, static_cast<int>(cols), static_cast<int>(cols / 16)};
    a.y = d_y;
    a.ystride = static_cast<int>(rows);
    a.status = device_status();
    if (!a.status) return GCUDA_E_CUDA;
    return launch_umma_gemm(a, static_cast<cudaStream_t>(stream));
}


size_t gcuda_op_q4_tiled_bytes(int64_t rows, int64_t cols) {
    const int64_t rows_pad = (rows + 31) / 32 * 32;
    return static_cast<size_t>(rows_pad / 16) * static_cast<size_t>(tile_bytes(static_cast<int>(cols)));
}

int gcuda_op_q4_relayout(const uint8_t *d_pack, int64_t rows, int64_t cols, uint8_t *d_tiles, void *stream) {
    if (!d_pack || !d_tiles || rows <= 0 || cols <= 0 || cols % 64) return GCUDA_E_ARG;
    const int64_t rows_pad = (rows + 31) / 32 * 32;
    const int64_t work = rows_pad / 16 * (cols / 64) * 32;
    const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, 148 * 32));
    k_relayout_q4<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_pack, rows, rows_pad, static_cast<int>(cols), d_tiles);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

int gcuda_op_quantize(const float *d_x, int n, int cols, int8_t *d_q, float *d_scale, int32_t *d_bsum, void *stream) {
    if (!d_x || n <= 0 || cols <= 0 || cols % 64) return GCUDA_E_ARG;
    const int64_t work = static_cast<int64_t>(n) * cols;
    const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, 148 * 16));
    k_quantize<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_x, n, cols, cols, d_q, d_scale, d_bsum);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

int gcuda_op_q4_gemv(const uint8_t *d_tiles, int64_t rows, int64_t cols, float global, const int8_t *d_q,
                     const float *d_scale, const int32_t *d_bsum, int n, float *d_y, void *stream) {
    if (!d_tiles || rows <= 0 || rows % 32 || cols <= 0 || cols % 64 || n < 1 || n > kMaxTok) return GCUDA_E_ARG;
    StaticGemv p{};
    p.units = nullptr;
    p.n_units = static_cast<int>(rows / 32);
    p.tiles = d_tiles;
    p.global = global;
    p.y = d_y;
    p.ystride = static_cast<int>(rows);
    p.mode = kStore;
    p.act = ActSet{d_q, d_scale, d_bsum, static_cast<int>(cols), n, static_cast<int>(cols), static_cast<int>(cols / 16)};
    p.ncols = n;
    p.allow_half = 1;
    p.status = device_status();
    if (!p.status) return GCUDA_E_CUDA;
    return launch_static_gemv(p, static_cast<cudaStream_t>(stream), false);
}

int gcuda_op_q4_dequant(const uint8_t *d_tiles, int64_t cols, float global, const int64_t *d_rows, int nrows,
                        float *d_out, void *stream) {
    if (!d_tiles || cols % 64 || nrows <= 0) return GCUDA_E_ARG;
    const int64_t work = static_cast<int64_t>(nrows) * cols;
    const int grid = static_cast<int>(std::min<int64_t>((work + 255) / 256, 148 * 16));
    k_dequant_rows<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_tiles, static_cast<int>(cols), global, d_rows,
                                                                        nrows, d_out);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

int gcuda_op_bf16_gemv(const uint16_t *d_w, int rows, int cols, const float *d_x, int n, float *d_y, void *stream) {
    uint32_t *status = device_status();
    if (!status) return GCUDA_E_CUDA;
    return launch_bf16_gemv(d_w, rows, cols, d_x, cols, n, d_y, rows, status, static_cast<cudaStream_t>(stream), false);
}

int gcuda_op_route_topk(const float *d_logits, int n, int E, int K, int *d_ids, float *d_weights, void *stream) {
    if (!d_logits || n < 1 || E < 1 || E > 1024 || K < 1 || K > E) return GCUDA_E_ARG;
    const int warps = 4;
    k_route_topk<<<(n + warps - 1) / warps, warps * 32, warps * E * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
        d_logits, n, E, K, d_ids, d_weights);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

size_t gcuda_op_route_out_bytes(void) { return sizeof(RouteOut); }

int gcuda_op_route_union(const float *d_logits, int n, int E, int K, void *d_out, size_t out_bytes, void *stream) {
    if (!d_logits || !d_out || n < 1 || n > kMaxTok || E < 1 || E > 1024 || K < 1 || K > 8 || K > E ||
        out_bytes < sizeof(RouteOut))
        return GCUDA_E_ARG;
    k_route<<<1, kRouteThreads, kMaxTok * E * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
        d_logits, n, E, K, static_cast<RouteOut *>(d_out), nullptr, 0, 1);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

int gcuda_op_norm_quant(const float *d_x, int n, int H, const float *d_w, float eps, float *d_hf, int8_t *d_q,
                        float *d_scale, int32_t *d_bsum, void *stream) {
    if (!d_x || !d_w || !d_q || !d_scale || !d_bsum || n < 1 || H < 16 || H % 16 || H > kNormThreads * kNormPer)
        return GCUDA_E_ARG;
    NormArgs a{};
    a.x = const_cast<float *>(d_x);   // (read only: the combine, which writes x, is off)
    a.w = d_w;
    a.eps = eps;
    a.H = H;
    a.n = n;
    a.hf = d_hf;
    a.q = d_q;
    a.scale = d_scale;
    a.bsum = d_bsum;
    return launch_ex(k_norm_quant, dim3(n), dim3(kNormThreads), 0, static_cast<cudaStream_t>(stream), false, a) ==
                   cudaSuccess
               ? GCUDA_OK
               : GCUDA_E_CUDA;
}

int gcuda_debug_expf_table(uint32_t first, int64_t count, float *d_out, void *stream) {
    if (!d_out || count < 1 || static_cast<uint64_t>(first) + static_cast<uint64_t>(count) > (1ull << 32))
        return GCUDA_E_ARG;
    k_expf_table<<<148 * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(first, count, d_out);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GCUDA_OK : GCUDA_E_CUDA;
}

int gcuda_op_greedy_verify(const float *d_target, const int *d_drafts, int S, int k, int V, uint64_t *d_scratch,
                           int *d_accepted, int *d_next, void *stream) {
    if (!d_target || !d_drafts || !d_scratch || !d_accepted || !d_next || S < 1 || k < 1 || V < 1 || S > 65535 ||
        static_cast<int64_t>(S) * (k + 1) > 65535)
        return GCUDA_E_ARG;   // (rows on the grid's y dimension)
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int rows = S * (k + 1);
    auto *best = reinterpret_cast<unsigned long long *>(d_scratch);
    if (cudaMemsetAsync(best, 0, sizeof(unsigned long long) * rows, st) != cudaSuccess) return GCUDA_E_CUDA;
    if (launch_ex(k_argmax_rows, dim3(argmax_slices(rows, sm_count()), rows), dim3(kArgmaxThreads), 0, st, false, d_target, V,
                  best) != cudaSuccess ||
        launch_ex(k_greedy_decide, dim3((S + 127) / 128), dim3(128), 0, st, false, best, d_drafts, S, k, d_accepted,
                  d_next) != cudaSuccess)
        return GCUDA_E_CUDA;
    return GCUDA_OK;
}

}  // extern "C"
