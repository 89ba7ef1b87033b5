// gemv_kernels.cuh - the launchable GEMV kernels over q4_gemv.cuh's unit stream, the load-time relayout, and the
// activation quantizer.
#pragma once

#include "gemv_core.cuh"

namespace gcu {

// ------------------------------------------------------------------------------------------- relayout ----
// pack rows [rows][cols/2 codes | cols/16 scales] -> 16-row tiles (q4_gemv.cuh's tile layout). rows_pad: rows
// rounded up to 32; padding rows get level codes of level -1 and scale byte 0 (they contribute 0).
// One thread per (tile, group, lane) word quadruple.
__global__ void k_relayout_q4(const uint8_t *__restrict__ src, int64_t rows, int64_t rows_pad, int cols,
                              uint8_t *__restrict__ dst) {
    const int ng = cols / 64;
    const int64_t tiles = rows_pad / 16;
    const int64_t total = tiles * ng * 32;
    const size_t rb = static_cast<size_t>(cols / 16) * 9;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int lane = static_cast<int>(i % 32);
        const int g = static_cast<int>((i / 32) % ng);
        const int64_t tile = i / (32 * ng);
        const int gid = lane >> 2, tig = lane & 3;
        const int64_t r0 = tile * 16 + gid, r1 = r0 + 8;
        uint8_t *out = dst + static_cast<size_t>(tile) * (ng * kGroupBytes) + static_cast<size_t>(g) * kGroupBytes;
        uint32_t words[4];
        for (int j = 0; j < 4; ++j) {
            const int b = 4 * g + j;
            uint32_t w = 0;
            for (int i2 = 0; i2 < 4; ++i2) {
                const int col = 16 * b + 4 * tig + i2;   // value index within the row
                uint32_t c0 = 7, c1 = 7;                   // padding: affine 7 = level -1 (scale 0)
                if (r0 < rows) {
                    const uint8_t byte = src[static_cast<size_t>(r0) * rb + col / 2];
                    const uint32_t c = (col & 1) ? (byte >> 4) : (byte & 15);
                    c0 = c < 8 ? c + 8 : 15 - c;
                }
                if (r1 < rows) {
                    const uint8_t byte = src[static_cast<size_t>(r1) * rb + col / 2];
                    const uint32_t c = (col & 1) ? (byte >> 4) : (byte & 15);
                    c1 = c < 8 ? c + 8 : 15 - c;
                }
                w |= (c0 | (c1 << 4)) << (8 * i2);
            }
            words[j] = w;
        }
        *reinterpret_cast<uint4 *>(out + lane * 16) = make_uint4(words[0], words[1], words[2], words[3]);
        // the scales: lane l < 16 writes row l's four bytes
        if (lane < 16) {
            const int64_t r = tile * 16 + lane;
            uint32_t s = 0;
            if (r < rows)
                for (int j = 0; j < 4; ++j)
                    s |= static_cast<uint32_t>(src[static_cast<size_t>(r) * rb + static_cast<size_t>(cols / 2) + 4 * g + j]) << (8 * j);
            *reinterpret_cast<uint32_t *>(out + 512 + lane * 4) = s;
        }
    }
}

// Row r of a tiled matrix back to floats: (level * 1) * (e4m3 * global) (engine/src/kernels.cpp:1214-1228) - the
// dequantized weights, for the bit-exactness check of the device copy. One thread per value.
__global__ void k_dequant_rows(const uint8_t *__restrict__ tiles, int cols, float global, const int64_t *__restrict__ rows,
                               int nrows, float *__restrict__ out) {
    const int ng = cols / 64;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < static_cast<int64_t>(nrows) * cols;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int k = static_cast<int>(i % cols);
        const int64_t r = rows[i / cols];
        const int64_t tile = r / 16;
        const int rr = static_cast<int>(r % 16), gid = rr & 7, hi = rr >> 3;
        const int b = k / 16, g = b / 4, j = b % 4, kk = k % 16, tig = kk / 4, i2 = kk % 4;
        const uint8_t *grp = tiles + static_cast<size_t>(tile) * ng * kGroupBytes + static_cast<size_t>(g) * kGroupBytes;
        const uint32_t w = *reinterpret_cast<const uint32_t *>(grp + (4 * gid + tig) * 16 + 4 * j);
        const uint32_t c = (w >> (8 * i2 + 4 * hi)) & 15;
        const int level = 2 * static_cast<int>(c) - 15;
        const uint8_t sb = grp[512 + rr * 4 + j];
        const float e4 = e4m3x2_to_float2(sb).x;
        out[i] = __fmul_rn(__fmul_rn(static_cast<float>(level), 1.0f), __fmul_rn(e4, global));
    }
}

// ------------------------------------------------------------------------------------------- quantize ----
// n vectors of cols floats (rows xstride apart) -> an ActSet (quantize_activation, engine/src/kernels.cpp:1254-1295).
// One half-warp per block of 16 values.
__global__ void k_quantize(const float *__restrict__ x, int n, int cols, int xstride, int8_t *__restrict__ q,
                           float *__restrict__ scale, int32_t *__restrict__ bsum) {
    const int nb = cols / 16;
    const int64_t total = static_cast<int64_t>(n) * nb * 16;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int k = static_cast<int>(i % 16);
        const int64_t blk = i / 16;
        const int t = static_cast<int>(blk / nb), b = static_cast<int>(blk % nb);
        const float v = x[static_cast<size_t>(t) * xstride + b * 16 + k];
        float amax = fabsf(v);
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        const int qv = max(-127, min(127, __float2int_rn(__fmul_rn(v, inv))));
        int s = qv;
        for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        q[static_cast<size_t>(t) * cols + b * 16 + k] = static_cast<int8_t>(qv);
        if (k == 0) {
            scale[static_cast<size_t>(t) * nb + b] = __fdiv_rn(amax, 127.0f);
            bsum[static_cast<size_t>(t) * nb + b] = s;
        }
    }
}

// ------------------------------------------------------------------------------------------- the static GEMV ----
// A table of units (built on the host), or one plain matrix, against one ActSet; units are dealt to the CTAs in turn. Every
// unit multiplies the same activations, so the CTA stages one image of all K (after the previous kernel ends) and
// every warp reads its groups from it.
struct StaticGemv {
    const GemvUnit *units;   // a unit table, or NULL: one plain matrix (below), units made on the fly
    int n_units;
    // the plain matrix: tiles (rows / 32 units of two adjacent tiles), y [ncols][ystride]
    const uint8_t *tiles;
    float global;
    float *y;
    int ystride, mode;
    ActSet act;
    int ncols;          // token columns (<= kMaxTok)
    int wpu, nslots;    // the launch shape (plan_static)
    int allow_half;     // the units may be split into one-tile units (no swiglu unit)
    int half;           // (the fan-in path) units of one tile: n_units * 2 of them
    int allow_split;    // the units' K may be split over warps (f32 sums in slice order: not the single chain's bits)
    uint32_t *status;
};

// K slices (stream_units with ks > 1): up to kSplitWarps warps a CTA, ks warps a unit, for launches with too few units
// to give every warp one (the verify step's projections). The rings (kSplitStages) hold a slice of up to
// kSplitStages - 2 groups whole, so all of it is requested before the previous kernel ends. ks a power of two, each
// slice an even number of groups; the xchg buffers after the warps' regions.
constexpr int kSplitWarps = 16;
constexpr int kSplitStages = 10;
__host__ __device__ inline size_t split_xchg_bytes(int slots, int ks) {
    return static_cast<size_t>(slots) * 2 * (ks - 1) * 1024;
}
inline bool plan_split(int cols, int n_units, int sms, GemvShape &r) {
    const int G = cols / 64;
    const int slots = (n_units + sms - 1) / sms;
    if (slots * 2 > kSplitWarps) return false;
    int ks = 1;
    while (ks * 2 <= 16 && ks * 2 * slots <= kSplitWarps && G % (4 * ks) == 0) ks *= 2;
    for (; ks >= 2; ks /= 2) {
        const int warps = ks * slots;
        const size_t smem = static_cast<size_t>(act_smem_bytes(cols)) + warps * stream_warp_bytes(kSplitStages, 0) +
                            split_xchg_bytes(slots, ks);
        if (smem <= static_cast<size_t>(kMaxDynSmem)) {
            r = GemvShape{ks, slots, G / ks, smem, kSplitStages};
            return true;
        }
    }
    return false;
}

inline bool plan_static(int cols, int n_units, int sms, GemvShape &r) {
    return plan_gemv(cols, cols, false, static_cast<size_t>(act_smem_bytes(cols)), (n_units + sms - 1) / sms, r);
}

// kStages: the streaming path's ring depth (a warp per unit, stream_units), 0: the fan-in (fan_units)
template <int kStages>
__global__ void __launch_bounds__((kStages ? stream_warps(kStages) : kFanWarps) * 32, 1) k_gemv_static(StaticGemv p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int cols = p.act.cols, wpu = p.wpu, nslots = p.nslots;
    uint8_t *img = smem;
    auto prelude = [&]() {
        // (the weights do not depend on the previous kernel: their first stages are already requested)
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;");
        stage_full(p.act, p.ncols, img);
        __syncthreads();
    };
    if (warp >= nslots * wpu) {   // (a warp without a slot helps stage the image)
        prelude();
        return;
    }
    const int slot = warp / wpu;
    const size_t tb = static_cast<size_t>(cols / 64) * kGroupBytes;
    auto unit_at = [&](int u, GemvUnit &U) {
        if (p.units) {
            U = p.units[u];
            U.tok_mask &= (1 << p.ncols) - 1;
            return true;
        }
        U.w0 = p.tiles + (2 * static_cast<size_t>(u)) * tb;
        U.w1 = U.w0 + tb;
        U.g0 = U.g1 = p.global;
        U.y0 = p.y + 32 * static_cast<size_t>(u);
        U.y1 = U.y0 + 16;
        U.ngroups = cols / 64;
        U.ystride = p.ystride;
        U.mode = p.mode;
        U.tok_mask = (1 << p.ncols) - 1;
        U.act_id = 0;
        for (int t = 0; t < kMaxTok; ++t) U.slot[t] = t;
        return true;
    };
    auto get = [&](int i, GemvUnit &U) -> bool {
        // CTA-major: unit u on CTA u % grid, so every SM holds the same count (+-1) whatever the slots' share
        const int u = blockIdx.x + gridDim.x * (slot + nslots * i);
        if (!p.half) return u < p.n_units && unit_at(u, U);
        // one-tile units: tile u % 2 of unit u / 2, as tile A
        if (u >= 2 * p.n_units || !unit_at(u >> 1, U)) return false;
        if (u & 1) {
            U.w0 = U.w1;
            U.g0 = U.g1;
            U.y0 = U.y1;
        }
        U.w1 = U.w0;
        U.y1 = nullptr;
        return true;
    };
    auto epi = [](const GemvUnit &U, const float(&y0)[4], const float(&y1)[4], int gid, int tig) {
        epi_store(U, y0, y1, gid, tig);
    };
    if constexpr (kStages > 0) {
        StreamCtx c;
        uint8_t *wbase = smem + act_smem_bytes(cols) + static_cast<size_t>(warp) * stream_warp_bytes(kStages, 0);
        c.e4p = reinterpret_cast<float *>(wbase);
        c.ring = wbase + 2048;
        c.img = img;
        c.img_ts = act_tstride(cols);
        c.ngroups = (cols / 64) / wpu;
        c.zero = static_cast<uint64_t>(static_cast<uint32_t>(wpu) >> 31);
        if (wpu > 1) {   // K slices: warp slot * wpu + kr walks slice kr of its slot's units
            c.ks = wpu;
            c.kr = warp % wpu;
            c.g0 = c.img_g0 = c.kr * c.ngroups;
            c.bar_id = 1 + slot;
            c.xchg = reinterpret_cast<uint4 *>(smem + act_smem_bytes(cols) +
                                               static_cast<size_t>(nslots * wpu) * stream_warp_bytes(kStages, 0) +
                                               split_xchg_bytes(slot, wpu));
        }
        stream_units<kStages>(get, c, [](const GemvUnit &) {}, epi, true, prelude);
    } else {
        FanCtx c;
        c.img = img;
        c.img_ts = act_tstride(cols);
        c.prod = smem + act_smem_bytes(cols);
        c.e4p = reinterpret_cast<float *>(c.prod + 2 * kFanSlotBytes);
        c.xchg = reinterpret_cast<float4 *>(c.prod + 2 * kFanSlotBytes + kFanProducers * 1024);
        c.ngroups = cols / 64;
        c.zero = static_cast<uint64_t>(static_cast<uint32_t>(nslots) >> 31);
        c.half = p.half != 0;
        fan_units(get, c, [](const GemvUnit &) { return false; }, [](const GemvUnit &, int, int) {}, epi, true, prelude);
    }
}

}  // namespace gcu

#include "layer_kernels.cuh"

namespace gcu {

}  // namespace gcu
