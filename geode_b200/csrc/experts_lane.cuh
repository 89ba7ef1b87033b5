// experts_lane.cuh - the MoE's experts at the verify step's few token rows (engine/src/model.cpp:4496-4543 for the
// routed experts of the union, 4554-4585 for the shared expert), one lane a weight row.
//
// At 5 rows and top-8 of 256 experts a routed expert serves about one token (40 picks over a union of ~38), so an MMA
// tile - which multiplies every token column - does several times the work each expert needs. Here lane r of a warp
// holds row r of its unit for the whole K: the row's codes times the activations of only the tokens that picked the
// expert (dp4a on the 4-bit codes), and the reference's chain over the row's blocks (engine/src/kernels.cpp:1304-1322:
// acc += float(isum_b) * (e4m3_b * ascale_b) in block order, y = acc * global) in that one thread, so every output is
// the reference's bits.
//
// A unit is two 16-row tiles: gate_up - gate tile j (lanes 0-15) and up tile j (lanes 16-31), whose SwiGLU meets in a
// shuffle, quantized into the pick's activation row; down - tiles 2j, 2j+1 (output rows 32 j + lane) into the pick's
// expert-output row. The shared expert is the last member. Warps take units in turn (CTA-major, so every SM gets a
// share); each warp streams its units through its own ring of bulk copies (cp.async.bulk, an mbarrier a stage,
// bounded waits) whose stage holds four 64-column groups of both tiles (4.6 KB): every pass round the ring (wait,
// refill) costs the warp a few hundred cycles whatever the stage's size, so a warp keeps HBM busy only with stages of
// kilobytes (measured on B200: about 1.0 TB/s with 576-byte stages at 4 warps an SM, about 4.5 TB/s with 4.6 KB). The
// activation rows are staged once per CTA.
//
// The weights in the "R16" layout (k_relayout_r16, from the tiled layout): per 16-row tile and 64-column group g, 576
// bytes - code chunk k (blocks 4 g + 2 k, + 1) at 256 k + 16 r for row r, whose byte 8 h + m (block 4 g + 2 k + h,
// m < 8) holds c'(16 b + m) in its low nibble and c'(16 b + 8 + m) in its high one; then at 512 + 4 r row r's four
// E4M3 scale bytes. c' is the affine code (level 2 c' - 15), so isum = 2 sum(c' q) - 15 bsum.
#pragma once

#include <algorithm>

#include "common.cuh"
#include "ep_exchange.cuh"
#include "layer_kernels.cuh"

namespace gcu {

constexpr int kLaneWarps = 12;                         // warps a CTA (one CTA an SM)
constexpr int kLaneMaxStages = 3;                      // ring stages a warp, at most
constexpr int kLaneTileGroup = 576;                    // a 16-row tile's 64-column group
constexpr int kLaneStageGroups = 4;                    // groups a stage (fewer when K has fewer)
constexpr int kLaneStageBytes = 2 * kLaneStageGroups * kLaneTileGroup;   // a stage: both tiles' groups

inline dim3 relayout_grid(int64_t items) {
    return dim3(static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, 65535))));
}

// Tiled (k_relayout_q4's layout) -> R16, one thread a (tile, group, row): the same bytes permuted within each tile
// group; the scales keep their place. `batch` matrices `bstride` bytes apart (a layer's experts at once).
__global__ void k_relayout_r16(const uint8_t *__restrict__ tiled, int64_t tiles, int cols, uint8_t *__restrict__ dst,
                               int batch = 1, size_t bstride = 0) {
    const int ng = cols / 64;
    const int64_t per = tiles * ng * 16, total = per * batch;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t bi = i / per, ii = i - bi * per;
        const int r = static_cast<int>(ii % 16);
        const int64_t tg = ii / 16;   // tile * ng + group
        const uint8_t *src = tiled + static_cast<size_t>(bi) * bstride + static_cast<size_t>(tg) * kLaneTileGroup;
        uint8_t *out = dst + static_cast<size_t>(bi) * bstride + static_cast<size_t>(tg) * kLaneTileGroup;
        // the tiled code of row r, value v (0..63 of the group): lane 4 (r % 8) + (v % 16) / 4, word v / 16, byte v % 4;
        // the low nibble for rows 0..7, the high for 8..15
        auto code = [&](int v) -> uint32_t {
            const int j = v >> 4, w = v & 15;
            const uint8_t byte = src[(4 * (r & 7) + (w >> 2)) * 16 + 4 * j + (w & 3)];
            return r < 8 ? (byte & 15u) : (byte >> 4);
        };
        uint32_t words[8];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t w = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int m = 4 * half + q;
                    w |= (code(16 * b + m) | (code(16 * b + 8 + m) << 4)) << (8 * q);
                }
                words[2 * b + half] = w;
            }
        }
        *reinterpret_cast<uint4 *>(out + 16 * r) = make_uint4(words[0], words[1], words[2], words[3]);
        *reinterpret_cast<uint4 *>(out + 256 + 16 * r) = make_uint4(words[4], words[5], words[6], words[7]);
        *reinterpret_cast<uint32_t *>(out + 512 + 4 * r) = *reinterpret_cast<const uint32_t *>(src + 512 + 4 * r);
    }
}

struct LaneArgs {
    const RouteOut *route;
    const uint8_t *experts;   // expert e at experts + e * stride: gate_up [2 ff][H], then down [H][ff] at down_off (R16)
    size_t stride, down_off;
    const float *globals;     // [E][2]: gate_up's, down's
    const uint8_t *sh_gate, *sh_up, *sh_down;   // the shared expert (R16; its ff = the routed experts')
    float sh_g0, sh_g1, sh_g2;
    int H, ff, K, n;
    ActSet hq;                // gate_up's input rows
    ActSet amid, shact;       // gate_up's outputs (pick rows, the shared expert's token rows), down's inputs
    float *eout, *shout;      // down's outputs: [n K][H] (pick rows), [n][H]
    int stages;               // ring stages a warp (lane_stages: as many as the shared memory holds)
    uint32_t *status;
    // expert parallelism (world > 1), down only: the picks' rows stored into every peer's slot for this layer too
    // (plain stores over NVLink), then the CTAs' last arrival raises this layer's flag in every peer (the step's
    // epoch) and waits, bounded, for every peer's - the exchange with no kernel of its own
    int rank, world, layer;
    float *peer_eout[kMaxEpWorld];     // the peers' slots for this layer (this rank's entry unused)
    uint32_t *flags;                   // this rank's flags [n_layers + 2][world], written by the peers
    uint32_t *peer_flags[kMaxEpWorld];
    const int *epoch;
    unsigned int *count;               // the CTAs' arrival counter (zero between launches)
};

// an image row: the cols int8 codes, then per block of 16 the (scale, bsum) pair
__host__ __device__ inline int lane_img_stride(int cols) { return cols + cols / 2; }
__host__ __device__ inline int lane_img_rows(bool up, int n, int K) { return up ? n : n * (K + 1); }
__host__ __device__ inline size_t lane_img_bytes(bool up, int n, int K, int cols) {
    return (static_cast<size_t>(lane_img_rows(up, n, K)) * lane_img_stride(cols) + 127) / 128 * 128;
}
__host__ __device__ inline size_t lane_smem_bytes(bool up, int n, int K, int cols, int stages) {
    return lane_img_bytes(up, n, K, cols) + static_cast<size_t>(kLaneWarps) * stages * (kLaneStageBytes + 8);
}
// the deepest ring (<= kLaneMaxStages) that fits beside the image in `avail` bytes of dynamic shared memory
inline int lane_stages(bool up, int n, int K, int cols, size_t avail) {
    const size_t img = lane_img_bytes(up, n, K, cols);
    if (avail <= img) return 0;
    const size_t per = static_cast<size_t>(kLaneWarps) * (kLaneStageBytes + 8);
    return static_cast<int>(std::min<size_t>(kLaneMaxStages, (avail - img) / per));
}

// rows r0.. of src into image rows img_row0..: every thread's loads issued before its stores (up to 8 items a thread
// in flight), so the staging costs one round trip rather than one per item
__device__ __forceinline__ void lane_stage_rows(const ActSet &src, int r0, int nrows, uint8_t *img, int img_row0,
                                                int cols) {
    const int nb = cols / 16, ist = lane_img_stride(cols), items = nrows * nb;
    for (int base = 0; base < items; base += 8 * blockDim.x) {
        uint4 q[8];
        float sc[8];
        int bs[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = base + k * blockDim.x + threadIdx.x;
            if (i < items) {
                const int r = i / nb, b = i - r * nb;
                q[k] = *reinterpret_cast<const uint4 *>(src.q + static_cast<size_t>(r0 + r) * src.qstride + 16 * b);
                sc[k] = src.scale[static_cast<size_t>(r0 + r) * src.sstride + b];
                bs[k] = src.bsum[static_cast<size_t>(r0 + r) * src.sstride + b];
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = base + k * blockDim.x + threadIdx.x;
            if (i < items) {
                const int r = i / nb, b = i - r * nb;
                uint8_t *row = img + static_cast<size_t>(img_row0 + r) * ist;
                *reinterpret_cast<uint4 *>(row + 16 * b) = q[k];
                *reinterpret_cast<uint2 *>(row + cols + 8 * b) = make_uint2(__float_as_uint(sc[k]), static_cast<uint32_t>(bs[k]));
            }
        }
    }
}

// The shared expert multiplies every token, the routed ones about one each: it is split into members of at most
// kLaneSharedToks tokens, so that no warp's unit holds several times another's work (its weights are read once per
// member - a few percent more bytes than once)
constexpr int kLaneSharedToks = 2;
constexpr int kLaneSharedMax = (kMaxTok + kLaneSharedToks - 1) / kLaneSharedToks;

// The route's members this rank computes, in shared memory for the CTA: expert, token mask, pick slots, globals
struct LaneRoute {
    int e[kMaxUnion + kLaneSharedMax];
    int mask[kMaxUnion + kLaneSharedMax];
    int slot[kMaxUnion + kLaneSharedMax][kMaxTok];
    float g[kMaxUnion + kLaneSharedMax][2];   // gate_up's (or the shared gate's, up's) / down's global
};

// kGS: 64-column groups a stage (4; 1 where K is not a multiple of 256)
template <bool kUp, int kGS>
__global__ void __launch_bounds__(kLaneWarps * 32) k_experts_lane(LaneArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ LaneRoute lr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cols = kUp ? a.H : a.ff, G = cols / 64, ist = lane_img_stride(cols);
    const int P = a.n * a.K;
    uint8_t *img = smem;
    const size_t ib = lane_img_bytes(kUp, a.n, a.K, cols);
    const int S = a.stages;
    uint8_t *ring = smem + ib + static_cast<size_t>(warp) * S * kLaneStageBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + ib + static_cast<size_t>(kLaneWarps) * S * kLaneStageBytes) +
                     warp * S;
    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(bars + s, 1);
        fence_barrier_init();
    }
    __syncwarp();
    // gate_up follows the route's kernel directly: the route after the dependent-launch wait; its activation rows
    // (the norm's, three kernels back, finished before the route's kernel passed its own wait and let this one start)
    // before it. Down follows gate_up, which passed its own wait only once the route's kernel had finished: down reads
    // the route and starts its weights' copies before its wait, and only the activation rows (gate_up's output) after
    if (kUp) {
        lane_stage_rows(a.hq, 0, a.n, img, 0, cols);
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;");
    }
    const RouteOut &R = *a.route;
    const int nu = R.n_own;
    const int per = kUp ? a.ff / 16 : a.H / 32;   // units a member
    const int nsh = (a.n + kLaneSharedToks - 1) / kLaneSharedToks;   // the shared expert's members, last
    const int total = (nu + nsh) * per;
    const int wg = blockIdx.x + gridDim.x * warp, NW = gridDim.x * kLaneWarps;
    const size_t tb = static_cast<size_t>(G) * kLaneTileGroup;
    // unit u's two tiles: member u / per, tile pair u % per; its expert from the route in global memory (the first
    // unit, before the shared copy is made) or in shared memory
    auto tiles_of = [&](int u, const uint8_t *&tA, const uint8_t *&tB, bool global) {
        const int m = u / per, j = u - m * per;
        if (m >= nu) {
            tA = kUp ? a.sh_gate + j * tb : a.sh_down + 2 * j * tb;
            tB = kUp ? a.sh_up + j * tb : tA + tb;
            return;
        }
        const uint8_t *base = a.experts + static_cast<size_t>(global ? R.own_ex[m] : lr.e[m]) * a.stride;
        tA = kUp ? base + j * tb : base + a.down_off + 2 * j * tb;
        tB = kUp ? base + (a.ff / 16 + j) * tb : tA + tb;
    };
    // a stage: kGS groups of tile A, then the same groups of tile B (two bulk copies)
    constexpr int gs = kGS;
    if (G % gs) {
        if (threadIdx.x == 0) atomicOr(a.status, kErrBadShape);
        if (!kUp) asm volatile("griddepcontrol.wait;" ::: "memory");   // (no kernel ends before its predecessor)
        return;
    }
    const uint32_t sbytes = static_cast<uint32_t>(gs) * kLaneTileGroup;
    // the producer (lane 0): its next stage's unit ordinal and first group, the unit's tiles (found when its first
    // stage is issued), the ring slot it fills, the stages issued
    int pk = 0, pg = 0, ps = 0, issued = 0;
    bool have = false;
    const uint8_t *ptA = nullptr, *ptB = nullptr;
    auto issue_next = [&](bool global) {
        const int u = wg + pk * NW;
        if (u >= total) return false;
        if (!have) {
            tiles_of(u, ptA, ptB, global);
            have = true;
        }
        uint8_t *dst = ring + ps * kLaneStageBytes;
        mbar_expect_tx(bars + ps, 2 * sbytes);
        bulk_g2s(dst, ptA + pg * kLaneTileGroup, sbytes, bars + ps);
        bulk_g2s(dst + sbytes, ptB + pg * kLaneTileGroup, sbytes, bars + ps);
        ++issued;
        if (++ps == S) ps = 0;
        pg += gs;
        if (pg == G) {
            pg = 0;
            ++pk;
            have = false;
        }
        return true;
    };
    // the first unit's copies at once, while the CTA copies the route and stages the activation rows
    if (lane == 0)
        while (issued < S && pk == 0 && issue_next(true)) {
        }
    for (int m = threadIdx.x; m < nu + nsh; m += blockDim.x) {
        if (m < nu) {
            const int su = R.own[m], e = R.ex[su];
            lr.e[m] = e;
            lr.mask[m] = R.mask[su];
            for (int t = 0; t < kMaxTok; ++t) lr.slot[m][t] = R.slot[su][t];
            lr.g[m][0] = kUp ? a.globals[2 * e] : a.globals[2 * e + 1];
            lr.g[m][1] = lr.g[m][0];
        } else {
            lr.e[m] = -1;
            lr.mask[m] = ((1 << kLaneSharedToks) - 1) << (kLaneSharedToks * (m - nu)) & ((1 << a.n) - 1);
            for (int t = 0; t < kMaxTok; ++t) lr.slot[m][t] = t;
            lr.g[m][0] = kUp ? a.sh_g0 : a.sh_g2;
            lr.g[m][1] = kUp ? a.sh_g1 : a.sh_g2;
        }
    }
    if (!kUp) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;");
        lane_stage_rows(a.amid, 0, P, img, 0, cols);
        lane_stage_rows(a.shact, 0, a.n, img, P, cols);
    }
    __syncthreads();
    if (lane == 0)
        while (issued < S && issue_next(false)) {
        }
    const int r = lane & 15;
    int st = 0;
    uint32_t ph = 0;   // the consumer's ring slot and its phase parity
    bool failed = false;
    for (int k = 0; !failed; ++k) {
        const int u = wg + k * NW;
        if (u >= total) break;
        const int m = u / per, j = u - m * per;
        const bool shared = m >= nu;
        // the unit's tokens: activation image rows and output rows
        int nt = 0, arow[kMaxTok], orow[kMaxTok];
        const int mask = lr.mask[m];
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
            arow[t] = 0;
            orow[t] = 0;
        }
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
            if (t < a.n && ((mask >> t) & 1)) {
                const int slot = lr.slot[m][t];
#pragma unroll
                for (int q = 0; q < kMaxTok; ++q)
                    if (q == nt) {
                        arow[q] = kUp ? t : (shared ? P + t : slot);
                        orow[q] = slot;
                    }
                ++nt;
            }
        }
        float acc[kMaxTok];
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) acc[t] = 0.0f;
        for (int g0 = 0; g0 < G; g0 += gs) {
            const bool ok = mbar_wait_bounded(bars + st, ph, a.status);
            if (!__all_sync(0xffffffffu, ok)) {
                // (status raised) the copies still in flight land, bounded, before the warp stops
                if (lane == 0)
                    for (int q = 1; q < S; ++q) {
                        const int sq = (st + q) % S;
                        mbar_wait_bounded(bars + sq, sq > st ? ph : ph ^ 1u, nullptr);
                    }
                failed = true;
                break;
            }
            // the stage's codes and E4M3 scales of this lane's row: gs groups of 4 blocks
            const uint8_t *sbase = ring + st * kLaneStageBytes + (lane >> 4) * sbytes;
            uint32_t wd[gs][8];
            float dw[gs][4];
#pragma unroll
            for (int gi = 0; gi < gs; ++gi) {
                const uint8_t *sp = sbase + gi * kLaneTileGroup;
                const uint4 c0 = ld_shared_v4(sp + 16 * r), c1 = ld_shared_v4(sp + 256 + 16 * r);
                const uint32_t sw = *reinterpret_cast<const uint32_t *>(sp + 512 + 4 * r);
                const float2 e01 = e4m3x2_to_float2(sw & 0xFFFFu), e23 = e4m3x2_to_float2(sw >> 16);
                dw[gi][0] = e01.x;
                dw[gi][1] = e01.y;
                dw[gi][2] = e23.x;
                dw[gi][3] = e23.y;
                wd[gi][0] = c0.x, wd[gi][1] = c0.y, wd[gi][2] = c0.z, wd[gi][3] = c0.w;
                wd[gi][4] = c1.x, wd[gi][5] = c1.y, wd[gi][6] = c1.z, wd[gi][7] = c1.w;
            }
            // per token: the stage's 4 gs products (independent), then added into the chain in block order (one body
            // for every token: the chains and rows indexed at run time)
#pragma unroll 1
            for (int t = 0; t < nt; ++t) {
                {
                    const uint8_t *row = img + static_cast<size_t>(arow[t]) * ist;
                    float p[4 * gs];
#pragma unroll
                    for (int q = 0; q < 4 * gs; ++q) {
                        const int gi = q >> 2, jb = q & 3, b = 4 * (g0 + gi) + jb;
                        const uint32_t lo = wd[gi][2 * jb], hi = wd[gi][2 * jb + 1];
                        const uint4 av = ld_shared_v4(row + 16 * b);
                        const uint2 pr = *reinterpret_cast<const uint2 *>(row + cols + 8 * b);
                        int d = __dp4a(static_cast<int>(lo & 0x0F0F0F0Fu), static_cast<int>(av.x), 0);
                        d = __dp4a(static_cast<int>(hi & 0x0F0F0F0Fu), static_cast<int>(av.y), d);
                        d = __dp4a(static_cast<int>((lo >> 4) & 0x0F0F0F0Fu), static_cast<int>(av.z), d);
                        d = __dp4a(static_cast<int>((hi >> 4) & 0x0F0F0F0Fu), static_cast<int>(av.w), d);
                        // float(isum) exactly, isum = 2 d - 15 bsum (|isum| < 2^22): the bits of 1.5 * 2^23 + isum
                        // less 1.5 * 2^23 - an integer add and a float subtraction
                        const float fi = __fsub_rn(__int_as_float(0x4B400000 + 2 * d - 15 * static_cast<int>(pr.y)), 12582912.0f);
                        p[q] = __fmul_rn(fi, __fmul_rn(dw[gi][jb], __uint_as_float(pr.x)));
                    }
                    float at = acc[t];
#pragma unroll
                    for (int q = 0; q < 4 * gs; ++q) at = __fadd_rn(at, p[q]);
                    acc[t] = at;
                }
            }
            __syncwarp();   // (every lane done with the stage: refill it)
            if (lane == 0) {
                fence_proxy_async();
                issue_next(false);
            }
            if (++st == S) {
                st = 0;
                ph ^= 1u;
            }
        }
        if (failed) break;
        const float gl = lr.g[m][lane >> 4];
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
            if (t >= nt) break;
            const float y = __fmul_rn(acc[t], gl);   // (acc * global * 1)
            if (kUp) {
                // a = silu(gate) * up (engine/src/model.cpp:4522-4524), the block of 16 (lanes 0-15) quantized as
                // quantize_activation (engine/src/kernels.cpp:1254-1295) into the output row's block j
                const float up = __shfl_down_sync(0xffffffffu, y, 16);
                const float av = lane < 16 ? __fmul_rn(silu_ref(y), up) : 0.0f;
                float amax = fabsf(av);
                for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                const int qv = max(-127, min(127, __float2int_rn(__fmul_rn(av, inv))));
                int sq = qv;
                for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (lane < 16) {
                    const ActSet &o = shared ? a.shact : a.amid;
                    const_cast<int8_t *>(o.q)[static_cast<size_t>(orow[t]) * o.qstride + 16 * j + lane] = static_cast<int8_t>(qv);
                    if (lane == 0) {
                        const_cast<float *>(o.scale)[static_cast<size_t>(orow[t]) * o.sstride + j] = __fdiv_rn(amax, 127.0f);
                        const_cast<int32_t *>(o.bsum)[static_cast<size_t>(orow[t]) * o.sstride + j] = sq;
                    }
                }
            } else {
                float *dst = shared ? a.shout : a.eout;
                const size_t at = static_cast<size_t>(orow[t]) * a.H + 32 * j + lane;
                dst[at] = y;
                if (!shared && a.world > 1) {
#pragma unroll
                    for (int s2 = 0; s2 < kMaxEpWorld; ++s2)
                        if (s2 < a.world && s2 != a.rank) a.peer_eout[s2][at] = y;
                }
            }
        }
    }
    if (!kUp && a.world > 1) {
        // every CTA's peer stores out before its arrival; the last to arrive tells the peers and waits for theirs
        __threadfence_system();
        __syncthreads();
        __shared__ int last;
        if (threadIdx.x == 0) last = atomicAdd(a.count, 1u) == gridDim.x - 1;
        __syncthreads();
        if (!last) return;
        const uint32_t ep = static_cast<uint32_t>(*reinterpret_cast<const volatile int *>(a.epoch));
        if (threadIdx.x == 0) *a.count = 0;
        const int s2 = threadIdx.x;
        if (s2 < a.world && s2 != a.rank) {
            st_release_sys(a.peer_flags[s2] + a.layer * a.world + a.rank, ep);
            const uint32_t *f = a.flags + a.layer * a.world + s2;
            bool ok = false;
            for (uint32_t it = 0; it < kExchangeWaitLimit && !ok; ++it) ok = ld_acquire_sys(f) == ep;
            if (!ok && a.status) atomicOr(a.status, kErrWaitTimeout);
        }
    }
}

// A route for ids given directly (the operator gcuda_op_moe_lane): the union of the picks in ascending expert order,
// each member's pick slots and token mask, every member this rank's. One CTA.
__global__ void k_route_from_ids(const int *__restrict__ ids, int n, int K, int E, RouteOut *out, uint32_t *status) {
    __shared__ uint32_t bits[32];
    __shared__ int mask[kMaxUnion], ex[kMaxUnion];
    if (threadIdx.x < 32) bits[threadIdx.x] = 0;
    if (threadIdx.x < kMaxUnion) mask[threadIdx.x] = 0;
    __syncthreads();
    const int P = n * K, pk = threadIdx.x;
    const int e = pk < P ? ids[pk] : -1;
    if (pk < P && (e < 0 || e >= E || e >= 1024)) atomicOr(status, kErrBadShape);
    const bool ok = pk < P && e >= 0 && e < E && e < 1024;
    if (ok) atomicOr(&bits[e >> 5], 1u << (e & 31));
    __syncthreads();
    int nu = 0;
    for (int i = 0; i < 32; ++i) nu += __popc(bits[i]);
    if (nu > kMaxUnion) {
        if (threadIdx.x == 0) atomicOr(status, kErrUnion);
        return;
    }
    if (ok) {
        const int w = e >> 5;
        int u = __popc(bits[w] & ((1u << (e & 31)) - 1u));
        for (int i = 0; i < w; ++i) u += __popc(bits[i]);
        ex[u] = e;
        out->ex[u] = e;
        out->slot[u][pk / K] = pk;
        out->ids[pk] = e;
        atomicOr(&mask[u], 1 << (pk / K));
    }
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < nu) {
        out->mask[threadIdx.x] = mask[threadIdx.x];
        out->own[threadIdx.x] = threadIdx.x;
        out->own_ex[threadIdx.x] = ex[threadIdx.x];
    }
    if (threadIdx.x == 0) {
        out->n_union = nu;
        out->n_own = nu;
    }
}

}  // namespace gcu
