// gemv_core.cuh - the q4 GEMV engine. A unit is two 16-row tiles x all K; its result per (row, token) is the
// reference's chain acc += float(isum_b) * (e4m3_b * ascale_b) over the blocks b in order (engine/src/kernels.cpp:
// 1316-1319), bit for bit. Two ways to run a launch:
//   - streaming (stream_units): a warp per unit, for launches with enough units to fill the SMs; the warp copies its
//     units' groups into its own shared-memory ring with cp.async and adds every product into the chain as it comes;
//   - fan-in (fan_units): for launches with few units; the whole CTA works on one unit, producer warps leave each
//     group's products in a shared slot and chain warps add the slots in block order.
// Both compute a group's products the same way (group_products): int8 mma.sync block sums of the codes as 16 c whose
// accumulator starts at 1.5 * 2^23 - 120 * bsum (so float(8 isum) is one subtraction), then f32x2 products.
#pragma once

#include "q4_gemv.cuh"

namespace gcu {

constexpr int kStageBytesR = 2 * kGroupBytes;   // a ring stage: one group of both tiles

// f32x2 (sm_100): two IEEE operations per instruction, each lane rounded on its own
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// a * b rounded once, as mul.rn.f32x2 - written as fma(a, b, z) with z a +0 pair the compiler cannot see is zero, so
// that no later pass contracts the product with the add that consumes it (ptxas was seen to fuse a mul.rn.f32x2 /
// add.rn.f32x2 pair). fma(a, b, +0) = round(a b), except that a -0 product becomes +0; the chains here start at +0
// and only add, so they never hold -0 and adding either zero leaves them unchanged.
__device__ __forceinline__ uint64_t f2_mul_sep(uint64_t a, uint64_t b, uint64_t z) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(z));
    return d;
}
__device__ __forceinline__ uint64_t pack2(uint32_t lo, uint32_t hi) { return static_cast<uint64_t>(hi) << 32 | lo; }
__device__ __forceinline__ float lo_f(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi_f(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }

// Activation images (stage_image below): an image's per-(group, tig) entry of accumulator inits and activation
// scales is kCsEntry bytes; a warp's own image of sg groups (launches whose units multiply different activations)
// takes warp_act_bytes(sg), the CTA's shared image of all K act_smem_bytes(K).
constexpr int kCsEntry = 96;
__host__ __device__ inline int slice_tstride(int sg) { return sg * 64 + (sg % 2 == 0 ? 64 : 0); }
__host__ __device__ inline int warp_act_bytes(int sg) { return kMaxTok * slice_tstride(sg) + sg * 4 * kCsEntry; }
// the whole-K image the CTA shares (act_tstride: token stride of the full image)
__host__ __device__ inline int act_tstride(int cols) { return (cols / 64) * 64 + ((cols / 64) % 2 == 0 ? 64 : 0); }
__host__ __device__ inline int act_smem_bytes(int cols) { return (kMaxTok * act_tstride(cols) + (cols / 64) * 4 * kCsEntry + 127) / 128 * 128; }
constexpr int kMaxDynSmem = 227 * 1024;

// A launch's shape: wpu warps per unit, nslots units at a time per CTA, the dynamic shared memory. The warps' regions
// (own: the groups of a per-warp image, 0 for none) follow `front` bytes (the CTA's shared image, or 0). Slots are
// dropped, then shorter chains taken, until it fits. False if no shape fits.
// A launch's shape: wpu = 1 and nslots warps per CTA (streaming, `stages` deep rings), or wpu = kFanWarps and one
// slot (fan-in, stages 0); sg the groups a unit's warp walks; the dynamic shared memory.
struct GemvShape {
    int wpu, nslots, sg;
    size_t smem;
    int stages = 0;
};
// The activation image of groups [g0, g0 + ng) of up to kMaxTok vectors (src(t) = the ActSet row of token column t, -1 =
// zeros), token stride ts: act word (t, gl, tig, j) at t * ts + (gl * 4 + tig) * 16 + 4 j (values 16 (4 g + j) + 4 tig
// .. + 3); cs per (gl, tig) kCsEntry bytes at kMaxTok * ts + (gl * 4 + tig) * kCsEntry: for each block j the mma's
// accumulator quad (cinit(2 tig), cinit(2 tig + 1), cinit(2 tig), cinit(2 tig + 1)), then (ascale(2 tig),
// ascale(2 tig + 1)) per block. cinit = 1.5 * 2^23 - 120 * bsum. Threads `me` of `nthr` share the blocks; a thread
// loads one block of every token (16 bytes each) before it stores any.
template <typename Src>
__device__ inline void stage_image(const ActSet &a, const Src &src, int g0, int ng, int ts, uint8_t *img, int me, int nthr) {
    // thread me takes blocks bl = me, me + nthr, ... of every token, four tokens' loads at a time
    const int nbl = ng * 4;
    int rows[kMaxTok];
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) rows[t] = src(t);
    constexpr int kT = 4;   // tokens whose loads are in flight together
    for (int bl = me; bl < nbl; bl += nthr)
#pragma unroll
    for (int t0 = 0; t0 < kMaxTok; t0 += kT) {
        const size_t b = static_cast<size_t>(g0) * 4 + bl;
        uint4 v[kT];
        int32_t bs[kT];
        float sc[kT];
#pragma unroll
        for (int u = 0; u < kT; ++u) {
            v[u] = make_uint4(0, 0, 0, 0);
            bs[u] = 0;
            sc[u] = 0.0f;
            if (rows[t0 + u] >= 0) {
                const size_t r = static_cast<size_t>(rows[t0 + u]);
                v[u] = *reinterpret_cast<const uint4 *>(a.q + r * a.qstride + 16 * b);
                bs[u] = a.bsum[r * a.sstride + b];
                sc[u] = a.scale[r * a.sstride + b];
            }
        }
        const int gl = bl >> 2, j = bl & 3;
#pragma unroll
        for (int u = 0; u < kT; ++u) {
            const int t = t0 + u;
            uint8_t *row = img + t * ts + gl * 64 + 4 * j;   // word (t, gl, tig, j) at + tig * 16
            *reinterpret_cast<uint32_t *>(row) = v[u].x;
            *reinterpret_cast<uint32_t *>(row + 16) = v[u].y;
            *reinterpret_cast<uint32_t *>(row + 32) = v[u].z;
            *reinterpret_cast<uint32_t *>(row + 48) = v[u].w;
            int32_t *base_cs = reinterpret_cast<int32_t *>(img + kMaxTok * ts + (gl * 4 + t / 2) * kCsEntry);
            const int32_t ci = static_cast<int32_t>(kBiasBits) - 120 * bs[u];
            base_cs[4 * j + (t % 2)] = ci;
            base_cs[4 * j + (t % 2) + 2] = ci;
            reinterpret_cast<float *>(base_cs)[16 + 2 * j + (t % 2)] = sc[u];
        }
    }
}

// a warp's own image of its K-slice (sel[t]: the ActSet row of column t, -1 = zeros)
__device__ inline void stage_slice(const ActSet &a, const int *sel, int g0, int sg, uint8_t *img) {
    stage_image(a, [&](int t) { return sel[t]; }, g0, sg, slice_tstride(sg), img, threadIdx.x & 31, 32);
}

// The CTA's image of all K for the first ncols vectors (zeros after them), token stride act_tstride(K). Every thread.
__device__ inline void stage_full(const ActSet &a, int ncols, uint8_t *img) {
    stage_image(a, [&](int t) { return t < ncols ? t : -1; }, 0, a.cols / 64, act_tstride(a.cols), img,
                static_cast<int>(threadIdx.x), static_cast<int>(blockDim.x));
}

// A group's scale word of (tile lane >> 4, row lane & 15) - the row's four blocks - to (e, e) float pairs in e4p, the
// layout group_products reads: [tile][block][gid][e(gid), e(gid), e(gid + 8), e(gid + 8)].
__device__ __forceinline__ void decode_scales(uint32_t word, int lane, float *e4p) {
    const int tile = lane >> 4, w = lane & 15;
    // E4M3 pairs through the hardware conversion (exact: every E4M3 value is an f16; 0x7F / 0xFF, the format's NaN,
    // decode as NaN as in engine/src/kernels.cpp:39-52)
    const float2 e01 = e4m3x2_to_float2(static_cast<uint16_t>(word & 0xFFFFu));
    const float2 e23 = e4m3x2_to_float2(static_cast<uint16_t>(word >> 16));
    const float e[4] = {e01.x, e01.y, e23.x, e23.y};
#pragma unroll
    for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float2 *>(e4p + ((tile * 4 + j) * 8 + (w & 7)) * 4 + (w >> 3) * 2) = make_float2(e[j], e[j]);
}

// One group of both tiles: for block j = 0..3 the products p[0..3] = tile A (row gid: the token pair (2 tig,
// 2 tig + 1), row gid + 8: the pair), tile B likewise, handed to sink(j, p) in block order.
// e4p: the group's scales as [tile][block][gid][e(gid), e(gid), e(gid+8), e(gid+8)] floats.
// wa / wb: the lane's 16 code bytes of tiles A and B.
// kOne: tile A only (p[2], p[3] left 0).
template <bool kOne = false, typename Sink>
__device__ __forceinline__ void group_products(const uint4 wa, const uint4 wb, const float *e4p, const uint8_t *act,
                                               const uint8_t *cs, int lane, uint64_t zero, const Sink &sink) {
    const int gid = lane >> 2;
    const uint4 av = ld_shared_v4(act);
    const uint4 s01 = ld_shared_v4(cs + 64);   // (as0, as1) for blocks 0, 1
    const uint4 s23 = ld_shared_v4(cs + 80);   // blocks 2, 3
    const uint32_t wA[4] = {wa.x, wa.y, wa.z, wa.w}, wB[4] = {wb.x, wb.y, wb.z, wb.w};
    const uint32_t bv[4] = {av.x, av.y, av.z, av.w};
    const uint64_t sp[4] = {pack2(s01.x, s01.y), pack2(s01.z, s01.w), pack2(s23.x, s23.y), pack2(s23.z, s23.w)};
    const uint64_t bias2 = pack2(__float_as_uint(kBiasF), __float_as_uint(kBiasF));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        int32_t dA[4], dB[4];
        (void)dB;
        const uint4 cq = ld_shared_v4(cs + 16 * j);   // the block's accumulator quad
        const int32_t cinit[4] = {static_cast<int32_t>(cq.x), static_cast<int32_t>(cq.y), static_cast<int32_t>(cq.z),
                                  static_cast<int32_t>(cq.w)};
        mma_u8s8_16816(dA, (wA[j] << 4) & 0xF0F0F0F0u, wA[j] & 0xF0F0F0F0u, bv[j], cinit);
        const uint4 eA = ld_shared_v4(e4p + ((0 * 4 + j) * 8 + gid) * 4);
        // float(8 isum) = bits(bias + 8 isum) - bias; p8 = float(8 isum) * (e4m3 * ascale) = 8 p exactly (a power of two:
        // the same rounding), and the chain of p8 is 8 times the chain of p; the epilogue multiplies by global / 8
        const uint64_t FAg = f2_sub(pack2(dA[0], dA[1]), bias2), FAh = f2_sub(pack2(dA[2], dA[3]), bias2);
        uint64_t p[4] = {f2_mul_sep(FAg, f2_mul(pack2(eA.x, eA.y), sp[j]), zero),
                         f2_mul_sep(FAh, f2_mul(pack2(eA.z, eA.w), sp[j]), zero), 0, 0};
        if constexpr (!kOne) {
            mma_u8s8_16816(dB, (wB[j] << 4) & 0xF0F0F0F0u, wB[j] & 0xF0F0F0F0u, bv[j], cinit);
            const uint4 eB = ld_shared_v4(e4p + ((1 * 4 + j) * 8 + gid) * 4);
            const uint64_t FBg = f2_sub(pack2(dB[0], dB[1]), bias2), FBh = f2_sub(pack2(dB[2], dB[3]), bias2);
            p[2] = f2_mul_sep(FBg, f2_mul(pack2(eB.x, eB.y), sp[j]), zero);
            p[3] = f2_mul_sep(FBh, f2_mul(pack2(eB.z, eB.w), sp[j]), zero);
        }
        sink(j, p);
    }
}

// the fan-in path's shape (fan_units below)
constexpr int kFanProducers = 16;
constexpr int kFanAhead = 4;   // a producer's items in flight
constexpr int kFanChains = 2;   // chain warps: tile A's sums, tile B's
constexpr int kFanWarps = kFanProducers + kFanChains;
constexpr int kFanThreads = kFanWarps * 32;
constexpr int kFanGroupBytes = 32 * 16 * 8;                      // a group's products: 32 lanes x 16 f32 pairs
constexpr int kFanSlotBytes = kFanProducers * kFanGroupBytes;
constexpr int kBarFull = 1, kBarEmpty = 3, kBarProducers = 5, kBarChains = 6;    // (+ slot)

// image (img_cols wide), then two product slots, then a KB of scale pairs per producer, then the chains' exchange
__host__ __device__ inline size_t fan_smem_bytes(int img_cols) {
    return static_cast<size_t>(act_smem_bytes(img_cols)) + 2 * kFanSlotBytes + kFanProducers * 1024 + 32 * 16;
}

// ------------------------------------------------------------------------------------------- streaming ----
// The path for launches with a warp per unit (wpu = 1): each warp (up to kStreamWarps) copies its units'
// groups (both tiles' 576 bytes) into its own ring of shared-memory stages with 16-byte cp.async copies, the
// stages ahead of the one it multiplies in flight, and adds every product into the chain as it comes. The copies hold
// no registers (so the CTA runs more warps) and their waits (cp.async.wait_group) always end: the copies land like
// any load.
constexpr int kStreamWarps = 24;
// ring depths: kDeepStages for launches with few units per SM (fewer warps, each with more copies in flight)
constexpr int kWideStages = 6, kDeepStages = 12;

// per warp: 1 KB of scale pairs, the ring, then the warp's own image (own groups, 0 for none)
__host__ __device__ inline int stream_warp_bytes(int stages, int own) {
    return 2048 + stages * kStageBytesR + (own ? (warp_act_bytes(own) + 127) / 128 * 128 : 0);
}
// warps per CTA on the streaming path: kStreamWarps (80 registers a thread) for wide launches, kDeepWarps (128) for
// the deep rings (kDeepStages, and the K slices' 10)
constexpr int kDeepWarps = 16;
__host__ __device__ constexpr int stream_warps(int stages) { return stages == kDeepStages || stages == 10 ? kDeepWarps : kStreamWarps; }

// A launch's shape: streaming (a warp per unit) when every CTA has kStreamMinUnits units or more, else the fan-in
// (stages 0; the CTA on one unit at a time, its image img_cols wide). units_per_cta: the units a CTA takes (all CTAs
// take the same share, +-1).
constexpr int kStreamMinUnits = 2;
inline bool plan_gemv(int cols, int img_cols, bool own_images, size_t front, int units_per_cta, GemvShape &r) {
    const size_t fan = fan_smem_bytes(img_cols);
    if (units_per_cta < kStreamMinUnits && cols >= 64 && fan <= static_cast<size_t>(kMaxDynSmem)) {
        r = GemvShape{kFanWarps, 1, cols / 64, fan, 0};
        return true;
    }
    if ((cols / 64) % 2 == 0) {
        const int g = cols / 64;
        const int stages = units_per_cta >= kStreamWarps ? kWideStages : kDeepStages;
        const size_t wb = static_cast<size_t>(stream_warp_bytes(stages, own_images ? g : 0));
        int ns = stream_warps(stages);
        if (units_per_cta > 0 && units_per_cta < ns) ns = units_per_cta;
        while (ns >= 1 && front + ns * wb > static_cast<size_t>(kMaxDynSmem)) --ns;
        if (g >= 1 && ns >= 1) {
            r = GemvShape{1, ns, g, front + ns * wb, stages};
            return true;
        }
    }
    if (cols >= 64 && fan <= static_cast<size_t>(kMaxDynSmem)) {
        r = GemvShape{kFanWarps, 1, cols / 64, fan, 0};
        return true;
    }
    return false;
}

__device__ __forceinline__ uint4 ldg_stream_v4(const uint8_t *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const uint8_t *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// (the same with constant offsets on both addresses)
template <int kDst, int kSrc>
__device__ __forceinline__ void cp_async16_off(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0+%2], [%1+%3], 16;" ::"r"(dst), "l"(src), "n"(kDst), "n"(kSrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// named barriers (bar.sync / bar.arrive over n threads)
__device__ __forceinline__ void bar_sync_n(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void bar_arrive_n(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }

struct StreamCtx {
    float *e4p;           // this warp's 2 KB of (e, e) pairs (two groups)
    uint8_t *ring;        // this warp's ring of stages of kStageBytesR
    const uint8_t *img;   // the activation image (token stride img_ts), groups from 0
    int img_ts;
    int ngroups;          // the groups this warp walks per unit (even): K / 64, or its K slice's
    uint64_t zero;        // a +0 pair from runtime values (f2_mul_sep)
    // K slices (ks > 1): the warps kr = 0 .. ks - 1 of a slice group walk groups [g0, g0 + ngroups) of the same units;
    // the chains of slices 1.. meet slice 0's at the unit's end through xchg (two buffers of (ks - 1) x 32 lanes x
    // 32 bytes) at named barrier bar_id (ks warps), added in slice order - f32 accumulation in that order, not the
    // single chain's. img_g0: the image's group of the slice's first group (g0 for a whole-K image, 0 for a slice's own)
    int ks = 1, kr = 0, g0 = 0, img_g0 = 0, bar_id = 0;
    uint4 *xchg = nullptr;
};

// get(i, U): the warp's i-th unit (false past the end); restage(U) (every lane) before a unit's first group; epi(U, y0,
// y1, gid, tig) after its last. `early`: the first copies go out before prelude() (weights do not depend on the
// previous kernel). Groups go two at a time (K / 64 even), both copies waited for, both groups' scales decoded, then
// both groups' products: two independent streams of tensor-core and f32 work for the scheduler.
template <int kStreamStages, typename GetUnit, typename Restage, typename Epi, typename Prelude>
__device__ void stream_units(const GetUnit &get, const StreamCtx &c, const Restage &restage, const Epi &epi, bool early,
                             const Prelude &prelude) {
    static_assert(kStreamStages % 2 == 0 && kStreamStages >= 4, "stages in pairs");
    const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int G = c.ngroups;
    // producer: this lane's copy sources in the current unit (codes of both tiles; lanes < 8 one 16-byte piece of the
    // scales), advanced a group (576 bytes) per copy. Every issue() commits one copy group (empty past the end): the
    // prologue kStreamStages - 2, then two per pair consumed, so when the pair (i, i + 1) is taken exactly
    // kStreamStages - 4 groups were committed after i + 1's. Item k lives in stage k % kStreamStages.
    const uint32_t ring_s = smem_addr(c.ring);
    const uint32_t st_end = ring_s + kStreamStages * kStageBytesR;
    const int sc_t = (lane >> 2) & 1, sc_k = lane & 3;   // (lanes < 8)
    const uint32_t d_code = lane * 16, d_sc = sc_t * kGroupBytes + 512 + 16 * sc_k;
    int pu = 0, pg = 0;
    uint32_t pdst = ring_s;
    const uint8_t *s0 = nullptr, *s1 = nullptr, *s2 = nullptr;
    bool p_ok;
    const size_t slice_off = static_cast<size_t>(c.g0) * kGroupBytes;
    auto unit_src = [&](int i) {
        GemvUnit T;
        p_ok = get(i, T);
        if (p_ok) {
            s0 = T.w0 + slice_off + lane * 16;
            s1 = T.w1 + slice_off + lane * 16;
            s2 = (sc_t ? T.w1 : T.w0) + slice_off + 512 + 16 * sc_k;
        }
    };
    // two groups (G is even: a pair never straddles two units), one copy group committed for each
    auto issue2 = [&]() {
        if (p_ok) {
            cp_async16(pdst + d_code, s0);
            cp_async16(pdst + kGroupBytes + d_code, s1);
            if (lane < 8) cp_async16(pdst + d_sc, s2);
            cp_async_commit();
            cp_async16_off<kStageBytesR, kGroupBytes>(pdst + d_code, s0);
            cp_async16_off<kStageBytesR, kGroupBytes>(pdst + kGroupBytes + d_code, s1);
            if (lane < 8) cp_async16_off<kStageBytesR, kGroupBytes>(pdst + d_sc, s2);
            cp_async_commit();
            s0 += 2 * kGroupBytes;
            s1 += 2 * kGroupBytes;
            s2 += 2 * kGroupBytes;
            pg += 2;
            if (pg == G) {
                pg = 0;
                unit_src(++pu);
            }
        } else {
            cp_async_commit();
            cp_async_commit();
        }
        pdst += 2 * kStageBytesR;
        if (pdst == st_end) pdst = ring_s;
    };
    // (get() may read the previous kernel's output: not before prelude() unless `early`)
    if (!early) prelude();
    unit_src(0);
    for (int k = 0; k < kStreamStages - 2; k += 2) issue2();
    if (early) prelude();
    // consumer
    int cu = 0, cg = 0;
    const uint8_t *st = c.ring;
    bool c_ok;
    {
        GemvUnit U;
        c_ok = get(0, U);
        if (c_ok) restage(U);
    }
    uint64_t acc[4] = {0, 0, 0, 0};
    auto chain = [&](int, const uint64_t (&p)[4]) {
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = f2_add(acc[q], p[q]);
    };
    const uint8_t *act0 = c.img + gid * c.img_ts + tig * 16 + c.img_g0 * 64;
    const uint8_t *cs0 = c.img + kMaxTok * c.img_ts + tig * kCsEntry + c.img_g0 * 4 * kCsEntry;
    const uint8_t *ring_end = c.ring + kStreamStages * kStageBytesR;
    int buf = 0;
    while (c_ok) {
        // items i, i + 1: kStreamStages - 4 groups committed after i + 1's may still fly
        cp_async_wait<kStreamStages - 4>();
        __syncwarp();
        const uint8_t *st1 = st + kStageBytesR;
        const int sc_off = (lane >> 4) * kGroupBytes + 512 + 4 * (lane & 15);
        decode_scales(*reinterpret_cast<const uint32_t *>(st + sc_off), lane, c.e4p);
        decode_scales(*reinterpret_cast<const uint32_t *>(st1 + sc_off), lane, c.e4p + 256);
        __syncwarp();
        group_products(ld_shared_v4(st + lane * 16), ld_shared_v4(st + kGroupBytes + lane * 16), c.e4p, act0 + cg * 64,
                       cs0 + cg * 4 * kCsEntry, lane, c.zero, chain);
        group_products(ld_shared_v4(st1 + lane * 16), ld_shared_v4(st1 + kGroupBytes + lane * 16), c.e4p + 256,
                       act0 + (cg + 1) * 64, cs0 + (cg + 1) * 4 * kCsEntry, lane, c.zero, chain);
        __syncwarp();   // every lane done with the stages and the scale pairs before they are refilled
        issue2();
        st = st1 + kStageBytesR == ring_end ? c.ring : st1 + kStageBytesR;
        cg += 2;
        if (cg == G) {
            // y = acc * global * 1 (engine/src/kernels.cpp:1320)
            GemvUnit U;
            get(cu, U);
            bool out = true;
            if (c.ks > 1) {
                uint4 *xb = c.xchg + (buf * (c.ks - 1)) * 64 + lane * 2;
                if (c.kr > 0) {
                    xb[(c.kr - 1) * 64] = make_uint4(static_cast<uint32_t>(acc[0]), static_cast<uint32_t>(acc[0] >> 32),
                                                     static_cast<uint32_t>(acc[1]), static_cast<uint32_t>(acc[1] >> 32));
                    xb[(c.kr - 1) * 64 + 1] = make_uint4(static_cast<uint32_t>(acc[2]), static_cast<uint32_t>(acc[2] >> 32),
                                                         static_cast<uint32_t>(acc[3]), static_cast<uint32_t>(acc[3] >> 32));
                    out = false;
                }
                bar_sync_n(c.bar_id, 32 * c.ks);
                if (c.kr == 0)
                    for (int r = 1; r < c.ks; ++r) {
                        const uint4 a01 = xb[(r - 1) * 64], a23 = xb[(r - 1) * 64 + 1];
                        acc[0] = f2_add(acc[0], pack2(a01.x, a01.y));
                        acc[1] = f2_add(acc[1], pack2(a01.z, a01.w));
                        acc[2] = f2_add(acc[2], pack2(a23.x, a23.y));
                        acc[3] = f2_add(acc[3], pack2(a23.z, a23.w));
                    }
                buf ^= 1;   // (the next unit's chains go to the other buffer: the barrier above orders its reuse)
            }
            if (out) {
                float y0[4] = {lo_f(acc[0]), hi_f(acc[0]), lo_f(acc[1]), hi_f(acc[1])};
                float y1[4] = {lo_f(acc[2]), hi_f(acc[2]), lo_f(acc[3]), hi_f(acc[3])};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    y0[i] = __fmul_rn(y0[i], __fmul_rn(U.g0, 0.125f));
                    y1[i] = __fmul_rn(y1[i], __fmul_rn(U.g1, 0.125f));
                }
                epi(U, y0, y1, gid, tig);
            }
            acc[0] = acc[1] = acc[2] = acc[3] = 0;
            cg = 0;
            c_ok = get(++cu, U);
            if (c_ok) restage(U);
        }
    }
    cp_async_wait<0>();   // (no copy in flight when the warp leaves: the stages are released with the CTA)
}

// ------------------------------------------------------------------------------------------- fan-in ----
// The path for launches with few units (latency-bound): the whole CTA works on one unit at a time. kFanProducers
// warps each take one group of a chunk (kFanProducers consecutive groups), multiply it and leave its products in a
// shared-memory slot; one chain warp then adds the chunk's products in block order (one f32x2 add per product, the
// only serial work) while the producers fill the other slot. Slots change hands through named barriers (FULL: the
// producers arrive, the chain warp waits; EMPTY: the reverse), which need no spinning and cannot be left waiting: every
// warp walks the same units and chunks.

struct FanCtx {
    uint8_t *img;       // the activation image (token stride img_ts)
    int img_ts;
    uint8_t *prod;      // two slots of kFanSlotBytes
    float *e4p;         // kFanProducers x 1 KB
    float4 *xchg;       // 32 lanes: tile B's sums, for the tile A chain warp's epilogue
    int ngroups;        // K / 64
    bool half;          // units of one tile (get() gives it as tile A, y1 = NULL; never a swiglu unit)
    uint64_t zero;      // a +0 pair from runtime values (f2_mul_sep)
};

// get(i, U): the CTA's i-th unit (false past the end); restage(U, me, nthr) by the producers (threads me of nthr)
// before a unit whose activations differ from the last one's (`changes(U)` true); epi(U, y0, y1, gid, tig) by the
// chain warp. `early`: the producers' first loads go out before prelude() (which every thread calls once).
template <typename GetUnit, typename Changes, typename Restage, typename Epi, typename Prelude>
__device__ void fan_units(const GetUnit &get, const FanCtx &c, const Changes &changes, const Restage &restage,
                          const Epi &epi, bool early, const Prelude &prelude) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int G = c.ngroups, nch = (G + kFanProducers - 1) / kFanProducers;
    if (warp < kFanProducers) {
        // producer: items (unit i, chunk k), group g = k * kFanProducers + warp; kFanAhead items' loads ahead in registers
        int pi = 0, pk = 0;
        const uint8_t *pw0 = nullptr, *pw1 = nullptr;
        bool p_ok;
        auto unit_ptrs = [&](int i) {
            GemvUnit T;
            p_ok = get(i, T);
            pw0 = T.w0;
            pw1 = T.w1;
        };
        uint4 ra[kFanAhead], rb[kFanAhead];
        uint32_t rs[kFanAhead];
        auto load = [&](int k) {
            if (!p_ok) return;
            const int g = pk * kFanProducers + warp;
            if (g < G) {
                const size_t off = static_cast<size_t>(g) * kGroupBytes;
                ra[k] = ldg_stream_v4(pw0 + off + lane * 16);
                if (!c.half) rb[k] = ldg_stream_v4(pw1 + off + lane * 16);
                rs[k] = ldg_stream_u32((lane < 16 ? pw0 : pw1) + off + 512 + 4 * (lane & 15));
            }
            if (++pk == nch) {
                pk = 0;
                unit_ptrs(++pi);
            }
        };
        // (get() may read the previous kernel's output: not before prelude() unless `early`)
        if (!early) prelude();
        unit_ptrs(0);
#pragma unroll
        for (int k = 0; k < kFanAhead; ++k) load(k);
        if (early) prelude();
        float *e4p = c.e4p + warp * 256;
        const uint8_t *act0 = c.img + gid * c.img_ts + tig * 16;
        const uint8_t *cs0 = c.img + kMaxTok * c.img_ts + tig * kCsEntry;
        // items in turn, kFanAhead per round so that the register buffers are indexed statically
        int item = 0, ci = 0, ck = 0;
        GemvUnit U;
        bool c_ok = get(0, U);
        while (c_ok) {
#pragma unroll
            for (int r = 0; r < kFanAhead; ++r) {
                if (!c_ok) break;
                if (ck == 0 && changes(U)) {
                    bar_sync_n(kBarProducers, kFanProducers * 32);   // every producer done with the old image
                    restage(U, static_cast<int>(threadIdx.x), kFanProducers * 32);
                    bar_sync_n(kBarProducers, kFanProducers * 32);
                }
                const int slot = item & 1;
                if (item >= 2) bar_sync_n(kBarEmpty + slot, kFanThreads);   // the chain warp read this slot
                const int g = ck * kFanProducers + warp;
                if (g < G) {
                    decode_scales(rs[r], lane, e4p);
                    __syncwarp();
                    uint4 *dst = reinterpret_cast<uint4 *>(c.prod + slot * kFanSlotBytes + warp * kFanGroupBytes) + lane;
                    auto put = [&](int j, const uint64_t (&p)[4]) {
                        dst[(2 * j) * 32] = make_uint4(static_cast<uint32_t>(p[0]), static_cast<uint32_t>(p[0] >> 32),
                                                       static_cast<uint32_t>(p[1]), static_cast<uint32_t>(p[1] >> 32));
                        dst[(2 * j + 1) * 32] = make_uint4(static_cast<uint32_t>(p[2]), static_cast<uint32_t>(p[2] >> 32),
                                                           static_cast<uint32_t>(p[3]), static_cast<uint32_t>(p[3] >> 32));
                    };
                    if (c.half)
                        group_products<true>(ra[r], ra[r], e4p, act0 + g * 64, cs0 + g * 4 * kCsEntry, lane, c.zero, put);
                    else
                        group_products<false>(ra[r], rb[r], e4p, act0 + g * 64, cs0 + g * 4 * kCsEntry, lane, c.zero, put);
                    __syncwarp();   // (the scale pairs are rewritten by the next group)
                }
                bar_arrive_n(kBarFull + slot, kFanThreads);
                load(r);
                ++item;
                if (++ck == nch) {
                    ck = 0;
                    c_ok = get(++ci, U);
                }
            }
        }
        // the chain warp's last two arrivals on EMPTY, consumed
        for (int j = item - 2; j < item; ++j)
            if (j >= 0) bar_sync_n(kBarEmpty + (j & 1), kFanThreads);
    } else {
        // chain warp h (0: tile A, 1: tile B) adds its tile's products (slot elements 2 j + h); tile B's sums go to
        // tile A's warp through shared memory, which runs the epilogue
        prelude();
        const int h = warp - kFanProducers;
        int item = 0;
        GemvUnit U;
        for (int i = 0; get(i, U); ++i) {
            uint64_t acc0 = 0, acc1 = 0;
#pragma unroll 1
            for (int k = 0; k < nch; ++k, ++item) {
                const int slot = item & 1;
                bar_sync_n(kBarFull + slot, kFanThreads);
                const int ng = min(kFanProducers, G - k * kFanProducers);
                // (half units: both chain warps read tile A's element; warp h adds its rows' half of it)
                const uint4 *src = reinterpret_cast<const uint4 *>(c.prod + slot * kFanSlotBytes) + (c.half ? 0 : h * 32) + lane;
                // two groups a round, alternating buffers: a group's four loads go out a round before its adds
                uint4 va[4], vb[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) va[j] = ld_shared_v4(src + (2 * j) * 32);
                int gl = 0;
#pragma unroll 1
                for (; gl + 2 <= ng; gl += 2) {
                    const uint4 *s1 = src + (gl + 1) * (kFanGroupBytes / 16);
#pragma unroll
                    for (int j = 0; j < 4; ++j) vb[j] = ld_shared_v4(s1 + (2 * j) * 32);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc0 = f2_add(acc0, pack2(va[j].x, va[j].y));
                        acc1 = f2_add(acc1, pack2(va[j].z, va[j].w));
                    }
                    if (gl + 2 < ng) {
                        const uint4 *s2 = src + (gl + 2) * (kFanGroupBytes / 16);
#pragma unroll
                        for (int j = 0; j < 4; ++j) va[j] = ld_shared_v4(s2 + (2 * j) * 32);
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc0 = f2_add(acc0, pack2(vb[j].x, vb[j].y));
                        acc1 = f2_add(acc1, pack2(vb[j].z, vb[j].w));
                    }
                }
                if (gl < ng) {   // (an odd count: the last group, already loaded)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc0 = f2_add(acc0, pack2(va[j].x, va[j].y));
                        acc1 = f2_add(acc1, pack2(va[j].z, va[j].w));
                    }
                }
                bar_arrive_n(kBarEmpty + slot, kFanThreads);
            }
            // y = acc * global * 1 (engine/src/kernels.cpp:1320). (Half units: warp 0 has all of tile A already; warp 1's
            // identical sums are not needed.)
            if (h == 1) c.xchg[lane] = make_float4(lo_f(acc0), hi_f(acc0), lo_f(acc1), hi_f(acc1));
            bar_sync_n(kBarChains, kFanChains * 32);
            if (h == 0) {
                const float4 yb = c.xchg[lane];
                float y0[4] = {lo_f(acc0), hi_f(acc0), lo_f(acc1), hi_f(acc1)};
                float y1[4] = {yb.x, yb.y, yb.z, yb.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    y0[q] = __fmul_rn(y0[q], __fmul_rn(U.g0, 0.125f));
                    y1[q] = __fmul_rn(y1[q], __fmul_rn(U.g1, 0.125f));
                }
                epi(U, y0, y1, gid, tig);
            }
            bar_sync_n(kBarChains, kFanChains * 32);   // (the exchange is free for the next unit)
        }
    }
}

}  // namespace gcu
