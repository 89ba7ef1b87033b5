// umma_gemm.cuh - the q4 product on the tcgen05 tensor core, bit for bit the reference's matvec_rows_q_ref
// (engine/src/kernels.cpp:1304-1322) for any number of token rows:
//   y[t][r] = (sum over blocks b in order of float(isum_b) * (e4m3[r][b] * ascale[t][b])) * global.
//
// The integer block sums come from int8 MMAs of K = 32 (two 16-value blocks): A = the weight codes as u8 (c' in
// 0..15, level = 2 c' - 15) for 128 rows, B = 2 NT "columns" per K-step, column 2t holding token t's 16 activations
// of the first block and zeros for the second, column 2t + 1 the reverse - so one MMA leaves each block's own sum
// sum_i c'_i q_i of every token in its own TMEM column, and isum = 2 D - 15 bsum (bsum: the activation block's sum).
// No accumulation in the tensor core: the float chain over the blocks, in block order, runs in the epilogue threads
// (one thread a row) with the reference's own operations, so the result is exact.
//
// Weights in the "U" layout (gcuda_op_q4_umma_relayout), the same 9/16 byte per value as the pack:
//   codes: for 128-row tile T and K-step ks (32 columns) 128 rows x 16 bytes at ((T * KS + ks) * 128 + r) * 16,
//          byte j = c'(column 32 ks + j) | c'(column 32 ks + 16 + j) << 4 - a row's K-step unpacks with two masks
//          into the two 16-byte halves the canonical K-major layout wants;
//   scales: after rows * cols / 2 code bytes, per tile, 64-column group g and row a 32-bit word of the four blocks'
//          E4M3 bytes at ((T * (cols / 64) + g) * 128 + r) * 4.
//
// A CTA (persistent over units = (tile, block of NT tokens)) runs four roles on its own rings:
//   warp 12 lane 0: per chunk of 8 K-steps, bulk copies (cp.async.bulk, mbarrier complete_tx) of the tile's packed
//              codes (16 KB) and of each token's 256 activations;
//   warps 8-11: per batch of 8 K-steps each thread unpacks its row into the batch's A (the K-major layout with the
//              128-byte swizzle: K-atoms of 8 rows x 128 bytes, four K-steps each; the tensor core reads it at full
//              shared-memory width, where the unswizzled layout made each MMA take about 200 ns) and the first 2N
//              threads write B's 16-byte pieces; one proxy fence a batch;
//   warp 13 lane 0: per batch, its 8 MMAs (descriptors 32 bytes further into the K-atom per step) into the TMEM
//              buffer of the current chunk (two buffers of 256 columns), a commit that frees the batch, a commit per
//              chunk that hands the buffer to the epilogue;
//   warps 0-7: two warps per TMEM lane quarter (the rows), each with half of the unit's tokens: per chunk its rows'
//              scale words, then its columns (tcgen05.ld, several K-steps before one wait) into its tokens' chains,
//              with the unit's per-token block sums and scales staged in shared memory; y = chain * global.
// Every wait is bounded: one that gives up sets kErrWaitTimeout in the status word and the CTA stops its units.
#pragma once

#include "common.cuh"
#include "gemv_core.cuh"
#include "q4_gemv.cuh"
#include "umma.cuh"

namespace gcu {

constexpr int kUmmaRows = 128;
constexpr int kUmmaStepBytes = kUmmaRows * 16;   // one tile's packed codes of one K-step
constexpr int kUmmaPackSteps = 8;                // K-steps per chunk of bulk copies
constexpr int kUmmaUnpackBatch = kUmmaPackSteps; // K-steps an unpacker thread writes before one proxy fence
constexpr int kUmmaEpiWarps = 8;                 // two per TMEM lane quarter, each half of the token columns
constexpr int kUmmaThreads = 32 * (kUmmaEpiWarps + 4 + 2);
constexpr int kUmmaMaxCols = 4096;
constexpr uint32_t kUmmaWaitLimit = 1u << 22;    // polls before a wait gives up (seconds at most)

__host__ __device__ inline size_t umma_code_bytes(int64_t rows, int64_t cols) {
    return static_cast<size_t>(rows) * static_cast<size_t>(cols) / 2;
}

template <int NT>
struct UmmaSmem {
    // A/B batches (8 K-steps each): as many as the shared memory holds next to the rest
    static constexpr int kABBatches = NT >= 8 ? 2 : 3;
    static constexpr int kPackStages = 4;
    static constexpr int N = 2 * NT;                              // MMA columns
    // a batch: two K-atoms of A (128 rows x 128 bytes = four K-steps each, 128-byte swizzle), then B's two K-atoms
    // (N rows x 128 bytes each); every atom 1024-byte aligned (the swizzle repeats every 8 rows of 128 bytes)
    static constexpr int kAAtomBytes = kUmmaRows * 128;
    static constexpr int kBAtomBytes = N * 128;
    static constexpr int kABBatchBytes = 2 * kAAtomBytes + 2 * kBAtomBytes;
    static constexpr int kActBytes = NT * kUmmaPackSteps * 32;    // the chunk's activations: NT tokens x 256 bytes
    static constexpr int kPackBytes = kUmmaPackSteps * kUmmaStepBytes + kActBytes;
    alignas(1024) uint8_t ab[kABBatches][kABBatchBytes];
    alignas(128) uint8_t packed[kPackStages][kPackBytes];
    // per token and K-step: the two blocks' activation sums, then their scales' bits (the epilogue's unit data)
    alignas(16) int4 tokdata[NT * (kUmmaMaxCols / 32)];
    uint64_t packed_full[kPackStages], packed_empty[kPackStages];
    uint64_t ab_full[kABBatches], ab_empty[kABBatches];
    uint64_t tm_full[2], tm_empty[2];
    uint32_t tmem_base;
    int abort;
    int epi_stop;   // the epilogue warps' common decision to stop after a unit
};

// A unit of the grouped form: one 128-row tile of one matrix (U layout) against up to NT token entries
// toklist[tok0 ..tok0 + nt) (activation row entry / act_div, output row entry).
struct UmmaUnit {
    const uint8_t *w;
    float global;
    int tile, nt, tok0;
};

struct UmmaGemmArgs {
    const uint8_t *w;   // U layout (the dense form: one matrix, every tile x every block of NT tokens)
    int rows, cols;     // every unit's matrix shape
    float global;
    ActSet act;         // activation row r: q at r * qstride, scale / bsum at r * sstride
    float *y;
    int ystride;        // y[output row * ystride + matrix row]
    uint32_t *status;
    // the grouped form (units != NULL): the unit table, its length (on the device), the token entries
    const UmmaUnit *units;
    const int *n_units;
    const int *toklist;
    int act_div;
};

// what a role needs of unit u: the matrix, its global, the tile, the token count and the first entry
struct UmmaUnitView {
    const uint8_t *w;
    float global;
    int tile, nt, tok0;
};

template <int NT>
__host__ __device__ constexpr size_t umma_smem_bytes() { return sizeof(UmmaSmem<NT>) + 1024; }

#if defined(__CUDA_ARCH__)
template <int NT>
__device__ __forceinline__ UmmaUnitView umma_unit(const UmmaGemmArgs &a, int u, int tblocks) {
    if (a.units) {
        const UmmaUnit U = a.units[u];
        return UmmaUnitView{U.w, U.global, U.tile, U.nt, U.tok0};
    }
    const int tb = u % tblocks;
    return UmmaUnitView{a.w, a.global, u / tblocks, min(NT, a.act.n - tb * NT), tb * NT};
}
// token entry i of a unit: its activation row and its output row
__device__ __forceinline__ int umma_entry(const UmmaGemmArgs &a, const UmmaUnitView &v, int i) {
    return a.units ? __ldg(a.toklist + v.tok0 + i) : v.tok0 + i;
}
__device__ __forceinline__ bool umma_give_up(volatile int *abort, uint32_t *status) {
    *abort = 1;
    if (status) atomicOr(status, kErrWaitTimeout);
    return false;
}
// a bounded wait that also stops when another role of the CTA gave up
__device__ __forceinline__ bool umma_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
    for (uint32_t i = 0; i < kUmmaWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *abort) return false;
    }
    return false;
}
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kUmmaEpiWarps) : "memory"); }
#endif

template <int NT>
__global__ void __launch_bounds__(kUmmaThreads, 1) k_umma_gemm(UmmaGemmArgs a) {
#if defined(__CUDA_ARCH__)
    extern __shared__ uint8_t smem_raw[];
    UmmaSmem<NT> &S = *reinterpret_cast<UmmaSmem<NT> *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int N = 2 * NT;
    constexpr int KT = 256 / N;         // K-steps per TMEM buffer (256 columns)
    constexpr int HT = NT / 2;          // tokens per epilogue warp
    constexpr int KB = NT >= 16 ? 1 : 4;   // K-steps whose TMEM loads go out together (a group)
    constexpr int kCodeBytes = kUmmaPackSteps * kUmmaStepBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KS = a.cols / 32, G = a.cols / 64;
    const int tiles = a.rows / kUmmaRows, tblocks = (a.act.n + NT - 1) / NT;
    const int units = a.units ? *a.n_units : tiles * tblocks;
    const int act_div = a.units ? a.act_div : 1;
    volatile int *abort = &S.abort;
    if (threadIdx.x == 0) {
        // (consumer barriers count warps: each warp's lanes finish, sync, then one lane arrives - 128 arrivals on one
        // barrier would serialise on its shared-memory word)
        for (int i = 0; i < UmmaSmem<NT>::kPackStages; ++i) mbar_init(&S.packed_full[i], 1), mbar_init(&S.packed_empty[i], 4);
        for (int i = 0; i < UmmaSmem<NT>::kABBatches; ++i) mbar_init(&S.ab_full[i], 4), mbar_init(&S.ab_empty[i], 1);
        for (int i = 0; i < 2; ++i) mbar_init(&S.tm_full[i], 1), mbar_init(&S.tm_empty[i], kUmmaEpiWarps);
        S.abort = 0;
        fence_barrier_init();
    }
    if (warp == kUmmaEpiWarps + 5) {
        tmem_alloc(&S.tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = S.tmem_base;

    if (warp == kUmmaEpiWarps + 4) {
        // ---- bulk copies: per chunk of 8 K-steps the tile's packed codes (16 KB) and each token's 256 activations
        if (lane == 0) {
            uint32_t s = 0, ph = 0;
            int last_ph[UmmaSmem<NT>::kPackStages];
            for (int i = 0; i < UmmaSmem<NT>::kPackStages; ++i) last_ph[i] = -1;
            for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x) {
                const UmmaUnitView U = umma_unit<NT>(a, u, tblocks);
                const int nt = U.nt;
                for (int pc = 0; pc < KS / kUmmaPackSteps && !*abort; ++pc) {
                    if (!umma_wait(&S.packed_empty[s], ph ^ 1, abort)) {
                        umma_give_up(abort, a.status);
                        break;
                    }
                    mbar_expect_tx(&S.packed_full[s], kCodeBytes + nt * kUmmaPackSteps * 32);
                    bulk_g2s(S.packed[s], U.w + (static_cast<size_t>(U.tile) * KS + static_cast<size_t>(pc) * kUmmaPackSteps) * kUmmaStepBytes,
                             kCodeBytes, &S.packed_full[s]);
                    for (int tok = 0; tok < nt; ++tok)
                        bulk_g2s(S.packed[s] + kCodeBytes + tok * kUmmaPackSteps * 32,
                                 a.act.q + static_cast<size_t>(umma_entry(a, U, tok) / act_div) * a.act.qstride +
                                     static_cast<size_t>(pc) * kUmmaPackSteps * 32,
                                 kUmmaPackSteps * 32, &S.packed_full[s]);
                    last_ph[s] = static_cast<int>(ph);
                    if (++s == UmmaSmem<NT>::kPackStages) s = 0, ph ^= 1;
                }
            }
            // no copy may still be writing this CTA's shared memory when it leaves (after a give-up the unpackers
            // stop consuming): wait for each stage's last fill, bounded
            for (int i = 0; i < UmmaSmem<NT>::kPackStages; ++i)
                if (last_ph[i] >= 0 && !mbar_wait(&S.packed_full[i], static_cast<uint32_t>(last_ph[i]), kUmmaWaitLimit))
                    umma_give_up(abort, a.status);
        }
    } else if (warp >= kUmmaEpiWarps && warp < kUmmaEpiWarps + 4) {
        // ---- unpack A (a thread a row), write B's 16-byte pieces from the staged activations
        const int t = threadIdx.x - 32 * kUmmaEpiWarps;
        uint32_t ps = 0, pph = 0, as = 0, aph = 0;
        const int ri = t & 7;
        const int n_ = t >> 1, c = t & 1, tok = n_ >> 1, h = n_ & 1;   // (this thread's B piece, t < 2N)
        constexpr int KU = kUmmaUnpackBatch, NB = UmmaSmem<NT>::kABBatches;
        // this thread's row in an A atom and its B row (128-byte swizzle: chunk q of the row at chunk q ^ (row % 8))
        const int a_row = (t >> 3) * 1024 + ri * 128, b_row = (n_ >> 3) * 1024 + (n_ & 7) * 128;
        for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x) {
            const int nt = umma_unit<NT>(a, u, tblocks).nt;
            bool ok = true;
            for (int k0 = 0; k0 < KS && ok; k0 += KU) {
                // KU K-steps at once (KS, the chunk and the ring are multiples of KU): their stages free, their packed
                // rows and activation pieces loaded, written, one fence, then their arrivals
                if ((k0 % kUmmaPackSteps) == 0 && !umma_wait(&S.packed_full[ps], pph, abort)) ok = false;
                if (ok && !umma_wait(&S.ab_empty[as], aph ^ 1, abort)) ok = false;
                ok = __all_sync(0xffffffffu, ok);   // (the warp syncs below: its lanes go on, or stop, together)
                if (!ok) {
                    umma_give_up(abort, a.status);
                    break;
                }
                uint4 x[KU], v[KU];
#pragma unroll
                for (int j = 0; j < KU; ++j) {
                    const int kp = (k0 + j) % kUmmaPackSteps;
                    x[j] = *reinterpret_cast<const uint4 *>(S.packed[ps] + (kp * kUmmaRows + t) * 16);
                    v[j] = make_uint4(0, 0, 0, 0);
                    if (t < 2 * N && c == h && tok < nt)
                        v[j] = *reinterpret_cast<const uint4 *>(S.packed[ps] + kCodeBytes + tok * kUmmaPackSteps * 32 + kp * 32 + 16 * c);
                }
#pragma unroll
                for (int j = 0; j < KU; ++j) {
                    constexpr uint32_t M4 = 0x0F0F0F0Fu;
                    const int ka = j >> 2, kq = j & 3;   // K-atom of the batch, K-step inside it (32 bytes)
                    uint8_t *A = S.ab[as] + ka * UmmaSmem<NT>::kAAtomBytes + a_row;
                    *reinterpret_cast<uint4 *>(A + (((2 * kq) ^ ri) << 4)) =
                        make_uint4(x[j].x & M4, x[j].y & M4, x[j].z & M4, x[j].w & M4);
                    *reinterpret_cast<uint4 *>(A + (((2 * kq + 1) ^ ri) << 4)) =
                        make_uint4((x[j].x >> 4) & M4, (x[j].y >> 4) & M4, (x[j].z >> 4) & M4, (x[j].w >> 4) & M4);
                    if (t < 2 * N)
                        *reinterpret_cast<uint4 *>(S.ab[as] + 2 * UmmaSmem<NT>::kAAtomBytes + ka * UmmaSmem<NT>::kBAtomBytes +
                                                   b_row + (((2 * kq + c) ^ (n_ & 7)) << 4)) = v[j];
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.ab_full[as]);
                if (((k0 + KU) % kUmmaPackSteps) == 0) {
                    if (lane == 0) mbar_arrive(&S.packed_empty[ps]);
                    if (++ps == UmmaSmem<NT>::kPackStages) ps = 0, pph ^= 1;
                }
                if (++as == NB) as = 0, aph ^= 1;
            }
        }
    } else if (warp == kUmmaEpiWarps + 5) {
        // ---- the MMAs
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_i8(kUmmaRows, N, false, true);
            uint32_t as = 0, aph = 0, tb_ = 0, tph = 0;
            int last_as = -1;   // the stage of the last MMA issued, and the phase its commit completes
            uint32_t last_aph = 0;
            constexpr int KU = kUmmaUnpackBatch, NB = UmmaSmem<NT>::kABBatches;
            for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x) {
                bool ok = true;
                for (int k0 = 0; k0 < KS && ok; k0 += KU) {
                    // one batch: its KU MMAs (a TMEM buffer handed over at each chunk's end, which may fall inside the
                    // batch), then one commit that frees the batch's stages
                    if (!umma_wait(&S.ab_full[as], aph, abort)) {
                        ok = umma_give_up(abort, a.status);
                        break;
                    }
                    tc_fence_after();
                    for (int j = 0; j < KU && ok; ++j) {
                        const int ks = k0 + j, kk = ks % KT;
                        if (kk == 0) {
                            if (!umma_wait(&S.tm_empty[tb_], tph ^ 1, abort)) {
                                ok = umma_give_up(abort, a.status);
                                break;
                            }
                            tc_fence_after();
                        }
                        // K-step j: K-atom j / 4, 32 bytes further into it per step
                        const uint32_t ab = smem_u32(S.ab[as]) + static_cast<uint32_t>((j & 3) * 32);
                        const uint32_t a_at = ab + static_cast<uint32_t>((j >> 2) * UmmaSmem<NT>::kAAtomBytes);
                        const uint32_t b_at = ab + static_cast<uint32_t>(2 * UmmaSmem<NT>::kAAtomBytes + (j >> 2) * UmmaSmem<NT>::kBAtomBytes);
                        umma_i8(tbase + tb_ * 256 + static_cast<uint32_t>(kk * N), umma_smem_desc_sw128(a_at, 1024),
                                umma_smem_desc_sw128(b_at, 1024), idesc, false);
                        if (kk == KT - 1 || ks == KS - 1) {
                            umma_commit(&S.tm_full[tb_]);
                            if (++tb_ == 2) tb_ = 0, tph ^= 1;
                        }
                    }
                    // (also after a give-up inside the batch: the commit then covers the MMAs it did issue)
                    umma_commit(&S.ab_empty[as]);
                    last_as = static_cast<int>(as);
                    last_aph = aph;
                    if (++as == NB) as = 0, aph ^= 1;
                }
            }
            // every MMA this thread issued has finished before the tensor memory is freed (its last commit covers
            // all earlier ones) - after a give-up too
            if (last_as >= 0 && !mbar_wait(&S.ab_empty[last_as], last_aph, kUmmaWaitLimit)) umma_give_up(abort, a.status);
        }
    } else {
        // ---- the epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its rows) and the columns of tokens
        // HT (w / 4) .. + HT - 1 of the unit's block
        const int quarter = warp & 3, half = warp >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        uint32_t tb_ = 0, tph = 0;
        // (every epilogue warp runs the same units: the named barriers below must see all of them, so whether to go
        // on after a unit is decided once, by thread 0, and read by all after the barrier)
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            const UmmaUnitView U = umma_unit<NT>(a, u, tblocks);
            const int T = U.tile, nt = U.nt;
            // the unit's per-token block data: (bsum, bsum, scale, scale) of blocks 2 ks, 2 ks + 1
            for (int i = threadIdx.x; i < NT * KS; i += 32 * kUmmaEpiWarps) {
                const int tk = i / KS, ks = i - tk * KS;
                int4 v = make_int4(0, 0, 0, 0);
                if (tk < nt) {
                    const size_t so = static_cast<size_t>(umma_entry(a, U, tk) / act_div) * a.act.sstride + 2 * ks;
                    const int2 bs = __ldg(reinterpret_cast<const int2 *>(a.act.bsum + so));
                    const float2 sc = __ldg(reinterpret_cast<const float2 *>(a.act.scale + so));
                    v = make_int4(bs.x, bs.y, __float_as_int(sc.x), __float_as_int(sc.y));
                }
                S.tokdata[tk * KS + ks] = v;
            }
            epi_sync();
            const int row = T * kUmmaRows + r;
            const uint32_t *sc = reinterpret_cast<const uint32_t *>(U.w + umma_code_bytes(a.rows, a.cols)) +
                                 static_cast<size_t>(T) * G * kUmmaRows + r;
            uint64_t acc[HT / 2];   // token pairs (2 tp, 2 tp + 1) of this warp's half, as f32x2
#pragma unroll
            for (int j = 0; j < HT / 2; ++j) acc[j] = 0;
            const uint64_t zero = static_cast<uint64_t>(static_cast<uint32_t>(a.rows) >> 31);   // +0 pair, runtime
            bool ok = true;
            for (int c0 = 0; c0 < KS && ok; c0 += KT) {
                const int kn = min(KT, KS - c0);
                uint32_t sw[(KT + 1) / 2];   // the row's scale words of the chunk's K-steps (two K-steps a word)
#pragma unroll
                for (int j = 0; j < (KT + 1) / 2; ++j)
                    sw[j] = 2 * j < kn ? __ldg(sc + static_cast<size_t>((c0 >> 1) + j) * kUmmaRows) : 0u;
                if (!__all_sync(0xffffffffu, umma_wait(&S.tm_full[tb_], tph, abort))) {   // (warp-uniform: syncs below)
                    ok = umma_give_up(abort, a.status);
                    break;
                }
                tc_fence_after();
                // groups of KB K-steps, two register buffers: the next group's TMEM loads are in flight while this
                // group's chains run (tcgen05.wait::ld waits for every load issued, so one group is waited at a time)
                uint32_t dA[KB][NT], dB[KB][NT];
                auto load_group = [&](int k0, uint32_t (&d)[KB][NT]) {
#pragma unroll
                    for (int j = 0; j < KB; ++j)
                        if (k0 + j < kn)
                            tmem_ld<NT>(tbase + lane_off + tb_ * 256 + static_cast<uint32_t>((k0 + j) * N + half * NT), d[j]);
                };
                auto chain_group = [&](int k0, const uint32_t (&d)[KB][NT]) {
#pragma unroll
                    for (int j = 0; j < KB; ++j) {
                        if (k0 + j >= kn) break;
                        const int kk = k0 + j, ks = c0 + kk;
                        const float2 e = e4m3x2_to_float2((sw[kk >> 1] >> (16 * (kk & 1))) & 0xFFFFu);
                        const uint64_t e0 = pack2(__float_as_uint(e.x), __float_as_uint(e.x));
                        const uint64_t e1 = pack2(__float_as_uint(e.y), __float_as_uint(e.y));
                        // two tokens at a time in f32x2 lanes (each lane rounded on its own, the product kept apart
                        // from the add); a token past the block's end has zero sums and scales and is not stored
#pragma unroll
                        for (int tp = 0; tp < HT / 2; ++tp) {
                            const int tk = half * HT + 2 * tp;
                            if (tk >= nt) break;   // (the unit's last pair may hold one token; none after it)
                            const int4 ta = S.tokdata[tk * KS + ks], tbd = S.tokdata[(tk + 1) * KS + ks];
                            const float fa0 = static_cast<float>(2 * static_cast<int32_t>(d[j][4 * tp]) - 15 * ta.x);
                            const float fb0 = static_cast<float>(2 * static_cast<int32_t>(d[j][4 * tp + 2]) - 15 * tbd.x);
                            const float fa1 = static_cast<float>(2 * static_cast<int32_t>(d[j][4 * tp + 1]) - 15 * ta.y);
                            const float fb1 = static_cast<float>(2 * static_cast<int32_t>(d[j][4 * tp + 3]) - 15 * tbd.y);
                            const uint64_t p0 = f2_mul_sep(pack2(__float_as_uint(fa0), __float_as_uint(fb0)),
                                                           f2_mul(e0, pack2(static_cast<uint32_t>(ta.z), static_cast<uint32_t>(tbd.z))), zero);
                            acc[tp] = f2_add(acc[tp], p0);
                            const uint64_t p1 = f2_mul_sep(pack2(__float_as_uint(fa1), __float_as_uint(fb1)),
                                                           f2_mul(e1, pack2(static_cast<uint32_t>(ta.w), static_cast<uint32_t>(tbd.w))), zero);
                            acc[tp] = f2_add(acc[tp], p1);
                        }
                    }
                };
                load_group(0, dA);
                tmem_wait_ld();
                for (int k0 = 0; k0 < kn; k0 += 2 * KB) {
                    if (k0 + KB < kn) load_group(k0 + KB, dB);
                    chain_group(k0, dA);
                    tmem_wait_ld();
                    if (k0 + KB < kn) {
                        if (k0 + 2 * KB < kn) load_group(k0 + 2 * KB, dA);
                        chain_group(k0 + KB, dB);
                        tmem_wait_ld();
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.tm_empty[tb_]);
                if (++tb_ == 2) tb_ = 0, tph ^= 1;
            }
            if (ok) {
#pragma unroll
                for (int tl = 0; tl < HT; ++tl) {
                    const int tk = half * HT + tl;
                    const float v = (tl & 1) ? hi_f(acc[tl >> 1]) : lo_f(acc[tl >> 1]);
                    if (tk < nt) a.y[static_cast<size_t>(umma_entry(a, U, tk)) * a.ystride + row] = __fmul_rn(v, U.global);
                }
            }
            if (threadIdx.x == 0) S.epi_stop = (!ok || *abort) ? 1 : 0;
            epi_sync();   // (every epilogue thread done with the unit's data before the next unit's goes in)
            if (S.epi_stop) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kUmmaEpiWarps + 5) {
        __syncwarp();
        tmem_dealloc(tbase, 512);
    }
#endif
}

// pack rows (C/2 code bytes, value 2j in the low nibble, then C/16 E4M3 bytes) -> the U layout; a thread per 16
// output bytes of codes or per scale word
__global__ void k_umma_relayout(const uint8_t *__restrict__ pack, int64_t rows, int64_t cols, uint8_t *__restrict__ u) {
    const int64_t KS = cols / 32, G = cols / 64, rb = cols / 2 + cols / 16;
    const int64_t n_code = rows * KS, n_sc = rows * G;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_code + n_sc;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        if (i < n_code) {
            const int64_t r = i % kUmmaRows, rest = i / kUmmaRows, ks = rest % KS, T = rest / KS;
            const uint8_t *src = pack + (T * kUmmaRows + r) * rb + ks * 16;   // values 32 ks .. 32 ks + 31
            auto code = [&](int v) {   // the pack's code of value v of this K-step, remapped so level = 2 c' - 15
                const int c = (src[v >> 1] >> ((v & 1) * 4)) & 15;
                return c < 8 ? c + 8 : 15 - c;
            };
            uint8_t out[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) out[j] = static_cast<uint8_t>(code(j) | (code(16 + j) << 4));
            *reinterpret_cast<uint4 *>(u + i * 16) = *reinterpret_cast<const uint4 *>(out);
        } else {
            const int64_t k = i - n_code;
            const int64_t r = k % kUmmaRows, rest = k / kUmmaRows, g = rest % G, T = rest / G;
            const uint8_t *s = pack + (T * kUmmaRows + r) * rb + cols / 2 + g * 4;
            const uint32_t w = s[0] | (s[1] << 8) | (s[2] << 16) | (static_cast<uint32_t>(s[3]) << 24);
            *reinterpret_cast<uint32_t *>(u + umma_code_bytes(rows, cols) + k * 4) = w;
        }
    }
}

}  // namespace gcu
