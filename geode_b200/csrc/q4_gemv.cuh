// q4_gemv.cuh - the weight GEMV of the verify step: up to 8 token columns against a q4 matrix, bit for bit the
// reference's int8 path (engine/src/kernels.cpp:1304-1322, matvec_rows_q_ref):
//     y[r] = (sum over blocks b, in order, of float(isum_b) * (e4m3(scale_rb) * ascale_b)) * global
// where isum_b is the integer dot product of block b's 16 weight levels with the token's 16 int8 activations.
//
// B200 mapping. The integer block sums run on the tensor cores (mma.sync m16n8k16 u8 x s8: 16 rows x one 16-value
// block x 8 token columns per instruction). The weights enter as 16 c (the affine code in a byte's high nibble, one
// AND / shift-and-AND per word), so with the accumulator started at 1.5 * 2^23 - 120 * bsum the result reads back as
// the exact float of 8 isum (level = 2c - 15: 16 c - 120 = 8 level) with one subtraction. Every product and sum of
// the per-(row, token) f32 chain is then 8 times the reference's, rounded the same way (a power of two, far from
// the format's limits), and the epilogue's global / 8 (exact) undoes it. The chain runs in block order with packed
// f32x2 operations (each lane IEEE, no contraction).
// Rows are relaid once at load time into 16-row tiles whose bytes a lane reads as its mma fragment. A launch runs
// its units (two tiles x all K) either a warp per unit with the weights streamed through per-warp cp.async rings, or -
// with few units - a CTA per unit whose producer warps compute the products and whose chain warps add them in order
// (gemv_core.cuh); either way no addition is reordered.
//
// Tile layout (per 16-row tile, per group of 4 blocks = 64 columns, 576 bytes):
//   bytes [0, 512):   lane l = 4 * gid + tig: 16 bytes = 4 words, word j for block 4g + j. Its low nibbles (byte i)
//                     hold the affine code of row gid, column 4 tig + i of that block; its high nibbles row gid + 8.
//   bytes [512, 576): the scale bytes, row r's four blocks at 4 r .. 4 r + 3.
// The affine code c' = c + 8 (c < 8) or 15 - c (c >= 8) of the pack's code c gives the level 2 c' - 15. The layout is
// a permutation of each tile's bytes (16 rows x 9/16 bytes per value): the bytes streamed equal the pack's.
#pragma once

#include "common.cuh"

namespace gcu {

constexpr int kGroupBytes = 576;           // one 16-row tile x 4 blocks
constexpr int kTileRows = 16;

__host__ __device__ inline int tile_bytes(int cols) { return (cols / 64) * kGroupBytes; }

// Activations quantized per 16 values (the engine's QAct): q [n][cols] int8, scale [n][cols/16] f32,
// bsum [n][cols/16] int32 (the block's sum of q), rows `stride` apart (elements).
struct ActSet {
    const int8_t *q;
    const float *scale;
    const int32_t *bsum;
    int cols, n;
    int qstride, sstride;   // between vectors: bytes of q, elements of scale / bsum
};

// Output handling of one unit (two 16-row tiles).
enum UnitMode : int {
    kStore = 0,        // y[t][row] = v
    kAccumulate = 1,   // y[t][row] += v (the residual add x += mix)
    kSwiglu = 2,       // tile 0 = gate rows, tile 1 = up rows: silu(g) * u quantized into an ActSet row per token
};

struct GemvUnit {
    const uint8_t *w0, *w1;   // the two tiles (tile layout)
    float g0, g1;             // the matrices' globals
    float *y0, *y1;           // row 0 of each tile in the output (y + t * ystride + r)
    int ngroups;              // cols / 64
    int ystride;              // elements between token rows of y
    int mode;
    int tok_mask;             // token columns written (bit t)
    // column t's output row: y + slot[t] * ystride (kStore, kAccumulate), or activation row slot[t] (kSwiglu)
    int slot[kMaxTok];
    int8_t *aq;
    float *as;
    int32_t *ab;
    int acols;                // the activation's width (the gate rows' count)
    int arow0;                // this unit's first value index in it
    int act_id;               // which activation vectors the unit multiplies (a warp restages when it changes)
};

// A block of 16 values spread over the 8 row lanes (gid) of one tig column group (v0 = value gid, v1 = value
// gid + 8), quantized as the engine's quantize_block (engine/src/kernels.cpp:1254-1267): s = amax / 127,
// q = clamp(lrint(x * (127 / amax)), +-127). Every lane of the warp must call it (shuffles).
struct Quant16 {
    int q0, q1, sum;
    float scale;
};
__device__ __forceinline__ Quant16 quant16_lanes(float v0, float v1) {
    float amax = fmaxf(fabsf(v0), fabsf(v1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 8));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 16));
    Quant16 r;
    r.scale = __fdiv_rn(amax, 127.0f);
    const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    r.q0 = max(-127, min(127, __float2int_rn(__fmul_rn(v0, inv))));
    r.q1 = max(-127, min(127, __float2int_rn(__fmul_rn(v1, inv))));
    int sum = r.q0 + r.q1;
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    sum += __shfl_xor_sync(0xffffffffu, sum, 8);
    sum += __shfl_xor_sync(0xffffffffu, sum, 16);
    r.sum = sum;
    return r;
}

// The plain epilogues: rows (gid, gid + 8) of each tile, token columns (2 tig, 2 tig + 1).
__device__ __forceinline__ void epi_store(const GemvUnit &U, const float (&y0)[4], const float (&y1)[4], int gid, int tig) {
    if (U.mode == kSwiglu) {
        // tile 0 = gate rows j, tile 1 = up rows j (j = arow0 + gid, + 8): a = silu(g) * u (engine/src/model.cpp:
        // 4522-4524, silu on std::exp), then the block of 16 quantized across the 8 gid lanes of each token column
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int t = 2 * tig + h;
            const bool on = ((U.tok_mask >> t) & 1) != 0;
            const float a0 = __fmul_rn(silu_ref(y0[h]), y1[h]);
            const float a1 = __fmul_rn(silu_ref(y0[2 + h]), y1[2 + h]);
            const Quant16 r = quant16_lanes(on ? a0 : 0.0f, on ? a1 : 0.0f);
            if (!on) continue;
            const size_t slot = static_cast<size_t>(U.slot[t]);
            int8_t *q = U.aq + slot * U.acols + U.arow0;
            q[gid] = static_cast<int8_t>(r.q0);
            q[gid + 8] = static_cast<int8_t>(r.q1);
            if (gid == 0) {
                U.as[slot * (U.acols / 16) + U.arow0 / 16] = r.scale;
                U.ab[slot * (U.acols / 16) + U.arow0 / 16] = r.sum;
            }
        }
        return;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int t = 2 * tig + h;
        if (t >= kMaxTok || !((U.tok_mask >> t) & 1)) continue;
        float *r0 = U.y0 + static_cast<size_t>(U.slot[t]) * U.ystride;
        if (U.mode == kAccumulate) {
            r0[gid] = __fadd_rn(r0[gid], y0[h]);
            r0[gid + 8] = __fadd_rn(r0[gid + 8], y0[2 + h]);
        } else {
            r0[gid] = y0[h];
            r0[gid + 8] = y0[2 + h];
        }
        if (!U.y1) continue;   // (a unit of one tile)
        float *r1 = U.y1 + static_cast<size_t>(U.slot[t]) * U.ystride;
        if (U.mode == kAccumulate) {
            r1[gid] = __fadd_rn(r1[gid], y1[h]);
            r1[gid + 8] = __fadd_rn(r1[gid + 8], y1[2 + h]);
        } else {
            r1[gid] = y1[h];
            r1[gid + 8] = y1[2 + h];
        }
    }
}

}  // namespace gcu
