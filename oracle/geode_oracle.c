/* geode_oracle.c - TEST INFRASTRUCTURE: the C restatement of the reference's CPU verify path (see geode_oracle.h).
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it, and only as the checker.
 *
 * Built with -ffp-contract=off: the reference's x86 build has no fused multiply-adds (-O3, no -mfma,
 * engine/CMakeLists.txt:45), and every float operation below is written in the reference's order, so results are
 * bit-identical to the reference on the same host libm (expf, log1pf, powf, sinf, cosf, sqrtf).
 */
#define _GNU_SOURCE
#include "geode_oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define KBLOCK 16

/* ---------------------------------------------------------------- formats (engine/src/kernels.cpp) ---- */

/* q4 levels in code order: the positive odd magnitudes, then their negatives (engine/src/kernels.cpp:30) */
static const int8_t kQ4[16] = {1, 3, 5, 7, 9, 11, 13, 15, -1, -3, -5, -7, -9, -11, -13, -15};

static float g_e4m3[256];
static pthread_once_t g_e4_once = PTHREAD_ONCE_INIT;

/* E4M3fn decoding (engine/src/kernels.cpp:39-52): exp 0 subnormal man/8 * 2^-6, else (1 + man/8) * 2^(exp-7);
 * 0x7F / 0xFF are NaN (no infinities). */
static void e4m3_init(void) {
    for (int b = 0; b < 256; ++b) {
        const int sign = b >> 7, ex = (b >> 3) & 15, man = b & 7;
        float x = ex == 0 ? ldexpf((float)man / 8.0f, -6) : ldexpf(1.0f + (float)man / 8.0f, ex - 7);
        if (ex == 15 && man == 7) x = NAN;
        g_e4m3[b] = sign ? -x : x;
    }
}

float go_e4m3_value(uint8_t b) {
    pthread_once(&g_e4_once, e4m3_init);
    return g_e4m3[b];
}

static inline size_t q4_row_bytes(int64_t cols) { return (size_t)(cols / KBLOCK) * 9; }

/* block b's 16 levels: byte j holds value 2j in its low nibble and 2j+1 in its high one (engine/src/kernels.cpp:82-90) */
static inline void block_ints(const uint8_t *codes, int b, int8_t *v) {
    const uint8_t *c = codes + b * 8;
    for (int j = 0; j < 8; ++j) {
        v[2 * j] = kQ4[c[j] & 15];
        v[2 * j + 1] = kQ4[c[j] >> 4];
    }
}

/* engine/src/kernels.cpp:1214-1228: (level * ls) * (e4m3 * global), ls = 1 for q4 */
void go_dequant_row(const go_q4 *w, int64_t r, float *out) {
    pthread_once(&g_e4_once, e4m3_init);
    const uint8_t *row = w->data + (size_t)r * q4_row_bytes(w->cols);
    const int nb = (int)(w->cols / KBLOCK);
    const uint8_t *scales = row + (size_t)nb * 8;
    for (int b = 0; b < nb; ++b) {
        int8_t v[KBLOCK];
        block_ints(row, b, v);
        const float s = g_e4m3[scales[b]] * w->global;
        for (int i = 0; i < KBLOCK; ++i) out[b * KBLOCK + i] = ((float)v[i] * 1.0f) * s;
    }
}

/* engine/src/kernels.cpp:1254-1267: per 16 values s = amax/127, q = clamp(lrint(x * 127/amax), +-127) */
void go_quantize_activation(const float *x, int64_t cols, int8_t *q, float *scale, int32_t *bsum) {
    const int64_t nb = cols / KBLOCK;
    for (int64_t b = 0; b < nb; ++b) {
        const float *xb = x + b * KBLOCK;
        float amax = 0.0f;
        for (int i = 0; i < KBLOCK; ++i) amax = fmaxf(amax, fabsf(xb[i]));
        const float s = amax / 127.0f, inv = amax > 0.0f ? 127.0f / amax : 0.0f;
        scale[b] = s;
        int32_t sum = 0;
        for (int i = 0; i < KBLOCK; ++i) {
            long v = lrintf(xb[i] * inv);
            if (v < -127) v = -127;
            if (v > 127) v = 127;
            q[b * KBLOCK + i] = (int8_t)v;
            sum += (int32_t)v;
        }
        if (bsum) bsum[b] = sum;
    }
}

/* engine/src/kernels.cpp:1304-1322: per row, blocks in order, acc += float(isum) * (e4m3 * ascale); y = acc*global*ls */
void go_matvec_q(const go_q4 *w, const int8_t *q, const float *scale, float *y, int64_t r0, int64_t r1) {
    pthread_once(&g_e4_once, e4m3_init);
    const int nb = (int)(w->cols / KBLOCK);
    const size_t rb = q4_row_bytes(w->cols);
    for (int64_t r = r0; r < r1; ++r) {
        const uint8_t *row = w->data + (size_t)r * rb;
        const uint8_t *scales = row + (size_t)nb * 8;
        float acc = 0.0f;
        for (int b = 0; b < nb; ++b) {
            int8_t v[KBLOCK];
            block_ints(row, b, v);
            int32_t s = 0;
            for (int i = 0; i < KBLOCK; ++i) s += v[i] * q[b * KBLOCK + i];
            acc += (float)s * (g_e4m3[scales[b]] * scale[b]);
        }
        y[r] = acc * w->global * 1.0f;
    }
}

static inline float bf16f(uint16_t v) {
    const uint32_t u = (uint32_t)v << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* engine/src/kernels.cpp:1449-1518 (and 1428-1435 when cols % 8): eight partial sums per row, combined as
 * ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7)); xs [n][cols], ys [n][rows] */
void go_matvec_bf16(const uint16_t *w, int64_t rows, int64_t cols, int n, const float *xs, float *ys) {
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t *row = w + r * cols;
        for (int t = 0; t < n; ++t) {
            const float *x = xs + (size_t)t * cols;
            if (cols % 8) {
                float acc = 0.0f;
                for (int64_t c = 0; c < cols; ++c) acc += bf16f(row[c]) * x[c];
                ys[(size_t)t * rows + r] = acc;
                continue;
            }
            float a[8] = {0};
            for (int64_t c = 0; c < cols; c += 8)
                for (int j = 0; j < 8; ++j) a[j] += bf16f(row[c + j]) * x[c + j];
            ys[(size_t)t * rows + r] = ((a[0] + a[4]) + (a[1] + a[5])) + ((a[2] + a[6]) + (a[3] + a[7]));
        }
    }
}

/* engine/src/kernels.cpp:1520-1529: the sum of squares in double, x * inv * (1 + w) */
void go_rmsnorm(const float *x, const float *w, float *out, int n, float eps, int zero_centered) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)x[i] * x[i];
    const float inv = 1.0f / sqrtf((float)(ss / n) + eps);
    if (!w) {
        for (int i = 0; i < n; ++i) out[i] = x[i] * inv;
        return;
    }
    for (int i = 0; i < n; ++i) out[i] = x[i] * inv * (zero_centered ? 1.0f + w[i] : w[i]);
}

/* engine/src/kernels.hpp:146-163: Cephes' expf (two-part ln 2 reduction, degree-6 polynomial) */
float go_fast_exp(float x) {
    x = fminf(fmaxf(x, -87.0f), 88.0f);
    const float n = floorf(x * 1.44269504088896341f + 0.5f);
    float r = x - n * 0.693359375f;
    r = r + n * 2.12194440e-4f;
    float p = 1.9875691500e-4f;
    p = p * r + 1.3981999507e-3f;
    p = p * r + 8.3334519073e-3f;
    p = p * r + 4.1665795894e-2f;
    p = p * r + 1.6666665459e-1f;
    p = p * r + 5.0000001201e-1f;
    p = p * r * r + r + 1.0f;
    uint32_t bits;
    memcpy(&bits, &p, 4);
    bits += (uint32_t)((int32_t)n) << 23;
    memcpy(&p, &bits, 4);
    return p;
}
static inline float silu_fast(float x) { return x / (1.0f + go_fast_exp(-x)); }
static inline float silu(float x) { return x / (1.0f + expf(-x)); }
static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
static inline float softplusf_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

/* ---------------------------------------------------------------- the router (engine/src/model.cpp:4021-4065) ---- */

/* softmax over E (float sum), the K largest probabilities (ties: the lower index - the reference's partial_sort
 * leaves their order unspecified), weights p_k / sum of the K (summed in pick order) */
void go_route_topk(const float *logits, int E, int K, int *ids, float *weights) {
    float *p = (float *)malloc(sizeof(float) * (size_t)E);
    float mx = logits[0];
    for (int e = 1; e < E; ++e)
        if (logits[e] > mx) mx = logits[e];
    float sum = 0.0f;
    for (int e = 0; e < E; ++e) sum += (p[e] = expf(logits[e] - mx));
    for (int e = 0; e < E; ++e) p[e] /= sum;
    char *used = (char *)calloc((size_t)E, 1);
    for (int i = 0; i < K; ++i) {
        int best = -1;
        for (int e = 0; e < E; ++e)
            if (!used[e] && (best < 0 || p[e] > p[best])) best = e;
        used[best] = 1;
        ids[i] = best;
    }
    float top = 0.0f;
    for (int i = 0; i < K; ++i) top += p[ids[i]];
    if (weights)
        for (int i = 0; i < K; ++i) weights[i] = p[ids[i]] / top;
    free(used);
    free(p);
}

/* ---------------------------------------------------------------- the q4 quantizer (engine/src/yue2_q4.cpp:72-114) ---- */

/* a non-negative float onto E4M3: the nearest positive code (ties to the even code), saturating at code 126 */
static uint8_t e4m3_byte(float x) {
    pthread_once(&g_e4_once, e4m3_init);
    if (!(x > 0.0f)) return 0;
    if (x >= g_e4m3[126]) return 126;
    int hi = 0; /* the first code with value > x (codes 0..126 ascending) */
    while (hi < 127 && !(g_e4m3[hi] > x)) ++hi;
    const int lo = hi - 1;
    const float dl = x - g_e4m3[lo], dh = g_e4m3[hi] - x;
    if (dl < dh) return (uint8_t)lo;
    if (dh < dl) return (uint8_t)hi;
    return (uint8_t)(lo % 2 == 0 ? lo : hi);
}

/* ten candidate scale codes (amax onto 15 and onto 13, two either side), the least squared error wins (the first of
 * equals); each value onto the nearest odd magnitude (exact ties to the even index) */
void go_q4_block(const float *x, float s2, uint8_t *scale_byte, uint8_t codes[16]) {
    pthread_once(&g_e4_once, e4m3_init);
    float amax = 0.0f;
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(x[i]));
    int cand[10], nc = 0;
    const float ts[2] = {15.0f, 13.0f};
    for (int t = 0; t < 2; ++t) {
        const int b0 = e4m3_byte(amax / (ts[t] * s2));
        for (int k = -2; k <= 2; ++k) {
            int c = b0 + k;
            if (c < 0) c = 0;
            if (c > 0x7E) c = 0x7E;
            cand[nc++] = c;
        }
    }
    float best = INFINITY;
    uint8_t tmp[16];
    for (int c = 0; c < nc; ++c) {
        const float scale = g_e4m3[cand[c]] * s2, safe = scale == 0.0f ? 1.0f : scale;
        float err = 0.0f;
        for (int i = 0; i < 16; ++i) {
            const float y = x[i] / safe, a = fminf(fabsf(y), 15.0f);
            int idx = (int)nearbyintf((a - 1.0f) * 0.5f);
            if (idx < 0) idx = 0;
            if (idx > 7) idx = 7;
            const int neg = y < 0.0f;
            const float qv = (float)(neg ? -(2 * idx + 1) : 2 * idx + 1) * scale;
            err += (qv - x[i]) * (qv - x[i]);
            tmp[i] = (uint8_t)(idx + (neg ? 8 : 0));
        }
        if (err < best) {
            best = err;
            *scale_byte = (uint8_t)cand[c];
            memcpy(codes, tmp, 16);
        }
    }
}

typedef struct {
    const float *w;
    int64_t r0, r1, cols;
    float s2;
    uint8_t *out;
} qjob;

static void *quantize_rows(void *arg) {
    const qjob *j = (const qjob *)arg;
    const int nb = (int)(j->cols / 16);
    const size_t rb = q4_row_bytes(j->cols);
    for (int64_t r = j->r0; r < j->r1; ++r) {
        uint8_t *row = j->out + (size_t)r * rb;
        for (int b = 0; b < nb; ++b) {
            uint8_t codes[16];
            go_q4_block(j->w + (size_t)r * j->cols + (size_t)b * 16, j->s2, &row[(size_t)nb * 8 + b], codes);
            for (int k = 0; k < 8; ++k) row[b * 8 + k] = (uint8_t)(codes[2 * k] | (codes[2 * k + 1] << 4));
        }
    }
    return NULL;
}

void go_quantize_q4(const float *w, int64_t rows, int64_t cols, float s2, uint8_t *out, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    pthread_t th[64];
    qjob jobs[64];
    const int64_t per = (rows + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        const int64_t r0 = t * per, r1 = r0 + per < rows ? r0 + per : rows;
        if (r0 >= r1) break;
        jobs[t] = (qjob){w, r0, r1, cols, s2, out};
        if (t == 0) continue;
        pthread_create(&th[t], NULL, quantize_rows, &jobs[t]);
        ++started;
    }
    if (rows > 0) quantize_rows(&jobs[0]);
    for (int t = 1; t <= started; ++t) pthread_join(th[t], NULL);
}

/* ---------------------------------------------------------------- the forward pass ---- */

typedef struct {
    int8_t *q;
    float *s;
} qact;

static qact qact_new(int64_t cols) {
    qact a = {(int8_t *)malloc((size_t)cols), (float *)malloc(sizeof(float) * (size_t)(cols / 16 + 1))};
    return a;
}
static void qact_free(qact a) {
    free(a.q);
    free(a.s);
}

/* Large products split by rows over threads (GEODE_ORACLE_THREADS, default the host's cores, at most 32): every row's
 * arithmetic is the same whichever thread runs it, so the results are the single-threaded ones bit for bit. */
typedef struct {
    const go_q4 *w;
    const int8_t *q;
    const float *s;
    float *y;
    int64_t r0, r1;
} mv_job;

static void *mv_run(void *p) {
    const mv_job *j = (const mv_job *)p;
    go_matvec_q(j->w, j->q, j->s, j->y, j->r0, j->r1);
    return NULL;
}

static int g_threads;
static pthread_once_t g_threads_once = PTHREAD_ONCE_INIT;
static void threads_init(void) {
    const char *e = getenv("GEODE_ORACLE_THREADS");
    long c = e ? atol(e) : sysconf(_SC_NPROCESSORS_ONLN);
    g_threads = c < 1 ? 1 : c > 32 ? 32 : (int)c;
}

static void matvec_rows(const go_q4 *w, const int8_t *q, const float *s, float *y) {
    pthread_once(&g_e4_once, e4m3_init);
    pthread_once(&g_threads_once, threads_init);
    const int T = g_threads;
    if (T <= 1 || w->rows * w->cols < ((int64_t)1 << 22)) {
        go_matvec_q(w, q, s, y, 0, w->rows);
        return;
    }
    pthread_t th[32];
    mv_job jb[32];
    int started[32] = {0};
    const int64_t chunk = (w->rows + T - 1) / T;
    for (int i = 0; i < T; ++i) {
        const int64_t r0 = (int64_t)i * chunk, r1 = r0 + chunk < w->rows ? r0 + chunk : w->rows;
        jb[i] = (mv_job){w, q, s, y, r0 < w->rows ? r0 : w->rows, r1};
        started[i] = jb[i].r0 < jb[i].r1 && pthread_create(&th[i], NULL, mv_run, &jb[i]) == 0;
        if (!started[i] && jb[i].r0 < jb[i].r1) mv_run(&jb[i]);   /* (no thread: this one does the rows) */
    }
    for (int i = 0; i < T; ++i)
        if (started[i]) pthread_join(th[i], NULL);
}

/* Model::matmul's int8 path (engine/src/model.cpp:3388-3397, 3422-3424): each token's activation quantized, then
 * matvec_rows_q over every row. xs [n][cols], ys [n][rows] */
static void matmul(const go_q4 *w, int n, const float *xs, float *ys) {
    qact a = qact_new(w->cols);
    for (int t = 0; t < n; ++t) {
        go_quantize_activation(xs + (size_t)t * w->cols, w->cols, a.q, a.s, NULL);
        matvec_rows(w, a.q, a.s, ys + (size_t)t * w->rows);
    }
    qact_free(a);
}

/* delta_strip (engine/src/model.cpp:3501-3524): one token through a strip of W columns of a head's state */
static void delta_strip(float *S, int dk, int W, int stride, const float *q, const float *k, const float *v,
                        float decay, float beta, float *out) {
    float mem[16] = {0}, o[16] = {0};
    for (int i = 0; i < dk; ++i) {
        float *row = S + (size_t)i * stride;
        const float ki = k[i];
        for (int j = 0; j < W; ++j) {
            row[j] *= decay;
            mem[j] += row[j] * ki;
        }
    }
    for (int j = 0; j < W; ++j) mem[j] = (v[j] - mem[j]) * beta;
    for (int i = 0; i < dk; ++i) {
        float *row = S + (size_t)i * stride;
        const float ki = k[i], qi = q[i];
        for (int j = 0; j < W; ++j) {
            row[j] += ki * mem[j];
            o[j] += row[j] * qi;
        }
    }
    for (int j = 0; j < W; ++j) out[j] = o[j];
}

/* Model::gdn (engine/src/model.cpp:3527-3688) for n tokens; h [n][H] -> mix [n][H] */
static void gdn_layer(const go_model *m, const go_layer *L, int gi, go_state *s, int n, const float *h, float *mix) {
    const go_config *c = &m->cfg;
    const int H = c->hidden, nk = c->gdn_k_heads, nv = c->gdn_v_heads, dk = c->gdn_k_dim, dv = c->gdn_v_dim,
              K = c->conv_kernel;
    const int kd = nk * dk, vd = nv * dv, conv_dim = 2 * kd + vd;
    float *proj = (float *)malloc(sizeof(float) * (size_t)n * conv_dim);
    float *z = (float *)malloc(sizeof(float) * (size_t)n * vd);
    float *a = (float *)malloc(sizeof(float) * (size_t)n * nv);
    float *b = (float *)malloc(sizeof(float) * (size_t)n * nv);
    float *core = (float *)malloc(sizeof(float) * (size_t)n * vd);
    matmul(&L->qkv, n, h, proj);
    matmul(&L->z, n, h, z);
    go_matvec_bf16(L->a, nv, H, n, h, a);
    go_matvec_bf16(L->b, nv, H, n, h, b);
    float *cs = s->conv + (size_t)gi * conv_dim * (K - 1);
    float *state = s->gdn + (size_t)gi * nv * dk * dv;
    const int rep = nv / nk;
    const float qscale = 1.0f / sqrtf((float)dk);
    /* the causal depthwise convolution over [state | input], then silu_fast (3555-3583) */
    for (int t = 0; t < n; ++t) {
        float *row = proj + (size_t)t * conv_dim;
        for (int ch = 0; ch < conv_dim; ++ch) {
            const float *w = L->conv + (size_t)ch * K;
            float *st = cs + (size_t)ch * (K - 1);
            const float in = row[ch];
            float acc = 0.0f;
            for (int k = 0; k < K - 1; ++k) acc += w[k] * st[k];
            acc += w[K - 1] * in;
            for (int k = 0; k + 1 < K - 1; ++k) st[k] = st[k + 1];
            if (K > 1) st[K - 2] = in;
            row[ch] = acc;
        }
        for (int ch = 0; ch < conv_dim; ++ch) row[ch] = silu_fast(row[ch]);
    }
    /* q, k L2-normalised per key head, q times 1/sqrt(dk) (3585-3602) */
    for (int t = 0; t < n; ++t)
        for (int kh = 0; kh < nk; ++kh) {
            float *mixed = proj + (size_t)t * conv_dim;
            float *q = mixed + kh * dk, *k = mixed + kd + kh * dk;
            float sq = 0.0f, sk = 0.0f;
            for (int j = 0; j < dk; ++j) {
                sq += q[j] * q[j];
                sk += k[j] * k[j];
            }
            const float iq = 1.0f / sqrtf(sq + 1e-6f), ik = 1.0f / sqrtf(sk + 1e-6f);
            for (int j = 0; j < dk; ++j) {
                q[j] = q[j] * iq * qscale;
                k[j] = k[j] * ik;
            }
        }
    /* beta and the decay (3604-3611) */
    for (int t = 0; t < n; ++t)
        for (int vh = 0; vh < nv; ++vh) {
            float *bb = b + (size_t)t * nv, *aa = a + (size_t)t * nv;
            bb[vh] = sigmoidf_(bb[vh]);
            aa[vh] = expf(-expf(L->A_log[vh]) * softplusf_(aa[vh] + L->dt_bias[vh]));
        }
    /* the gated delta rule in 16-column strips (3644-3666; the state [nv][dv/16][dk][16]) */
    const int strips = dv / 16;
    for (int vh = 0; vh < nv; ++vh)
        for (int st = 0; st < strips; ++st) {
            const int j0 = st * 16, kh = vh / rep;
            float *S = state + (size_t)vh * dk * dv + (size_t)j0 * dk;
            for (int t = 0; t < n; ++t) {
                const float *mixed = proj + (size_t)t * conv_dim;
                delta_strip(S, dk, 16, 16, mixed + kh * dk, mixed + kd + kh * dk, mixed + 2 * kd + vh * dv + j0,
                            a[(size_t)t * nv + vh], b[(size_t)t * nv + vh], core + (size_t)t * vd + (size_t)vh * dv + j0);
            }
        }
    /* gated RMSNorm o / rms(o) * w * silu_fast(z) (3670-3682) */
    for (int t = 0; t < n; ++t)
        for (int vh = 0; vh < nv; ++vh) {
            float *o = core + (size_t)t * vd + (size_t)vh * dv;
            float ss = 0.0f;
            for (int j = 0; j < dv; ++j) ss += o[j] * o[j];
            const float inv = 1.0f / sqrtf(ss / (float)dv + c->eps);
            const float *zz = z + (size_t)t * vd + vh * dv;
            for (int j = 0; j < dv; ++j) o[j] = o[j] * inv * L->gnorm[j] * silu_fast(zz[j]);
        }
    matmul(&L->out, n, core, mix);
    free(proj);
    free(z);
    free(a);
    free(b);
    free(core);
}

/* quant_kv_row (engine/src/model.cpp:3767-3774): amax/127, nearbyint (round half even), clamp +-127 */
static void quant_kv_row(const float *x, int n, int8_t *q, float *scale) {
    float amax = 0.0f;
    for (int i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    for (int i = 0; i < n; ++i) {
        float v = nearbyintf(x[i] * inv);
        if (v < -127.0f) v = -127.0f;
        if (v > 127.0f) v = 127.0f;
        q[i] = (int8_t)v;
    }
    *scale = amax / 127.0f;
}

/* Model::attention + attend<int8_t> + attend_heads (engine/src/model.cpp:3690-3743, 3778-3856, 3899-4019) */
static void attn_layer(const go_model *m, const go_layer *L, int ai, go_state *s, int n, const float *h, float *mix) {
    const go_config *c = &m->cfg;
    const int nh = c->n_heads, nkv = c->n_kv_heads, hd = c->head_dim, half = c->rope_dim / 2;
    const int kv_row = nkv * hd, qw = nh * 2 * hd;
    float *qs = (float *)malloc(sizeof(float) * (size_t)n * qw);
    float *ks = (float *)malloc(sizeof(float) * (size_t)n * kv_row);
    float *vs = (float *)malloc(sizeof(float) * (size_t)n * kv_row);
    float *core = (float *)malloc(sizeof(float) * (size_t)n * nh * hd);
    matmul(&L->q, n, h, qs);
    matmul(&L->k, n, h, ks);
    matmul(&L->v, n, h, vs);
    float *inv_freq = (float *)malloc(sizeof(float) * (size_t)(half > 0 ? half : 1));
    float *cosv = (float *)malloc(sizeof(float) * (size_t)(half > 0 ? half : 1));
    float *sinv = (float *)malloc(sizeof(float) * (size_t)(half > 0 ? half : 1));
    /* engine/src/model.cpp:737-740 */
    for (int i = 0; i < half; ++i) inv_freq[i] = 1.0f / powf(c->rope_theta, (float)(2 * i) / (float)c->rope_dim);
    for (int t = 0; t < n; ++t) {
        const int p = s->pos + t; /* text: the three M-RoPE streams are one position (rope_pos, 1746-1759) */
        for (int i = 0; i < half; ++i) {
            const float f = (float)p * inv_freq[i];
            cosv[i] = cosf(f);
            sinv[i] = sinf(f);
        }
        for (int hh = 0; hh < nh + nkv; ++hh) {
            float *x = hh < nh ? qs + (size_t)t * qw + (size_t)hh * 2 * hd : ks + (size_t)t * kv_row + (size_t)(hh - nh) * hd;
            go_rmsnorm(x, hh < nh ? L->q_norm : L->k_norm, x, hd, c->eps, 1);
            for (int i = 0; i < half; ++i) {
                const float x1 = x[i], x2 = x[i + half];
                x[i] = x1 * cosv[i] - x2 * sinv[i];
                x[i + half] = x2 * cosv[i] + x1 * sinv[i];
            }
        }
    }
    /* the batch's K and V rows stored (3782-3797) */
    int8_t *kbase = s->kv + (size_t)ai * 2 * s->ctx * kv_row;
    int8_t *vbase = kbase + (size_t)s->ctx * kv_row;
    float *ksbase = s->kvs + (size_t)ai * 2 * s->ctx * nkv;
    float *vsbase = ksbase + (size_t)s->ctx * nkv;
    for (int t = 0; t < n; ++t) {
        const int p = s->pos + t;
        for (int kh = 0; kh < nkv; ++kh) {
            quant_kv_row(ks + (size_t)t * kv_row + kh * hd, hd, kbase + (size_t)p * kv_row + kh * hd, &ksbase[(size_t)p * nkv + kh]);
            quant_kv_row(vs + (size_t)t * kv_row + kh * hd, hd, vbase + (size_t)p * kv_row + kh * hd, &vsbase[(size_t)p * nkv + kh]);
        }
    }
    const int group = nh / nkv, blk = c->attn_block;
    const float scale = 1.0f / sqrtf((float)hd);
    const int maxp = s->pos + n;
    float *sc = (float *)malloc(sizeof(float) * (size_t)(blk < maxp ? blk : maxp));
    const int nbmax = (maxp + blk - 1) / blk;
    float *parts = (float *)malloc(sizeof(float) * (size_t)nbmax * (hd + 2));
    for (int t = 0; t < n; ++t) {
        const int P = s->pos + t, nbt = P / blk + 1;
        for (int h0 = 0; h0 < nh; ++h0) {
            const int kh = h0 / group;
            const float *q = qs + (size_t)t * qw + (size_t)h0 * 2 * hd;
            for (int b = 0; b < nbt; ++b) {
                const int p0 = b * blk, p1 = P + 1 < p0 + blk ? P + 1 : p0 + blk, np = p1 - p0;
                float mx = -INFINITY;
                for (int pp = 0; pp < np; ++pp) {
                    const int8_t *k = kbase + (size_t)(p0 + pp) * kv_row + kh * hd;
                    float acc[8] = {0};
                    for (int i = 0; i < hd; i += 8)
                        for (int j = 0; j < 8; ++j) acc[j] += q[i + j] * (float)k[i + j];
                    const float dot = ((acc[0] + acc[4]) + (acc[1] + acc[5])) + ((acc[2] + acc[6]) + (acc[3] + acc[7]));
                    const float f = scale * ksbase[(size_t)(p0 + pp) * nkv + kh];
                    const float sv = dot * f;
                    sc[pp] = sv;
                    mx = fmaxf(mx, sv);
                }
                float sum = 0.0f;
                for (int pp = 0; pp < np; ++pp) {
                    sc[pp] = expf(sc[pp] - mx);
                    sum += sc[pp];
                }
                for (int pp = 0; pp < np; ++pp) sc[pp] *= vsbase[(size_t)(p0 + pp) * nkv + kh];
                float *dst = parts + (size_t)b * (hd + 2);
                dst[hd] = mx;
                dst[hd + 1] = sum;
                for (int i = 0; i < hd; i += 8) {
                    float acc[8] = {0};
                    for (int pp = 0; pp < np; ++pp) {
                        const int8_t *v = vbase + (size_t)(p0 + pp) * kv_row + kh * hd + i;
                        const float w = sc[pp];
                        for (int j = 0; j < 8; ++j) acc[j] += w * (float)v[j];
                    }
                    memcpy(dst + i, acc, sizeof acc);
                }
            }
            /* the blocks joined in order, softmax's division, the gate (3832-3853) */
            float *o = core + (size_t)t * nh * hd + (size_t)h0 * hd;
            const float *gate = qs + (size_t)t * qw + (size_t)h0 * 2 * hd + hd;
            float sum = parts[hd + 1];
            if (nbt == 1) {
                memcpy(o, parts, sizeof(float) * (size_t)hd);
            } else {
                float mx = -INFINITY;
                for (int b = 0; b < nbt; ++b) mx = fmaxf(mx, parts[(size_t)b * (hd + 2) + hd]);
                for (int j = 0; j < hd; ++j) o[j] = 0.0f;
                sum = 0.0f;
                for (int b = 0; b < nbt; ++b) {
                    const float *pq = parts + (size_t)b * (hd + 2);
                    const float f = expf(pq[hd] - mx);
                    sum += pq[hd + 1] * f;
                    for (int j = 0; j < hd; ++j) o[j] += pq[j] * f;
                }
            }
            const float inv = 1.0f / sum;
            for (int j = 0; j < hd; ++j) o[j] = o[j] * inv * sigmoidf_(gate[j]);
        }
    }
    matmul(&L->o, n, core, mix);
    free(sc);
    free(parts);
    free(inv_freq);
    free(cosv);
    free(sinv);
    free(qs);
    free(ks);
    free(vs);
    free(core);
}

/* Model::moe's int8 path (engine/src/model.cpp:4123-4585); the dense MLP (4128-4151). h [n][H] -> out [n][H] */
static void mlp_layer(const go_model *m, const go_layer *L, int l, int n, const float *h, float *out, const go_trace *tr) {
    const go_config *c = &m->cfg;
    const int H = c->hidden, E = c->n_experts, K = c->top_k, ff = c->moe_ff, sff = c->shared_ff;
    float *sg = (float *)malloc(sizeof(float) * (size_t)n * sff);
    float *su = (float *)malloc(sizeof(float) * (size_t)n * sff);
    float *sh = (float *)malloc(sizeof(float) * (size_t)n * H);
    matmul(&L->sh_gate, n, h, sg);
    matmul(&L->sh_up, n, h, su);
    for (size_t i = 0; i < (size_t)n * sff; ++i) sg[i] = silu(sg[i]) * su[i];
    if (c->dense) {
        matmul(&L->sh_down, n, sg, out);
        free(sg);
        free(su);
        free(sh);
        return;
    }
    matmul(&L->sh_down, n, sg, sh);
    float *lg = (float *)malloc(sizeof(float) * (size_t)n * E);
    go_matvec_bf16(L->router, E, H, n, h, lg);
    int *ids = (int *)malloc(sizeof(int) * (size_t)n * K);
    float *w = (float *)malloc(sizeof(float) * (size_t)n * K);
    for (int t = 0; t < n; ++t) go_route_topk(lg + (size_t)t * E, E, K, ids + (size_t)t * K, w + (size_t)t * K);
    /* each pick: gate_up on the token's quantized h, silu(gate) * up, quantized again, down (4496-4543) */
    float *y = (float *)malloc(sizeof(float) * (size_t)n * K * H);
    float *gu = (float *)malloc(sizeof(float) * 2 * (size_t)ff);
    const size_t gu_bytes = (size_t)(2 * ff) * q4_row_bytes(H);
    for (int t = 0; t < n; ++t)
        for (int k = 0; k < K; ++k) {
            const int e = ids[(size_t)t * K + k];
            const uint8_t *blk = L->experts + (size_t)e * L->expert_stride;
            go_q4 gw = {blk, 2 * ff, H, L->expert_scales[2 * e]};
            go_q4 dw = {blk + gu_bytes, H, ff, L->expert_scales[2 * e + 1]};
            matmul(&gw, 1, h + (size_t)t * H, gu);
            for (int i = 0; i < ff; ++i) gu[i] = silu(gu[i]) * gu[ff + i];
            matmul(&dw, 1, gu, y + ((size_t)t * K + k) * H);
        }
    /* per token: sigmoid(shared gate . h) * shared + the routed outputs in rank order (4554-4585) */
    for (int t = 0; t < n; ++t) {
        const float *ht = h + (size_t)t * H;
        float gs = 0.0f;
        for (int i = 0; i < H; ++i) gs += bf16f(L->shared_gate[i]) * ht[i];
        gs = sigmoidf_(gs);
        float *o = out + (size_t)t * H;
        for (int i = 0; i < H; ++i) o[i] = gs * sh[(size_t)t * H + i];
        for (int k = 0; k < K; ++k) {
            const float wk = w[(size_t)t * K + k];
            if (wk == 0.0f) continue;
            const float *yy = y + ((size_t)t * K + k) * H;
            for (int i = 0; i < H; ++i) o[i] += wk * yy[i];
        }
        if (tr && tr->ids) {
            memcpy(tr->ids + ((size_t)l * n + t) * K, ids + (size_t)t * K, sizeof(int) * (size_t)K);
            memcpy(tr->weights + ((size_t)l * n + t) * K, w + (size_t)t * K, sizeof(float) * (size_t)K);
            tr->gate[(size_t)l * n + t] = gs;
        }
    }
    free(sg);
    free(su);
    free(sh);
    free(lg);
    free(ids);
    free(w);
    free(y);
    free(gu);
}

/* One routed pick of Model::moe (engine/src/model.cpp:4496-4543) by itself: the expert block (gate_up [2 ff][H] q4
 * rows, then down [H][ff]) on one token's h: gate_up on the quantized h, silu(gate) * up, quantized again, down. */
void go_expert_pair(const uint8_t *blk, float g_gu, float g_dn, int H, int ff, const float *h, float *y) {
    float *gu = (float *)malloc(sizeof(float) * 2 * (size_t)ff);
    go_q4 gw = {blk, 2 * ff, H, g_gu};
    go_q4 dw = {blk + (size_t)(2 * ff) * q4_row_bytes(H), H, ff, g_dn};
    matmul(&gw, 1, h, gu);
    for (int i = 0; i < ff; ++i) gu[i] = silu(gu[i]) * gu[ff + i];
    matmul(&dw, 1, gu, y);
    free(gu);
}

/* Model::forward_batch (engine/src/model.cpp:5235-5413) without images, for the verify pass */
int go_forward(const go_model *m, go_state *s, const int *toks, int n, float *logits, float *hidden, const go_trace *tr) {
    const go_config *c = &m->cfg;
    const int H = c->hidden;
    if (n <= 0 || s->pos + n > s->ctx) return -1;
    float *x = (float *)malloc(sizeof(float) * (size_t)n * H);
    float *h = (float *)malloc(sizeof(float) * (size_t)n * H);
    float *mix = (float *)malloc(sizeof(float) * (size_t)n * H);
    float *moe = (float *)malloc(sizeof(float) * (size_t)n * H);
    for (int t = 0; t < n; ++t) {
        if (toks[t] < 0 || toks[t] >= m->embed.rows) {
            free(x), free(h), free(mix), free(moe);
            return -1;
        }
        go_dequant_row(&m->embed, toks[t], x + (size_t)t * H);
    }
    int gi = 0, ai = 0;
    for (int l = 0; l < c->n_layers; ++l) {
        const go_layer *L = &m->layers[l];
        if (tr && tr->x) memcpy(tr->x + (size_t)l * n * H, x, sizeof(float) * (size_t)n * H);
        for (int t = 0; t < n; ++t) go_rmsnorm(x + (size_t)t * H, L->in_norm, h + (size_t)t * H, H, c->eps, 1);
        if (L->attn) attn_layer(m, L, ai++, s, n, h, mix);
        else gdn_layer(m, L, gi++, s, n, h, mix);
        for (int t = 0; t < n; ++t) {
            float *xr = x + (size_t)t * H;
            for (int i = 0; i < H; ++i) xr[i] += mix[(size_t)t * H + i];
            go_rmsnorm(xr, L->post_norm, h + (size_t)t * H, H, c->eps, 1);
        }
        mlp_layer(m, L, l, n, h, moe, tr);
        for (size_t i = 0; i < (size_t)n * H; ++i) x[i] += moe[i];
        if (tr && tr->mixer) {
            memcpy(tr->mixer + (size_t)l * n * H, mix, sizeof(float) * (size_t)n * H);
            memcpy(tr->moe + (size_t)l * n * H, moe, sizeof(float) * (size_t)n * H);
            memcpy(tr->out + (size_t)l * n * H, x, sizeof(float) * (size_t)n * H);
        }
    }
    for (int t = 0; t < n; ++t) go_rmsnorm(x + (size_t)t * H, m->final_norm, h + (size_t)t * H, H, c->eps, 1);
    if (hidden) memcpy(hidden, h, sizeof(float) * (size_t)n * H);
    if (logits) matmul(&m->lm_head, n, h, logits);
    s->pos += n;
    free(x);
    free(h);
    free(mix);
    free(moe);
    return 0;
}

/* Model::forward_mtp (engine/src/model.cpp:4965-5039) on the CPU path: the fc input per position, the layer's
 * attention over its own KV slot (the main layers' attention, at positions pos..), its MLP (expert layer n_layers),
 * the logits of the last position after mtp.norm */
int go_forward_mtp(const go_model *m, const go_mtp *mtp, int8_t *kv, float *kvs, int ctx, const int *next,
                   const float *hidden, int n, int pos, float *logits, float *out_hidden) {
    const go_config *c = &m->cfg;
    const int H = c->hidden;
    if (n <= 0 || pos < 0 || pos + n > ctx || !mtp || !kv || !kvs) return -1;
    for (int t = 0; t < n; ++t)
        if (next[t] < 0 || next[t] >= m->embed.rows) return -1;
    float *in = (float *)malloc(sizeof(float) * (size_t)n * 2 * H);
    float *e = (float *)malloc(sizeof(float) * (size_t)H);
    float *x = (float *)malloc(sizeof(float) * (size_t)n * H);
    float *h = (float *)malloc(sizeof(float) * (size_t)n * H);
    float *mix = (float *)malloc(sizeof(float) * (size_t)n * H);
    float *moe = (float *)malloc(sizeof(float) * (size_t)n * H);
    /* [norm_e(embedding) | norm_h(hidden)] per position, then fc (5008-5024) */
    for (int t = 0; t < n; ++t) {
        float *row = in + (size_t)t * 2 * H;
        go_dequant_row(&m->embed, next[t], e);
        go_rmsnorm(e, mtp->pre_e, row, H, c->eps, 1);
        go_rmsnorm(hidden + (size_t)t * H, mtp->pre_h, row + H, H, c->eps, 1);
    }
    matmul(&mtp->fc, n, in, x);
    const go_layer *L = &mtp->layer;
    for (int t = 0; t < n; ++t) go_rmsnorm(x + (size_t)t * H, L->in_norm, h + (size_t)t * H, H, c->eps, 1);
    /* the attention at the MTP layer's positions pos.. over its own KV (apos_ = pos, 5029-5032) */
    go_state v = {pos, ctx, NULL, NULL, kv, kvs};
    attn_layer(m, L, 0, &v, n, h, mix);
    for (int t = 0; t < n; ++t) {
        float *xr = x + (size_t)t * H;
        for (int i = 0; i < H; ++i) xr[i] += mix[(size_t)t * H + i];
        go_rmsnorm(xr, L->post_norm, h + (size_t)t * H, H, c->eps, 1);
    }
    mlp_layer(m, L, c->n_layers, n, h, moe, NULL);
    for (size_t i = 0; i < (size_t)n * H; ++i) x[i] += moe[i];
    if (logits || out_hidden) {
        go_rmsnorm(x + (size_t)(n - 1) * H, mtp->norm, h, H, c->eps, 1);
        if (out_hidden) memcpy(out_hidden, h, sizeof(float) * (size_t)H);
        if (logits) matmul(&m->lm_head, 1, h, logits);
    }
    free(in);
    free(e);
    free(x);
    free(h);
    free(mix);
    free(moe);
    return 0;
}

/* ---------------------------------------------------------------- sampling ---- */

/* MT19937-64 (Matsumoto & Nishimura 2000; the std::mt19937_64 of the C++ standard, [rand.predef]) */
void go_mt64_seed(go_mt64 *g, uint64_t seed) {
    g->mt[0] = seed;
    for (int i = 1; i < 312; ++i) g->mt[i] = 6364136223846793005ULL * (g->mt[i - 1] ^ (g->mt[i - 1] >> 62)) + (uint64_t)i;
    g->mti = 312;
}

uint64_t go_mt64_next(go_mt64 *g) {
    static const uint64_t mag[2] = {0ULL, 0xB5026F5AA96619E9ULL};
    const uint64_t UM = 0xFFFFFFFF80000000ULL, LM = 0x7FFFFFFFULL;
    if (g->mti >= 312) {
        int i;
        for (i = 0; i < 312 - 156; ++i) {
            const uint64_t x = (g->mt[i] & UM) | (g->mt[i + 1] & LM);
            g->mt[i] = g->mt[i + 156] ^ (x >> 1) ^ mag[(int)(x & 1ULL)];
        }
        for (; i < 311; ++i) {
            const uint64_t x = (g->mt[i] & UM) | (g->mt[i + 1] & LM);
            g->mt[i] = g->mt[i + (156 - 312)] ^ (x >> 1) ^ mag[(int)(x & 1ULL)];
        }
        const uint64_t x = (g->mt[311] & UM) | (g->mt[0] & LM);
        g->mt[311] = g->mt[155] ^ (x >> 1) ^ mag[(int)(x & 1ULL)];
        g->mti = 0;
    }
    uint64_t x = g->mt[g->mti++];
    x ^= (x >> 29) & 0x5555555555555555ULL;
    x ^= (x << 17) & 0x71D67FFFEDA60000ULL;
    x ^= (x << 37) & 0xFFF7EEE000000000ULL;
    x ^= (x >> 43);
    return x;
}

/* generate_canonical<double, 53> over a 64-bit engine as libstdc++ computes it (one draw: x / 2^64, a result
 * of 1 pulled down below 1) */
double go_canonical(go_mt64 *g) {
    const double r = 18446744073709551616.0; /* 2^64 */
    double ret = (double)go_mt64_next(g) / r;
    if (ret >= 1.0) ret = nextafter(1.0, 0.0);
    return ret;
}

typedef struct {
    float v;
    int i;
} cand_t;

static int cand_cmp(const void *a, const void *b) {
    const cand_t *x = (const cand_t *)a, *y = (const cand_t *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return x->i - y->i; /* equal logits: the lower token first (the reference's partial_sort: unspecified) */
}

/* engine/src/sampler.cpp:16-50 with the uniform given: greedy = the first maximum; else the top k (1024 when off)
 * by logit, exp((l - max) / T) in float summed in double, the top-p prefix, r = u * kept, the first with r <= 0 */
int go_sample(const float *logits, int n, float temperature, float top_p, int top_k, double u) {
    if (temperature <= 0.0f) {
        int best = 0;
        for (int i = 1; i < n; ++i)
            if (logits[i] > logits[best]) best = i;
        return best;
    }
    int k = top_k > 0 ? top_k : 1024;
    if (k > n) k = n;
    cand_t *c = (cand_t *)malloc(sizeof(cand_t) * (size_t)n);
    for (int i = 0; i < n; ++i) c[i] = (cand_t){logits[i], i};
    qsort(c, (size_t)n, sizeof(cand_t), cand_cmp);
    const float mx = c[0].v;
    double sum = 0.0;
    for (int i = 0; i < k; ++i) {
        c[i].v = expf((c[i].v - mx) / temperature);
        sum += c[i].v;
    }
    int keep = k;
    if (top_p < 1.0f) {
        double acc = 0.0;
        for (int i = 0; i < k; ++i) {
            acc += c[i].v / sum;
            if (acc >= top_p) {
                keep = i + 1;
                break;
            }
        }
    }
    double kept = 0.0;
    for (int i = 0; i < keep; ++i) kept += c[i].v;
    double r = u * (kept - 0.0) + 0.0;
    int out = c[keep - 1].i;
    for (int i = 0; i < keep; ++i) {
        r -= c[i].v;
        if (r <= 0.0) {
            out = c[i].i;
            break;
        }
    }
    free(c);
    return out;
}

/* engine/src/geode.cpp:327-350: rows sampled in order (one draw per sampled row when not greedy); draft i+1 stands
 * while row i's sample is that draft and no stop token. Each row goes through geode_generate's sample()
 * (engine/src/geode.cpp:246-255): with a presence penalty, the penalty is first subtracted from the row's logit of
 * every token in seen (in/out: the answer's tokens so far, each once, in the order first sampled; room for n more),
 * and the sample joins seen when it is new (only while the penalty is on, as the engine's is_seen). The rows are not
 * modified (each is sampled from a copy). */
int go_accept_seen(const float *rows, int n, int V, const int *batch, float temperature, float top_p, int top_k,
                   uint64_t seed, const int *stops, int n_stops, float penalty, int *seen, int *n_seen, int *next,
                   int *samples) {
    go_mt64 g;
    go_mt64_seed(&g, seed);
    for (int i = 0; i < n; ++i) samples[i] = -1;
    int kept = 1;
    *next = -1;
    const int on = penalty != 0.0f;
    float *row = on ? (float *)malloc(sizeof(float) * (size_t)V) : NULL;
    unsigned char *is_seen = on ? (unsigned char *)calloc((size_t)V, 1) : NULL;
    if (on && (!row || !is_seen)) {
        free(row);
        free(is_seen);
        return -1;
    }
    if (on)
        for (int j = 0; j < *n_seen; ++j)
            if (seen[j] >= 0 && seen[j] < V) is_seen[seen[j]] = 1;
    for (int i = 0; i < n; ++i) {
        const float *lg = rows + (size_t)i * V;
        if (on) {
            memcpy(row, lg, sizeof(float) * (size_t)V);
            for (int j = 0; j < *n_seen; ++j) row[seen[j]] -= penalty;
            lg = row;
        }
        const double u = temperature > 0.0f ? go_canonical(&g) : 0.0;
        const int y = go_sample(lg, V, temperature, top_p, top_k, u);
        samples[i] = y;
        if (on && y >= 0 && y < V && !is_seen[y]) {
            is_seen[y] = 1;
            seen[(*n_seen)++] = y;
        }
        int stop = 0;
        for (int s = 0; s < n_stops; ++s) stop |= stops[s] == y;
        if (i + 1 < n && y == batch[i + 1] && !stop) {
            ++kept;
            continue;
        }
        *next = y;
        break;
    }
    free(row);
    free(is_seen);
    return kept;
}

int go_accept(const float *rows, int n, int V, const int *batch, float temperature, float top_p, int top_k,
              uint64_t seed, const int *stops, int n_stops, int *next, int *samples) {
    int none = 0;
    return go_accept_seen(rows, n, V, batch, temperature, top_p, top_k, seed, stops, n_stops, 0.0f, NULL, &none, next,
                          samples);
}

/* ---------------------------------------------------------------- rejection sampling (not in the reference) ---- */

/* Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3", SC 2011) */
void go_philox4x32(uint64_t key, uint64_t counter_hi, uint64_t counter_lo, uint32_t out[4]) {
    uint32_t c0 = (uint32_t)counter_lo, c1 = (uint32_t)(counter_lo >> 32), c2 = (uint32_t)counter_hi,
             c3 = (uint32_t)(counter_hi >> 32);
    uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0, n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c1 = (uint32_t)p1;
        c3 = (uint32_t)p0;
        c0 = n0;
        c2 = n2;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0, out[1] = c1, out[2] = c2, out[3] = c3;
}

/* a double in [0, 1) from two 32-bit words (53 bits) */
static double u53(uint32_t a, uint32_t b) {
    return (double)(((uint64_t)a << 21) ^ ((uint64_t)b >> 11)) * (1.0 / 9007199254740992.0);
}

/* the filtered distribution of one row: top-k (1024 when off) by logit, weights fast_exp((l - max) * (1/T)),
 * the top-p prefix; returns the kept count, ids/probs (probs = weight / sum of kept, in double) in logit order */
static int filtered(const float *logits, int V, float temperature, float top_p, int top_k, int *ids, double *probs) {
    int k = top_k > 0 ? top_k : 1024;
    if (k > V) k = V;
    cand_t *c = (cand_t *)malloc(sizeof(cand_t) * (size_t)V);
    for (int i = 0; i < V; ++i) c[i] = (cand_t){logits[i], i};
    qsort(c, (size_t)V, sizeof(cand_t), cand_cmp);
    const float mx = c[0].v, it = 1.0f / temperature;
    double sum = 0.0;
    double *w = (double *)malloc(sizeof(double) * (size_t)k);
    for (int i = 0; i < k; ++i) {
        w[i] = (double)go_fast_exp((c[i].v - mx) * it);
        sum += w[i];
    }
    int keep = k;
    if (top_p < 1.0f) {
        double acc = 0.0;
        for (int i = 0; i < k; ++i) {
            acc += w[i] / sum;
            if (acc >= top_p) {
                keep = i + 1;
                break;
            }
        }
    }
    double kept = 0.0;
    for (int i = 0; i < keep; ++i) kept += w[i];
    for (int i = 0; i < keep; ++i) {
        ids[i] = c[i].i;
        probs[i] = w[i] / kept;
    }
    free(w);
    free(c);
    return keep;
}

static double prob_of(const int *ids, const double *p, int n, int tok) {
    for (int i = 0; i < n; ++i)
        if (ids[i] == tok) return p[i];
    return 0.0;
}

/* Speculative sampling (Leviathan et al. 2023, Algorithm 1; Chen et al. 2023): draft i accepted when
 * u_i * q(d_i) < p(d_i) (u_i < min(1, p/q)); the first rejection resamples from norm(max(0, p - q)); all accepted:
 * a bonus token from the last target row. Uniforms: Philox4x32-10, key = seed, counter = (seq, row): word 0-1 the
 * acceptance draw, 2-3 the resample draw. Resampling walks the support in ascending token id. */
int go_spec_reject(const float *target, const float *draft, int n_drafts, int V, const int *drafts,
                   float temperature, float top_p, int top_k, uint64_t seed, uint64_t seq, int *next) {
    const int cap = 1024 < V ? 1024 : V;
    int *pid = (int *)malloc(sizeof(int) * (size_t)cap), *qid = (int *)malloc(sizeof(int) * (size_t)cap);
    double *pp = (double *)malloc(sizeof(double) * (size_t)cap), *qp = (double *)malloc(sizeof(double) * (size_t)cap);
    int accepted = 0;
    *next = -1;
    for (int i = 0; i <= n_drafts; ++i) {
        uint32_t r[4];
        go_philox4x32(seed, seq, (uint64_t)i, r);
        const double ua = u53(r[0], r[1]), ur = u53(r[2], r[3]);
        const int np = filtered(target + (size_t)i * V, V, temperature, top_p, top_k, pid, pp);
        if (i == n_drafts) { /* every draft accepted: the bonus token from the target row */
            /* ascending token id walk over the target's support */
            int best = -1;
            double acc = 0.0, total = 0.0;
            for (int j = 0; j < np; ++j) total += pp[j];
            const double lim = ur * total;
            for (int tok = 0, left = np; left > 0 && tok < V; ++tok) {
                const double pv = prob_of(pid, pp, np, tok);
                if (pv <= 0.0) continue;
                --left;
                acc += pv;
                best = tok;
                if (acc > lim) break;
            }
            *next = best;
            break;
        }
        const int nq = filtered(draft + (size_t)i * V, V, temperature, top_p, top_k, qid, qp);
        const int d = drafts[i];
        const double pd = prob_of(pid, pp, np, d), qd = prob_of(qid, qp, nq, d);
        if (qd > 0.0 && ua * qd < pd) {
            ++accepted;
            continue;
        }
        /* the residual max(0, p - q) over p's support (q > p elsewhere gives 0) */
        double total = 0.0;
        for (int j = 0; j < np; ++j) {
            const double rv = pp[j] - prob_of(qid, qp, nq, pid[j]);
            if (rv > 0.0) total += rv;
        }
        int best = -1;
        if (total > 0.0) {
            const double lim = ur * total;
            double acc = 0.0;
            for (int tok = 0; tok < V; ++tok) {
                const double pv = prob_of(pid, pp, np, tok);
                if (pv <= 0.0) continue;
                const double rv = pv - prob_of(qid, qp, nq, tok);
                if (rv <= 0.0) continue;
                acc += rv;
                best = tok;
                if (acc > lim) break;
            }
        } else { /* p == q on the support: sample from p */
            const double lim = ur;
            double acc = 0.0;
            for (int tok = 0; tok < V; ++tok) {
                const double pv = prob_of(pid, pp, np, tok);
                if (pv <= 0.0) continue;
                acc += pv;
                best = tok;
                if (acc > lim) break;
            }
        }
        *next = best;
        break;
    }
    free(pid);
    free(qid);
    free(pp);
    free(qp);
    return accepted;
}

/* ------------------------------------------------------------------ the exp premise (test infrastructure) ---- */

/* The kernels stand in (float)exp((double)x) for the reference's float exp (std::exp on a float calls glibc's
 * expf): in route_topk's softmax (engine/src/model.cpp:4021-4065), the Sampler's weights (engine/src/sampler.cpp:
 * 16-50), the Gated DeltaNet's decay and the SwiGLU / sigmoid gates. These count, over float bit patterns, where that
 * stand-in differs from glibc's expf - computed here on the host (go_expf_mismatch) or read from a table the device
 * computed (go_expf_check_table). Two NaNs count as equal; every other pair is compared bit for bit. The first `cap`
 * differing patterns go to first[]. */
/* glibc's expf restated (the ARM optimized-routines expf by Szabolcs Nagy, in glibc since 2.27; the multiply-adds
 * fused as in glibc's FMA build): x * 32/ln2 = k + r, 2^(k/32) from a table of 2^(i/32) (the double nearest each,
 * its exponent field less i << 47), 2^(r/32) by a cubic in double, one rounding to float. The kernels' expf_ref is
 * the same sequence. */
static const uint64_t go_exp2_table[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

float go_expf_restated(float x) {
    uint32_t ux;
    memcpy(&ux, &x, 4);
    const uint32_t top = (ux >> 20) & 0x7ffu;
    if (top >= 0x42bu) {
        if (ux == 0xff800000u) return 0.0f;
        if (top >= 0x7f8u) return x + x;
        if (x > 0x1.62e42ep6f) return INFINITY;
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double inv_ln2_32 = 0x1.71547652b82fep+0 * 32.0, shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0, c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0,
                 c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double xd = (double)x;
    double kd = fma(inv_ln2_32, xd, shift);
    uint64_t ki;
    memcpy(&ki, &kd, 8);
    kd -= shift;
    const double r = fma(inv_ln2_32, xd, -kd);
    const uint64_t t = go_exp2_table[ki & 31u] + (ki << 47);
    double s;
    memcpy(&s, &t, 8);
    const double z = fma(c0, r, c1);
    const double y = fma(z, r * r, fma(c2, r, 1.0));
    return (float)(y * s);
}

typedef struct {
    uint64_t lo, hi;
    const float *vals;   /* NULL: computed here (restated: go_expf_restated, else (float)exp((double)x)) */
    int restated;
    uint64_t count;
    uint32_t first[16];
    int nfirst;
} expf_job;

static void *expf_run(void *p) {
    expf_job *j = (expf_job *)p;
    for (uint64_t b = j->lo; b < j->hi; ++b) {
        const uint32_t bits = (uint32_t)b;
        float x;
        memcpy(&x, &bits, 4);
        const float want = expf(x);
        const float got = j->vals ? j->vals[b - j->lo] : j->restated ? go_expf_restated(x) : (float)exp((double)x);
        uint32_t wb, gb;
        memcpy(&wb, &want, 4);
        memcpy(&gb, &got, 4);
        if (wb != gb && !(want != want && got != got)) {
            if (j->nfirst < 16) j->first[j->nfirst++] = bits;
            ++j->count;
        }
    }
    return NULL;
}

static uint64_t expf_sweep(uint64_t lo, uint64_t n, const float *vals, int restated, int threads, uint32_t *first,
                           int cap) {
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    expf_job jobs[64];
    pthread_t th[64];
    int started[64];
    for (int t = 0; t < threads; ++t) {
        jobs[t].lo = lo + n * (uint64_t)t / (uint64_t)threads;
        jobs[t].hi = lo + n * (uint64_t)(t + 1) / (uint64_t)threads;
        jobs[t].vals = vals ? vals + (jobs[t].lo - lo) : NULL;
        jobs[t].restated = restated;
        jobs[t].count = 0;
        jobs[t].nfirst = 0;
        started[t] = pthread_create(&th[t], NULL, expf_run, &jobs[t]) == 0;
        if (!started[t]) expf_run(&jobs[t]);
    }
    uint64_t total = 0;
    int k = 0;
    for (int t = 0; t < threads; ++t) {
        if (started[t]) pthread_join(th[t], NULL);
        total += jobs[t].count;
        for (int i = 0; i < jobs[t].nfirst && k < cap; ++i) first[k++] = jobs[t].first[i];
    }
    return total;
}

uint64_t go_expf_mismatch(uint64_t lo, uint64_t hi, int restated, int threads, uint32_t *first, int cap) {
    return hi > lo ? expf_sweep(lo, hi - lo, NULL, restated, threads, first, cap) : 0;
}

uint64_t go_expf_check_table(uint64_t lo, uint64_t n, const float *vals, int threads, uint32_t *first, int cap) {
    return expf_sweep(lo, n, vals, 0, threads, first, cap);
}
