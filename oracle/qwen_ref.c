/* ORACLE — test infrastructure only (tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py). The product never links it.
 *
 * A plain-C restatement of the reference's behavioural model
 *   legacy_100mhz_closed/src/PC/model_backend.py:14-115
 * with the rounding variants of
 *   legacy_100mhz_closed/src/software/interactive/tests/rtl_numeric_reference.py:6-32
 * and the per-token-per-head KV8 rule (amax/127 fp32 scale, round-half-even
 * codes clamped to +-127) used by the B200 engine's KV cache.
 *
 * Fixed evaluation order (so that results do not depend on thread count):
 *   linear:  per output, fp32 sum over k in increasing order (every product
 *            bf16 x int8 is exact in fp32, so FMA or not gives the same sum)
 *   scores:  per (row, head, key), fmaf over d in increasing order
 *   softmax: max, e = expf(s - max), Z = sequential sum, P = bf16(e * (1/Z))
 *   context: per (row, head, d), fmaf over keys in increasing order
 * REF_EXACT replaces every order-dependent fp32 sum by an exact integer sum
 * on a grid fixed by the data (projections, the RMSNorm sum of squares, the
 * softmax sum and, with REF_KV8, the KV8 context) and expf by ref_qexp, a
 * fixed sequence of IEEE fp32 operations, so that any implementation doing
 * the same integer sums and the same fp32 operations matches bit for bit.
 * Build with -ffp-contract=off (oracle/Makefile).
 */
#include "qwen_ref.h"

#include "assets.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define NL 24
#define HID 896
#define FFN 4864
#define VOC 151936
#define QH 14
#define KVH 2
#define HD 64
#define QKV 1152

/* Projection table: out, in, SCALE.BIN offset, DESC.BIN byte offset
 * (model_backend.py:29-32). */
static const unsigned P_OUT[7] = {896, 128, 128, 896, 4864, 4864, 896};
static const unsigned P_IN[7] = {896, 896, 896, 896, 896, 896, 4864};
static const unsigned P_SCALE[7] = {0, 896, 1024, 1152, 2048, 6912, 11776};
static const unsigned P_FIELD[7] = {40, 48, 56, 80, 96, 104, 120};
enum { PQ, PK, PV, PO, PG, PU, PD };

struct ref_model {
    int8_t *w[NL][7];  /* logical [out][in] */
    int8_t *wt[NL][7]; /* transposed [in][out] */
    int8_t *lm, *lmt;
    float *scale, *bias, *gamma;
    uint16_t *embed;
    unsigned mode, capacity, position;
    float *rope; /* [capacity][64] */
    float *kf[NL], *vf[NL];         /* bf16 KV: [cap][2][64] */
    int8_t *kc[NL], *vc[NL];        /* KV8: [2][cap][64] */
    float *ks[NL], *vs[NL];         /* KV8: [2][cap] */
    /* KV8 caches of nslots sequences: kc/vc [slot][2][cap][64], ks/vs
     * [slot][2][cap]; slot 0 is the sequence of the single-sequence calls,
     * whose position is `position`; spos[s] holds the others' */
    unsigned nslots, *spos;
    /* REF_RTL_KV (allocated when the mode is set): the low K16 plane klo
     * [slot][2][cap][64] beside kc (the high plane), the K block locks
     * klock [slot][2][cap/256 rounded up] and the V layer locks vlock [slot][2] */
    int8_t *klo[NL];
    uint8_t *klock[NL], *vlock[NL];
    int dump_layer;
    float *dq, *dk, *dv, *dctx, *dh, *dm, *dy;
};

/* ---------------------------------------------------------------- rounding */
static inline uint32_t f2u(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    return u;
}
static inline float u2f(uint32_t u) {
    float x;
    memcpy(&x, &u, 4);
    return x;
}
/* torch .to(bfloat16): round to nearest even (model_backend.py:45). */
static inline float bf_rne(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return u2f(0x7fc00000u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return u2f(u & 0xffff0000u);
}
/* rtl_numeric_reference.py:6-12: half away from zero, FTZ, canonical NaN. */
static inline float bf_rnd8(float x) {
    uint32_t b = f2u(x);
    uint32_t upper = ((b >> 16) + ((b >> 15) & 1u)) & 0xffffu;
    uint32_t e = (b >> 23) & 0xffu;
    if (e == 0) upper = (b >> 16) & 0x8000u;
    if (e == 255 && (b & 0x7fffffu)) upper = 0x7fc0u;
    return u2f(upper << 16);
}
float ref_bf(float x, unsigned mode) { return (mode & REF_RND8) ? bf_rnd8(x) : bf_rne(x); }
static inline float bfm(float x, unsigned mode) { return (mode & REF_RND8) ? bf_rnd8(x) : bf_rne(x); }
static inline float bf2f(uint16_t b) { return u2f((uint32_t)b << 16); }

void ref_set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

/* ------------------------------------------------------------------- loader */
static void *slurp(const char *root, const char *name, size_t expect, char *err, size_t errlen) {
    char path[4096];
    snprintf(path, sizeof(path), "%s/QWEN25/%s", root, name);
    FILE *f = fopen(path, "rb");
    if (!f) {
        snprintf(err, errlen, "cannot open %s", path);
        return NULL;
    }
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    rewind(f);
    void *p = NULL;
    if (expect == 0 || (long)expect == n) {
        p = malloc((size_t)n + 1);
        if (p && fread(p, 1, (size_t)n, f) != (size_t)n) {
            free(p);
            p = NULL;
        }
        if (p) ((char *)p)[n] = 0;
    } else {
        snprintf(err, errlen, "wrong size %s", path);
    }
    fclose(f);
    return p;
}

/* model_backend.py:51-55: physical [C/128][I/128][4][128][2][16] -> logical [C][I]. */
static void unpack_tiles(const int8_t *raw, unsigned columns, unsigned inner, int8_t *out) {
#pragma omp parallel for schedule(static)
    for (long c = 0; c < (long)columns; ++c) {
        unsigned cb = (unsigned)c / 128, ci = (unsigned)c % 128, a = ci / 64, b = (ci % 64) / 16, d = ci % 16;
        for (unsigned i = 0; i < inner; ++i) {
            unsigned ib = i / 128, e = i % 128;
            size_t off = (((((size_t)cb * (inner / 128) + ib) * 4 + b) * 128 + e) * 2 + a) * 16 + d;
            out[(size_t)c * inner + i] = raw[off];
        }
    }
}

static int8_t *transpose_i8(const int8_t *w, unsigned out, unsigned in) {
    int8_t *t = (int8_t *)malloc((size_t)out * in);
    if (!t) return NULL;
#pragma omp parallel for schedule(static)
    for (long i = 0; i < (long)in; ++i)
        for (unsigned o = 0; o < out; ++o) t[(size_t)i * out + o] = w[(size_t)o * in + i];
    return t;
}

static float *bf16_file(const char *root, const char *name, size_t count, char *err, size_t errlen) {
    uint16_t *raw = (uint16_t *)slurp(root, name, count * 2, err, errlen);
    if (!raw) return NULL;
    float *f = (float *)malloc(count * sizeof(float));
    for (size_t i = 0; f && i < count; ++i) f[i] = bf2f(raw[i]);
    free(raw);
    return f;
}

void ref_rope_table(unsigned positions, float *table) {
    /* model_backend.py:41: 1 / 1e6^(2i/64) in fp32; phase = pos * inv (fp32). */
    float inv[32];
    for (int i = 0; i < 32; ++i) inv[i] = 1.0f / (float)pow(1000000.0, (double)(2 * i) / 64.0);
    for (unsigned p = 0; p < positions; ++p)
        for (int i = 0; i < 32; ++i) {
            float phase = (float)p * inv[i];
            table[(size_t)p * 64 + i] = (float)cos((double)phase);
            table[(size_t)p * 64 + 32 + i] = (float)sin((double)phase);
        }
}

ref_model *ref_open(const char *root, unsigned capacity, char *err, size_t errlen) {
    ref_model *m = (ref_model *)calloc(1, sizeof(ref_model));
    if (!m) return NULL;
    m->capacity = capacity ? capacity : 256;
    m->dump_layer = -1;
    m->nslots = 1;
    m->spos = (unsigned *)calloc(1, sizeof(unsigned));
    char *cfg = (char *)slurp(root, "CONFIG.JSON", 0, err, errlen);
    if (!cfg) goto fail;
    /* model_backend.py:19 asserts hidden/layers/vocab. */
    if (!strstr(cfg, "\"hidden\": 896") || !strstr(cfg, "\"layers\": 24") || !strstr(cfg, "\"vocab\": 151936")) {
        snprintf(err, errlen, "CONFIG.JSON is not Qwen2.5-0.5B (hidden 896, 24 layers, vocab 151936)");
        free(cfg);
        goto fail;
    }
    free(cfg);
    m->scale = bf16_file(root, "SCALE.BIN", 304128 + VOC, err, errlen);
    m->bias = bf16_file(root, "BIAS.BIN", NL * QKV, err, errlen);
    m->gamma = bf16_file(root, "GAMMA.BIN", NL * 1792 + HID, err, errlen);
    m->embed = (uint16_t *)slurp(root, "EMBED.BIN", (size_t)VOC * HID * 2, err, errlen);
    if (!m->scale || !m->bias || !m->gamma || !m->embed) goto fail;
    {
        uint8_t *desc = (uint8_t *)slurp(root, "DESC.BIN", 0, err, errlen);
        int8_t *packed = (int8_t *)slurp(root, "WEIGHTS.BIN", 0, err, errlen);
        if (!desc || !packed) {
            free(desc);
            free(packed);
            goto fail;
        }
        size_t packed_size = (size_t)24 * 14909440ULL;
        for (int l = 0; l < NL; ++l)
            for (int p = 0; p < 7; ++p) {
                uint64_t address;
                memcpy(&address, desc + l * 256 + P_FIELD[p], 8);
                uint64_t off = address - 0x41000000ULL;
                size_t bytes = (size_t)P_OUT[p] * P_IN[p];
                if (address < 0x41000000ULL || off + bytes > packed_size) {
                    snprintf(err, errlen, "descriptor %d/%u outside WEIGHTS.BIN", l, P_FIELD[p]);
                    free(desc);
                    free(packed);
                    goto fail;
                }
                m->w[l][p] = (int8_t *)malloc(bytes);
                unpack_tiles(packed + off, P_OUT[p], P_IN[p], m->w[l][p]);
                m->wt[l][p] = transpose_i8(m->w[l][p], P_OUT[p], P_IN[p]);
            }
        free(desc);
        free(packed);
        int8_t *lm = (int8_t *)slurp(root, "LMW.BIN", (size_t)VOC * HID, err, errlen);
        if (!lm) goto fail;
        m->lm = (int8_t *)malloc((size_t)VOC * HID);
        unpack_tiles(lm, VOC, HID, m->lm);
        free(lm);
        m->lmt = transpose_i8(m->lm, VOC, HID);
    }
    m->rope = (float *)malloc((size_t)m->capacity * 64 * sizeof(float));
    ref_rope_table(m->capacity, m->rope);
    for (int l = 0; l < NL; ++l) {
        m->kf[l] = (float *)calloc((size_t)m->capacity * KVH * HD, sizeof(float));
        m->vf[l] = (float *)calloc((size_t)m->capacity * KVH * HD, sizeof(float));
        m->kc[l] = (int8_t *)calloc((size_t)m->capacity * KVH * HD, 1);
        m->vc[l] = (int8_t *)calloc((size_t)m->capacity * KVH * HD, 1);
        m->ks[l] = (float *)calloc((size_t)m->capacity * KVH, sizeof(float));
        m->vs[l] = (float *)calloc((size_t)m->capacity * KVH, sizeof(float));
    }
    return m;
fail:
    ref_close(m);
    return NULL;
}

void ref_close(ref_model *m) {
    if (!m) return;
    for (int l = 0; l < NL; ++l) {
        for (int p = 0; p < 7; ++p) {
            free(m->w[l][p]);
            free(m->wt[l][p]);
        }
        free(m->kf[l]);
        free(m->vf[l]);
        free(m->kc[l]);
        free(m->vc[l]);
        free(m->ks[l]);
        free(m->vs[l]);
        free(m->klo[l]);
        free(m->klock[l]);
        free(m->vlock[l]);
    }
    free(m->lm);
    free(m->lmt);
    free(m->scale);
    free(m->bias);
    free(m->gamma);
    free(m->embed);
    free(m->rope);
    free(m->spos);
    free(m);
}

static unsigned rtl_blocks(const ref_model *m) { return (m->capacity + 255) / 256; }
/* (Re)allocates the RTL-format arrays for the current slots, zeroed. */
static int rtl_alloc(ref_model *m) {
    for (int l = 0; l < NL; ++l) {
        free(m->klo[l]);
        free(m->klock[l]);
        free(m->vlock[l]);
        m->klo[l] = (int8_t *)calloc((size_t)m->nslots * m->capacity * KVH * HD, 1);
        m->klock[l] = (uint8_t *)calloc((size_t)m->nslots * KVH * rtl_blocks(m), 1);
        m->vlock[l] = (uint8_t *)calloc((size_t)m->nslots * KVH, 1);
        if (!m->klo[l] || !m->klock[l] || !m->vlock[l]) return -1;
    }
    return 0;
}
void ref_set_mode(ref_model *m, unsigned mode) {
    if ((mode & REF_RTL_KV) && !m->klo[0] && rtl_alloc(m)) mode &= ~REF_RTL_KV;
    m->mode = mode;
}
void ref_clear(ref_model *m) { m->position = 0; } /* model_backend.py:57-60 */
unsigned ref_position(const ref_model *m) { return m->position; }
const int8_t *ref_weight(const ref_model *m, int layer, int proj) { return m->w[layer][proj]; }
const float *ref_scale(const ref_model *m) { return m->scale; }
const float *ref_bias(const ref_model *m) { return m->bias; }
const float *ref_gamma(const ref_model *m) { return m->gamma; }
const int8_t *ref_lm_weight(const ref_model *m) { return m->lm; }
const uint16_t *ref_embedding(const ref_model *m) { return m->embed; }

void ref_set_dump(ref_model *m, int layer, float *q, float *k, float *v, float *ctx, float *h, float *mid,
                  float *y) {
    m->dump_layer = layer;
    m->dq = q;
    m->dk = k;
    m->dv = v;
    m->dctx = ctx;
    m->dh = h;
    m->dm = mid;
    m->dy = y;
}

/* -------------------------------------------------------------- operators */
static float eps_of(unsigned mode) {
    return (mode & REF_CSR_EPS) ? u2f(0x35860000u) : 1e-6f; /* rtl_numeric_reference.py:18 */
}

/* exp(x) in fp32 by Cody-Waite range reduction and a degree-7 Taylor
 * polynomial (W. J. Cody, W. Waite, Software Manual for the Elementary
 * Functions, 1980): n = rint(x * log2 e), r = x - n*ln2 with ln2 split into a
 * 15-bit head and a tail (two fmas), exp(x) = 2^n * sum_{k<=7} r^k/k! by
 * Horner's rule in fmas, 2^n applied as two exact power-of-two factors. Every
 * step is one IEEE fp32 operation, so a device version written with the same
 * operations returns the same bits. |r| <= 0.347, truncation r^8/8! < 2^-27;
 * within 1 ulp of exp over the range the model uses (tests/test_exact_mode.py). */
static inline float pow2f(int n) { return u2f((uint32_t)(n + 127) << 23); } /* -126 <= n <= 127 */
float ref_qexp(float x) {
    if (!(x >= -104.0f)) return 0.0f; /* exp(-104) is below half the smallest subnormal; NaN -> 0 */
    if (x > 88.75f) return INFINITY;
    const float n = rintf(x * 1.44269504f);
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.42860677e-6f, r);
    float p = 1.98412698e-4f;
    p = fmaf(p, r, 1.38888889e-3f);
    p = fmaf(p, r, 8.33333333e-3f);
    p = fmaf(p, r, 4.16666667e-2f);
    p = fmaf(p, r, 1.66666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int)n, n1 = ni < -126 ? -126 : (ni > 127 ? 127 : ni);
    return (p * pow2f(n1)) * pow2f(ni - n1);
}
static inline float exp_m(float x, unsigned mode) { return (mode & REF_EXACT) ? ref_qexp(x) : expf(x); }

/* Exponent of the largest magnitude of v[0..n) (0 when all are zero). */
static int max_exponent(const float *v, unsigned n) {
    float amax = 0.0f;
    for (unsigned i = 0; i < n; ++i)
        if (fabsf(v[i]) > amax) amax = fabsf(v[i]);
    return amax > 0.0f ? ilogbf(amax) : 0;
}

/* model_backend.py:69-71. REF_EXACT: the sum of squares is exact on the grid
 * of the row's 21-bit alignment: X = rint(x * 2^(20-E)) (|X| < 2^21),
 * ss = RN32(sum X^2) * 2^(2E-40) (the integer sum is below 2^52). */
void ref_rmsnorm(const float *x, unsigned rows, const float *gamma, float eps, unsigned mode, float *out) {
    for (unsigned r = 0; r < rows; ++r) {
        const float *xr = x + (size_t)r * HID;
        float ss = 0.0f;
        if (mode & REF_EXACT) {
            const int e = max_exponent(xr, HID);
            int64_t s2 = 0;
            for (unsigned i = 0; i < HID; ++i) {
                const int64_t xi = (int64_t)rintf(ldexpf(xr[i], 20 - e));
                s2 += xi * xi;
            }
            ss = ldexpf((float)s2, 2 * e - 40);
        } else {
            for (unsigned i = 0; i < HID; ++i) ss += xr[i] * xr[i];
        }
        float mean = ss / (float)HID;
        float rs = 1.0f / sqrtf(mean + eps);
        for (unsigned i = 0; i < HID; ++i) out[(size_t)r * HID + i] = bfm(bfm(xr[i] * rs, mode) * gamma[i], mode);
    }
}

static void accum_t(const float *x, unsigned rows, unsigned K, const int8_t *wt, unsigned N, float *acc) {
    const unsigned NB = 256, RB = 16;
    long nblocks = (N + NB - 1) / NB;
#pragma omp parallel for schedule(static)
    for (long nb = 0; nb < nblocks; ++nb) {
        unsigned n0 = (unsigned)nb * NB, nn = N - n0 < NB ? N - n0 : NB;
        float wf[256];
        float a[16][256];
        for (unsigned r0 = 0; r0 < rows; r0 += RB) {
            unsigned rb = rows - r0 < RB ? rows - r0 : RB;
            for (unsigned r = 0; r < rb; ++r)
                for (unsigned j = 0; j < nn; ++j) a[r][j] = 0.0f;
            for (unsigned k = 0; k < K; ++k) {
                const int8_t *wr = wt + (size_t)k * N + n0;
                for (unsigned j = 0; j < nn; ++j) wf[j] = (float)wr[j];
                for (unsigned r = 0; r < rb; ++r) {
                    float xk = x[(size_t)(r0 + r) * K + k];
                    for (unsigned j = 0; j < nn; ++j) a[r][j] += xk * wf[j];
                }
            }
            for (unsigned r = 0; r < rb; ++r)
                memcpy(acc + (size_t)(r0 + r) * N + n0, a[r], nn * sizeof(float));
        }
    }
}

/* Projection sums in the accelerator's order (REF_EXACT). The RTL GEMM array
 * multiplies block-aligned activation mantissas by the int8 codes and sums
 * them as integers (src/rtl/qwen_gemm_array_i.sv header: INT24 segment sums
 * with a block exponent). Restated with one 28-bit alignment per activation
 * row: E = exponent of max|x[r][:]| (max in [2^E, 2^E+1)),
 * X[k] = rint(x[r][k] * 2^(26-E)) (|X| < 2^27), the dot product with the
 * codes is exact (int64), and acc = RN32(dot) * 2^(E-26). Exact integer sums
 * make the result independent of summation order and of how K is split. */
static int align_row(const float *xr, unsigned K, int32_t *X) {
    float amax = 0.0f;
    for (unsigned k = 0; k < K; ++k)
        if (fabsf(xr[k]) > amax) amax = fabsf(xr[k]);
    const int e = amax > 0.0f ? ilogbf(amax) : 0;
    for (unsigned k = 0; k < K; ++k) X[k] = (int32_t)rintf(ldexpf(xr[k], 26 - e));
    return e;
}
static void accum_exact(const float *x, unsigned rows, unsigned K, const int8_t *w, int transposed, unsigned N,
                        float *acc) {
    for (unsigned r = 0; r < rows; ++r) {
        int32_t *X = (int32_t *)malloc(K * sizeof(int32_t));
        const int e = align_row(x + (size_t)r * K, K, X);
#pragma omp parallel for schedule(static)
        for (long n = 0; n < (long)N; ++n) {
            int64_t s = 0;
            if (transposed)
                for (unsigned k = 0; k < K; ++k) s += (int64_t)X[k] * w[(size_t)k * N + n];
            else
                for (unsigned k = 0; k < K; ++k) s += (int64_t)X[k] * w[(size_t)n * K + k];
            acc[(size_t)r * N + n] = ldexpf((float)s, e - 26);
        }
        free(X);
    }
}

/* Same sums from a row-major weight w[n][k] (operator-level entry). */
static void accum_rowmajor(const float *x, unsigned rows, unsigned K, const int8_t *w, unsigned N, float *acc) {
#pragma omp parallel for schedule(static)
    for (long n = 0; n < (long)N; ++n)
        for (unsigned r = 0; r < rows; ++r) {
            float s = 0.0f;
            const int8_t *wr = w + (size_t)n * K;
            const float *xr = x + (size_t)r * K;
            for (unsigned k = 0; k < K; ++k) s += xr[k] * (float)wr[k];
            acc[(size_t)r * N + n] = s;
        }
}

/* model_backend.py:62-64: bf16(bf16(x W^T) * scale). */
static void epi_linear(float *acc, unsigned rows, unsigned N, const float *scale, unsigned mode) {
    for (size_t i = 0; i < (size_t)rows * N; ++i) acc[i] = bfm(bfm(acc[i], mode) * scale[i % N], mode);
}
/* model_backend.py:66-67 (two roundings) or rtl_numeric_reference.py:27-32 (one). */
static void epi_bias(float *acc, unsigned rows, unsigned N, const float *scale, const float *bias, unsigned mode) {
    for (size_t i = 0; i < (size_t)rows * N; ++i) {
        unsigned n = (unsigned)(i % N);
        if (mode & REF_FUSED_BIAS)
            acc[i] = bfm(bfm(acc[i], mode) * scale[n] + bias[n], mode);
        else
            acc[i] = bfm(bfm(bfm(acc[i], mode) * scale[n], mode) + bias[n], mode);
    }
}

/* Raw sums of a projection from the transposed weight wt[k][n]. */
static void accum(const float *x, unsigned rows, unsigned K, const int8_t *wt, unsigned N, float *acc, unsigned mode) {
    if (mode & REF_EXACT)
        accum_exact(x, rows, K, wt, 1, N, acc);
    else
        accum_t(x, rows, K, wt, N, acc);
}

void ref_linear(const float *x, unsigned rows, unsigned k, const int8_t *w, const float *scale, unsigned n,
                unsigned mode, float *out) {
    if (mode & REF_EXACT)
        accum_exact(x, rows, k, w, 0, n, out);
    else
        accum_rowmajor(x, rows, k, w, n, out);
    epi_linear(out, rows, n, scale, mode);
}

void ref_linear_bias(const float *x, unsigned rows, unsigned k, const int8_t *w, const float *scale,
                     const float *bias, unsigned n, unsigned mode, float *out) {
    if (mode & REF_EXACT)
        accum_exact(x, rows, k, w, 0, n, out);
    else
        accum_rowmajor(x, rows, k, w, n, out);
    epi_bias(out, rows, n, scale, bias, mode);
}

/* model_backend.py:73-78 with the fp32 cos/sin table. */
static void rope_rows(float *x, unsigned rows, unsigned heads, const uint32_t *positions, const float *table,
                      unsigned mode, float *out) {
    for (unsigned r = 0; r < rows; ++r) {
        const float *cs = table + (size_t)positions[r] * 64;
        for (unsigned h = 0; h < heads; ++h) {
            const float *xi = x + ((size_t)r * heads + h) * HD;
            float *yo = out + ((size_t)r * heads + h) * HD;
            float tmp[HD];
            for (int i = 0; i < HD; ++i) {
                float c = cs[i & 31], s = cs[32 + (i & 31)];
                float rot = i < 32 ? -xi[i + 32] : xi[i - 32];
                float a = xi[i] * c;
                float b = rot * s;
                tmp[i] = bfm(a + b, mode);
            }
            memcpy(yo, tmp, sizeof(tmp));
        }
    }
}

void ref_rope(const float *x, unsigned rows, unsigned heads, const uint32_t *positions, unsigned mode, float *out) {
    unsigned maxp = 0;
    for (unsigned r = 0; r < rows; ++r)
        if (positions[r] > maxp) maxp = positions[r];
    float *table = (float *)malloc((size_t)(maxp + 1) * 64 * sizeof(float));
    ref_rope_table(maxp + 1, table);
    float *tmp = (float *)malloc((size_t)rows * heads * HD * sizeof(float));
    memcpy(tmp, x, (size_t)rows * heads * HD * sizeof(float));
    rope_rows(tmp, rows, heads, positions, table, mode, out);
    free(tmp);
    free(table);
}

/* KV8 rule per (token, kv head): s = amax/127 (fp32), code = clamp(rne(x/s), +-127);
 * an all-zero vector gets s = 0 and zero codes. */
void ref_kv8_quant(const float *x, unsigned rows, int8_t *codes, float *scales) {
    for (unsigned r = 0; r < rows; ++r) {
        const float *xr = x + (size_t)r * HD;
        float amax = 0.0f;
        for (int d = 0; d < HD; ++d) {
            float a = fabsf(xr[d]);
            if (a > amax) amax = a;
        }
        float s = amax / 127.0f;
        scales[r] = s;
        for (int d = 0; d < HD; ++d) {
            float q = s > 0.0f ? nearbyintf(xr[d] / s) : 0.0f;
            if (q > 127.0f) q = 127.0f;
            if (q < -127.0f) q = -127.0f;
            codes[(size_t)r * HD + d] = (int8_t)q;
        }
    }
}

/* model_backend.py:97-102 for one (row, head) once the scores are known:
 * P = bf(softmax(S)) over keys 0..visible-1 (causal mask), ctx = bf(P.v); val
 * reads the (dequantised) cache through its view. */
typedef float (*kv_at)(const void *view, unsigned t, unsigned d);

/* Softmax of scratch[0..visible) in place: E = exp(S - max). REF_EXACT: E by
 * ref_qexp and the sum exact on the 2^-40 grid, Z = RN32(sum rint(E * 2^40))
 * * 2^-40 (E <= 1, so the integer sum stays below 2^56); else expf and a
 * sequential fp32 sum. Returns 1/Z. */
static float softmax_exp(float *scratch, unsigned visible, unsigned mode) {
    float mx = -INFINITY;
    for (unsigned t = 0; t < visible; ++t)
        if (scratch[t] > mx) mx = scratch[t];
    float z = 0.0f;
    if (mode & REF_EXACT) {
        int64_t zi = 0;
        for (unsigned t = 0; t < visible; ++t) {
            scratch[t] = ref_qexp(scratch[t] - mx);
            zi += (int64_t)llrintf(ldexpf(scratch[t], 40));
        }
        z = ldexpf((float)zi, -40);
    } else {
        for (unsigned t = 0; t < visible; ++t) {
            scratch[t] = expf(scratch[t] - mx);
            z += scratch[t];
        }
    }
    return 1.0f / z;
}

static void attend_finish(float *scratch, unsigned visible, kv_at val, const void *vview, unsigned mode, float *out) {
    const float inv = softmax_exp(scratch, visible, mode);
    float acc[HD];
    for (unsigned d = 0; d < HD; ++d) acc[d] = 0.0f;
    for (unsigned t = 0; t < visible; ++t) {
        float p = bfm(scratch[t] * inv, mode);
        for (unsigned d = 0; d < HD; ++d) acc[d] = fmaf(p, val(vview, t, d), acc[d]);
    }
    for (unsigned d = 0; d < HD; ++d) out[d] = bfm(acc[d], mode);
}

/* KV8 context in the accelerator's order (REF_KV8 | REF_EXACT). The array
 * folds the per-token V scale into the probability before the reduction over
 * tokens (src/rtl/kv8_v_pscale.sv:1-20, p'[t] = p[t] * m[t]) and sums p'
 * against the int8 codes as block-aligned integers. Restated with one 28-bit
 * alignment per (row, head):
 *   P[t] = bf16(E[t] / Z),  w[t] = RN32(P[t] * vscale[t])
 *   E_h  = exponent of RN32(bf16(1/Z) * max_t vscale[t]), a bound of every
 *          w[t] (E[t] <= 1 and rounding is monotone), known before any w[t]
 *   W[t] = rint(w[t] * 2^(26-E_h)) (|W| < 2^27)
 *   ctx[d] = bf16(RN32(sum_t W[t] * code[t][d]) * 2^(E_h-26))
 * with the sum exact in int64 (below 2^49 for 32768 keys). */
static void attend_finish_kv8_exact(float *scratch, unsigned visible, const int8_t *vcodes, const float *vscales,
                                    unsigned mode, float *out) {
    const float inv = softmax_exp(scratch, visible, mode);
    float vmax = 0.0f;
    for (unsigned t = 0; t < visible; ++t)
        if (vscales[t] > vmax) vmax = vscales[t];
    const float bound = bfm(inv, mode) * vmax;
    const int e = bound > 0.0f ? ilogbf(bound) : 0;
    int64_t acc[HD];
    for (unsigned d = 0; d < HD; ++d) acc[d] = 0;
    for (unsigned t = 0; t < visible; ++t) {
        const float w = bfm(scratch[t] * inv, mode) * vscales[t];
        const int64_t wi = (int64_t)rintf(ldexpf(w, 26 - e));
        for (unsigned d = 0; d < HD; ++d) acc[d] += wi * vcodes[(size_t)t * HD + d];
    }
    for (unsigned d = 0; d < HD; ++d) out[d] = bfm(ldexpf((float)acc[d], e - 26), mode);
}

/* model_backend.py:97 with a cache read through a view: S = bf(q.k/8), the
 * dot product an fp32 fma chain over d ascending. */
static void attend(const float *q, unsigned visible, kv_at key, const void *kview, kv_at val, const void *vview,
                   unsigned mode, float *out) {
    float *scratch = (float *)malloc(visible * sizeof(float));
    for (unsigned t = 0; t < visible; ++t) {
        float acc = 0.0f;
        for (unsigned d = 0; d < HD; ++d) acc = fmaf(q[d], key(kview, t, d), acc);
        scratch[t] = bfm(acc / 8.0f, mode);
    }
    attend_finish(scratch, visible, val, vview, mode, out);
    free(scratch);
}

/* KV8 scores in the accelerator's order: the array sums q against the int8
 * codes in block-aligned integers (src/rtl/kv8_v_pscale.sv:40-44, INT24
 * accumulator normalised to the block maximum) and the per-token K scale
 * multiplies the finished sum (src/rtl/kv8_score_scale8.sv:6-12). Restated
 * with 28-bit alignment: E = the exponent of max|q| (max|q| in [2^E, 2^E+1)),
 * Q[d] = rint(q[d] * 2^(26-E)) (|Q| < 2^27), dot = sum_d Q[d] * code[t][d]
 * exactly (int64), and
 *   S[t] = bf16(RN32(RN32(dot) * 2^(E-26) * kscale[t]) / 8).
 * Exact integer sums make the result independent of summation order. */
/* With klo (REF_RTL_KV) the K code of dim d is the 16-bit 256 * kcodes[d] +
 * klo[d] of the accelerator's two planes, the same formula otherwise. */
static void kv_scores(const float *q, unsigned visible, const int8_t *kcodes, const int8_t *klo, const float *kscales,
                      unsigned mode, float *scores) {
    float amax = 0.0f;
    for (unsigned d = 0; d < HD; ++d)
        if (fabsf(q[d]) > amax) amax = fabsf(q[d]);
    const int e = amax > 0.0f ? ilogbf(amax) : 0;
    int32_t qi[HD];
    for (unsigned d = 0; d < HD; ++d) qi[d] = (int32_t)rintf(ldexpf(q[d], 26 - e));
    for (unsigned t = 0; t < visible; ++t) {
        int64_t acc = 0;
        if (klo)
            for (unsigned d = 0; d < HD; ++d)
                acc += (int64_t)qi[d] * (256 * (int32_t)kcodes[(size_t)t * HD + d] + klo[(size_t)t * HD + d]);
        else
            for (unsigned d = 0; d < HD; ++d) acc += (int64_t)qi[d] * kcodes[(size_t)t * HD + d];
        const float dot = ldexpf((float)acc, e - 26);
        scores[t] = bfm(dot * kscales[t] / 8.0f, mode);
    }
}
void ref_kv8_scores(const float *q, unsigned visible, const int8_t *kcodes, const float *kscales, unsigned mode,
                    float *scores) {
    kv_scores(q, visible, kcodes, NULL, kscales, mode, scores);
}

/* KV8 view: codes [t][64], scales [t]; dequantised value = code * scale (fp32). */
typedef struct kv8_view { const int8_t *codes; const float *scales; } kv8_view;
static float kv8_at(const void *c, unsigned t, unsigned d) {
    const kv8_view *v = (const kv8_view *)c;
    return (float)v->codes[(size_t)t * HD + d] * v->scales[t];
}
/* bf16 view: data [t][2][64], pre-offset to one KV head. */
typedef struct bf_view { const float *data; } bf_view;
static float bf_at(const void *c, unsigned t, unsigned d) {
    const bf_view *v = (const bf_view *)c;
    return v->data[(size_t)t * KVH * HD + d];
}

void ref_attention_kv8(const float *q, unsigned rows, const uint32_t *positions, const int8_t *kcodes,
                       const float *kscales, const int8_t *vcodes, const float *vscales, unsigned capacity,
                       unsigned mode, float *ctx) {
#pragma omp parallel for schedule(dynamic)
    for (long rh = 0; rh < (long)rows * QH; ++rh) {
        unsigned r = (unsigned)rh / QH, h = (unsigned)rh % QH, g = h / 7; /* repeat_interleave(7), :97-98 */
        const unsigned visible = positions[r] + 1;
        kv8_view vv = {vcodes + (size_t)g * capacity * HD, vscales + (size_t)g * capacity};
        float *scratch = (float *)malloc(visible * sizeof(float));
        ref_kv8_scores(q + ((size_t)r * QH + h) * HD, visible, kcodes + (size_t)g * capacity * HD,
                       kscales + (size_t)g * capacity, mode, scratch);
        if (mode & REF_EXACT)
            attend_finish_kv8_exact(scratch, visible, vv.codes, vv.scales, mode,
                                    ctx + (size_t)r * HID + (size_t)h * HD);
        else
            attend_finish(scratch, visible, kv8_at, &vv, mode, ctx + (size_t)r * HID + (size_t)h * HD);
        free(scratch);
    }
}

void ref_attention_bf16(const float *q, unsigned rows, const uint32_t *positions, const float *k, const float *v,
                        unsigned mode, float *ctx) {
#pragma omp parallel for schedule(dynamic)
    for (long rh = 0; rh < (long)rows * QH; ++rh) {
        unsigned r = (unsigned)rh / QH, h = (unsigned)rh % QH, g = h / 7;
        bf_view kv = {k + (size_t)g * HD}, vv = {v + (size_t)g * HD};
        attend(q + ((size_t)r * QH + h) * HD, positions[r] + 1, bf_at, &kv, bf_at, &vv, mode,
               ctx + (size_t)r * HID + (size_t)h * HD);
    }
}

/* model_backend.py:106: bf16(bf16(silu(gate)) * up), silu(g) = g / (1 + exp(-g))
 * (exp by ref_qexp under REF_EXACT). */
void ref_swiglu(const float *gate, const float *up, unsigned count, unsigned mode, float *out) {
    for (unsigned i = 0; i < count; ++i) {
        float g = gate[i];
        float s = g / (1.0f + exp_m(-g, mode));
        out[i] = bfm(bfm(s, mode) * up[i], mode);
    }
}

/* Greedy token, highest index on ties (model_backend.py:113-114). */
static uint32_t argmax_last(const float *v, unsigned n) {
    uint32_t best = 0;
    for (unsigned i = 1; i < n; ++i)
        if (v[i] >= v[best]) best = i;
    return best;
}

static void lm_head_rows(const ref_model *m, const float *x, unsigned n, unsigned mode, uint32_t *tokens,
                         float *logits);
uint32_t ref_lm_head(const ref_model *m, const float *x, unsigned mode, float *logits) {
    uint32_t tok = 0;
    lm_head_rows(m, x, 1, mode, &tok, logits);
    return tok;
}

int ref_kv8_state(const ref_model *m, int layer, int8_t *kcodes, float *kscales, int8_t *vcodes, float *vscales) {
    unsigned n = m->position;
    for (int g = 0; g < KVH; ++g) {
        memcpy(kcodes + (size_t)g * n * HD, m->kc[layer] + (size_t)g * m->capacity * HD, (size_t)n * HD);
        memcpy(vcodes + (size_t)g * n * HD, m->vc[layer] + (size_t)g * m->capacity * HD, (size_t)n * HD);
        memcpy(kscales + (size_t)g * n, m->ks[layer] + (size_t)g * m->capacity, n * sizeof(float));
        memcpy(vscales + (size_t)g * n, m->vs[layer] + (size_t)g * m->capacity, n * sizeof(float));
    }
    return (int)n;
}

/* The engine's seeded KV8 fill (its fill_kv_kernel), restated so both sides
 * hold identical caches: per (layer, K|V, kv head) a key
 * seed * 0x100000001B3 + (4 layer + 2 (V?1:0) + head) * 0x9E3779B9, code of
 * (t, d) = hash(key + 64 t + d) % 255 - 127, scale of t =
 * 0.01 + 0.02 * (hash(~key + t) & 0xffff) / 65536, with the SplitMix64
 * finaliser as the hash (upper 32 bits of its output). */
static uint32_t fill_hash(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return (uint32_t)((x ^ (x >> 31)) >> 16);
}

static size_t slot_codes(const ref_model *m, unsigned slot) { return (size_t)slot * KVH * m->capacity * HD; }
static size_t slot_scales(const ref_model *m, unsigned slot) { return (size_t)slot * KVH * m->capacity; }

static int fill_slot(ref_model *m, unsigned slot, unsigned length, uint64_t seed) {
    if (length > m->capacity || slot >= m->nslots) return -1;
#pragma omp parallel for schedule(static)
    for (int l = 0; l < NL; ++l)
        for (int which = 0; which < 2; ++which)
            for (int g = 0; g < KVH; ++g) {
                const uint64_t key = seed * 0x100000001B3ULL + ((uint64_t)l * 4 + (uint64_t)which * 2 + g) * 0x9E3779B9ULL;
                int8_t *codes = (which ? m->vc[l] : m->kc[l]) + slot_codes(m, slot) + (size_t)g * m->capacity * HD;
                float *scales = (which ? m->vs[l] : m->ks[l]) + slot_scales(m, slot) + (size_t)g * m->capacity;
                for (unsigned t = 0; t < length; ++t) {
                    for (int d = 0; d < HD; ++d)
                        codes[(size_t)t * HD + d] = (int8_t)((int)(fill_hash(key + (uint64_t)t * HD + d) % 255u) - 127);
                    scales[t] = 0.01f + 0.02f * (float)(fill_hash(~key + t) & 0xffff) / 65536.0f;
                }
            }
    if (slot == 0)
        m->position = length;
    else
        m->spos[slot] = length;
    return 0;
}

int ref_fill_kv_synthetic(ref_model *m, unsigned length, uint64_t seed) { return fill_slot(m, 0, length, seed); }
int ref_fill_kv_synthetic_slot(ref_model *m, unsigned slot, unsigned length, uint64_t seed) {
    return fill_slot(m, slot, length, seed);
}

int ref_set_slots(ref_model *m, unsigned nslots) {
    if (!nslots) return -1;
    unsigned *sp = (unsigned *)calloc(nslots, sizeof(unsigned));
    if (!sp) return -1;
    for (int l = 0; l < NL; ++l) {
        free(m->kc[l]);
        free(m->vc[l]);
        free(m->ks[l]);
        free(m->vs[l]);
        m->kc[l] = (int8_t *)calloc((size_t)nslots * m->capacity * KVH * HD, 1);
        m->vc[l] = (int8_t *)calloc((size_t)nslots * m->capacity * KVH * HD, 1);
        m->ks[l] = (float *)calloc((size_t)nslots * m->capacity * KVH, sizeof(float));
        m->vs[l] = (float *)calloc((size_t)nslots * m->capacity * KVH, sizeof(float));
        if (!m->kc[l] || !m->vc[l] || !m->ks[l] || !m->vs[l]) {
            free(sp);
            return -1;
        }
    }
    free(m->spos);
    m->spos = sp;
    m->nslots = nslots;
    m->position = 0;
    if (m->klo[0] && rtl_alloc(m)) return -1;
    return 0;
}

/* ------------------------------------------------------------------ forward */
/* KV8 attention of rows whose sequences sit in different slots. */
static void attention_slots(const ref_model *m, int l, const float *q, unsigned rows, const uint32_t *pos,
                            const uint32_t *slot, unsigned mode, float *ctx) {
#pragma omp parallel for schedule(dynamic)
    for (long rh = 0; rh < (long)rows * QH; ++rh) {
        const unsigned r = (unsigned)rh / QH, h = (unsigned)rh % QH;
        const unsigned g = h / 7, visible = pos[r] + 1; /* repeat_interleave(7), model_backend.py:97-98 */
        const int8_t *kc = m->kc[l] + slot_codes(m, slot[r]) + (size_t)g * m->capacity * HD;
        const int8_t *vc = m->vc[l] + slot_codes(m, slot[r]) + (size_t)g * m->capacity * HD;
        const float *ks = m->ks[l] + slot_scales(m, slot[r]) + (size_t)g * m->capacity;
        const float *vs = m->vs[l] + slot_scales(m, slot[r]) + (size_t)g * m->capacity;
        kv8_view vv = {vc, vs};
        float *scratch = (float *)malloc(visible * sizeof(float));
        float *out = ctx + (size_t)r * HID + (size_t)h * HD;
        const int8_t *klo =
            (mode & REF_RTL_KV) ? m->klo[l] + slot_codes(m, slot[r]) + (size_t)g * m->capacity * HD : NULL;
        kv_scores(q + ((size_t)r * QH + h) * HD, visible, kc, klo, ks, mode, scratch);
        if (mode & REF_EXACT)
            attend_finish_kv8_exact(scratch, visible, vc, vs, mode, out);
        else
            attend_finish(scratch, visible, kv8_at, &vv, mode, out);
        free(scratch);
    }
}

/* Final norm + LM head + greedy argmax of n rows x [n][896] (weights
 * streamed once for all rows; each row's sums are those of a one-row call). */
static void lm_head_rows(const ref_model *m, const float *x, unsigned n, unsigned mode, uint32_t *tokens,
                         float *logits) {
    float *h = (float *)malloc((size_t)n * HID * sizeof(float));
    ref_rmsnorm(x, n, m->gamma + 43008, eps_of(mode), mode, h);
    float *acc = (float *)malloc((size_t)n * VOC * sizeof(float));
    float *pre = (float *)malloc((size_t)VOC * sizeof(float));
    accum(h, n, HID, m->lmt, VOC, acc, mode);
    const float *s = m->scale + 304128;
    for (unsigned r = 0; r < n; ++r) {
        float *a = acc + (size_t)r * VOC;
        for (unsigned j = 0; j < VOC; ++j) {
            pre[j] = bfm(a[j], mode) * s[j];
            a[j] = bfm(pre[j], mode);
        }
        tokens[r] = (mode & REF_ARGMAX_F32) ? argmax_last(pre, VOC) : argmax_last(a, VOC);
        if (logits) memcpy(logits + (size_t)r * VOC, a, (size_t)VOC * sizeof(float));
    }
    free(h);
    free(acc);
    free(pre);
}

/* REF_RTL_KV append of one (token, KV head): the accelerator's K16 and V
 * formats (ref_k16_quant, ref_v8_quant below) into the caches, the K code as
 * its two planes kc (high) / klo (low) with the scale m16 * 2^(lock - 142),
 * V as codes with the scale m8 * 2^(lock - 134). A 256-token block's first
 * token sets its K lock, the token at position 0 the V lock; a later V token
 * of a slot without a V lock is quantised as a first token and sets none. */
static void rtl_append(ref_model *m, int l, unsigned slot, int g, unsigned t, const float *kr, const float *vr) {
    uint16_t kb[HD], vb[HD];
    for (int d = 0; d < HD; ++d) {
        kb[d] = (uint16_t)(f2u(kr[d]) >> 16);
        vb[d] = (uint16_t)(f2u(vr[d]) >> 16);
    }
    const size_t cs = slot_codes(m, slot) + ((size_t)g * m->capacity + t) * HD;
    const size_t ss = slot_scales(m, slot) + (size_t)g * m->capacity + t;
    uint8_t *klk = m->klock[l] + ((size_t)slot * KVH + g) * rtl_blocks(m) + t / 256;
    uint16_t m16;
    uint8_t etab, m8;
    int clip;
    ref_k16_quant(kb, t % 256 == 0, klk, m->kc[l] + cs, m->klo[l] + cs, &m16, &etab, &clip);
    m->ks[l][ss] = ldexpf((float)m16, (int)*klk - 142);
    uint8_t *vlk = m->vlock[l] + (size_t)slot * KVH + g;
    uint8_t lock = *vlk;
    uint16_t vsc;
    const int first = t == 0 || lock == 0;
    ref_v8_quant(vb, first, &lock, m->vc[l] + cs, &m8, &vsc, &clip);
    if (t == 0) *vlk = lock;
    m->vs[l][ss] = ldexpf((float)m8, (int)lock - 134);
}

/* The RTL-format K planes and locks of one layer's first n tokens of a slot:
 * klo [2][n][64], klock [2][cap/256 rounded up], vlock [2]. */
int ref_rtl_kv_state(const ref_model *m, int layer, unsigned slot, unsigned n, int8_t *klo, uint8_t *klock,
                     uint8_t *vlock) {
    if (!m->klo[0] || layer < 0 || layer >= NL || slot >= m->nslots || n > m->capacity) return -1;
    for (int g = 0; g < KVH; ++g) {
        if (klo)
            memcpy(klo + (size_t)g * n * HD, m->klo[layer] + slot_codes(m, slot) + (size_t)g * m->capacity * HD,
                   (size_t)n * HD);
        if (klock)
            memcpy(klock + (size_t)g * rtl_blocks(m), m->klock[layer] + ((size_t)slot * KVH + g) * rtl_blocks(m),
                   rtl_blocks(m));
        if (vlock) vlock[g] = m->vlock[layer][(size_t)slot * KVH + g];
    }
    return 0;
}

/* The forward of model_backend.py:80-115 over `rows` rows, row r being token
 * ids[r] of the sequence in slot slot[r] at position pos[r] (rows of one
 * sequence in increasing positions); the LM head runs on the nlm rows listed
 * in lm_rows. */
static void run_rows(ref_model *m, unsigned rows, const uint32_t *ids, const uint32_t *pos, const uint32_t *slot,
                     unsigned nlm, const uint32_t *lm_rows, uint32_t *tokens, float *logits) {
    const unsigned mode = m->mode;
    const float eps = eps_of(mode);
    float *x = (float *)malloc((size_t)rows * HID * sizeof(float));
    float *h = (float *)malloc((size_t)rows * HID * sizeof(float));
    float *q = (float *)malloc((size_t)rows * HID * sizeof(float));
    float *k = (float *)malloc((size_t)rows * KVH * HD * sizeof(float));
    float *v = (float *)malloc((size_t)rows * KVH * HD * sizeof(float));
    float *ctx = (float *)malloc((size_t)rows * HID * sizeof(float));
    float *gu = (float *)malloc((size_t)rows * FFN * 2 * sizeof(float));
    float *mid = (float *)malloc((size_t)rows * FFN * sizeof(float));
    float *tmp = (float *)malloc((size_t)rows * FFN * sizeof(float));
    for (unsigned r = 0; r < rows; ++r)
        for (unsigned i = 0; i < HID; ++i) x[(size_t)r * HID + i] = bf2f(m->embed[(size_t)ids[r] * HID + i]);
    for (int l = 0; l < NL; ++l) {
        const float *sc = m->scale + (size_t)l * 12672;
        const float *bias = m->bias + (size_t)l * QKV;
        ref_rmsnorm(x, rows, m->gamma + (size_t)l * 1792, eps, mode, h);
        /* q, k, v projections with bias (model_backend.py:91-93) */
        accum(h, rows, HID, m->wt[l][PQ], 896, q, mode);
        epi_bias(q, rows, 896, sc + P_SCALE[PQ], bias, mode);
        accum(h, rows, HID, m->wt[l][PK], 128, k, mode);
        epi_bias(k, rows, 128, sc + P_SCALE[PK], bias + 896, mode);
        accum(h, rows, HID, m->wt[l][PV], 128, v, mode);
        epi_bias(v, rows, 128, sc + P_SCALE[PV], bias + 1024, mode);
        rope_rows(q, rows, QH, pos, m->rope, mode, q);
        rope_rows(k, rows, KVH, pos, m->rope, mode, k);
        /* append to the cache (model_backend.py:95-96) */
        for (unsigned r = 0; r < rows; ++r)
            for (int g = 0; g < KVH; ++g) {
                const float *kr = k + ((size_t)r * KVH + g) * HD, *vr = v + ((size_t)r * KVH + g) * HD;
                const size_t t = pos[r];
                if (slot[r] == 0) {
                    memcpy(m->kf[l] + (t * KVH + g) * HD, kr, HD * sizeof(float));
                    memcpy(m->vf[l] + (t * KVH + g) * HD, vr, HD * sizeof(float));
                }
                const size_t cs = slot_codes(m, slot[r]) + ((size_t)g * m->capacity + t) * HD;
                const size_t ss = slot_scales(m, slot[r]) + (size_t)g * m->capacity + t;
                if (mode & REF_RTL_KV)
                    rtl_append(m, l, slot[r], g, (unsigned)t, kr, vr);
                else {
                    ref_kv8_quant(kr, 1, m->kc[l] + cs, m->ks[l] + ss);
                    ref_kv8_quant(vr, 1, m->vc[l] + cs, m->vs[l] + ss);
                }
            }
        if (mode & REF_KV8) {
            attention_slots(m, l, q, rows, pos, slot, mode, ctx);
        } else {
#pragma omp parallel for schedule(dynamic)
            for (long rh = 0; rh < (long)rows * QH; ++rh) {
                unsigned r = (unsigned)rh / QH, hh = (unsigned)rh % QH, g = hh / 7;
                bf_view kv = {m->kf[l] + (size_t)g * HD}, vv = {m->vf[l] + (size_t)g * HD};
                attend(q + ((size_t)r * QH + hh) * HD, pos[r] + 1, bf_at, &kv, bf_at, &vv, mode,
                       ctx + (size_t)r * HID + (size_t)hh * HD);
            }
        }
        if (l == m->dump_layer) {
            if (m->dq) memcpy(m->dq, q, (size_t)rows * HID * sizeof(float));
            if (m->dk) memcpy(m->dk, k, (size_t)rows * 128 * sizeof(float));
            if (m->dv) memcpy(m->dv, v, (size_t)rows * 128 * sizeof(float));
            if (m->dctx) memcpy(m->dctx, ctx, (size_t)rows * HID * sizeof(float));
        }
        /* O projection + residual (model_backend.py:103) */
        accum(ctx, rows, HID, m->wt[l][PO], HID, tmp, mode);
        epi_linear(tmp, rows, HID, sc + P_SCALE[PO], mode);
        for (size_t i = 0; i < (size_t)rows * HID; ++i) x[i] = bfm(x[i] + tmp[i], mode);
        if (l == m->dump_layer && m->dh) memcpy(m->dh, x, (size_t)rows * HID * sizeof(float));
        /* FFN (model_backend.py:104-107) */
        ref_rmsnorm(x, rows, m->gamma + (size_t)l * 1792 + 896, eps, mode, h);
        float *gate = gu, *up = gu + (size_t)rows * FFN;
        accum(h, rows, HID, m->wt[l][PG], FFN, gate, mode);
        epi_linear(gate, rows, FFN, sc + P_SCALE[PG], mode);
        accum(h, rows, HID, m->wt[l][PU], FFN, up, mode);
        epi_linear(up, rows, FFN, sc + P_SCALE[PU], mode);
        ref_swiglu(gate, up, rows * FFN, mode, mid);
        accum(mid, rows, FFN, m->wt[l][PD], HID, tmp, mode);
        epi_linear(tmp, rows, HID, sc + P_SCALE[PD], mode);
        for (size_t i = 0; i < (size_t)rows * HID; ++i) x[i] = bfm(x[i] + tmp[i], mode);
        if (l == m->dump_layer) {
            if (m->dm) memcpy(m->dm, mid, (size_t)rows * FFN * sizeof(float));
            if (m->dy) memcpy(m->dy, x, (size_t)rows * HID * sizeof(float));
        }
    }
    /* final norm + LM head + argmax (model_backend.py:108-114) */
    float *xl = (float *)malloc((size_t)nlm * HID * sizeof(float));
    for (unsigned i = 0; i < nlm; ++i) memcpy(xl + (size_t)i * HID, x + (size_t)lm_rows[i] * HID, HID * sizeof(float));
    lm_head_rows(m, xl, nlm, mode, tokens, logits);
    free(xl);
    free(x);
    free(h);
    free(q);
    free(k);
    free(v);
    free(ctx);
    free(gu);
    free(mid);
    free(tmp);
}

int ref_forward(ref_model *m, const uint32_t *ids, unsigned rows, unsigned position, uint32_t *token,
                float *logits) {
    if (position != m->position || rows == 0 || position + rows > m->capacity) return -8;
    for (unsigned r = 0; r < rows; ++r)
        if (ids[r] >= VOC) return -1;
    uint32_t *pos = (uint32_t *)malloc(rows * sizeof(uint32_t));
    uint32_t *slot = (uint32_t *)calloc(rows, sizeof(uint32_t));
    for (unsigned r = 0; r < rows; ++r) pos[r] = position + r;
    const uint32_t last = rows - 1;
    uint32_t tok = 0;
    run_rows(m, rows, ids, pos, slot, 1, &last, &tok, logits);
    m->position = position + rows;
    if (token) *token = tok;
    free(pos);
    free(slot);
    return 0;
}

int ref_decode_batch(ref_model *m, unsigned n, const uint32_t *slots, const uint32_t *ids, uint32_t *tokens,
                     float *logits) {
    if (!n || !(m->mode & REF_KV8)) return -1;
    uint32_t *pos = (uint32_t *)malloc(n * sizeof(uint32_t));
    uint32_t *rows = (uint32_t *)malloc(n * sizeof(uint32_t));
    char *seen = (char *)calloc(m->nslots, 1);
    int rc = 0;
    for (unsigned r = 0; r < n && !rc; ++r) {
        if (slots[r] >= m->nslots || seen[slots[r]] || ids[r] >= VOC) rc = -1;
        else {
            seen[slots[r]] = 1;
            pos[r] = slots[r] == 0 ? m->position : m->spos[slots[r]];
            if (pos[r] >= m->capacity) rc = -8;
        }
        rows[r] = r;
    }
    if (!rc) {
        run_rows(m, n, ids, pos, slots, n, rows, tokens, logits);
        for (unsigned r = 0; r < n; ++r) {
            if (slots[r] == 0)
                m->position += 1;
            else
                m->spos[slots[r]] += 1;
        }
    }
    free(pos);
    free(rows);
    free(seen);
    return rc;
}

int ref_synth_write(const char *root, uint64_t seed) {
    qa_model m;
    if (qa_alloc(&m)) {
        qa_free(&m);
        return -6;
    }
    qa_generate(seed, &m);
    const int rc = qa_write(&m, root, seed);
    qa_free(&m);
    return rc;
}

void ref_synth_prompt(uint64_t seed, unsigned n, uint32_t *ids) { qa_prompt(seed, n, ids); }

/* ------------------------------------------------ RTL-format K16 quantiser
 * The accelerator's own KV8 K format, restated from src/rtl/kv8_k_quant.sv
 * with the K chain's parameters (MARGIN 8 as src/rtl/storage/
 * qwen25_qkv_controller.v:1908 instantiates the chain, MTOP 65535, RSHIFT 24,
 * CODE_EXTRA 8) and the block lock of src/rtl/kv8_k_write_chain.sv:503-600
 * (the first token of each 256-token block fixes the exponent of that
 * (layer, head, block); later tokens are quantised against it):
 *   maxmag = max_d (k & 0x7fff), E = maxmag >> 7, M8 = 0x80 | (maxmag & 0x7f)
 *   first : eb = E > 9 ? E - 8 : 1, m = ceil(M8 * 2^8 / 127),
 *           lock = published exponent ((eb > 10 ? eb - 10 : 0) + 10, 255 top)
 *   later : s = E - lock, n = M8 * 2^s (saturating at s > 15, 0 below -15),
 *           m = min(ceil(n / 127), 65535)
 *   R = floor((2^24 + floor(m / 2)) / m) (2^24 when m = 0)
 *   per dim: N = M8d * 2^(Ed - lock) (0 for Ed = 0, 0xffffff above a shift
 *   of 15), q16 = (N * R + 2^15) >> 16 clamped to 32639, published as two
 *   int8 planes hi = (q16 + 128) >> 8, lo = q16 mod 256, both negated for a
 *   negative k (two's complement bytes: 256 * hi + lo = q16 except where the
 *   low byte is 0x80 on a negative value, as in the RTL).
 * Exponent-table byte: kexp(lock) (src/rtl/kv8_k_write_chain.sv:416-438);
 * clip: m == 0, m == 65535 or the normalised exponent at 255. */
static unsigned k16_norm_exp(unsigned eb) { return eb <= 3 ? 1 : (eb > 258 ? 255 : eb - 3); }
static unsigned k16_kexp(unsigned eb) {
    const unsigned t = k16_norm_exp(eb);
    return t <= 9 ? 1 : t - 8;
}

void ref_k16_quant(const uint16_t *k, int first, uint8_t *lock, int8_t *hi, int8_t *lo, uint16_t *m16,
                   uint8_t *etab, int *clip) {
    unsigned maxmag = 0;
    for (int d = 0; d < HD; ++d)
        if ((k[d] & 0x7fffu) > maxmag) maxmag = k[d] & 0x7fffu;
    const unsigned E = maxmag >> 7, M8 = 0x80u | (maxmag & 0x7fu);
    unsigned eb, m;
    if (first) {
        const unsigned eb_r = E > 9 ? E - 8 : 1;
        const unsigned num = M8 << 8;
        m = num / 127 + (num % 127 != 0);
        const unsigned ob = eb_r > 10 ? eb_r - 10 : 0;
        *lock = (uint8_t)(ob > 245 ? 255 : ob + 10);
        eb = *lock;
    } else {
        eb = *lock;
        const int s = (int)E - (int)eb;
        uint32_t n;
        if (s > 15) n = 0x7fffffu;
        else if (s < -15) n = 0;
        else if (s < 0) n = M8 >> (-s);
        else n = M8 << s;
        const uint32_t quo = n / 127, rem = n % 127;
        m = (quo > 65535u || (quo == 65535u && rem != 0)) ? 65535u : quo + (rem != 0);
    }
    const uint64_t R = m == 0 ? (1ull << 24) : ((1ull << 24) + (m >> 1)) / m;
    for (int i = 0; i < HD; ++i) {
        const unsigned kk = k[i], e = (kk >> 7) & 0xffu, mm = 0x80u | (kk & 0x7fu);
        const int d = (int)e - (int)eb;
        uint32_t nn;
        if (e == 0) nn = 0;
        else if (d >= 0) nn = d > 15 ? 0xffffffu : mm << d;
        else nn = (-d) >= 8 ? 0 : mm >> (-d);
        const uint64_t qv = ((uint64_t)nn * R + (1ull << 15)) >> 16;
        const unsigned qmag = ((qv >> 16) != 0 || (qv & 0xffffu) > 32639u) ? 32639u : (unsigned)qv;
        const uint8_t hu = (uint8_t)(((qmag + 128u) >> 8) & 0xffu), lu = (uint8_t)(qmag & 0xffu);
        const int neg = (kk >> 15) & 1;
        hi[i] = (int8_t)(neg ? (uint8_t)(0u - hu) : hu);
        lo[i] = (int8_t)(neg ? (uint8_t)(0u - lu) : lu);
    }
    *m16 = (uint16_t)m;
    *etab = (uint8_t)k16_kexp(eb);
    *clip = m == 0 || m == 65535u || k16_norm_exp(eb) == 255;
}

/* ------------------------------------------------ RTL-format V quantiser
 * The accelerator's own KV8 V format, restated from src/rtl/kv8_v_quant.sv
 * with the V chain's margin (MARGIN 2: src/rtl/storage/
 * qwen25_qkv_controller.v:1951, and the V case of
 * src/verification/tb_kv8_quant_pipeline.sv) and the layer lock of
 * src/rtl/kv8_v_write_chain.sv:387-468 (the first token of a request fixes
 * the exponent of that (layer, head); every token keeps its own 8-bit
 * mantissa):
 *   maxmag = max_d (v & 0x7fff), E = maxmag >> 7, M8 = 0x80 | (maxmag & 0x7f)
 *   first : eb = E > 3 ? E - 2 : 1, m = ceil(M8 * 2^2 / 127) (5..9),
 *           lock = max(eb, 10) (the table convention round trip of
 *           kv8_v_quant.sv:110 and kv8_v_write_chain.sv:302: eb - 10
 *           floored at 0, plus 10)
 *   later : s = E - lock, n = M8 * 2^s (0x7fffff above s = 15, 0 below -15),
 *           m = ceil(n / 127), 255 when that exceeds 255
 *   R = floor((2^16 + floor(m / 2)) / m) (2^16 when m = 0)
 *   per dim: N = (M8d * 2^(Ed - lock)) mod 2^24 (the 24-bit shifter of
 *   kv8_v_quant.sv:279-281, without a clamp; 0 for Ed = 0),
 *   q = min((N * R + 2^15) >> 16, 127), negated for a negative v.
 * The dequantised value is code * m * 2^(lock - 134); the layer's published
 * scale is the bf16 2^(lock - 134) (m = 1, kv8_v_write_chain.sv:306-332,
 * 421-437). clip: m == 0 or m == 255 (the chain's witness). */
void ref_v8_quant(const uint16_t *v, int first, uint8_t *lock, int8_t *codes, uint8_t *m8, uint16_t *scale_bf16,
                  int *clip) {
    unsigned maxmag = 0;
    for (int d = 0; d < HD; ++d)
        if ((v[d] & 0x7fffu) > maxmag) maxmag = v[d] & 0x7fffu;
    const unsigned E = maxmag >> 7, M8 = 0x80u | (maxmag & 0x7fu);
    unsigned eb, m;
    if (first) {
        const unsigned eb_calc = E > 3 ? E - 2 : 1;
        const unsigned num = M8 << 2;
        m = num / 127 + (num % 127 != 0);
        eb = eb_calc > 10 ? eb_calc : 10;
        *lock = (uint8_t)eb;
    } else {
        eb = *lock;
        const int s = (int)E - (int)eb;
        uint32_t n;
        if (s > 15) n = 0x7fffffu;
        else if (s < -15) n = 0;
        else if (s < 0) n = M8 >> (-s);
        else n = M8 << s;
        const uint32_t quo = n / 127, rem = n % 127;
        m = (quo > 255u || (quo == 255u && rem != 0)) ? 255u : quo + (rem != 0);
    }
    const uint64_t R = m == 0 ? (1ull << 16) : ((1ull << 16) + (m >> 1)) / m;
    for (int i = 0; i < HD; ++i) {
        const unsigned vv = v[i], e = (vv >> 7) & 0xffu, mm = 0x80u | (vv & 0x7fu);
        const int d = (int)e - (int)eb;
        uint32_t nn;
        if (e == 0) nn = 0;
        else if (d >= 0) nn = d >= 24 ? 0 : (mm << d) & 0xffffffu;
        else nn = (-d) >= 8 ? 0 : mm >> (-d);
        const uint64_t qv = ((uint64_t)nn * R + (1ull << 15)) >> 16;
        const uint8_t q = (uint8_t)(qv > 127 ? 127 : qv);
        codes[i] = (int8_t)((vv >> 15) & 1u ? (uint8_t)(0u - q) : q);
    }
    *m8 = (uint8_t)m;
    *scale_bf16 = (uint16_t)(eb > 7 ? (eb - 7u) << 7 : 0);
    *clip = m == 0 || m == 255u;
}
