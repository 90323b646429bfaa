/* Seeded synthetic Qwen2.5-0.5B assets in the reference's SD-card format, and
 * the reader that loads that format (real or synthetic) into logical arrays.
 *
 * Quantisation rule: legacy_100mhz_closed/src/software/interactive/tests/
 * validate_model_weights.py:38-39 (scale = bf16(max(amax,1e-12)/127),
 * code = round_half_even(w/scale) clamped to +-127).
 * Physical weight tiling: model_backend.py:51-55.
 */
#include "assets.h"

#include <errno.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

const qa_proj_shape qa_proj[QA_NPROJ] = {
    {896, 896, 0, 5},      /* q    model_backend.py:30 field 40 */
    {128, 896, 896, 6},    /* k    field 48 */
    {128, 896, 1024, 7},   /* v    field 56 */
    {896, 896, 1152, 10},  /* o    model_backend.py:31 field 80 */
    {4864, 896, 2048, 12}, /* gate field 96 */
    {4864, 896, 6912, 13}, /* up   model_backend.py:32 field 104 */
    {896, 4864, 11776, 15} /* down field 120 */
};

uint16_t qa_f2bf(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float qa_bf2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Counter-based generator: SplitMix64 finaliser over (stream key, counter). */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
static inline uint64_t stream_key(uint64_t seed, uint64_t tensor) {
    return mix64(seed * 0xD1B54A32D192ED03ULL + mix64(tensor));
}
static inline uint64_t draw(uint64_t key, uint64_t counter) {
    return mix64(key + counter * 0x9E3779B97F4A7C15ULL);
}
/* Element i of an N(0, sigma) stream: Box-Muller on the pair (i/2). */
static inline float gauss(uint64_t key, uint64_t i, double sigma) {
    uint64_t p = i >> 1;
    double u1 = ((double)(draw(key, 2 * p) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(draw(key, 2 * p + 1) >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1));
    double a = 6.283185307179586476925286766559 * u2;
    double z = (i & 1) ? r * sin(a) : r * cos(a);
    return (float)(sigma * z);
}

enum { T_LAYER = 16, T_BIAS = 7, T_EMBED = 100000, T_PROMPT = 200000 };

/* validate_model_weights.py:38-39 on one output channel. */
static uint16_t quantise_row(const float *w, unsigned n, int8_t *q) {
    float amax = 0.0f;
    for (unsigned i = 0; i < n; ++i) {
        float a = fabsf(w[i]);
        if (a > amax) amax = a;
    }
    if (amax < 1e-12f) amax = 1e-12f;
    uint16_t sb = qa_f2bf(amax / 127.0f);
    float s = qa_bf2f(sb);
    for (unsigned i = 0; i < n; ++i) {
        float v = nearbyintf(w[i] / s);
        if (v > 127.0f) v = 127.0f;
        if (v < -127.0f) v = -127.0f;
        q[i] = (int8_t)v;
    }
    return sb;
}

int qa_alloc(qa_model *m) {
    memset(m, 0, sizeof(*m));
    for (int l = 0; l < QA_LAYERS; ++l)
        for (int p = 0; p < QA_NPROJ; ++p) {
            m->w[l][p] = (int8_t *)malloc((size_t)qa_proj[p].out * qa_proj[p].in);
            if (!m->w[l][p]) return -6;
        }
    m->lmw = (int8_t *)malloc((size_t)QA_VOCAB * QA_HIDDEN);
    m->scale = (uint16_t *)calloc(QA_SCALE_COUNT, 2);
    m->bias = (uint16_t *)calloc((size_t)QA_LAYERS * QA_BIAS_LAYER, 2);
    m->gamma = (uint16_t *)calloc(QA_GAMMA_COUNT, 2);
    m->embed = (uint16_t *)malloc((size_t)QA_VOCAB * QA_HIDDEN * 2);
    if (!m->lmw || !m->scale || !m->bias || !m->gamma || !m->embed) return -6;
    return 0;
}

void qa_free(qa_model *m) {
    for (int l = 0; l < QA_LAYERS; ++l)
        for (int p = 0; p < QA_NPROJ; ++p) free(m->w[l][p]);
    free(m->lmw);
    free(m->scale);
    free(m->bias);
    free(m->gamma);
    free(m->embed);
    memset(m, 0, sizeof(*m));
}

int qa_generate(uint64_t seed, qa_model *m) {
    for (int l = 0; l < QA_LAYERS; ++l) {
        for (int p = 0; p < QA_NPROJ; ++p) {
            const unsigned out = qa_proj[p].out, in = qa_proj[p].in;
            const uint64_t key = stream_key(seed, (uint64_t)l * T_LAYER + (uint64_t)p);
            int8_t *dst = m->w[l][p];
            uint16_t *sc = m->scale + (size_t)l * QA_SCALE_LAYER + qa_proj[p].scale_off;
#pragma omp parallel
            {
                float *row = (float *)malloc(sizeof(float) * in);
#pragma omp for schedule(static)
                for (long r = 0; r < (long)out; ++r) {
                    for (unsigned i = 0; i < in; ++i) row[i] = gauss(key, (uint64_t)r * in + i, 0.02);
                    sc[r] = quantise_row(row, in, dst + (size_t)r * in);
                }
                free(row);
            }
        }
        const uint64_t bkey = stream_key(seed, (uint64_t)l * T_LAYER + T_BIAS);
        for (unsigned i = 0; i < QA_BIAS_LAYER; ++i)
            m->bias[(size_t)l * QA_BIAS_LAYER + i] = qa_f2bf(gauss(bkey, i, 0.02));
    }
    for (unsigned i = 0; i < QA_GAMMA_COUNT; ++i) m->gamma[i] = 0x3f80; /* 1.0 */
    const uint64_t ekey = stream_key(seed, T_EMBED);
#pragma omp parallel
    {
        float *row = (float *)malloc(sizeof(float) * QA_HIDDEN);
#pragma omp for schedule(static)
        for (long r = 0; r < (long)QA_VOCAB; ++r) {
            uint16_t *e = m->embed + (size_t)r * QA_HIDDEN;
            for (unsigned i = 0; i < QA_HIDDEN; ++i) {
                e[i] = qa_f2bf(gauss(ekey, (uint64_t)r * QA_HIDDEN + i, 0.02));
                row[i] = qa_bf2f(e[i]);
            }
            m->scale[QA_SCALE_LM + r] = quantise_row(row, QA_HIDDEN, m->lmw + (size_t)r * QA_HIDDEN);
        }
        free(row);
    }
    return 0;
}

void qa_prompt(uint64_t seed, unsigned n, uint32_t *ids) {
    const uint64_t key = stream_key(seed, T_PROMPT);
    for (unsigned i = 0; i < n; ++i) ids[i] = (uint32_t)(((draw(key, i) >> 32) * (uint64_t)QA_VOCAB) >> 32);
}

/* Offset of logical (c, i) inside the physical 128x128 tiling (model_backend.py:53-54). */
static inline size_t phys_offset(unsigned c, unsigned i, unsigned in) {
    unsigned cb = c >> 7, cin = c & 127, a = cin >> 6, b = (cin & 63) >> 4, d = cin & 15;
    unsigned ib = i >> 7, e = i & 127;
    return (((((size_t)cb * (in >> 7) + ib) * 4 + b) * 128 + e) * 2 + a) * 16 + d;
}

static void pack(const int8_t *logical, unsigned out, unsigned in, int8_t *phys) {
#pragma omp parallel for schedule(static)
    for (long c = 0; c < (long)out; ++c)
        for (unsigned i = 0; i < in; ++i) phys[phys_offset((unsigned)c, i, in)] = logical[(size_t)c * in + i];
}

static void unpack(const int8_t *phys, unsigned out, unsigned in, int8_t *logical) {
#pragma omp parallel for schedule(static)
    for (long c = 0; c < (long)out; ++c)
        for (unsigned i = 0; i < in; ++i) logical[(size_t)c * in + i] = phys[phys_offset((unsigned)c, i, in)];
}

static int write_file(const char *dir, const char *name, const void *data, size_t bytes) {
    char path[4096];
    snprintf(path, sizeof(path), "%s/%s", dir, name);
    FILE *f = fopen(path, "wb");
    if (!f) return -7;
    size_t w = fwrite(data, 1, bytes, f);
    int bad = fclose(f) != 0 || w != bytes;
    return bad ? -7 : 0;
}

static size_t proj_offset(int l, int p) {
    size_t off = (size_t)l * QA_LAYER_BYTES;
    for (int j = 0; j < p; ++j) off += (size_t)qa_proj[j].out * qa_proj[j].in;
    return off;
}

int qa_write(const qa_model *m, const char *root, uint64_t seed) {
    char dir[4096];
    snprintf(dir, sizeof(dir), "%s/QWEN25", root);
    mkdir(root, 0755);
    if (mkdir(dir, 0755) && errno != EEXIST) return -7;
    char cfg[1024];
    int n = snprintf(cfg, sizeof(cfg),
                     "{\n  \"hidden\": 896,\n  \"layers\": 24,\n  \"vocab\": 151936,\n  \"ffn\": 4864,\n"
                     "  \"q_heads\": 14,\n  \"kv_heads\": 2,\n  \"head_dimension\": 64,\n"
                     "  \"rms_epsilon_bf16\": \"0x3586\",\n"
                     "  \"decoding\": \"greedy latest-token-index on ties\",\n"
                     "  \"synthetic\": {\"seed\": %llu, \"weights\": \"fp32 N(0,0.02) -> int8 per-output-channel\"}\n}\n",
                     (unsigned long long)seed);
    int rc = write_file(dir, "CONFIG.JSON", cfg, (size_t)n);
    uint64_t desc[QA_LAYERS * 32];
    memset(desc, 0, sizeof(desc));
    for (int l = 0; l < QA_LAYERS; ++l) {
        uint64_t *d = desc + l * 32;
        d[1] = ((uint64_t)l << 32) | 0x380;
        d[2] = 0x40010000ULL + (uint64_t)l * QA_SCALE_LAYER * 2;
        d[3] = 0x40100000ULL + (uint64_t)l * QA_BIAS_LAYER * 2;
        d[4] = 0x40110000ULL + (uint64_t)l * QA_GAMMA_LAYER * 2;
        for (int p = 0; p < QA_NPROJ; ++p) d[qa_proj[p].desc_field] = QA_WEIGHTS_BASE + proj_offset(l, p);
        d[11] = 0x71700000ULL;
        d[14] = 0x71800000ULL;
        d[16] = 0x71b00000ULL;
        d[17] = l + 1 < QA_LAYERS ? 0x40000000ULL + (uint64_t)(l + 1) * 256 : 0;
        d[18] = 0x57000000ULL;
    }
    rc = rc ? rc : write_file(dir, "DESC.BIN", desc, sizeof(desc));
    rc = rc ? rc : write_file(dir, "SCALE.BIN", m->scale, (size_t)QA_SCALE_COUNT * 2);
    rc = rc ? rc : write_file(dir, "BIAS.BIN", m->bias, (size_t)QA_LAYERS * QA_BIAS_LAYER * 2);
    rc = rc ? rc : write_file(dir, "GAMMA.BIN", m->gamma, (size_t)QA_GAMMA_COUNT * 2);
    rc = rc ? rc : write_file(dir, "EMBED.BIN", m->embed, (size_t)QA_VOCAB * QA_HIDDEN * 2);
    if (rc) return rc;
    int8_t *buf = (int8_t *)malloc((size_t)QA_LAYERS * QA_LAYER_BYTES);
    if (!buf) return -6;
    for (int l = 0; l < QA_LAYERS; ++l)
        for (int p = 0; p < QA_NPROJ; ++p) pack(m->w[l][p], qa_proj[p].out, qa_proj[p].in, buf + proj_offset(l, p));
    rc = write_file(dir, "WEIGHTS.BIN", buf, (size_t)QA_LAYERS * QA_LAYER_BYTES);
    if (!rc) {
        pack(m->lmw, QA_VOCAB, QA_HIDDEN, buf);
        rc = write_file(dir, "LMW.BIN", buf, (size_t)QA_VOCAB * QA_HIDDEN);
    }
    free(buf);
    return rc;
}

static void *read_file(const char *dir, const char *name, size_t expect, char *err, size_t errlen) {
    char path[4096];
    snprintf(path, sizeof(path), "%s/%s", dir, name);
    FILE *f = fopen(path, "rb");
    if (!f) {
        snprintf(err, errlen, "cannot open %s", path);
        return NULL;
    }
    fseek(f, 0, SEEK_END);
    long size = ftell(f);
    rewind(f);
    if (size < 0 || (size_t)size != expect) {
        snprintf(err, errlen, "wrong size %s: %ld (expected %zu)", path, size, expect);
        fclose(f);
        return NULL;
    }
    void *data = malloc(expect);
    if (data && fread(data, 1, expect, f) != expect) {
        free(data);
        data = NULL;
        snprintf(err, errlen, "short read %s", path);
    }
    fclose(f);
    return data;
}

int qa_read(const char *root, qa_model *m, char *err, size_t errlen) {
    char dir[4096];
    snprintf(dir, sizeof(dir), "%s/QWEN25", root);
    if (qa_alloc(m)) {
        snprintf(err, errlen, "out of host memory");
        return -6;
    }
    uint64_t *desc = (uint64_t *)read_file(dir, "DESC.BIN", QA_LAYERS * 256, err, errlen);
    uint16_t *scale = (uint16_t *)read_file(dir, "SCALE.BIN", (size_t)QA_SCALE_COUNT * 2, err, errlen);
    uint16_t *bias = (uint16_t *)read_file(dir, "BIAS.BIN", (size_t)QA_LAYERS * QA_BIAS_LAYER * 2, err, errlen);
    uint16_t *gamma = (uint16_t *)read_file(dir, "GAMMA.BIN", (size_t)QA_GAMMA_COUNT * 2, err, errlen);
    uint16_t *embed = (uint16_t *)read_file(dir, "EMBED.BIN", (size_t)QA_VOCAB * QA_HIDDEN * 2, err, errlen);
    int8_t *weights = (int8_t *)read_file(dir, "WEIGHTS.BIN", (size_t)QA_LAYERS * QA_LAYER_BYTES, err, errlen);
    int8_t *lmw = (int8_t *)read_file(dir, "LMW.BIN", (size_t)QA_VOCAB * QA_HIDDEN, err, errlen);
    int rc = 0;
    if (!desc || !scale || !bias || !gamma || !embed || !weights || !lmw) rc = -7;
    for (int l = 0; !rc && l < QA_LAYERS; ++l)
        for (int p = 0; !rc && p < QA_NPROJ; ++p) {
            uint64_t addr = desc[l * 32 + qa_proj[p].desc_field];
            size_t bytes = (size_t)qa_proj[p].out * qa_proj[p].in;
            if (addr < QA_WEIGHTS_BASE || addr - QA_WEIGHTS_BASE + bytes > (size_t)QA_LAYERS * QA_LAYER_BYTES) {
                snprintf(err, errlen, "DESC.BIN layer %d field %u out of WEIGHTS.BIN", l, qa_proj[p].desc_field * 8);
                rc = -7;
                break;
            }
            unpack(weights + (addr - QA_WEIGHTS_BASE), qa_proj[p].out, qa_proj[p].in, m->w[l][p]);
        }
    if (!rc) {
        unpack(lmw, QA_VOCAB, QA_HIDDEN, m->lmw);
        memcpy(m->scale, scale, (size_t)QA_SCALE_COUNT * 2);
        memcpy(m->bias, bias, (size_t)QA_LAYERS * QA_BIAS_LAYER * 2);
        memcpy(m->gamma, gamma, (size_t)QA_GAMMA_COUNT * 2);
        memcpy(m->embed, embed, (size_t)QA_VOCAB * QA_HIDDEN * 2);
    }
    free(desc);
    free(scale);
    free(bias);
    free(gamma);
    free(embed);
    free(weights);
    free(lmw);
    if (rc) qa_free(m);
    return rc;
}
