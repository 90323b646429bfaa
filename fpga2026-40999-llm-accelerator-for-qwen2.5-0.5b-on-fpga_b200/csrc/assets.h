/* Host-side model assets: the reference's SD-card package format (QWEN25/<NAME>.BIN)
 * and a seeded synthetic generator that writes it.
 *
 * Format (legacy_100mhz_closed/src/PC/model_backend.py:18-55, board_parameters.h:18-26):
 *   CONFIG.JSON  hidden/layers/vocab (model_backend.py:18-19)
 *   DESC.BIN     24 x 256 B layer descriptors; u64 byte-offset fields 40/48/56/80/96/104/120
 *                hold the DDR address (0x41000000 + offset into WEIGHTS.BIN) of
 *                q/k/v/o/gate/up/down (model_backend.py:29-35)
 *   SCALE.BIN    bf16 per-output-channel scales, layer stride 12672, LM head at 304128
 *   BIAS.BIN     bf16 q/k/v biases, layer stride 1152
 *   GAMMA.BIN    bf16 RMSNorm gains, attn at l*1792, ffn at l*1792+896, final at 43008
 *   WEIGHTS.BIN  int8 codes in 128x128 physical tiles [C/128][I/128][4][128][2][16]
 *   LMW.BIN      int8 LM-head codes, same tiling (model_backend.py:39-40,51-55)
 *   EMBED.BIN    bf16 [151936][896] (model_backend.py:23)
 */
#ifndef QWEN_B200_ASSETS_H
#define QWEN_B200_ASSETS_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define QA_LAYERS 24
#define QA_HIDDEN 896
#define QA_FFN 4864
#define QA_VOCAB 151936
#define QA_SCALE_LAYER 12672
#define QA_SCALE_LM 304128
#define QA_SCALE_COUNT (QA_SCALE_LM + QA_VOCAB)
#define QA_BIAS_LAYER 1152
#define QA_GAMMA_LAYER 1792
#define QA_GAMMA_FINAL 43008
#define QA_GAMMA_COUNT (QA_GAMMA_FINAL + QA_HIDDEN)
#define QA_WEIGHTS_BASE 0x41000000ULL
#define QA_LAYER_BYTES 14909440ULL

/* Projection order inside a layer: q, k, v, o, gate, up, down. */
enum { QA_Q, QA_K, QA_V, QA_O, QA_GATE, QA_UP, QA_DOWN, QA_NPROJ };

typedef struct qa_proj_shape { unsigned out, in, scale_off, desc_field; } qa_proj_shape;
extern const qa_proj_shape qa_proj[QA_NPROJ];

/* Logical (unpacked, row-major [out][in]) host copy of every asset. */
typedef struct qa_model {
    int8_t *w[QA_LAYERS][QA_NPROJ];
    int8_t *lmw;          /* [VOCAB][HIDDEN] */
    uint16_t *scale;      /* SCALE.BIN contents, bf16 bits */
    uint16_t *bias;       /* BIAS.BIN */
    uint16_t *gamma;      /* GAMMA.BIN */
    uint16_t *embed;      /* EMBED.BIN */
} qa_model;

int qa_alloc(qa_model *m);
void qa_free(qa_model *m);
/* Seeded synthetic weights: fp32 N(0, 0.02) -> int8 per-output-channel with
 * bf16-representable scales; gains 1.0; q/k/v bias N(0, 0.02) in bf16; tied
 * embedding (EMBED = bf16(W), LMW = int8 of the same bf16 values). */
int qa_generate(uint64_t seed, qa_model *m);
/* Write <root>/QWEN25/{CONFIG.JSON,DESC.BIN,...} in the reference format. */
int qa_write(const qa_model *m, const char *root, uint64_t seed);
/* Read the reference format back into logical arrays. 0 on success, -7 on I/O
 * or size errors (message in err). */
int qa_read(const char *root, qa_model *m, char *err, size_t errlen);
/* Seeded uniform prompt ids in [0, VOCAB). */
void qa_prompt(uint64_t seed, unsigned n, uint32_t *ids);

/* bf16 helpers shared by host code (round to nearest even). */
uint16_t qa_f2bf(float x);
float qa_bf2f(uint16_t b);

#ifdef __cplusplus
}
#endif
#endif
