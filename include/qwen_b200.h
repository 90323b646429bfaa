/* libqwen_b200 — B200 (sm_100a) engine for the Qwen2.5-0.5B W8A16 / KV8 decode
 * path that the reference runs in KV260 programmable logic.
 *
 * The boundary keeps the reference's host call surface:
 *   - the qgen_ops CSR protocol (src/software/generation.h:5-18): write / read /
 *     embedding callbacks, START at 0x10, status at 0x18, token at 0x1f8;
 *   - the behavioural model's Model.forward(ids, position) / clear()
 *     (legacy_100mhz_closed/src/PC/model_backend.py:57-115);
 *   - one operator-level entry per PL stage (embedding, RMSNorm, W8A16 GEMM,
 *     RoPE, KV8 quantise-append, GQA attention, SwiGLU FFN, LM head + argmax).
 * Plain C types only: bf16 tensors are uint16_t bit patterns, device pointers
 * are CUDA global-memory addresses, streams are cudaStream_t passed as void*.
 * One handle per GPU; a handle is not thread-safe; one host thread per handle.
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* Model geometry (legacy_100mhz_closed/board/deployment/QWEN25/CONFIG.JSON). */
#define QWEN_B200_LAYERS 24
#define QWEN_B200_HIDDEN 896
#define QWEN_B200_FFN 4864
#define QWEN_B200_Q_HEADS 14
#define QWEN_B200_KV_HEADS 2
#define QWEN_B200_HEAD_DIM 64
#define QWEN_B200_QKV 1152
#define QWEN_B200_VOCAB 151936

/* Status codes. -1..-5 keep the meanings of src/software/generation.h:16. */
#define QWEN_B200_OK 0
#define QWEN_B200_EINVAL (-1)   /* bad input */
#define QWEN_B200_ETIMEOUT (-2) /* a bounded device wait expired */
#define QWEN_B200_EDEVICE (-3)  /* CUDA error (the reference's "PL error") */
#define QWEN_B200_ETOKEN (-4)   /* produced token id >= vocab */
#define QWEN_B200_EOUTPUT (-5)  /* output buffer error */
#define QWEN_B200_ENOMEM (-6)   /* device or host allocation failed */
#define QWEN_B200_EIO (-7)      /* asset file missing or of the wrong size */
#define QWEN_B200_ESTATE (-8)   /* KV position mismatch (model_backend.py:82-83) */
#define QWEN_B200_ESCRATCH (-9) /* request larger than the fixed no-allocation scratch */

/* CSR map emulated by qwen_b200_csr_read/write (src/software/README.md CSR
 * table; src/rtl/qwen25_compute_cfg.v, qwen25_result_regs.v). */
#define QWEN_B200_CSR_ID 0x0000
#define QWEN_B200_CSR_VERSION 0x0008
#define QWEN_B200_CSR_CONTROL 0x0010 /* bit0 START, bit3 CLEAR */
#define QWEN_B200_CSR_STATUS 0x0018  /* done <=> (s & 0x46) == 0x44; bit3 error */
#define QWEN_B200_CSR_ERROR 0x0030  /* 1 bad request, 2 CUDA error, 3 no model, 4 START while busy,
                                        5 a bounded device wait expired */
#define QWEN_B200_CSR_RUN_MODE 0x0080 /* 0 prefill (clears the context), 1 decode */
#define QWEN_B200_CSR_SEQ_LEN 0x0088
#define QWEN_B200_CSR_CONTEXT_LEN 0x0090
#define QWEN_B200_CSR_TOKEN_POS 0x0098
#define QWEN_B200_CSR_BEST_TOKEN 0x01f8
#define QWEN_B200_ID_VALUE 0x515732354b563236ULL
#define QWEN_B200_VERSION_VALUE 0x10000ULL

typedef struct qwen_b200 qwen_b200;

typedef struct qwen_b200_config {
    int device;           /* CUDA device ordinal */
    uint32_t max_seqs;    /* sequence slots (KV caches) */
    uint32_t max_context; /* KV capacity per slot, tokens (reference firmware: 256) */
    uint32_t max_rows;    /* rows per forward chunk; longer prompts are chunked */
    float rms_eps;        /* RMSNorm epsilon, 1e-6 (model_backend.py:71) */
    uint32_t flags;       /* 0, or QWEN_B200_FLAG_RTL_KV */
} qwen_b200_config;

/* The accelerator's own KV cache format instead of the engine's KV8 rule:
 * K as 16-bit codes in two int8 planes with a 16-bit mantissa per (token,
 * head) and an exponent locked per 256-token block (src/rtl/kv8_k_quant.sv,
 * kv8_k_write_chain.sv), V as 8-bit codes with an 8-bit mantissa per (token,
 * head) and an exponent locked per (layer, head) by a request's first token
 * (kv8_v_quant.sv at margin 2, kv8_v_write_chain.sv), the same rules as
 * qwen_b200_op_k16_append / qwen_b200_op_v8_append. Attention reads them
 * with the engine's exact arithmetic (the K code of a dim is 256 * high +
 * low, the scales m16 * 2^(lock - 142) and m8 * 2^(lock - 134)), so tokens and
 * logits equal the oracle's in the same mode. For RTL numeric comparisons:
 * every step takes the per-kernel path and the attention kernel for long
 * rows, and qwen_b200_fill_kv_synthetic is not available. */
#define QWEN_B200_FLAG_RTL_KV 1u

/* ---- handle lifecycle ------------------------------------------------------ */
/* Fills defaults: device 0, 1 slot, 256-token context, 256 rows, eps 1e-6. */
void qwen_b200_default_config(qwen_b200_config *cfg);
/* Allocates nothing on the device until assets are loaded. */
int qwen_b200_open(const qwen_b200_config *cfg, qwen_b200 **out);
int qwen_b200_close(qwen_b200 *h);
/* Loads <sd_root>/QWEN25/{DESC,SCALE,BIAS,GAMMA,WEIGHTS,LMW,EMBED}.BIN (the
 * reference's SD package, main.c:88-104 / board_parameters.h:18-26). */
int qwen_b200_load_assets(qwen_b200 *h, const char *sd_root);
/* Same model as qwen_b200_synth_write(seed) would write, generated in memory. */
int qwen_b200_load_synthetic(qwen_b200 *h, uint64_t seed);
const char *qwen_b200_last_error(const qwen_b200 *h);
/* The configuration the handle was opened with (defaults filled in). */
int qwen_b200_get_config(const qwen_b200 *h, qwen_b200_config *cfg);

/* ---- seeded synthetic assets (no checkpoint is available offline) ---------- */
/* Writes the <sd_root>/QWEN25 files in the reference format from a seed: fp32
 * N(0,0.02) weights quantised per output channel with the rule of
 * legacy_.../tests/validate_model_weights.py:38-39, gains 1.0, bf16 biases. */
int qwen_b200_synth_write(const char *sd_root, uint64_t seed);
/* n uniform prompt ids in [0, 151936) from the seed. */
void qwen_b200_synth_prompt(uint64_t seed, uint32_t n, uint32_t *ids);

/* ---- sequence level (model_backend.py:57-115) ------------------------------ */
/* Model.clear(): the slot's position returns to 0. */
int qwen_b200_reset(qwen_b200 *h, uint32_t slot);
int qwen_b200_position(const qwen_b200 *h, uint32_t slot, uint32_t *position);
/* Model.forward(ids, position): rows tokens at position..position+rows-1 of one
 * slot; returns the greedy token of the last row (highest index on ties) and,
 * if logits != NULL, its 151936 bf16 logits. ESTATE when position differs from
 * the slot's position or the capacity would overflow. Host buffers. */
int qwen_b200_forward(qwen_b200 *h, uint32_t slot, const uint32_t *ids, uint32_t rows, uint32_t position,
                      uint32_t *token, uint16_t *logits);
/* Prefill of n sequences in one call (batched prompt processing): sequence
 * i is lens[i] ids (the sequences' ids concatenated in `ids`) appended to slot
 * slots[i] at its current position (0 after qwen_b200_reset). The rows of all
 * sequences go through the layers together, max_rows at a time (a chunk may
 * hold rows of several sequences; each row attends to its own slot's keys
 * up to its position). tokens_out (nullable) [n]: the greedy token after each
 * sequence; hidden_out (nullable, host) [n][896] bf16: each sequence's last
 * hidden row before the final RMSNorm (the input of qwen_b200_lm_head_range,
 * e.g. on other GPUs). At least one of the two. With tokens_out NULL the LM
 * head is not run. The reference feeds a prompt in row groups through the
 * same layer sequence (src/rtl/storage/qwen25_qkv_controller.v:400-474;
 * model_backend.py:80-115 for several ids at once). Host buffers. */
int qwen_b200_prefill(qwen_b200 *h, uint32_t n, const uint32_t *slots, const uint32_t *lens, const uint32_t *ids,
                      uint32_t *tokens_out, uint16_t *hidden_out);
/* Final RMSNorm + LM head over the vocabulary rows [begin, end) of the
 * resident tied head + greedy argmax, for rows hidden rows (d_hidden: device
 * bf16 [rows][896], before the final norm): d_values[r] is the best bf16
 * logit of row r (as fp32) and d_indices[r] its global token id, highest id
 * on ties (model_backend.py:108-114). begin and end are multiples of 128
 * (151936 is one). Shards of the vocabulary combine by taking, per row, the
 * largest value and then the highest index: the vocab-sharded LM head of
 * several GPUs. Enqueued on `stream` (device buffers, no synchronisation);
 * calls on one handle must not overlap other work of that handle. */
int qwen_b200_lm_head_range(qwen_b200 *h, const uint16_t *d_hidden, uint32_t rows, uint32_t begin, uint32_t end,
                            float *d_values, uint32_t *d_indices, void *stream);
/* One decode step for n slots (one token each, each at its own position).
 * Host buffers; the host->device and device->host copies are inside the call.
 * The forward is replayed from a CUDA graph per (n, context bucket of 128):
 * the first step of a bucket launches the kernels directly and captures them.
 * Changing qwen_b200_set_persistent_decode drops the captured graphs. */
int qwen_b200_decode_step(qwen_b200 *h, const uint32_t *slots, const uint32_t *tokens_in, uint32_t n,
                          uint32_t *tokens_out);
/* The same step, also returning every row's 151936 bf16 logits in
 * logits[n][151936] (host buffer). Runs the kernels directly (no graph);
 * the device buffer for the logits is allocated at the first call. */
int qwen_b200_decode_step_logits(qwen_b200 *h, const uint32_t *slots, const uint32_t *tokens_in, uint32_t n,
                                 uint32_t *tokens_out, uint16_t *logits);
/* The same step for slots 0..n-1 with device-resident token arrays, enqueued
 * on `stream` (a cudaStream_t; NULL is the CUDA default stream); d_tokens_out is written on the
 * device and ids are not range-checked on the host. The first call for a given
 * (n, context bucket of 128, buffers) runs eagerly and captures a CUDA graph
 * that later calls replay. */
int qwen_b200_decode_step_device(qwen_b200 *h, const uint32_t *d_tokens_in, uint32_t n, uint32_t *d_tokens_out,
                                 void *stream);
/* Fills the first `length` KV entries of every layer of a slot with seeded
 * synthetic KV8 codes/scales and sets its position to `length` (bench set-up
 * for long contexts whose prefill is not under test). */
int qwen_b200_fill_kv_synthetic(qwen_b200 *h, uint32_t slot, uint32_t length, uint64_t seed);
/* Copies one layer's KV8 cache of a slot to host: codes [2][n][64], scales [2][n]. */
int qwen_b200_read_kv(qwen_b200 *h, uint32_t slot, uint32_t layer, uint32_t n, int8_t *kcodes, float *kscales,
                      int8_t *vcodes, float *vscales);
/* QWEN_B200_FLAG_RTL_KV handles: the low K planes klo [2][n][64], the K
 * block locks klock [2][ceil(max_context / 256)] and the V layer locks
 * vlock [2] of one layer and slot (nullable outputs). */
int qwen_b200_read_kv_rtl(qwen_b200 *h, uint32_t slot, uint32_t layer, uint32_t n, int8_t *klo, uint8_t *klock,
                          uint8_t *vlock);
/* Records the bf16 tensors of one layer (q k v context h m y, rows x dims) at
 * the next forward into host buffers (the reference's RTL_DUMP_LAYERS names,
 * src/verification/rtl_bridge.cpp:109-171). layer < 0 disables. */
int qwen_b200_set_dump(qwen_b200 *h, int layer, uint16_t *q, uint16_t *k, uint16_t *v, uint16_t *ctx,
                       uint16_t *hbuf, uint16_t *mid, uint16_t *y);

/* Single-row forwards and decode steps can run as one persistent
 * cooperative launch of one CTA per SM: every layer, the LM head and the
 * argmax, weights streamed into shared memory ahead of use, phases separated
 * by grid barriers; same arithmetic (and bits) as the per-kernel path.
 * enable = 1 (default): the persistent launch for contexts up to 96 keys,
 * where it is the faster path; 2: up to 1024 keys; 0: always the per-kernel
 * path. */
int qwen_b200_set_persistent_decode(qwen_b200 *h, int enable);
/* Test switch for the error path of the bounded device waits (reference:
 * the -2 / -3 returns of src/software/generation.c:21-25). While enabled, the
 * persistent single-row step waits at its last grid barrier for one arrival
 * more than its CTAs make, with a short limit (a few milliseconds), at a
 * point where no bulk copy or tensor-core operation is in flight: the wait
 * expires, the kernel returns normally, and the call reports
 * QWEN_B200_ETIMEOUT (qwen_b200_forward) or CSR status 8 with error code 5.
 * The device stays usable. Default off; toggling drops captured graphs. */
int qwen_b200_test_expire_wait(qwen_b200 *h, int enable);

/* Kernel classes reported by qwen_b200_profile_decode. */
#define QWEN_B200_KCLASSES 9 /* 0 embedding, 1 RMSNorm+QKV+RoPE+KV8 append, 2 attention,
                                3 O proj+residual, 4 RMSNorm+gate/up+SiLU*mul, 5 down+residual,
                                6 LM head+argmax, 7 bookkeeping (row gathers, position updates),
                                8 persistent batch-1 step (every layer + LM head + argmax) */
/* One decode step of slots 0..n-1 (host buffers, like qwen_b200_decode_step)
 * with CUDA events around every kernel launch on the launching stream: ms[c]
 * is the summed device time of class c, launches[c] its launch count. */
int qwen_b200_profile_decode(qwen_b200 *h, const uint32_t *tokens_in, uint32_t n, uint32_t *tokens_out, float *ms,
                             uint32_t *launches);
/* Kernels enqueued by the last forward / decode step (a replayed graph
 * launches the same number). */
uint32_t qwen_b200_step_launches(const qwen_b200 *h);

/* ---- continuous batching (beyond the reference's one request at a time) ---- */
/* A scheduler over one handle. The reference serves one request at a time
 * (src/software/main.c:243-265). Here requests queue and share the GPU: each
 * qwen_b200_sched_step admits waiting requests into free slots (first come,
 * first served), prefills up to prefill_budget prompt tokens of admitted
 * requests together (a longer prompt continues in the next steps), runs one
 * batched decode step for every request that has a token, and retires
 * requests at max_new tokens or at an end-of-text id (151643 / 151645, the
 * stop ids of src/software/generation.c). Every request's tokens equal those
 * of the request run alone. Single-threaded, like the handle; an error
 * returned by a step leaves the scheduler unusable. */
typedef struct qwen_b200_sched qwen_b200_sched;
int qwen_b200_sched_open(qwen_b200 *h, uint32_t prefill_budget, qwen_b200_sched **out);
int qwen_b200_sched_close(qwen_b200_sched *s);
/* Queues a prompt; QWEN_B200_ESTATE when n + max_new exceeds a slot's capacity. */
int qwen_b200_sched_submit(qwen_b200_sched *s, const uint32_t *ids, uint32_t n, uint32_t max_new,
                           uint32_t *request_id);
/* One scheduling step; *running (nullable) = requests not yet finished. */
int qwen_b200_sched_step(qwen_b200_sched *s, uint32_t *running);
/* Tokens produced so far (up to cap copied), and whether the request is
 * finished; a finished request's result can be read once. */
int qwen_b200_sched_result(qwen_b200_sched *s, uint32_t request_id, uint32_t *tokens, uint32_t cap,
                           uint32_t *count, int *done);

/* ---- CSR protocol: drop-in for struct qgen_ops (generation.h:5-14) ---------- */
/* ops.context = handle; ops.write = qwen_b200_csr_write; ops.read =
 * qwen_b200_csr_read; ops.embedding = qwen_b200_embedding. Slot 0 is used.
 * START (0x10 bit0) enqueues the forward and returns at once; 0x18 reads 2
 * while it runs, 0x44 when the token is ready, 8 on error (code at 0x30; a
 * device wait that expired during the forward reads 8 with code 5). */
void qwen_b200_csr_write(void *h, unsigned offset, uint64_t value);
uint64_t qwen_b200_csr_read(void *h, unsigned offset);
/* main.c:114-125 copy_embedding: records token id for ACT_IN row `row`. */
void qwen_b200_embedding(void *h, unsigned token, unsigned row);
/* main.c:162-170 reset_context. */
void qwen_b200_clear(void *h);

/* ---- operator level: device pointers, enqueued on `stream` ----------------- */
/* x[r] = embed[ids[r]] (main.c:114-125). */
int qwen_b200_op_embed(const uint16_t *embed, const uint32_t *ids, uint32_t rows, uint16_t *x, void *stream);
/* out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * gamma), x [rows][896]
 * (model_backend.py:69-71; AFU src/rtl/afu/qwen25_afu.v:75-125). */
int qwen_b200_op_rmsnorm(const uint16_t *x, const uint16_t *gamma, uint32_t rows, float eps, uint16_t *out,
                         void *stream);
/* y = bf16(bf16(x W^T) * scale) [+ bias: bf16(. + bias)], W int8 row-major [n][k]
 * (model_backend.py:62-67; GEMM src/rtl/qwen25_gemm_i.sv). k is 896 or 4864;
 * n a multiple of 4. */
int qwen_b200_op_gemm_w8a16(const uint16_t *x, uint32_t rows, uint32_t k, const int8_t *w, const float *scale,
                            uint32_t n, const uint16_t *bias, uint16_t *y, void *stream);
/* y = bf16(y + bf16(bf16(x W^T) * scale)): O / down projection + residual
 * (model_backend.py:103,107). */
int qwen_b200_op_gemm_w8a16_residual(const uint16_t *x, uint32_t rows, uint32_t k, const int8_t *w,
                                     const float *scale, uint32_t n, uint16_t *y, void *stream);
/* Tensor-core (tcgen05 kind::i8) form of the same projection (the engine's
 * form for 2 rows and more; rows >= 1 accepted),
 * with the GEMV's exact integer sums: every activation row is aligned to the
 * exponent of its largest |x| as a 28-bit integer held in four int8 limb
 * planes, each limb plane is multiplied with the row-major int8 weight
 * [n][k] on the tensor cores into int32 accumulators, the four are folded to
 * one exact int64 sum per output and rounded once to fp32
 * (src/rtl/qwen_gemm_array_i.sv header: block-aligned integer sums).
 * k is 896 or 4864, n % 128 == 0. epi: 0 plain, 1 + bias, 2 residual (y
 * in/out), 3 SiLU(gate)*up over interleaved gate/up rows (y [rows][n/2]).
 * The workspace holds the limb planes and exponents; its first 4 bytes become
 * non-zero if a bounded pipeline wait expired. */
size_t qwen_b200_gemm_tc_workspace(uint32_t rows, uint32_t n, uint32_t k);
int qwen_b200_op_gemm_w8a16_tc(const uint16_t *x, uint32_t rows, uint32_t k, const int8_t *w,
                               const float *scale, uint32_t n, const uint16_t *bias, int epi, uint16_t *y,
                               void *workspace, size_t workspace_bytes, void *stream);
/* Host-side cos/sin table [positions][64] (cos 0..31, sin 32..63) for
 * theta_i = 1e6^(-2i/64) (model_backend.py:41). */
void qwen_b200_rope_table(uint32_t positions, float *table);
/* In-place split-half RoPE on x [rows][heads][64] (model_backend.py:73-78;
 * src/rtl/rope/qwen25_rope.v). table: device copy of qwen_b200_rope_table. */
int qwen_b200_op_rope(uint16_t *x, uint32_t rows, uint32_t heads, const uint32_t *positions, const float *table,
                      void *stream);
/* KV8 quantise-append: kv [rows][2][64] bf16 -> codes[slot][2][capacity][64],
 * scales[slot][2][capacity] at positions[r] (scale = amax/127, code =
 * clamp(rne(x/scale), +-127)). */
int qwen_b200_op_kv8_append(const uint16_t *kv, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                            int8_t *codes, float *scales, uint32_t capacity, void *stream);
/* The accelerator's own K cache format (its K16 KV8 path,
 * src/rtl/kv8_k_quant.sv with the K chain's parameters and the 256-token
 * block lock of src/rtl/kv8_k_write_chain.sv:503-600), as an alternative
 * cache format for RTL numeric parity: k [rows][2][64] bf16 (post-RoPE) of
 * rows at positions[r] < capacity of slot slots[r] -> two int8 code planes
 * hi, lo [slot][2][capacity][64] (k ~ (256 hi + lo) * m * 2^(lock - 142)),
 * 16-bit mantissas m16 [slot][2][capacity] and the block exponent locks
 * lock [slot][2][ceil(capacity / 256)], set by each block's first token. A
 * call may hold a block's later tokens only if its first token is in the same
 * call or was appended before. Integer arithmetic, bit-identical to the
 * oracle's restatement. */
int qwen_b200_op_k16_append(const uint16_t *k, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                            int8_t *hi, int8_t *lo, uint16_t *m16, uint8_t *lock, uint32_t capacity, void *stream);
/* The accelerator's own V cache format (its KV8 V path, src/rtl/kv8_v_quant.sv
 * at the V chain's margin 2, src/rtl/storage/qwen25_qkv_controller.v:1951,
 * with the layer lock of src/rtl/kv8_v_write_chain.sv:387-468), the partner
 * of qwen_b200_op_k16_append: v [rows][2][64] bf16 of rows at positions[r] <
 * capacity of slot slots[r] -> int8 codes [slot][2][capacity][64], 8-bit
 * per-token mantissas m8 [slot][2][capacity] and the layer's exponent lock
 * lock [slot][2] (v ~ code * m * 2^(lock - 134)). The lock is set by the
 * slot's token at position 0 (the RTL restarts it at a request's token 0);
 * later tokens need it set, in the same call or before (a later token whose
 * lock is still 0 is quantised as a first token and sets nothing). Integer
 * arithmetic, bit-identical to the oracle's restatement. */
int qwen_b200_op_v8_append(const uint16_t *v, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                           int8_t *codes, uint8_t *m8, uint8_t *lock, uint32_t capacity, void *stream);
/* Fused attention block input: RMSNorm + QKV GEMM + bias + RoPE + KV8 append.
 * x [rows][896]; w [1152][896] (q|k|v rows); q_out [rows][896] post-RoPE. */
int qwen_b200_op_qkv(const uint16_t *x, uint32_t rows, const uint16_t *gamma, float eps, const int8_t *w,
                     const float *scale, const uint16_t *bias, const uint32_t *slots, const uint32_t *positions,
                     const float *table, uint16_t *q_out, int8_t *kcodes, float *kscales, int8_t *vcodes,
                     float *vscales, uint32_t capacity, void *stream);
/* GQA attention over a KV8 cache (model_backend.py:97-102; src/rtl/attention/
 * qwen25_attention.v): q [rows][14][64]; row r of slot slots[r] sees keys
 * 0..positions[r]; ctx [rows][896]. Workspace from qwen_b200_attention_workspace. */
size_t qwen_b200_attention_workspace(uint32_t rows, uint32_t capacity);
/* max_len: an upper bound of positions[r] + 1 over all rows (capacity is
 * always valid; a tight bound launches fewer context chunks). */
int qwen_b200_op_attention(const uint16_t *q, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                           uint32_t max_len, const int8_t *kcodes, const float *kscales, const int8_t *vcodes,
                           const float *vscales, uint32_t capacity, uint16_t *ctx, void *workspace,
                           size_t workspace_bytes, void *stream);
/* Attention without any device allocation. This entry point has no
 * counterpart in the reference. It is for callers that cannot call cudaMalloc
 * at the point they run attention: hosts that hand every byte of the GPU to
 * their own memory pool up front (as the reference's firmware works inside
 * fixed DDR windows, src/verification/board_parameters.h), code whose
 * latency budget does not allow the implicit device synchronisation that
 * cudaMalloc / cudaFree can cause, and plugins that do not own the process's
 * allocator. Instead of a caller workspace it uses one fixed scratch array of
 * QWEN_B200_NOALLOC_SCRATCH_BYTES per GPU, built into the library: every GPU
 * that loads the library holds it until the process exits. Requests whose
 * scratch need, qwen_b200_attention_workspace(rows, capacity), exceeds that
 * size are rejected with QWEN_B200_ESCRATCH before anything is launched (for
 * example 64 rows at capacity 2048 fit; 64 rows at capacity 8192 do not).
 * The first call on each device looks up the scratch's device address with
 * that device current; make that first call before any stream capture. The
 * address is remembered per device and CUDA context: a call in a new context
 * (after cudaDeviceReset, or with another driver context made current on the
 * device) looks it up again, so that call too should come before any
 * capture. All
 * calls on a device share the one array and it keeps the last call's
 * contents: each call zeroes the parts that must start at zero, but calls
 * whose executions overlap on the GPU (different streams, or different host
 * threads) race on it and must be serialised by the caller. No cudaMalloc,
 * cudaFree or allocating library routine is called. Arguments and result
 * are those of qwen_b200_op_attention. */
#define QWEN_B200_NOALLOC_SCRATCH_BYTES (16u << 20)
int qwen_b200_op_attention_noalloc(const uint16_t *q, uint32_t rows, const uint32_t *slots,
                                   const uint32_t *positions, uint32_t max_len, const int8_t *kcodes,
                                   const float *kscales, const int8_t *vcodes, const float *vscales,
                                   uint32_t capacity, uint16_t *ctx, void *stream);
/* The same attention in one launch with no workspace (the form the engine
 * uses): one CTA, or a thread-block cluster of up to 16 splitting the
 * context, per (row, KV head); both products run on the tensor cores and the
 * clusters exchange the softmax statistics and partial contexts over
 * distributed shared memory; results are independent of scheduling. Rows of
 * up to 8 x 2304 keys (16 x 2304 for small batches, where the GPU places a
 * 16-CTA cluster) keep each lane's scores in its own shared-memory words (a
 * 12-warp CTA), others a 4-warp CTA with a shared score array.
 * max_len <= 32768 (the model's context limit); q, kcodes, vcodes 16-byte
 * aligned, ctx 8-byte aligned (QWEN_B200_EINVAL otherwise). */
int qwen_b200_op_attention_cluster(const uint16_t *q, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                                   uint32_t max_len, const int8_t *kcodes, const float *kscales, const int8_t *vcodes,
                                   const float *vscales, uint32_t capacity, uint16_t *ctx, void *stream);
/* Attention of the prefill rows of one sequence, query tiles on the tensor
 * cores (the engine's form for prompt chunks of 16 rows and more): rows
 * r = 0 .. rows-1 are positions pos0 + r (each sees keys 0 .. pos0 + r), q
 * [rows][14][64] post-RoPE, the sequence's KV8 cache of this layer kcodes /
 * vcodes [2][capacity][64], kscales / vscales [2][capacity] with the rows' own
 * keys already appended; ctx [rows][896]. Query tiles of 4 rows x 7 heads
 * score against 128-key chunks with tcgen05.mma (kind::i8), and the context
 * is a second tcgen05 product of the softmax weights' byte planes with the V
 * codes; a cluster of up to 8 CTAs splits a prefix, so pos0 + rows <= 8192.
 * Bit-identical to qwen_b200_op_attention_cluster. Workspace from
 * qwen_b200_attention_prefill_workspace (zeroed once: its first 4 bytes
 * become non-zero if a bounded wait expired); the call synchronises the
 * stream. */
size_t qwen_b200_attention_prefill_workspace(uint32_t rows);
int qwen_b200_op_attention_prefill(const uint16_t *q, uint32_t rows, uint32_t pos0, const int8_t *kcodes,
                                   const float *kscales, const int8_t *vcodes, const float *vscales, uint32_t capacity,
                                   uint16_t *ctx, void *workspace, size_t workspace_bytes, void *stream);
/* SwiGLU FFN input half: mid = bf16(bf16(silu(g)) * u) with g, u from
 * RMSNorm(x) (gamma NULL: no norm) times the interleaved gate/up weight
 * w_gu [2*4864][896] (row 2j gate j, row 2j+1 up j) and scales s_gu [2*4864]
 * (model_backend.py:104-106; AFU op 13, qwen25_afu.v:81,172-180). */
int qwen_b200_op_swiglu(const uint16_t *x, uint32_t rows, const uint16_t *gamma, float eps, const int8_t *w_gu,
                        const float *s_gu, uint16_t *mid, void *stream);
/* Final RMSNorm (gamma NULL: none) + LM head + greedy argmax, highest index on
 * ties (model_backend.py:108-114; qwen25_bf16_argmax.v). logits (nullable)
 * [rows][vocab] bf16. Workspace from qwen_b200_lm_head_workspace. */
size_t qwen_b200_lm_head_workspace(uint32_t rows, uint32_t vocab);
int qwen_b200_op_lm_head_argmax(const uint16_t *x, uint32_t rows, const uint16_t *gamma, float eps,
                                const int8_t *w, const float *scale, uint32_t vocab, uint16_t *logits,
                                uint32_t *tokens, void *workspace, size_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif
#endif
