// Host-side launchers of the sm_100a kernels. Every launcher enqueues on the
// given stream and returns 0 or a QWEN_B200_* status (-1 bad shape, -3 CUDA).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

namespace qb {

enum Epi { EPI_PLAIN = 0, EPI_BIAS = 1, EPI_RESIDUAL = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4 };

// y = epi(bf16(bf16(norm?(x) W^T) * scale)); W int8 row-major [n][k].
// EPI_SWIGLU: W holds interleaved gate/up rows, y is [rows][n/2].
// gamma != nullptr fuses the RMSNorm prologue (k must be 896).
int launch_gemv(int epi, const uint16_t *x, int rows, int k, const uint16_t *gamma, float eps, const int8_t *w,
                const float *scale, const uint16_t *bias, int n, uint16_t *y, cudaStream_t st);

// RMSNorm + QKV + bias + RoPE + KV8 append (one CTA per 64-row head block).
struct QkvArgs {
    const uint16_t *x;
    int rows;
    const uint16_t *gamma;
    float eps;
    const int8_t *w;       // [1152][896]
    const float *scale;    // [1152]
    const uint16_t *bias;  // [1152]
    const uint32_t *slots, *positions;
    const float *table;    // [capacity][64]
    uint16_t *q_out;       // [rows][896]
    int8_t *kc, *vc;       // [slots][2][cap][64]
    float *ks, *vs;        // [slots][2][cap]
    int cap;
    uint16_t *kv_out;      // nullable [rows][256]: post-RoPE k (128) | v (128), bf16
};
int launch_qkv(const QkvArgs &a, cudaStream_t st);

// Persistent batch-1 decode step (decode1.cu): every layer, the LM head and
// the argmax in one cooperative launch of one CTA per SM.
#define QB_NL 24
#define QB_D1_MAX_KEYS 1024  // context keys held in shared memory by the attention phase
// Default limit of the persistent path: beyond about 100 keys its attention
// phase (two CTAs) is slower than the per-kernel path (measured single-row
// step, host timed: 0.76 against 0.85 ms at 65 keys, 0.91 against 0.85 at
// 128, 3.02 against 0.92 at 1001).
#define QB_D1_AUTO_KEYS 96
struct D1Layer {
    const int8_t *qkv, *o, *gu, *d;
    const float *s_qkv, *s_o, *s_gu, *s_d;
    const uint16_t *bias, *g_attn, *g_ffn;
};
struct D1Args {
    const D1Layer *layers;  // [24], device memory
    const int8_t *lmw;
    const float *s_lm;
    const uint16_t *g_final;
    const float *rope;                 // [capacity][64]
    int8_t *kc, *vc;                   // layer 0 of [layer][slot][2][cap][64]
    float *ks, *vs;                    // layer 0 of [layer][slot][2][cap]
    size_t codes_per_layer, scales_per_layer;
    int cap;
    const uint32_t *meta;              // ids | slots | positions of the row (n = 1)
    const uint16_t *embed;             // [151936][896]: layer 0 reads the token's row itself
    const uint32_t *tok_in;            // nullable: a device-resident step, token tok_in[0] in slot 0 at
    uint32_t *slot_pos;                // position slot_pos[0], which the launch advances (else meta)
    uint16_t *x, *qkv, *ctx, *mid;     // [896] residual, [1152], [896], [4864]
    uint16_t *logits;                  // nullable [151936]
    uint32_t *tokens;                  // [1]
    float *cand_v;                     // [grid] per-CTA best value
    uint32_t *cand_i;                  // [grid] per-CTA best index
    unsigned *bar;                     // [0] arrivals, [1] launches: monotonic, zeroed once
    unsigned *err;                     // error flag of the bounded waits
    float eps;
    // test switch (host-set): the last grid barrier waits for one arrival
    // more than the grid makes, with a short limit, so that bounded wait
    // expires (code 20) with nothing asynchronous in flight
    int expire_last_barrier;
};
// max_len within [1, limit] (limit <= QB_D1_MAX_KEYS) and a grid of enough SMs.
int decode1_supported(int max_len, int limit = QB_D1_MAX_KEYS);
size_t decode1_smem_bytes();
int launch_decode1(const D1Args &a, cudaStream_t st);

// Final RMSNorm + LM head + argmax. part: [rows][nblocks] (value, index).
size_t lm_head_workspace(int rows, int vocab);
// n_base is added to every reported index (w, scale and logits are those of
// the rows [n_base, n_base + vocab) of a larger head); values (nullable)
// receives each row's best logit.
int launch_lm_head(const uint16_t *x, int rows, const uint16_t *gamma, float eps, const int8_t *w,
                   const float *scale, int vocab, uint16_t *logits, uint32_t *tokens, void *ws, size_t ws_bytes,
                   cudaStream_t st, int n_base = 0, float *values = nullptr, unsigned *err = nullptr);

// Attention over a KV8 cache (two passes + last-block combine). The
// workspace is laid out for ws_rows rows (>= rows); its completion counters
// must be zero before the first launch and are left zero by every launch
// (clear_counters zeroes them first).
size_t attention_workspace(int rows, int cap);
int launch_attention(const uint16_t *q, int rows, const uint32_t *slots, const uint32_t *positions, int max_len,
                     const int8_t *kc, const float *ks, const int8_t *vc, const float *vs, int cap, uint16_t *ctx,
                     void *ws, size_t ws_bytes, int ws_rows, bool clear_counters, cudaStream_t st);

// Single-launch attention: one thread-block cluster per (row, KV head) over
// the row's context; no workspace. max_len <= 32768; q, kc, vc 16-byte and ctx
// 8-byte aligned. A bounded wait that expires records code 11/12 in *err (a
// library-internal flag when err is null). klo (nullable, 16-byte aligned):
// the low planes of 16-bit K codes (the accelerator's K16 format: the code
// of a dim is 256 * kc + klo); such calls always take this kernel.
int launch_attention_cluster(const uint16_t *q, int rows, const uint32_t *slots, const uint32_t *positions,
                             int max_len, const int8_t *kc, const float *ks, const int8_t *vc, const float *vs, int cap,
                             uint16_t *ctx, unsigned *err, cudaStream_t st, const int8_t *klo = nullptr);
// The same attention with transposed tensor-core scores kept lane-private in
// shared memory (attention_rs.cu: CTAs of 12 warps, up to 8 per row for
// long contexts); 0 when launched, 1 when a row needs more than 8 CTAs (the
// caller then uses the kernel above), negative on a launch error.
int launch_attention_rs(const uint16_t *q, int rows, const uint32_t *slots, const uint32_t *positions, int max_len,
                        const int8_t *kc, const float *ks, const int8_t *vc, const float *vs, int cap, uint16_t *ctx,
                        unsigned *err, cudaStream_t st);

int launch_embed(const uint16_t *embed, const uint32_t *ids, int rows, uint16_t *x, cudaStream_t st);
int launch_rmsnorm(const uint16_t *x, const uint16_t *gamma, int rows, float eps, uint16_t *out, cudaStream_t st);
// Activation rows as the int8 limb planes of their 28-bit alignment (the
// operand of the exact tensor-core projections): limbs[l][row][k] at
// l * plane + row * ld + k, exponent ex[row]. The RMSNorm variant also writes
// the bf16 row to out unless out is null.
int launch_rmsnorm_limbs(const uint16_t *x, const uint16_t *gamma, int rows, float eps, uint16_t *out,
                         int8_t *limbs, size_t plane, int ld, int *ex, cudaStream_t st);
int launch_act_quant(const uint16_t *x, int rows, int k, int8_t *limbs, size_t plane, int ld, int *ex,
                     cudaStream_t st);
int launch_rope(uint16_t *x, int rows, int heads, const uint32_t *positions, const float *table, cudaStream_t st);
int launch_kv8_append(const uint16_t *kv, int rows, const uint32_t *slots, const uint32_t *positions, int8_t *codes,
                      float *scales, int cap, cudaStream_t st);
int launch_gather_rows(const uint16_t *x, const uint32_t *rows_idx, int n, uint16_t *out, cudaStream_t st);
// Decode-step bookkeeping for slots 0..n-1: ids/slots/positions from the
// device position table, and the table's advance after the step.
int launch_decode_prologue(const uint32_t *tokens_in, int n, const uint32_t *slot_pos, uint32_t *ids,
                           uint32_t *slots, uint32_t *positions, cudaStream_t st);
int launch_decode_epilogue(int n, uint32_t *slot_pos, cudaStream_t st);
// The accelerator's own K cache format (kv8_rtl.cu): hi/lo code planes
// [slot][2][cap][64], 16-bit mantissas [slot][2][cap], one exponent lock per
// 256-token block [slot][2][ceil(cap / 256)].
int launch_k16_append(const uint16_t *k, int rows, const uint32_t *slots, const uint32_t *positions, int8_t *hi,
                      int8_t *lo, uint16_t *m16, uint8_t *lock, int cap, cudaStream_t st);
// Query-tiled prefill attention (attention_tile.cu): a tile is up to 4
// consecutive positions of one slot (row0: its first row in q / ctx); tiles
// are grouped by the number of 1024-key CTAs their prefix needs (splits),
// each group one launch of clusters of that size. The K codes are read
// through kmap, a 2D tensor map of [rows][64] int8 (64-byte swizzle, box
// 128 rows) in which key t of (slot, KV head g) is row krow0 + (slot * 2 + g)
// * cap + t.
struct AtTile {
    int row0, nq, slot, pos0;
};
struct AtGroup {
    int splits, kpc, first, count;
};
int attention_tile_plan(int rows, const uint32_t *slots, const uint32_t *positions, AtTile *tiles,
                        std::vector<AtGroup> &groups);
int launch_attention_tiles(const CUtensorMap &kmap, long long krow0, const AtTile *d_tiles, const AtGroup &grp,
                           const uint16_t *q, const int8_t *vc, const float *ks, const float *vs, int cap,
                           uint16_t *ctx, unsigned *err, cudaStream_t st);
int make_kcache_map(CUtensorMap *map, const int8_t *kc, long long rows);
// The engine's RTL KV mode (kv8_rtl.cu): kv [rows][256] post-RoPE k | v (bf16)
// appended in the accelerator's K16 and V formats into one layer's caches:
// kc / klo the high / low K planes, ks = m16 * 2^(lock - 142), vc, vs = m8 *
// 2^(lock - 134); klock [slot][2][ceil(cap / 256)], vlock [slot][2].
int launch_rtl_kv_append(const uint16_t *kv, int rows, const uint32_t *slots, const uint32_t *positions, int8_t *kc,
                         int8_t *klo, float *ks, uint8_t *klock, int8_t *vc, float *vs, uint8_t *vlock, int cap,
                         cudaStream_t st);
// The accelerator's own V cache format (kv8_rtl.cu): codes [slot][2][cap][64],
// per-token mantissas m8 [slot][2][cap], layer locks [slot][2].
int launch_v8_append(const uint16_t *v, int rows, const uint32_t *slots, const uint32_t *positions, int8_t *codes,
                     uint8_t *m8, uint8_t *lock, int cap, cudaStream_t st);
// Seeded synthetic KV8 contents for positions [0, length) of one slot, all layers.
int launch_fill_kv(int8_t *kc, float *ks, int8_t *vc, float *vs, int layers, int nslots, int slot, int cap,
                   int length, uint64_t seed, cudaStream_t st);

// ---- tcgen05 exact W8A16 GEMM (rows > 8): row-major int8 weights [n][k] by
// TMA times the int8 limb planes of the activation rows (see
// launch_rmsnorm_limbs / launch_act_quant) -> exact int32/int64 sums.
struct TcArgs {
    const float *scale;
    const uint16_t *bias;
    uint16_t *y;
    const int *ex;  // row exponents of the activation limbs
    int M, N, K, kc_per_split, splits;
    unsigned *err;
    long long *part;  // split-K partial tiles [tile][split][64 rows][128 channels] (splits > 1)
    float *pv;
    uint32_t *pi;
    int nblk;
    uint16_t *logits;
    int n_base;  // LM head: first row of the weight map this launch covers
};
struct TcArgmax {
    float *pv;
    uint32_t *pi;
    int nblk;         // = n / 128 partial candidates per row
    uint16_t *logits; // nullable [rows][n]
    int n_base = 0;   // the n channels are rows [n_base, n_base + n) of the weight map
};
// Tensor maps: weights [n][k] int8 row-major; limbs[l][row][k] with planes
// `plane` bytes apart, rows `ld` bytes apart, rows_alloc rows.
int make_weight_map(CUtensorMap *map, const int8_t *w, int n, int k);
int make_limb_map(CUtensorMap *map, const int8_t *limbs, int rows_alloc, int ld, size_t plane, int k);
int tc_pick_splits(int rows, int n, int k);
// Workspace: a 256-byte error flag (zero before the first launch; clear
// zeroes it first).
size_t tc_gemm_workspace(int rows, int n, int splits);
int launch_gemm_tc(int epi, const CUtensorMap &wmap, const CUtensorMap &lmap, const int *ex, int rows, int k,
                   const float *scale, const uint16_t *bias, int n, uint16_t *y, int splits, void *ws,
                   size_t ws_bytes, bool clear, const TcArgmax *am, cudaStream_t st);
int launch_argmax_reduce(const float *pv, const uint32_t *pi, int rows, int nblk, uint32_t *tokens, cudaStream_t st,
                         float *values = nullptr);
// RoPE + KV8 append for the q|k|v rows produced by the tensor-core QKV GEMM
// (qkv [rows][1152], bias already added).
int launch_rope_kv8(const uint16_t *qkv, int rows, const uint32_t *slots, const uint32_t *positions,
                    const float *table, uint16_t *q_out, int8_t *kc, float *ks, int8_t *vc, float *vs, int cap,
                    uint16_t *kv_out, cudaStream_t st);

}  // namespace qb
