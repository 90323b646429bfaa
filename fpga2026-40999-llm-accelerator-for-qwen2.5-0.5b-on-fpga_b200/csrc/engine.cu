// libqwen_b200 host engine: owns the device copy of the model and the KV8
// caches, sequences the per-layer kernels (the role of the PL's layer FSM,
// src/rtl/storage/qwen25_qkv_controller.v:123-136), emulates the CSR protocol
// of src/software/generation.c:5-39 and exports the C ABI of qwen_b200.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "assets.h"
#include "common.cuh"
#include "kernels.h"
#include "qwen_b200.h"

using namespace qb;

namespace {

constexpr int NL = QWEN_B200_LAYERS;
constexpr int HID = QWEN_B200_HIDDEN;
constexpr int FFN = QWEN_B200_FFN;
constexpr int VOC = QWEN_B200_VOCAB;
constexpr int QKVN = QWEN_B200_QKV;
constexpr int CSR_IDS = 256;  // ACT_IN rows addressable through the embedding callback

struct LayerW {
    int8_t *qkv, *o, *gu, *d;  // [1152][896], [896][896], [9728][896] gate/up interleaved, [896][4864]
    CUtensorMap mqkv, mo, mgu, md;  // tensor maps of the same weights for the tensor-core GEMM
    float *s_qkv, *s_o, *s_gu, *s_d;
    uint16_t *bias, *g_attn, *g_ffn;
};

// Rows at or above which a step uses the tcgen05 GEMMs instead of the GEMVs.
// The GEMV family's integer work grows with every row (four limb planes per
// row and weight word) and it streams the weights once per 4-row tile, while
// the tensor-core step costs the same from 1 to 64 rows: batched decode steps
// at 500-key contexts measured 1.26 / 2.18 / 2.76 ms with GEMVs at 2 / 4 / 8
// rows against 1.18 ms at 16 rows on the tensor cores (0.86 ms for one row
// with GEMVs). Single rows keep the GEMVs (and the persistent kernel).
constexpr int TC_MIN_ROWS = 2;

enum CsrState { CSR_IDLE = 0, CSR_BUSY = 1, CSR_DONE = 2, CSR_ERROR = 3 };

}  // namespace

struct qwen_b200 {
    qwen_b200_config cfg{};
    std::string err;
    bool loaded = false;
    int R = 0;  // activation rows
    cudaStream_t stream = nullptr, cap_stream = nullptr;
    std::vector<void *> dev_allocs;
    // model
    LayerW L[NL];
    uint16_t *g_final = nullptr, *embed = nullptr;
    int8_t *lmw = nullptr;
    CUtensorMap mlm;
    float *s_lm = nullptr, *rope = nullptr;
    // KV8 caches: codes [layer][slot][2][cap][64], scales [layer][slot][2][cap]
    int8_t *kc = nullptr, *vc = nullptr;
    float *ks = nullptr, *vs = nullptr;
    // QWEN_B200_FLAG_RTL_KV: low K planes (layout of kc), K block locks
    // [layer][slot][2][nblk], V layer locks [layer][slot][2], and the
    // post-RoPE k | v rows [R][256] the append reads
    bool rtl = false;
    int8_t *klo = nullptr;
    uint8_t *klock = nullptr, *vlock = nullptr;
    uint16_t *rtl_kv = nullptr;
    // query-tiled prefill attention: the K caches of all layers as one tensor
    // map, and the tile plan of the forward being enqueued (host staging,
    // device copy, launch groups)
    CUtensorMap kmap;
    bool kmap_ok = false;
    AtTile *d_tiles = nullptr, *h_tiles = nullptr;
    std::vector<AtGroup> tgroups;
    bool tplan = false;
    // activations
    uint16_t *x = nullptr, *q = nullptr, *ctx = nullptr, *mid = nullptr, *xl = nullptr, *logits = nullptr;
    uint16_t *blogits = nullptr;  // [R][vocab] logits of batched steps that return them
    uint16_t *hn = nullptr, *qkvb = nullptr;  // normalised rows / q|k|v rows of the tensor-core path
    void *tc_ws = nullptr;                    // error flags of the bounded waits
    size_t tc_ws_bytes = 0;
    // activation rows as int8 limb planes [4][R][4864] and row exponents [R]
    // (operand of the tensor-core projections), with their tensor maps for
    // k = 896 and k = 4864
    int8_t *limbs = nullptr;
    int *lex = nullptr;
    size_t limb_plane = 0;
    CUtensorMap lmap_hid, lmap_ffn;
    uint32_t *meta = nullptr;  // [4][R]: ids | slots | positions | logit rows
    // persistent batch-1 decode: per-layer pointers, barrier counter and the
    // per-CTA argmax candidates
    int persistent = 1;  // 0 per-kernel, 1 persistent up to QB_D1_AUTO_KEYS keys, 2 up to QB_D1_MAX_KEYS
    bool expire_wait = false;  // test switch: the persistent step's last barrier times out
    D1Layer *d1_layers = nullptr;
    unsigned *d1_bar = nullptr;
    float *d1_cand_v = nullptr;
    uint32_t *d1_cand_i = nullptr;
    uint32_t *tokens = nullptr, *slot_pos = nullptr;
    void *lm_ws = nullptr;
    size_t lm_ws_bytes = 0;
    // pinned staging
    uint32_t *h_meta = nullptr, *h_tokens = nullptr, *h_slot_pos = nullptr, *h_flag = nullptr;
    std::vector<uint32_t> pos;  // host mirror of every slot's position
    // decode graphs keyed by (n, context bucket, tokens_in, tokens_out)
    std::map<std::tuple<uint32_t, uint32_t, const void *, const void *>, cudaGraphExec_t> graphs;
    // host-buffer decode steps: the forward over the staged ids / slots /
    // positions, keyed by (n, context bucket), with its launch count
    std::map<std::pair<uint32_t, uint32_t>, std::pair<cudaGraphExec_t, uint32_t>> host_graphs;
    // layer dump (tests): device buffers and host destinations
    int dump_layer = -1;
    uint16_t *dump_host[7] = {};
    uint16_t *d_dump = nullptr;  // [R][896 q | 256 kv | 896 ctx | 896 h | 4864 mid | 896 y]
    // per-kernel-class CUDA events (profiled steps) and the launch count of the
    // last enqueued step
    bool prof = false;
    std::vector<cudaEvent_t> prof_ev[QWEN_B200_KCLASSES];
    size_t prof_used[QWEN_B200_KCLASSES] = {};
    uint32_t nlaunch = 0;
    // CSR protocol state (slot 0)
    uint64_t regs[128] = {};
    uint32_t csr_ids[CSR_IDS] = {};
    int csr_state = CSR_IDLE;
    uint64_t csr_error = 0;
    uint32_t csr_token = 0;
    cudaEvent_t csr_event = nullptr;
    cudaEvent_t staged = nullptr;  // the last host->device copy out of h_meta has been read
};

namespace {

int fail(qwen_b200 *h, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    h->err = buf;
    return code;
}

#define CK(call)                                                                                       \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess) return fail(h, QWEN_B200_EDEVICE, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)
#define RK(call)                                                                           \
    do {                                                                                   \
        int r_ = (call);                                                                   \
        if (r_) return fail(h, r_, "%s failed (%d): %s", #call, r_, cudaGetErrorString(cudaGetLastError())); \
    } while (0)

int dalloc(qwen_b200 *h, void **p, size_t bytes) {
    if (cudaMalloc(p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(h, QWEN_B200_ENOMEM, "cudaMalloc(%zu) failed", bytes);
    }
    h->dev_allocs.push_back(*p);
    return 0;
}

// Brackets one kernel launch of class c with a pair of events on stream st
// when a profiled step is running; counts launches either way.
struct LaunchScope {
    qwen_b200 *h;
    int c;
    cudaStream_t st;
    LaunchScope(qwen_b200 *h_, int c_, cudaStream_t st_, uint32_t kernels) : h(h_), c(c_), st(st_) {
        h->nlaunch += kernels;
        if (h->prof) record();
    }
    ~LaunchScope() {
        if (h->prof) record();
    }
    void record() {
        auto &pool = h->prof_ev[c];
        if (h->prof_used[c] == pool.size()) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            pool.push_back(e);
        }
        cudaEventRecord(pool[h->prof_used[c]++], st);
        pdl_break();
    }
};

constexpr size_t DUMP_COLS = 896 + 256 + 896 + 896 + 4864 + 896;

size_t kv_layer_codes(const qwen_b200 *h) { return (size_t)h->cfg.max_seqs * 2 * h->cfg.max_context * 64; }
size_t kv_layer_scales(const qwen_b200 *h) { return (size_t)h->cfg.max_seqs * 2 * h->cfg.max_context; }
// Context bucket of a captured decode step (the upper bound of its longest
// row's keys that the graph was recorded for): 64 keys, within which a
// single-row step takes the persistent kernel, then multiples of 128.
uint32_t context_bucket(uint32_t max_len) { return max_len <= 64 ? 64u : (max_len + 127) / 128 * 128; }
size_t rtl_klock_layer(const qwen_b200 *h) { return (size_t)h->cfg.max_seqs * 2 * ((h->cfg.max_context + 255) / 256); }

int allocate(qwen_b200 *h) {
    const qwen_b200_config &c = h->cfg;
    h->R = (int)std::max(c.max_rows, c.max_seqs);
    const size_t R = (size_t)h->R;
    CK(cudaSetDevice(c.device));
    CK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&h->cap_stream, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&h->csr_event, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&h->staged, cudaEventDisableTiming));
    void *p;
    int rc;
    // weights: one block per layer
    const size_t lw = (size_t)QKVN * HID + (size_t)HID * HID + (size_t)2 * FFN * HID + (size_t)HID * FFN;
    if ((rc = dalloc(h, &p, lw * NL))) return rc;
    for (int l = 0; l < NL; ++l) {
        int8_t *b = (int8_t *)p + lw * l;
        h->L[l].qkv = b;
        h->L[l].o = b + (size_t)QKVN * HID;
        h->L[l].gu = h->L[l].o + (size_t)HID * HID;
        h->L[l].d = h->L[l].gu + (size_t)2 * FFN * HID;
    }
    for (int l = 0; l < NL; ++l) {
        LayerW &W = h->L[l];
        if (make_weight_map(&W.mqkv, W.qkv, QKVN, HID) || make_weight_map(&W.mo, W.o, HID, HID) ||
            make_weight_map(&W.mgu, W.gu, 2 * FFN, HID) || make_weight_map(&W.md, W.d, HID, FFN))
            return fail(h, QWEN_B200_EDEVICE, "cannot encode the weight tensor maps");
    }
    const size_t ls = QKVN + HID + 2 * FFN + HID;
    if ((rc = dalloc(h, &p, ls * NL * sizeof(float)))) return rc;
    for (int l = 0; l < NL; ++l) {
        float *b = (float *)p + ls * l;
        h->L[l].s_qkv = b;
        h->L[l].s_o = b + QKVN;
        h->L[l].s_gu = h->L[l].s_o + HID;
        h->L[l].s_d = h->L[l].s_gu + 2 * FFN;
    }
    const size_t lb = QKVN + 2 * HID;
    if ((rc = dalloc(h, &p, (lb * NL + HID) * 2))) return rc;
    for (int l = 0; l < NL; ++l) {
        uint16_t *b = (uint16_t *)p + lb * l;
        h->L[l].bias = b;
        h->L[l].g_attn = b + QKVN;
        h->L[l].g_ffn = b + QKVN + HID;
    }
    h->g_final = (uint16_t *)p + lb * NL;
    if ((rc = dalloc(h, (void **)&h->embed, (size_t)VOC * HID * 2))) return rc;
    if ((rc = dalloc(h, (void **)&h->lmw, (size_t)VOC * HID))) return rc;
    if (make_weight_map(&h->mlm, h->lmw, VOC, HID)) return fail(h, QWEN_B200_EDEVICE, "cannot encode the LM-head map");
    if ((rc = dalloc(h, (void **)&h->s_lm, (size_t)VOC * 4))) return rc;
    if ((rc = dalloc(h, (void **)&h->rope, (size_t)c.max_context * 64 * 4))) return rc;
    // KV8 caches
    if ((rc = dalloc(h, (void **)&h->kc, kv_layer_codes(h) * NL))) return rc;
    if ((rc = dalloc(h, (void **)&h->vc, kv_layer_codes(h) * NL))) return rc;
    if ((rc = dalloc(h, (void **)&h->ks, kv_layer_scales(h) * NL * 4))) return rc;
    if ((rc = dalloc(h, (void **)&h->vs, kv_layer_scales(h) * NL * 4))) return rc;
    CK(cudaMemset(h->kc, 0, kv_layer_codes(h) * NL));
    CK(cudaMemset(h->vc, 0, kv_layer_codes(h) * NL));
    CK(cudaMemset(h->ks, 0, kv_layer_scales(h) * NL * 4));
    CK(cudaMemset(h->vs, 0, kv_layer_scales(h) * NL * 4));
    h->kmap_ok = make_kcache_map(&h->kmap, h->kc, (long long)(kv_layer_codes(h) / 64) * NL) == 0;
    if ((rc = dalloc(h, (void **)&h->d_tiles, R * sizeof(AtTile)))) return rc;
    CK(cudaMallocHost((void **)&h->h_tiles, R * sizeof(AtTile)));
    if (h->rtl) {
        if ((rc = dalloc(h, (void **)&h->klo, kv_layer_codes(h) * NL))) return rc;
        if ((rc = dalloc(h, (void **)&h->klock, rtl_klock_layer(h) * NL))) return rc;
        if ((rc = dalloc(h, (void **)&h->vlock, (size_t)c.max_seqs * 2 * NL))) return rc;
        if ((rc = dalloc(h, (void **)&h->rtl_kv, R * 256 * 2))) return rc;
        CK(cudaMemset(h->klo, 0, kv_layer_codes(h) * NL));
        CK(cudaMemset(h->klock, 0, rtl_klock_layer(h) * NL));
        CK(cudaMemset(h->vlock, 0, (size_t)c.max_seqs * 2 * NL));
    }
    // activations
    if ((rc = dalloc(h, (void **)&h->x, R * HID * 2))) return rc;
    if ((rc = dalloc(h, (void **)&h->q, R * HID * 2))) return rc;
    if ((rc = dalloc(h, (void **)&h->ctx, R * HID * 2))) return rc;
    if ((rc = dalloc(h, (void **)&h->mid, R * FFN * 2))) return rc;
    if ((rc = dalloc(h, (void **)&h->xl, R * HID * 2))) return rc;
    if ((rc = dalloc(h, (void **)&h->hn, R * HID * 2))) return rc;
    if ((rc = dalloc(h, (void **)&h->qkvb, R * QKVN * 2))) return rc;
    h->limb_plane = R * FFN;
    if ((rc = dalloc(h, (void **)&h->limbs, 4 * h->limb_plane))) return rc;
    if ((rc = dalloc(h, (void **)&h->lex, R * 4))) return rc;
    if (make_limb_map(&h->lmap_hid, h->limbs, h->R, FFN, h->limb_plane, HID) ||
        make_limb_map(&h->lmap_ffn, h->limbs, h->R, FFN, h->limb_plane, FFN))
        return fail(h, QWEN_B200_EDEVICE, "cannot encode the limb tensor maps");
    // error word + split-K partial tiles: the split plan keeps tiles x splits
    // within one CTA per SM whenever it splits
    h->tc_ws_bytes = 256 + (size_t)148 * 64 * 128 * 8;
    if ((rc = dalloc(h, &h->tc_ws, h->tc_ws_bytes))) return rc;
    CK(cudaMemset(h->tc_ws, 0, h->tc_ws_bytes));
    if ((rc = dalloc(h, (void **)&h->logits, (size_t)VOC * 2))) return rc;
    if ((rc = dalloc(h, (void **)&h->meta, R * 4 * 4))) return rc;
    if ((rc = dalloc(h, (void **)&h->d1_layers, NL * sizeof(D1Layer)))) return rc;
    if ((rc = dalloc(h, (void **)&h->d1_bar, 256))) return rc;
    CK(cudaMemset(h->d1_bar, 0, 256));  // the persistent launch's arrival and launch counters
    if ((rc = dalloc(h, (void **)&h->d1_cand_v, 1024 * 4))) return rc;
    if ((rc = dalloc(h, (void **)&h->d1_cand_i, 1024 * 4))) return rc;
    if ((rc = dalloc(h, (void **)&h->tokens, R * 4))) return rc;
    if ((rc = dalloc(h, (void **)&h->slot_pos, (size_t)c.max_seqs * 4))) return rc;
    CK(cudaMemset(h->slot_pos, 0, (size_t)c.max_seqs * 4));
    h->lm_ws_bytes = lm_head_workspace(h->R, VOC);
    if ((rc = dalloc(h, &h->lm_ws, h->lm_ws_bytes))) return rc;
    CK(cudaMallocHost((void **)&h->h_meta, R * 4 * 4));
    CK(cudaMallocHost((void **)&h->h_tokens, R * 4));
    CK(cudaMallocHost((void **)&h->h_slot_pos, (size_t)c.max_seqs * 4));
    CK(cudaMallocHost((void **)&h->h_flag, 16));
    h->pos.assign(c.max_seqs, 0);
    std::vector<float> table((size_t)c.max_context * 64);
    qwen_b200_rope_table(c.max_context, table.data());
    CK(cudaMemcpy(h->rope, table.data(), table.size() * 4, cudaMemcpyHostToDevice));
    return 0;
}

int upload(qwen_b200 *h, const qa_model &m) {
    std::vector<int8_t> gu((size_t)2 * FFN * HID), qkv((size_t)QKVN * HID);
    std::vector<float> s(QKVN + HID + 2 * FFN + HID);
    std::vector<uint16_t> b(QKVN + 2 * HID);
    for (int l = 0; l < NL; ++l) {
        memcpy(qkv.data(), m.w[l][QA_Q], (size_t)896 * HID);
        memcpy(qkv.data() + (size_t)896 * HID, m.w[l][QA_K], (size_t)128 * HID);
        memcpy(qkv.data() + (size_t)1024 * HID, m.w[l][QA_V], (size_t)128 * HID);
        for (int j = 0; j < FFN; ++j) {
            memcpy(gu.data() + (size_t)(2 * j) * HID, m.w[l][QA_GATE] + (size_t)j * HID, HID);
            memcpy(gu.data() + (size_t)(2 * j + 1) * HID, m.w[l][QA_UP] + (size_t)j * HID, HID);
        }
        const uint16_t *sc = m.scale + (size_t)l * QA_SCALE_LAYER;
        for (int i = 0; i < QKVN; ++i) s[i] = qa_bf2f(sc[i]);  // q@0 k@896 v@1024
        for (int i = 0; i < HID; ++i) s[QKVN + i] = qa_bf2f(sc[1152 + i]);
        for (int j = 0; j < FFN; ++j) {
            s[QKVN + HID + 2 * j] = qa_bf2f(sc[2048 + j]);
            s[QKVN + HID + 2 * j + 1] = qa_bf2f(sc[6912 + j]);
        }
        for (int i = 0; i < HID; ++i) s[QKVN + HID + 2 * FFN + i] = qa_bf2f(sc[11776 + i]);
        memcpy(b.data(), m.bias + (size_t)l * QA_BIAS_LAYER, QKVN * 2);
        memcpy(b.data() + QKVN, m.gamma + (size_t)l * QA_GAMMA_LAYER, (size_t)2 * HID * 2);
        const LayerW &W = h->L[l];
        CK(cudaMemcpy(W.qkv, qkv.data(), qkv.size(), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(W.o, m.w[l][QA_O], (size_t)HID * HID, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(W.gu, gu.data(), gu.size(), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(W.d, m.w[l][QA_DOWN], (size_t)HID * FFN, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(W.s_qkv, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(W.bias, b.data(), b.size() * 2, cudaMemcpyHostToDevice));
    }
    D1Layer d1[NL];
    for (int l = 0; l < NL; ++l) {
        const LayerW &W = h->L[l];
        d1[l] = D1Layer{W.qkv, W.o, W.gu, W.d, W.s_qkv, W.s_o, W.s_gu, W.s_d, W.bias, W.g_attn, W.g_ffn};
    }
    CK(cudaMemcpy(h->d1_layers, d1, sizeof(d1), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(h->g_final, m.gamma + QA_GAMMA_FINAL, HID * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(h->embed, m.embed, (size_t)VOC * HID * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(h->lmw, m.lmw, (size_t)VOC * HID, cudaMemcpyHostToDevice));
    std::vector<float> slm(VOC);
    for (int i = 0; i < VOC; ++i) slm[i] = qa_bf2f(m.scale[QA_SCALE_LM + i]);
    CK(cudaMemcpy(h->s_lm, slm.data(), (size_t)VOC * 4, cudaMemcpyHostToDevice));
    return 0;
}

int ensure_device(qwen_b200 *h) {
    if (!h->loaded) return fail(h, QWEN_B200_EINVAL, "no assets loaded");
    CK(cudaSetDevice(h->cfg.device));
    return 0;
}

// Exact tensor-core GEMM y = epi(x W^T) for n rows whose limbs are in
// h->limbs (k = 896 or 4864) with exponents h->lex.
int tc_gemm(qwen_b200 *h, int epi, int n, int k, const CUtensorMap &wmap, const float *scale, const uint16_t *bias,
            int nout, uint16_t *y, const TcArgmax *am, cudaStream_t st) {
    const int splits = am ? 1 : tc_pick_splits(n, nout, k);
    RK(launch_gemm_tc(epi, wmap, k == HID ? h->lmap_hid : h->lmap_ffn, h->lex, n, k, scale, bias, nout, y, splits,
                      h->tc_ws, h->tc_ws_bytes, false, am, st));
    return 0;
}

int make_limbs(qwen_b200 *h, const uint16_t *x, int n, int k, cudaStream_t st) {
    RK(launch_act_quant(x, n, k, h->limbs, h->limb_plane, FFN, h->lex, st));
    return 0;
}

int norm_limbs(qwen_b200 *h, const uint16_t *x, const uint16_t *gamma, int n, float eps, cudaStream_t st) {
    RK(launch_rmsnorm_limbs(x, gamma, n, eps, nullptr, h->limbs, h->limb_plane, FFN, h->lex, st));
    return 0;
}

// Reads the error flag that tcgen05 kernels set when a bounded wait expires.
int check_device_flags(qwen_b200 *h) {
    unsigned flag = 0;
    CK(cudaMemcpy(&flag, h->tc_ws, 4, cudaMemcpyDeviceToHost));
    if (flag) {
        cudaMemset(h->tc_ws, 0, 4);
        // a persistent launch that gave up waiting may have left its barrier
        // counters off their launch stride: start them again
        if (h->d1_bar) cudaMemset(h->d1_bar, 0, 256);
        return fail(h, QWEN_B200_ETIMEOUT, "a pipeline wait on the device timed out (code %u)", flag);
    }
    return 0;
}

// Final RMSNorm + LM head over the vocabulary rows [begin, end) + greedy
// argmax (highest index on ties, model_backend.py:108-114) for nlog rows of
// xin: tokens_dst[r] the best global index, values_dst[r] (nullable) its bf16
// logit as fp32, logits_dst (nullable) [nlog][end - begin].
int lm_head_rows(qwen_b200 *h, const uint16_t *xin, int nlog, int begin, int end, uint16_t *logits_dst,
                 uint32_t *tokens_dst, float *values_dst, cudaStream_t st) {
    const float eps = h->cfg.rms_eps;
    const int width = end - begin;
    if (nlog >= TC_MIN_ROWS) {
        LaunchScope ls(h, 6, st, 3);
        int rc = norm_limbs(h, xin, h->g_final, nlog, eps, st);
        if (rc) return rc;
        const int nblk = width / 128;
        TcArgmax am;
        am.pv = reinterpret_cast<float *>(h->lm_ws);
        am.pi = reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(h->lm_ws) + (size_t)nlog * nblk * 4);
        am.nblk = nblk;
        am.logits = logits_dst;
        am.n_base = begin;
        rc = tc_gemm(h, EPI_ARGMAX, nlog, HID, h->mlm, h->s_lm + begin, nullptr, width, nullptr, &am, st);
        if (rc) return rc;
        RK(launch_argmax_reduce(am.pv, am.pi, nlog, nblk, tokens_dst, st, values_dst));
    } else {
        LaunchScope ls(h, 6, st, 2);
        RK(launch_lm_head(xin, nlog, h->g_final, eps, h->lmw + (size_t)begin * HID, h->s_lm + begin, width,
                          logits_dst, tokens_dst, h->lm_ws, h->lm_ws_bytes, st, begin, values_dst,
                          reinterpret_cast<unsigned *>(h->tc_ws)));
    }
    return 0;
}

// Rows per forward chunk from which prompt rows take the query-tiled
// attention (shorter chunks keep the per-row kernels).
constexpr int TILE_MIN_ROWS = 16;

// Plans the query tiles of a forward chunk of m rows (host slots and
// positions) and enqueues the copy of the tile list; the next run_forward
// uses them. Needs the rows' pinned staging to stay untouched until the
// chunk's staging event.
int prepare_tiles(qwen_b200 *h, int m, const uint32_t *slots, const uint32_t *positions, cudaStream_t st) {
    h->tplan = false;
    if (m < TILE_MIN_ROWS || h->rtl || !h->kmap_ok) return 0;
    if (attention_tile_plan(m, slots, positions, h->h_tiles, h->tgroups)) return 0;
    int ntiles = 0;
    for (const AtGroup &g : h->tgroups) ntiles += g.count;
    CK(cudaMemcpyAsync(h->d_tiles, h->h_tiles, (size_t)ntiles * sizeof(AtTile), cudaMemcpyHostToDevice, st));
    h->tplan = true;
    return 0;
}

// One forward over R rows whose ids/slots/positions are at meta[0..3R) with
// stride n (ids n | slots n | positions n | logit rows n). nlog rows get the
// LM head: rows listed at meta+3n, or all rows when identity. Without
// lm_head the nlog rows are only gathered into h->xl (identity false).
// Whether a forward of n rows (max_len keys at most) runs as the persistent
// single-row launch.
static bool uses_decode1(const qwen_b200 *h, int n, int max_len, int nlog, bool identity) {
    const bool dump = h->dump_layer >= 0 && h->d_dump;
    return n == 1 && nlog == 1 && identity && !dump && h->persistent && !h->rtl &&
           decode1_supported(max_len, h->persistent == 1 ? QB_D1_AUTO_KEYS : QB_D1_MAX_KEYS);
}

// tok_in / slot_pos (device-resident single-row steps, uses_decode1 true):
// the persistent launch reads the token and the position itself and advances
// the position, in place of the step's prologue and epilogue kernels.
int run_forward(qwen_b200 *h, int n, int max_len, int nlog, bool identity, uint16_t *logits_dst, uint32_t *tokens_dst,
                cudaStream_t st, bool lm_head = true, const uint32_t *tok_in = nullptr, uint32_t *slot_pos = nullptr) {
    const uint32_t *ids = h->meta, *slots = h->meta + n, *positions = h->meta + 2 * n, *lrows = h->meta + 3 * n;
    const int cap = (int)h->cfg.max_context;
    const float eps = h->cfg.rms_eps;
    const bool dump = h->dump_layer >= 0 && h->d_dump;
    PdlChain chain;  // consecutive kernels of the forward overlap one another
    if (lm_head && uses_decode1(h, n, max_len, nlog, identity)) {
        // one row: the embedding, every layer, the LM head and the argmax in
        // one persistent launch
        D1Args a;
        a.layers = h->d1_layers;
        a.lmw = h->lmw;
        a.s_lm = h->s_lm;
        a.g_final = h->g_final;
        a.rope = h->rope;
        a.kc = h->kc;
        a.vc = h->vc;
        a.ks = h->ks;
        a.vs = h->vs;
        a.codes_per_layer = kv_layer_codes(h);
        a.scales_per_layer = kv_layer_scales(h);
        a.cap = cap;
        a.meta = h->meta;
        a.embed = h->embed;
        a.tok_in = tok_in;
        a.slot_pos = tok_in ? slot_pos : nullptr;
        a.x = h->x;
        a.qkv = h->qkvb;
        a.ctx = h->ctx;
        a.mid = h->mid;
        a.logits = logits_dst;
        a.tokens = tokens_dst;
        a.cand_v = h->d1_cand_v;
        a.cand_i = h->d1_cand_i;
        a.bar = h->d1_bar;
        a.err = reinterpret_cast<unsigned *>(h->tc_ws);
        a.eps = eps;
        a.expire_last_barrier = h->expire_wait ? 1 : 0;
        LaunchScope ls(h, 8, st, 1);
        RK(launch_decode1(a, st));
        return 0;
    }
    if (tok_in) return fail(h, QWEN_B200_EINVAL, "device-resident token input needs the persistent single-row launch");
    {
        LaunchScope ls(h, 0, st, 1);
        RK(launch_embed(h->embed, ids, n, h->x, st));
    }
    for (int l = 0; l < NL; ++l) {
        const LayerW &W = h->L[l];
        int8_t *kc = h->kc + kv_layer_codes(h) * l, *vc = h->vc + kv_layer_codes(h) * l;
        float *ks = h->ks + kv_layer_scales(h) * l, *vs = h->vs + kv_layer_scales(h) * l;
        uint16_t *dq = nullptr;
        if (dump && l == h->dump_layer) dq = h->d_dump;
        QkvArgs a;
        a.x = h->x;
        a.rows = n;
        a.gamma = W.g_attn;
        a.eps = eps;
        a.w = W.qkv;
        a.scale = W.s_qkv;
        a.bias = W.bias;
        a.slots = slots;
        a.positions = positions;
        a.table = h->rope;
        a.q_out = h->q;
        a.kc = kc;
        a.vc = vc;
        a.ks = ks;
        a.vs = vs;
        a.cap = cap;
        a.kv_out = dq ? dq + (size_t)n * 896 : (h->rtl ? h->rtl_kv : nullptr);
        int8_t *klo = h->rtl ? h->klo + kv_layer_codes(h) * l : nullptr;
        if (n >= TC_MIN_ROWS) {
            LaunchScope ls(h, 1, st, 3);
            int rc = norm_limbs(h, h->x, W.g_attn, n, eps, st);
            if (!rc) rc = tc_gemm(h, EPI_BIAS, n, HID, W.mqkv, W.s_qkv, W.bias, QKVN, h->qkvb, nullptr, st);
            if (rc) return rc;
            RK(launch_rope_kv8(h->qkvb, n, slots, positions, h->rope, h->q, kc, ks, vc, vs, cap, a.kv_out, st));
        } else {
            LaunchScope ls(h, 1, st, 1);
            RK(launch_qkv(a, st));
        }
        if (h->rtl) {
            // the accelerator's formats over the engine-format codes just written
            LaunchScope ls(h, 1, st, 2);
            RK(launch_rtl_kv_append(a.kv_out, n, slots, positions, kc, klo, ks,
                                    h->klock + rtl_klock_layer(h) * l, vc, vs,
                                    h->vlock + (size_t)h->cfg.max_seqs * 2 * l, cap, st));
        }
        if (h->tplan) {
            // prefill rows: query tiles on the tensor cores, one launch per split group
            LaunchScope ls(h, 2, st, (uint32_t)h->tgroups.size());
            const long long krow0 = (long long)(kv_layer_codes(h) / 64) * l;
            for (const AtGroup &grp : h->tgroups)
                RK(launch_attention_tiles(h->kmap, krow0, h->d_tiles, grp, h->q, vc, ks, vs, cap, h->ctx,
                                          reinterpret_cast<unsigned *>(h->tc_ws), st));
        } else {
            LaunchScope ls(h, 2, st, 1);
            RK(launch_attention_cluster(h->q, n, slots, positions, max_len, kc, ks, vc, vs, cap, h->ctx,
                                        reinterpret_cast<unsigned *>(h->tc_ws), st, klo));
        }
        if (dq) {
            CK(cudaMemcpyAsync(dq, h->q, (size_t)n * 896 * 2, cudaMemcpyDeviceToDevice, st));
            CK(cudaMemcpyAsync(dq + (size_t)n * 1152, h->ctx, (size_t)n * 896 * 2, cudaMemcpyDeviceToDevice, st));
            pdl_break();
        }
        {
            LaunchScope ls(h, 3, st, n >= TC_MIN_ROWS ? 2 : 1);
            if (n >= TC_MIN_ROWS) {
                int rc = make_limbs(h, h->ctx, n, HID, st);
                if (!rc) rc = tc_gemm(h, EPI_RESIDUAL, n, HID, W.mo, W.s_o, nullptr, HID, h->x, nullptr, st);
                if (rc) return rc;
            } else {
                RK(launch_gemv(EPI_RESIDUAL, h->ctx, n, HID, nullptr, 0.f, W.o, W.s_o, nullptr, HID, h->x, st));
            }
        }
        if (dq) {
            CK(cudaMemcpyAsync(dq + (size_t)n * 2048, h->x, (size_t)n * 896 * 2, cudaMemcpyDeviceToDevice, st));
            pdl_break();
        }
        if (n >= TC_MIN_ROWS) {
            LaunchScope ls(h, 4, st, 2);
            int rc = norm_limbs(h, h->x, W.g_ffn, n, eps, st);
            if (!rc) rc = tc_gemm(h, EPI_SWIGLU, n, HID, W.mgu, W.s_gu, nullptr, 2 * FFN, h->mid, nullptr, st);
            if (rc) return rc;
        } else {
            LaunchScope ls(h, 4, st, 1);
            RK(launch_gemv(EPI_SWIGLU, h->x, n, HID, W.g_ffn, eps, W.gu, W.s_gu, nullptr, 2 * FFN, h->mid, st));
        }
        if (n >= TC_MIN_ROWS) {
            LaunchScope ls(h, 5, st, 2);
            int rc = make_limbs(h, h->mid, n, FFN, st);
            if (!rc) rc = tc_gemm(h, EPI_RESIDUAL, n, FFN, W.md, W.s_d, nullptr, HID, h->x, nullptr, st);
            if (rc) return rc;
        } else {
            LaunchScope ls(h, 5, st, 1);
            RK(launch_gemv(EPI_RESIDUAL, h->mid, n, FFN, nullptr, 0.f, W.d, W.s_d, nullptr, HID, h->x, st));
        }
        if (dq) {
            CK(cudaMemcpyAsync(dq + (size_t)n * 2944, h->mid, (size_t)n * FFN * 2, cudaMemcpyDeviceToDevice, st));
            CK(cudaMemcpyAsync(dq + (size_t)n * 7808, h->x, (size_t)n * 896 * 2, cudaMemcpyDeviceToDevice, st));
            pdl_break();
        }
    }
    if (nlog > 0) {
        const uint16_t *xin = h->x;
        if (!identity) {
            LaunchScope ls(h, 7, st, 1);
            RK(launch_gather_rows(h->x, lrows, nlog, h->xl, st));
            xin = h->xl;
        }
        if (lm_head) return lm_head_rows(h, xin, nlog, 0, VOC, logits_dst, tokens_dst, nullptr, st);
    }
    return 0;
}

int sync_slot_positions(qwen_b200 *h, cudaStream_t st) {
    memcpy(h->h_slot_pos, h->pos.data(), h->pos.size() * 4);
    CK(cudaMemcpyAsync(h->slot_pos, h->h_slot_pos, h->pos.size() * 4, cudaMemcpyHostToDevice, st));
    return 0;
}

// Copies dump buffers of one forward chunk (rows [r0, r0+n)) to the host.
int copy_dump(qwen_b200 *h, int n, int r0) {
    uint16_t *d = h->d_dump;
    uint16_t **o = h->dump_host;
    struct Part {
        uint16_t *dst;
        size_t off, cols, pitch_cols, col0;
    } parts[7] = {
        {o[0], 0, 896, 896, 0},          {o[1], (size_t)n * 896, 128, 256, 0},
        {o[2], (size_t)n * 896, 128, 256, 128}, {o[3], (size_t)n * 1152, 896, 896, 0},
        {o[4], (size_t)n * 2048, 896, 896, 0}, {o[5], (size_t)n * 2944, 4864, 4864, 0},
        {o[6], (size_t)n * 7808, 896, 896, 0}};
    for (const Part &p : parts) {
        if (!p.dst) continue;
        CK(cudaMemcpy2D(p.dst + (size_t)r0 * p.cols, p.cols * 2, d + p.off + p.col0, p.pitch_cols * 2, p.cols * 2,
                        (size_t)n, cudaMemcpyDeviceToHost));
    }
    return 0;
}

void csr_start(qwen_b200 *h) {
    auto error = [&](uint64_t code) {
        h->csr_state = CSR_ERROR;
        h->csr_error = code;
    };
    // Error codes at 0x30: 1 malformed request, 2 CUDA error, 3 no model
    // loaded, 4 START while busy, 5 a bounded device wait expired (the
    // reference's PL-error path, generation.c:21-25).
    if (h->csr_state == CSR_BUSY) return error(4);
    const uint64_t mode = h->regs[0x80 / 8] & 1, rows = h->regs[0x88 / 8], ctxlen = h->regs[0x90 / 8],
                   position = h->regs[0x98 / 8];
    const uint32_t cached = h->loaded ? h->pos[0] : 0;
    if (rows == 0 || rows > CSR_IDS || rows > std::max(h->cfg.max_rows, h->cfg.max_seqs) ||
        ctxlen != position + rows || position + rows > h->cfg.max_context)
        return error(1);
    if (mode == 0 ? position != 0 : position != cached) return error(1);
    for (uint64_t i = 0; i < rows; ++i)
        if (h->csr_ids[i] >= (uint32_t)VOC) return error(1);
    if (!h->loaded || cudaSetDevice(h->cfg.device) != cudaSuccess) return error(3);
    if (mode == 0) h->pos[0] = 0;
    const int n = (int)rows;
    for (int i = 0; i < n; ++i) {
        h->h_meta[i] = h->csr_ids[i];
        h->h_meta[n + i] = 0;
        h->h_meta[2 * n + i] = (uint32_t)position + (uint32_t)i;
    }
    h->h_meta[3 * n] = (uint32_t)(n - 1);
    cudaStream_t st = h->stream;
    bool ok = cudaMemcpyAsync(h->meta, h->h_meta, (size_t)(3 * n + 1) * 4, cudaMemcpyHostToDevice, st) == cudaSuccess;
    ok = ok && run_forward(h, n, (int)(position + rows), 1, n == 1, nullptr, h->tokens, st) == 0;
    ok = ok && cudaMemcpyAsync(h->h_tokens, h->tokens, 4, cudaMemcpyDeviceToHost, st) == cudaSuccess;
    // the bounded-wait error flag travels with the token
    ok = ok && cudaMemcpyAsync(h->h_flag + 1, h->tc_ws, 4, cudaMemcpyDeviceToHost, st) == cudaSuccess;
    ok = ok && cudaEventRecord(h->csr_event, st) == cudaSuccess;
    if (!ok) return error(2);
    h->pos[0] = (uint32_t)(position + rows);
    h->csr_state = CSR_BUSY;
}

}  // namespace

// ============================================================== C ABI
extern "C" {

void qwen_b200_default_config(qwen_b200_config *cfg) {
    if (!cfg) return;
    cfg->device = 0;
    cfg->max_seqs = 1;
    cfg->max_context = 256;
    cfg->max_rows = 256;
    cfg->rms_eps = 1e-6f;
    cfg->flags = 0;
}

int qwen_b200_open(const qwen_b200_config *cfg, qwen_b200 **out) {
    if (!out) return QWEN_B200_EINVAL;
    *out = nullptr;
    qwen_b200_config c;
    qwen_b200_default_config(&c);
    if (cfg) c = *cfg;
    if (c.max_seqs == 0 || c.max_context == 0 || c.max_rows == 0 || c.device < 0 || !(c.rms_eps > 0.f) ||
        (c.flags & ~QWEN_B200_FLAG_RTL_KV))
        return QWEN_B200_EINVAL;
    qwen_b200 *h = new (std::nothrow) qwen_b200();
    if (!h) return QWEN_B200_ENOMEM;
    h->cfg = c;
    h->rtl = (c.flags & QWEN_B200_FLAG_RTL_KV) != 0;
    *out = h;
    return QWEN_B200_OK;
}

int qwen_b200_close(qwen_b200 *h) {
    if (!h) return QWEN_B200_EINVAL;
    if (h->loaded) {
        cudaSetDevice(h->cfg.device);
        cudaDeviceSynchronize();
        for (auto &kv : h->graphs) cudaGraphExecDestroy(kv.second);
        for (auto &kv : h->host_graphs) cudaGraphExecDestroy(kv.second.first);
        for (auto &pool : h->prof_ev)
            for (cudaEvent_t e : pool) cudaEventDestroy(e);
        for (void *p : h->dev_allocs) cudaFree(p);
        if (h->d_dump) cudaFree(h->d_dump);
        cudaFreeHost(h->h_meta);
        cudaFreeHost(h->h_tokens);
        cudaFreeHost(h->h_slot_pos);
        cudaFreeHost(h->h_flag);
        cudaFreeHost(h->h_tiles);
        if (h->csr_event) cudaEventDestroy(h->csr_event);
        if (h->staged) cudaEventDestroy(h->staged);
        if (h->stream) cudaStreamDestroy(h->stream);
        if (h->cap_stream) cudaStreamDestroy(h->cap_stream);
    }
    delete h;
    return QWEN_B200_OK;
}

const char *qwen_b200_last_error(const qwen_b200 *h) { return h ? h->err.c_str() : "null handle"; }

int qwen_b200_get_config(const qwen_b200 *h, qwen_b200_config *cfg) {
    if (!h || !cfg) return QWEN_B200_EINVAL;
    *cfg = h->cfg;
    return QWEN_B200_OK;
}

static int load_model(qwen_b200 *h, qa_model &m) {
    int rc = allocate(h);
    if (!rc) rc = upload(h, m);
    qa_free(&m);
    if (!rc) {
        CK(cudaDeviceSynchronize());
        h->loaded = true;
    }
    return rc;
}

int qwen_b200_load_assets(qwen_b200 *h, const char *sd_root) {
    if (!h || !sd_root) return QWEN_B200_EINVAL;
    if (h->loaded) return fail(h, QWEN_B200_EINVAL, "assets already loaded");
    qa_model m;
    char err[512] = "";
    int rc = qa_read(sd_root, &m, err, sizeof(err));
    if (rc) return fail(h, rc, "%s", err);
    return load_model(h, m);
}

int qwen_b200_load_synthetic(qwen_b200 *h, uint64_t seed) {
    if (!h) return QWEN_B200_EINVAL;
    if (h->loaded) return fail(h, QWEN_B200_EINVAL, "assets already loaded");
    qa_model m;
    if (qa_alloc(&m)) {
        qa_free(&m);
        return fail(h, QWEN_B200_ENOMEM, "host allocation failed");
    }
    qa_generate(seed, &m);
    return load_model(h, m);
}

int qwen_b200_synth_write(const char *sd_root, uint64_t seed) {
    if (!sd_root) return QWEN_B200_EINVAL;
    qa_model m;
    if (qa_alloc(&m)) {
        qa_free(&m);
        return QWEN_B200_ENOMEM;
    }
    qa_generate(seed, &m);
    int rc = qa_write(&m, sd_root, seed);
    qa_free(&m);
    return rc;
}

void qwen_b200_synth_prompt(uint64_t seed, uint32_t n, uint32_t *ids) {
    if (ids) qa_prompt(seed, n, ids);
}

void qwen_b200_rope_table(uint32_t positions, float *table) {
    // 1 / 1e6^(2i/64) rounded to fp32, phase = pos * inv in fp32, cos/sin of
    // that fp32 phase rounded to fp32 (model_backend.py:41,74-76).
    float inv[32];
    for (int i = 0; i < 32; ++i) inv[i] = 1.0f / (float)pow(1000000.0, (double)(2 * i) / 64.0);
    for (uint32_t p = 0; p < positions; ++p)
        for (int i = 0; i < 32; ++i) {
            const float phase = (float)p * inv[i];
            table[(size_t)p * 64 + i] = (float)cos((double)phase);
            table[(size_t)p * 64 + 32 + i] = (float)sin((double)phase);
        }
}

// Captured steps have the engine's switches built in: drops them.
static void drop_graphs(qwen_b200 *h) {
    if (!h->loaded) return;
    cudaSetDevice(h->cfg.device);
    cudaDeviceSynchronize();
    for (auto &kv : h->graphs) cudaGraphExecDestroy(kv.second);
    for (auto &kv : h->host_graphs) cudaGraphExecDestroy(kv.second.first);
    h->graphs.clear();
    h->host_graphs.clear();
}

int qwen_b200_set_persistent_decode(qwen_b200 *h, int enable) {
    if (!h) return QWEN_B200_EINVAL;
    const int p = enable <= 0 ? 0 : (enable == 1 ? 1 : 2);
    if (p != h->persistent) drop_graphs(h);  // captured steps have the previous choice built in
    h->persistent = p;
    return QWEN_B200_OK;
}

int qwen_b200_test_expire_wait(qwen_b200 *h, int enable) {
    if (!h) return QWEN_B200_EINVAL;
    const bool e = enable != 0;
    if (e != h->expire_wait) drop_graphs(h);
    h->expire_wait = e;
    return QWEN_B200_OK;
}

int qwen_b200_reset(qwen_b200 *h, uint32_t slot) {
    if (!h || slot >= h->cfg.max_seqs) return QWEN_B200_EINVAL;
    if (!h->loaded) return QWEN_B200_OK;
    h->pos[slot] = 0;
    CK(cudaSetDevice(h->cfg.device));
    return sync_slot_positions(h, h->stream) ? QWEN_B200_EDEVICE : QWEN_B200_OK;
}

int qwen_b200_position(const qwen_b200 *h, uint32_t slot, uint32_t *position) {
    if (!h || !position || slot >= h->cfg.max_seqs) return QWEN_B200_EINVAL;
    *position = h->loaded ? h->pos[slot] : 0;
    return QWEN_B200_OK;
}

int qwen_b200_forward(qwen_b200 *h, uint32_t slot, const uint32_t *ids, uint32_t rows, uint32_t position,
                      uint32_t *token, uint16_t *logits) {
    if (!h) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    if (!ids || slot >= h->cfg.max_seqs) return fail(h, QWEN_B200_EINVAL, "bad slot or ids");
    for (uint32_t i = 0; i < rows; ++i)
        if (ids[i] >= (uint32_t)VOC) return fail(h, QWEN_B200_EINVAL, "token id %u >= vocab", ids[i]);
    if (position != h->pos[slot] || rows == 0 || (uint64_t)position + rows > h->cfg.max_context)
        return fail(h, QWEN_B200_ESTATE, "KV position mismatch pos=%u cached=%u ids=%u", position, h->pos[slot],
                    rows);
    cudaStream_t st = h->stream;
    for (uint32_t c0 = 0; c0 < rows; c0 += (uint32_t)h->cfg.max_rows) {
        const int n = (int)std::min<uint32_t>(h->cfg.max_rows, rows - c0);
        const bool last = c0 + (uint32_t)n == rows;
        // the previous chunk's copy out of the pinned staging buffer must have
        // happened before the buffer is rewritten
        if (c0) CK(cudaEventSynchronize(h->staged));
        for (int i = 0; i < n; ++i) {
            h->h_meta[i] = ids[c0 + i];
            h->h_meta[n + i] = slot;
            h->h_meta[2 * n + i] = position + c0 + (uint32_t)i;
        }
        h->h_meta[3 * n] = (uint32_t)(n - 1);
        CK(cudaMemcpyAsync(h->meta, h->h_meta, (size_t)(3 * n + 1) * 4, cudaMemcpyHostToDevice, st));
        if ((rc = prepare_tiles(h, n, h->h_meta + n, h->h_meta + 2 * n, st))) return rc;
        CK(cudaEventRecord(h->staged, st));
        rc = run_forward(h, n, (int)(position + c0 + (uint32_t)n), last ? 1 : 0, n == 1,
                         last && logits ? h->logits : nullptr, h->tokens, st);
        h->tplan = false;
        if (rc) return rc;
        if (h->dump_layer >= 0 && h->d_dump) {
            CK(cudaStreamSynchronize(st));
            if ((rc = copy_dump(h, n, (int)c0))) return rc;
        }
    }
    CK(cudaMemcpyAsync(h->h_tokens, h->tokens, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if ((rc = check_device_flags(h))) return rc;
    if (logits) CK(cudaMemcpy(logits, h->logits, (size_t)VOC * 2, cudaMemcpyDeviceToHost));
    h->pos[slot] = position + rows;
    if ((rc = sync_slot_positions(h, st))) return rc;
    if (h->h_tokens[0] >= (uint32_t)VOC) return fail(h, QWEN_B200_ETOKEN, "token %u", h->h_tokens[0]);
    if (token) *token = h->h_tokens[0];
    return QWEN_B200_OK;
}

// One decode step of n slots from host buffers; with logits != NULL the
// forward runs directly (no graph) and every row's logits come back too.
static int decode_step_impl(qwen_b200 *h, const uint32_t *slots, const uint32_t *tokens_in, uint32_t n,
                            uint32_t *tokens_out, uint16_t *logits) {
    if (!h) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    if (!slots || !tokens_in || !tokens_out || n == 0 || n > h->cfg.max_seqs || (int)n > h->R)
        return fail(h, QWEN_B200_EINVAL, "bad decode batch");
    std::vector<char> seen(h->cfg.max_seqs, 0);
    uint32_t max_len = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (slots[i] >= h->cfg.max_seqs || seen[slots[i]]) return fail(h, QWEN_B200_EINVAL, "bad or repeated slot");
        seen[slots[i]] = 1;
        if (tokens_in[i] >= (uint32_t)VOC) return fail(h, QWEN_B200_EINVAL, "token id %u >= vocab", tokens_in[i]);
        if (h->pos[slots[i]] >= h->cfg.max_context) return fail(h, QWEN_B200_ESTATE, "slot %u is full", slots[i]);
        max_len = std::max(max_len, h->pos[slots[i]] + 1);
    }
    cudaStream_t st = h->stream;
    for (uint32_t i = 0; i < n; ++i) {
        h->h_meta[i] = tokens_in[i];
        h->h_meta[n + i] = slots[i];
        h->h_meta[2 * n + i] = h->pos[slots[i]];
    }
    CK(cudaMemcpyAsync(h->meta, h->h_meta, (size_t)3 * n * 4, cudaMemcpyHostToDevice, st));
    // steps of one batch size and context bucket replay one graph of the
    // forward (it reads the staged ids / slots / positions on the device);
    // the first such step runs the launches directly and captures them (a
    // profiled step always runs them directly, between its events)
    const uint32_t bound = context_bucket(max_len);
    const int bucket_len = (int)std::min<uint32_t>(bound, h->cfg.max_context);
    const auto key = std::make_pair(n, bound);
    auto it = (h->prof || logits) ? h->host_graphs.end() : h->host_graphs.find(key);
    if (logits && !h->blogits) {
        // every row's logits: allocated at the first such step
        if ((rc = dalloc(h, (void **)&h->blogits, (size_t)h->R * VOC * 2))) return rc;
    }
    if (it != h->host_graphs.end()) {
        CK(cudaGraphLaunch(it->second.first, st));
        h->nlaunch = it->second.second;
    } else if (h->prof || logits) {
        h->nlaunch = 0;
        if ((rc = run_forward(h, (int)n, bucket_len, (int)n, true, logits ? h->blogits : nullptr, h->tokens, st)))
            return rc;
    } else {
        h->nlaunch = 0;
        if ((rc = run_forward(h, (int)n, bucket_len, (int)n, true, nullptr, h->tokens, st))) return rc;
        cudaGraph_t graph;
        CK(cudaStreamBeginCapture(h->cap_stream, cudaStreamCaptureModeThreadLocal));
        h->nlaunch = 0;
        rc = run_forward(h, (int)n, bucket_len, (int)n, true, nullptr, h->tokens, h->cap_stream);
        cudaError_t e = cudaStreamEndCapture(h->cap_stream, &graph);
        if (rc) return rc;
        if (e != cudaSuccess) return fail(h, QWEN_B200_EDEVICE, "graph capture: %s", cudaGetErrorString(e));
        cudaGraphExec_t exec;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail(h, QWEN_B200_EDEVICE, "graph instantiate: %s", cudaGetErrorString(e));
        h->host_graphs[key] = std::make_pair(exec, h->nlaunch);
    }
    CK(cudaMemcpyAsync(h->h_tokens, h->tokens, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(h->h_flag, h->tc_ws, 4, cudaMemcpyDeviceToHost, st));  // bounded-wait error flag
    CK(cudaStreamSynchronize(st));
    if (*h->h_flag) {
        cudaMemset(h->tc_ws, 0, 4);
        return fail(h, QWEN_B200_ETIMEOUT, "a pipeline wait on the device timed out (code %u)", *h->h_flag);
    }
    if (logits) CK(cudaMemcpy(logits, h->blogits, (size_t)n * VOC * 2, cudaMemcpyDeviceToHost));
    for (uint32_t i = 0; i < n; ++i) {
        h->pos[slots[i]] += 1;
        tokens_out[i] = h->h_tokens[i];
    }
    if ((rc = sync_slot_positions(h, st))) return rc;
    for (uint32_t i = 0; i < n; ++i)
        if (tokens_out[i] >= (uint32_t)VOC) return fail(h, QWEN_B200_ETOKEN, "token %u", tokens_out[i]);
    return QWEN_B200_OK;
}

int qwen_b200_decode_step(qwen_b200 *h, const uint32_t *slots, const uint32_t *tokens_in, uint32_t n,
                          uint32_t *tokens_out) {
    return decode_step_impl(h, slots, tokens_in, n, tokens_out, nullptr);
}

int qwen_b200_decode_step_logits(qwen_b200 *h, const uint32_t *slots, const uint32_t *tokens_in, uint32_t n,
                                 uint32_t *tokens_out, uint16_t *logits) {
    if (!logits) return h ? fail(h, QWEN_B200_EINVAL, "logits buffer is NULL") : QWEN_B200_EINVAL;
    return decode_step_impl(h, slots, tokens_in, n, tokens_out, logits);
}

int qwen_b200_prefill(qwen_b200 *h, uint32_t n, const uint32_t *slots, const uint32_t *lens, const uint32_t *ids,
                      uint32_t *tokens_out, uint16_t *hidden_out) {
    if (!h) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    if (!slots || !lens || !ids || n == 0 || n > h->cfg.max_seqs || (!tokens_out && !hidden_out))
        return fail(h, QWEN_B200_EINVAL, "bad prefill request");
    std::vector<char> seen(h->cfg.max_seqs, 0);
    size_t total = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (slots[i] >= h->cfg.max_seqs || seen[slots[i]] || lens[i] == 0)
            return fail(h, QWEN_B200_EINVAL, "bad or repeated slot, or empty sequence");
        seen[slots[i]] = 1;
        if ((uint64_t)h->pos[slots[i]] + lens[i] > h->cfg.max_context)
            return fail(h, QWEN_B200_ESTATE, "slot %u: %u + %u tokens exceed the capacity", slots[i], h->pos[slots[i]],
                        lens[i]);
        total += lens[i];
    }
    for (size_t t = 0; t < total; ++t)
        if (ids[t] >= (uint32_t)VOC) return fail(h, QWEN_B200_EINVAL, "token id %u >= vocab", ids[t]);
    // every row: (sequence, position); rows of all sequences go through the
    // layers together, max_rows at a time
    std::vector<uint32_t> rseq(total), rpos(total);
    for (uint32_t i = 0, t = 0; i < n; ++i)
        for (uint32_t j = 0; j < lens[i]; ++j, ++t) {
            rseq[t] = i;
            rpos[t] = h->pos[slots[i]] + j;
        }
    cudaStream_t st = h->stream;
    const size_t chunk = h->cfg.max_rows;
    uint32_t done = 0;
    for (size_t c0 = 0; c0 < total; c0 += chunk) {
        const int m = (int)std::min(chunk, total - c0);
        if (c0) CK(cudaEventSynchronize(h->staged));  // the pinned staging buffer is free again
        int nl = 0, max_len = 0;
        for (int r = 0; r < m; ++r) {
            const size_t t = c0 + r;
            h->h_meta[r] = ids[t];
            h->h_meta[m + r] = slots[rseq[t]];
            h->h_meta[2 * m + r] = rpos[t];
            max_len = std::max(max_len, (int)rpos[t] + 1);
            if (t + 1 == total || rseq[t + 1] != rseq[t]) h->h_meta[3 * m + nl++] = (uint32_t)r;  // a last row
        }
        CK(cudaMemcpyAsync(h->meta, h->h_meta, (size_t)(3 * m + nl) * 4, cudaMemcpyHostToDevice, st));
        if ((rc = prepare_tiles(h, m, h->h_meta + m, h->h_meta + 2 * m, st))) return rc;
        CK(cudaEventRecord(h->staged, st));
        h->nlaunch = 0;
        rc = run_forward(h, m, max_len, nl, false, nullptr, h->tokens + done, st, tokens_out != nullptr);
        h->tplan = false;
        if (rc) return rc;
        if (hidden_out && nl)
            CK(cudaMemcpyAsync(hidden_out + (size_t)done * HID, h->xl, (size_t)nl * HID * 2, cudaMemcpyDeviceToHost,
                               st));
        done += (uint32_t)nl;
    }
    if (tokens_out) CK(cudaMemcpyAsync(h->h_tokens, h->tokens, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(h->h_flag, h->tc_ws, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (*h->h_flag) {
        cudaMemset(h->tc_ws, 0, 4);
        return fail(h, QWEN_B200_ETIMEOUT, "a pipeline wait on the device timed out (code %u)", *h->h_flag);
    }
    for (uint32_t i = 0; i < n; ++i) h->pos[slots[i]] += lens[i];
    if ((rc = sync_slot_positions(h, st))) return rc;
    if (tokens_out)
        for (uint32_t i = 0; i < n; ++i) {
            if (h->h_tokens[i] >= (uint32_t)VOC) return fail(h, QWEN_B200_ETOKEN, "token %u", h->h_tokens[i]);
            tokens_out[i] = h->h_tokens[i];
        }
    return QWEN_B200_OK;
}

int qwen_b200_lm_head_range(qwen_b200 *h, const uint16_t *d_hidden, uint32_t rows, uint32_t begin, uint32_t end,
                            float *d_values, uint32_t *d_indices, void *stream) {
    if (!h) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    if (!d_hidden || !d_values || !d_indices || rows == 0 || (int)rows > h->R)
        return fail(h, QWEN_B200_EINVAL, "bad LM-head request");
    if (begin >= end || end > (uint32_t)VOC || begin % 128 || end % 128)
        return fail(h, QWEN_B200_EINVAL, "vocabulary range [%u, %u) is not whole 128-row tiles of [0, %d)", begin,
                    end, VOC);
    cudaStream_t st = (cudaStream_t)stream;
    CK(cudaMemcpyAsync(h->xl, d_hidden, (size_t)rows * HID * 2, cudaMemcpyDeviceToDevice, st));
    h->nlaunch = 0;
    return lm_head_rows(h, h->xl, (int)rows, (int)begin, (int)end, nullptr, d_indices, d_values, st);
}

static int enqueue_device_step(qwen_b200 *h, const uint32_t *d_in, int n, int max_len, uint32_t *d_out,
                               cudaStream_t st) {
    uint32_t *ids = h->meta, *slots = h->meta + n, *positions = h->meta + 2 * n;
    h->nlaunch = 0;
    if (uses_decode1(h, n, max_len, n, true))  // one launch reads the token and advances the position
        return run_forward(h, n, max_len, n, true, nullptr, d_out, st, true, d_in, h->slot_pos);
    PdlChain chain;  // prologue, the layers and the epilogue overlap one another
    {
        LaunchScope ls(h, 7, st, 1);
        RK(launch_decode_prologue(d_in, n, h->slot_pos, ids, slots, positions, st));
    }
    int rc = run_forward(h, n, max_len, n, true, nullptr, d_out, st);
    if (rc) return rc;
    LaunchScope ls(h, 7, st, 1);
    RK(launch_decode_epilogue(n, h->slot_pos, st));
    return 0;
}

int qwen_b200_decode_step_device(qwen_b200 *h, const uint32_t *d_tokens_in, uint32_t n, uint32_t *d_tokens_out,
                                 void *stream) {
    if (!h) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    if (!d_tokens_in || !d_tokens_out || n == 0 || n > h->cfg.max_seqs || (int)n > h->R)
        return fail(h, QWEN_B200_EINVAL, "bad decode batch");
    uint32_t max_len = 0;
    for (uint32_t i = 0; i < n; ++i) {
        if (h->pos[i] >= h->cfg.max_context) return fail(h, QWEN_B200_ESTATE, "slot %u is full", i);
        max_len = std::max(max_len, h->pos[i] + 1);
    }
    const uint32_t bound = context_bucket(max_len);
    const int bucket_len = (int)std::min<uint32_t>(bound, h->cfg.max_context);
    cudaStream_t st = (cudaStream_t)stream;  // NULL: the CUDA default stream
    const auto key = std::make_tuple(n, bound, (const void *)d_tokens_in, (const void *)d_tokens_out);
    auto it = h->graphs.find(key);
    if (it != h->graphs.end()) {
        CK(cudaGraphLaunch(it->second, st));
    } else {
        if ((rc = enqueue_device_step(h, d_tokens_in, (int)n, bucket_len, d_tokens_out, st))) return rc;
        cudaGraph_t graph;
        CK(cudaStreamBeginCapture(h->cap_stream, cudaStreamCaptureModeThreadLocal));
        rc = enqueue_device_step(h, d_tokens_in, (int)n, bucket_len, d_tokens_out, h->cap_stream);
        cudaError_t e = cudaStreamEndCapture(h->cap_stream, &graph);
        if (rc) return rc;
        if (e != cudaSuccess) return fail(h, QWEN_B200_EDEVICE, "graph capture: %s", cudaGetErrorString(e));
        cudaGraphExec_t exec;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail(h, QWEN_B200_EDEVICE, "graph instantiate: %s", cudaGetErrorString(e));
        h->graphs[key] = exec;
    }
    for (uint32_t i = 0; i < n; ++i) h->pos[i] += 1;
    return QWEN_B200_OK;
}

int qwen_b200_fill_kv_synthetic(qwen_b200 *h, uint32_t slot, uint32_t length, uint64_t seed) {
    if (!h) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    if (slot >= h->cfg.max_seqs || length == 0 || length > h->cfg.max_context)
        return fail(h, QWEN_B200_EINVAL, "bad slot or length");
    if (h->rtl) return fail(h, QWEN_B200_ESTATE, "synthetic KV fill is not available in the RTL KV format");
    RK(launch_fill_kv(h->kc, h->ks, h->vc, h->vs, NL, (int)h->cfg.max_seqs, (int)slot, (int)h->cfg.max_context,
                      (int)length, seed, h->stream));
    h->pos[slot] = length;
    if ((rc = sync_slot_positions(h, h->stream))) return rc;
    CK(cudaStreamSynchronize(h->stream));
    return QWEN_B200_OK;
}

int qwen_b200_read_kv_rtl(qwen_b200 *h, uint32_t slot, uint32_t layer, uint32_t n, int8_t *klo, uint8_t *klock,
                          uint8_t *vlock) {
    if (!h) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    if (!h->rtl) return fail(h, QWEN_B200_ESTATE, "the handle does not hold the RTL KV format");
    if (slot >= h->cfg.max_seqs || layer >= (uint32_t)NL || n > h->cfg.max_context)
        return fail(h, QWEN_B200_EINVAL, "bad slot/layer/length");
    CK(cudaStreamSynchronize(h->stream));
    const size_t cap = h->cfg.max_context, nblk = (cap + 255) / 256;
    for (int g = 0; g < 2; ++g) {
        const size_t row = ((size_t)slot * 2 + g) * cap;
        if (klo)
            CK(cudaMemcpy(klo + (size_t)g * n * 64, h->klo + kv_layer_codes(h) * layer + row * 64, (size_t)n * 64,
                          cudaMemcpyDeviceToHost));
        if (klock)
            CK(cudaMemcpy(klock + (size_t)g * nblk, h->klock + rtl_klock_layer(h) * layer + ((size_t)slot * 2 + g) * nblk,
                          nblk, cudaMemcpyDeviceToHost));
    }
    if (vlock)
        CK(cudaMemcpy(vlock, h->vlock + (size_t)h->cfg.max_seqs * 2 * layer + (size_t)slot * 2, 2,
                      cudaMemcpyDeviceToHost));
    return QWEN_B200_OK;
}

int qwen_b200_read_kv(qwen_b200 *h, uint32_t slot, uint32_t layer, uint32_t n, int8_t *kcodes, float *kscales,
                      int8_t *vcodes, float *vscales) {
    if (!h) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    if (slot >= h->cfg.max_seqs || layer >= (uint32_t)NL || n > h->cfg.max_context)
        return fail(h, QWEN_B200_EINVAL, "bad slot/layer/length");
    CK(cudaStreamSynchronize(h->stream));
    const size_t cap = h->cfg.max_context;
    for (int g = 0; g < 2; ++g) {
        const size_t row = ((size_t)slot * 2 + g) * cap;
        if (kcodes)
            CK(cudaMemcpy(kcodes + (size_t)g * n * 64, h->kc + kv_layer_codes(h) * layer + row * 64, (size_t)n * 64,
                          cudaMemcpyDeviceToHost));
        if (vcodes)
            CK(cudaMemcpy(vcodes + (size_t)g * n * 64, h->vc + kv_layer_codes(h) * layer + row * 64, (size_t)n * 64,
                          cudaMemcpyDeviceToHost));
        if (kscales)
            CK(cudaMemcpy(kscales + (size_t)g * n, h->ks + kv_layer_scales(h) * layer + row, (size_t)n * 4,
                          cudaMemcpyDeviceToHost));
        if (vscales)
            CK(cudaMemcpy(vscales + (size_t)g * n, h->vs + kv_layer_scales(h) * layer + row, (size_t)n * 4,
                          cudaMemcpyDeviceToHost));
    }
    return QWEN_B200_OK;
}

int qwen_b200_set_dump(qwen_b200 *h, int layer, uint16_t *q, uint16_t *k, uint16_t *v, uint16_t *ctx,
                       uint16_t *hbuf, uint16_t *mid, uint16_t *y) {
    if (!h || layer >= NL) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    h->dump_layer = layer;
    uint16_t *ptrs[7] = {q, k, v, ctx, hbuf, mid, y};
    memcpy(h->dump_host, ptrs, sizeof(ptrs));
    if (layer >= 0 && !h->d_dump) CK(cudaMalloc((void **)&h->d_dump, (size_t)h->R * DUMP_COLS * 2));
    return QWEN_B200_OK;
}

int qwen_b200_profile_decode(qwen_b200 *h, const uint32_t *tokens_in, uint32_t n, uint32_t *tokens_out,
                             float *ms, uint32_t *launches) {
    if (!h || !ms || !launches) return QWEN_B200_EINVAL;
    int rc = ensure_device(h);
    if (rc) return rc;
    std::vector<uint32_t> slots(n);
    for (uint32_t i = 0; i < n; ++i) slots[i] = i;
    for (int c = 0; c < QWEN_B200_KCLASSES; ++c) h->prof_used[c] = 0;
    h->prof = true;
    rc = qwen_b200_decode_step(h, slots.data(), tokens_in, n, tokens_out);
    h->prof = false;
    if (rc) return rc;
    CK(cudaStreamSynchronize(h->stream));
    for (int c = 0; c < QWEN_B200_KCLASSES; ++c) {
        float total = 0.f;
        for (size_t i = 0; i + 1 < h->prof_used[c]; i += 2) {
            float t = 0.f;
            CK(cudaEventElapsedTime(&t, h->prof_ev[c][i], h->prof_ev[c][i + 1]));
            total += t;
        }
        ms[c] = total;
        launches[c] = (uint32_t)(h->prof_used[c] / 2);
    }
    return QWEN_B200_OK;
}

uint32_t qwen_b200_step_launches(const qwen_b200 *h) { return h ? h->nlaunch : 0; }

// ----------------------------------------------------------------- CSR protocol
void qwen_b200_csr_write(void *ctx, unsigned offset, uint64_t value) {
    qwen_b200 *h = (qwen_b200 *)ctx;
    if (!h || offset % 8 || offset / 8 >= 128) return;
    h->regs[offset / 8] = value;
    if (offset != QWEN_B200_CSR_CONTROL) return;
    if (value & 8u) {  // CLEAR: drop a latched error / finished result
        if (h->csr_state != CSR_BUSY) h->csr_state = CSR_IDLE;
        h->csr_error = 0;
    }
    if (value & 1u) csr_start(h);
    h->regs[offset / 8] = 0;  // the control register reads back 0 (no IRQ)
}

uint64_t qwen_b200_csr_read(void *ctx, unsigned offset) {
    qwen_b200 *h = (qwen_b200 *)ctx;
    if (!h) return 0;
    switch (offset) {
        case QWEN_B200_CSR_ID: return QWEN_B200_ID_VALUE;
        case QWEN_B200_CSR_VERSION: return QWEN_B200_VERSION_VALUE;
        case QWEN_B200_CSR_STATUS:
            if (h->csr_state == CSR_BUSY) {
                cudaSetDevice(h->cfg.device);
                cudaError_t e = cudaEventQuery(h->csr_event);
                if (e == cudaErrorNotReady) return 0x2;
                if (e != cudaSuccess) {
                    h->csr_state = CSR_ERROR;
                    h->csr_error = 2;
                } else if (h->h_flag[1]) {
                    // a bounded wait on the device expired: the token is not valid
                    cudaMemsetAsync(h->tc_ws, 0, 4, h->stream);
                    h->h_flag[1] = 0;
                    h->csr_state = CSR_ERROR;
                    h->csr_error = 5;
                } else {
                    h->csr_token = h->h_tokens[0];
                    h->csr_state = CSR_DONE;
                }
            }
            if (h->csr_state == CSR_ERROR) return 0x8;
            if (h->csr_state == CSR_DONE) return 0x44;
            return 0x0;
        case QWEN_B200_CSR_ERROR: return h->csr_error;
        case QWEN_B200_CSR_BEST_TOKEN: return h->csr_token & 0x3ffffu;
        default: return (offset % 8 || offset / 8 >= 128) ? 0 : h->regs[offset / 8];
    }
}

void qwen_b200_embedding(void *ctx, unsigned token, unsigned row) {
    qwen_b200 *h = (qwen_b200 *)ctx;
    if (h && row < CSR_IDS) h->csr_ids[row] = token;
}

void qwen_b200_clear(void *ctx) {
    qwen_b200 *h = (qwen_b200 *)ctx;
    if (!h) return;
    if (h->csr_state == CSR_BUSY && h->loaded) {
        cudaSetDevice(h->cfg.device);
        cudaEventSynchronize(h->csr_event);
    }
    h->csr_state = CSR_IDLE;
    h->csr_error = 0;
    qwen_b200_reset(h, 0);
}

// ------------------------------------------------------------ operator level
int qwen_b200_op_embed(const uint16_t *embed, const uint32_t *ids, uint32_t rows, uint16_t *x, void *stream) {
    if (!embed || !ids || !x) return QWEN_B200_EINVAL;
    return launch_embed(embed, ids, (int)rows, x, (cudaStream_t)stream);
}

int qwen_b200_op_rmsnorm(const uint16_t *x, const uint16_t *gamma, uint32_t rows, float eps, uint16_t *out,
                         void *stream) {
    if (!x || !gamma || !out) return QWEN_B200_EINVAL;
    return launch_rmsnorm(x, gamma, (int)rows, eps, out, (cudaStream_t)stream);
}

int qwen_b200_op_gemm_w8a16(const uint16_t *x, uint32_t rows, uint32_t k, const int8_t *w, const float *scale,
                            uint32_t n, const uint16_t *bias, uint16_t *y, void *stream) {
    if (!x || !w || !scale || !y) return QWEN_B200_EINVAL;
    return launch_gemv(bias ? EPI_BIAS : EPI_PLAIN, x, (int)rows, (int)k, nullptr, 0.f, w, scale, bias, (int)n, y,
                       (cudaStream_t)stream);
}

int qwen_b200_op_gemm_w8a16_residual(const uint16_t *x, uint32_t rows, uint32_t k, const int8_t *w,
                                     const float *scale, uint32_t n, uint16_t *y, void *stream) {
    if (!x || !w || !scale || !y) return QWEN_B200_EINVAL;
    return launch_gemv(EPI_RESIDUAL, x, (int)rows, (int)k, nullptr, 0.f, w, scale, nullptr, (int)n, y,
                       (cudaStream_t)stream);
}

int qwen_b200_op_rope(uint16_t *x, uint32_t rows, uint32_t heads, const uint32_t *positions, const float *table,
                      void *stream) {
    if (!x || !positions || !table) return QWEN_B200_EINVAL;
    return launch_rope(x, (int)rows, (int)heads, positions, table, (cudaStream_t)stream);
}

int qwen_b200_op_kv8_append(const uint16_t *kv, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                            int8_t *codes, float *scales, uint32_t capacity, void *stream) {
    if (!kv || !slots || !positions || !codes || !scales) return QWEN_B200_EINVAL;
    return launch_kv8_append(kv, (int)rows, slots, positions, codes, scales, (int)capacity, (cudaStream_t)stream);
}

int qwen_b200_op_k16_append(const uint16_t *k, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                            int8_t *hi, int8_t *lo, uint16_t *m16, uint8_t *lock, uint32_t capacity, void *stream) {
    if (!k || !slots || !positions || !hi || !lo || !m16 || !lock || !rows || !capacity) return QWEN_B200_EINVAL;
    return launch_k16_append(k, (int)rows, slots, positions, hi, lo, m16, lock, (int)capacity, (cudaStream_t)stream);
}

int qwen_b200_op_v8_append(const uint16_t *v, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                           int8_t *codes, uint8_t *m8, uint8_t *lock, uint32_t capacity, void *stream) {
    if (!v || !slots || !positions || !codes || !m8 || !lock || !rows || !capacity) return QWEN_B200_EINVAL;
    return launch_v8_append(v, (int)rows, slots, positions, codes, m8, lock, (int)capacity, (cudaStream_t)stream);
}

int qwen_b200_op_qkv(const uint16_t *x, uint32_t rows, const uint16_t *gamma, float eps, const int8_t *w,
                     const float *scale, const uint16_t *bias, const uint32_t *slots, const uint32_t *positions,
                     const float *table, uint16_t *q_out, int8_t *kcodes, float *kscales, int8_t *vcodes,
                     float *vscales, uint32_t capacity, void *stream) {
    if (!x || !gamma || !w || !scale || !bias || !slots || !positions || !table || !q_out || !kcodes || !kscales ||
        !vcodes || !vscales)
        return QWEN_B200_EINVAL;
    QkvArgs a;
    a.x = x;
    a.rows = (int)rows;
    a.gamma = gamma;
    a.eps = eps;
    a.w = w;
    a.scale = scale;
    a.bias = bias;
    a.slots = slots;
    a.positions = positions;
    a.table = table;
    a.q_out = q_out;
    a.kc = kcodes;
    a.vc = vcodes;
    a.ks = kscales;
    a.vs = vscales;
    a.cap = (int)capacity;
    a.kv_out = nullptr;
    return launch_qkv(a, (cudaStream_t)stream);
}

size_t qwen_b200_attention_workspace(uint32_t rows, uint32_t capacity) {
    return attention_workspace((int)rows, (int)capacity);
}

int qwen_b200_op_attention(const uint16_t *q, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                           uint32_t max_len, const int8_t *kcodes, const float *kscales, const int8_t *vcodes,
                           const float *vscales, uint32_t capacity, uint16_t *ctx, void *workspace,
                           size_t workspace_bytes, void *stream) {
    if (!q || !slots || !positions || !kcodes || !kscales || !vcodes || !vscales || !ctx || !workspace)
        return QWEN_B200_EINVAL;
    return launch_attention(q, (int)rows, slots, positions, (int)max_len, kcodes, kscales, vcodes, vscales,
                            (int)capacity, ctx, workspace, workspace_bytes, (int)rows, true, (cudaStream_t)stream);
}

int qwen_b200_op_attention_cluster(const uint16_t *q, uint32_t rows, const uint32_t *slots, const uint32_t *positions,
                                   uint32_t max_len, const int8_t *kcodes, const float *kscales, const int8_t *vcodes,
                                   const float *vscales, uint32_t capacity, uint16_t *ctx, void *stream) {
    if (!q || !slots || !positions || !kcodes || !kscales || !vcodes || !vscales || !ctx) return QWEN_B200_EINVAL;
    return launch_attention_cluster(q, (int)rows, slots, positions, (int)max_len, kcodes, kscales, vcodes, vscales,
                                    (int)capacity, ctx, nullptr, (cudaStream_t)stream);
}

size_t qwen_b200_attention_prefill_workspace(uint32_t rows) { return 256 + (size_t)rows * sizeof(AtTile); }

int qwen_b200_op_attention_prefill(const uint16_t *q, uint32_t rows, uint32_t pos0, const int8_t *kcodes,
                                   const float *kscales, const int8_t *vcodes, const float *vscales, uint32_t capacity,
                                   uint16_t *ctx, void *workspace, size_t workspace_bytes, void *stream) {
    if (!q || !kcodes || !kscales || !vcodes || !vscales || !ctx || !workspace || !rows || !capacity)
        return QWEN_B200_EINVAL;
    if ((uint64_t)pos0 + rows > capacity || workspace_bytes < qwen_b200_attention_prefill_workspace(rows))
        return QWEN_B200_EINVAL;
    std::vector<uint32_t> slots(rows, 0u), pos(rows);
    for (uint32_t r = 0; r < rows; ++r) pos[r] = pos0 + r;
    std::vector<AtTile> tiles(rows);
    std::vector<AtGroup> groups;
    if (attention_tile_plan((int)rows, slots.data(), pos.data(), tiles.data(), groups)) return QWEN_B200_EINVAL;
    CUtensorMap kmap;
    if (make_kcache_map(&kmap, kcodes, 2ll * capacity)) return QWEN_B200_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    AtTile *d_tiles = reinterpret_cast<AtTile *>(reinterpret_cast<char *>(workspace) + 256);
    int ntiles = 0;
    for (const AtGroup &g : groups) ntiles += g.count;
    if (cudaMemcpyAsync(d_tiles, tiles.data(), (size_t)ntiles * sizeof(AtTile), cudaMemcpyHostToDevice, st) !=
        cudaSuccess)
        return QWEN_B200_EDEVICE;
    for (const AtGroup &g : groups) {
        const int rc = launch_attention_tiles(kmap, 0, d_tiles, g, q, vcodes, kscales, vscales, (int)capacity, ctx,
                                              reinterpret_cast<unsigned *>(workspace), st);
        if (rc) return rc == -1 ? QWEN_B200_EINVAL : QWEN_B200_EDEVICE;
    }
    // the host tile list must outlive the copy out of it
    return cudaStreamSynchronize(st) == cudaSuccess ? QWEN_B200_OK : QWEN_B200_EDEVICE;
}

int qwen_b200_op_swiglu(const uint16_t *x, uint32_t rows, const uint16_t *gamma, float eps, const int8_t *w_gu,
                        const float *s_gu, uint16_t *mid, void *stream) {
    if (!x || !w_gu || !s_gu || !mid) return QWEN_B200_EINVAL;
    return launch_gemv(EPI_SWIGLU, x, (int)rows, HID, gamma, eps, w_gu, s_gu, nullptr, 2 * FFN, mid,
                       (cudaStream_t)stream);
}

// Workspace of the standalone tensor-core GEMM: 256-byte error word, the
// split-K partial tiles of its split plan, the activation rows' four int8
// limb planes [4][rows][k] and their exponents [rows].
size_t qwen_b200_gemm_tc_workspace(uint32_t rows, uint32_t n, uint32_t k) {
    if (!rows || n % 128 || (k != HID && k != FFN)) return 256 + 4 * (size_t)rows * k + 4 * (size_t)rows;
    return tc_gemm_workspace((int)rows, (int)n, tc_pick_splits((int)rows, (int)n, (int)k)) + 4 * (size_t)rows * k +
           4 * (size_t)rows;
}

int qwen_b200_op_gemm_w8a16_tc(const uint16_t *x, uint32_t rows, uint32_t k, const int8_t *w,
                               const float *scale, uint32_t n, const uint16_t *bias, int epi, uint16_t *y,
                               void *workspace, size_t workspace_bytes, void *stream) {
    if (!x || !w || !scale || !y || !workspace || epi < EPI_PLAIN || epi > EPI_SWIGLU || !rows) return QWEN_B200_EINVAL;
    if (epi == EPI_BIAS && !bias) return QWEN_B200_EINVAL;
    if ((k != HID && k != FFN) || n % 128) return QWEN_B200_EINVAL;
    if (workspace_bytes < qwen_b200_gemm_tc_workspace(rows, n, k)) return QWEN_B200_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t plane = (size_t)rows * k;
    const int splits = tc_pick_splits((int)rows, (int)n, (int)k);
    int8_t *limbs = reinterpret_cast<int8_t *>(workspace) + tc_gemm_workspace((int)rows, (int)n, splits);
    int *ex = reinterpret_cast<int *>(limbs + 4 * plane);
    CUtensorMap wmap, lmap;
    if (make_weight_map(&wmap, w, (int)n, (int)k) || make_limb_map(&lmap, limbs, (int)rows, (int)k, plane, (int)k))
        return QWEN_B200_EINVAL;
    int rc = launch_act_quant(x, (int)rows, (int)k, limbs, plane, (int)k, ex, st);
    if (rc) return rc;
    return launch_gemm_tc(epi, wmap, lmap, ex, (int)rows, (int)k, scale, bias, (int)n, y, splits, workspace,
                          workspace_bytes, true, nullptr, st);
}

size_t qwen_b200_lm_head_workspace(uint32_t rows, uint32_t vocab) { return lm_head_workspace((int)rows, (int)vocab); }

int qwen_b200_op_lm_head_argmax(const uint16_t *x, uint32_t rows, const uint16_t *gamma, float eps,
                                const int8_t *w, const float *scale, uint32_t vocab, uint16_t *logits,
                                uint32_t *tokens, void *workspace, size_t workspace_bytes, void *stream) {
    if (!x || !w || !scale || !tokens || !workspace) return QWEN_B200_EINVAL;
    return launch_lm_head(x, (int)rows, gamma, eps, w, scale, (int)vocab, logits, tokens, workspace,
                          workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"
