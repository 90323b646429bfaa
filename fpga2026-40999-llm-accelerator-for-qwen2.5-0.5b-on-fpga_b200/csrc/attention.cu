// GQA decode/prefill attention over the int8 (KV8) cache, split over context
// chunks of 128 keys so that long contexts spread across all SMs.
//
// Arithmetic contract (legacy_100mhz_closed/src/PC/model_backend.py:97-102
// over the KV8 cache in the accelerator's order, oracle ref_kv8_scores):
//   S[t]  = bf16(RN32(RN32(Q . kcode[t]) * 2^(E-26) * kscale[t]) / 8), q
//           aligned to its largest exponent E as 28-bit integers
//           Q[d] = rint(q[d] * 2^(26-E)), the dot product exact (four int8
//           limbs of Q against the codes with dp4a, combined in int64)
//   P[t]  = bf16(exp(S[t] - max S) * (1 / sum exp(S - max S)))
//   ctx   = bf16(sum_t P[t] * (vcode[t][d] * vscale[t]))
// Query head h reads KV head h / 7 (repeat_interleave(7), model_backend.py:97-98).
// The exact bf16 rounding of P needs the global max and sum before P.V, so:
//   pass 1 (score):  S for the chunk -> workspace, chunk max m_c and
//                    l_c = sum exp(S - m_c)
//   pass 2 (pv):     global max / sum from all chunk stats, P for the chunk,
//                    partial P.V -> workspace; the last CTA of a (row, kv head)
//                    adds the partials in chunk order and writes ctx.
// Cache layout: codes [slot][kv head][capacity][64] int8, scales
// [slot][kv head][capacity] fp32.
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "qwen_b200.h"

namespace qb {

constexpr int AT = 128;  // keys per chunk

struct AttnArgs {
    const uint16_t *q;
    const uint32_t *slots, *positions;
    const int8_t *kc, *vc;
    const float *ks, *vs;
    int cap;
    uint16_t *ctx;
    float *S;           // [rows][14][cap]
    float2 *stats;      // [rows][14][nck]
    float *part;        // [rows][14][nck][64]
    unsigned *counters; // [rows][2]
    int nck;            // chunk capacity = ceil(cap / AT)
};

struct AttnLayout {
    size_t cnt_off, s_off, st_off, part_off, total;
};

// Workspace regions for up to `rows` rows. The layout depends only on the
// workspace's row capacity, never on the rows of one launch, so the completion
// counters (first region) are never overwritten by another launch's scores.
static AttnLayout attn_layout(int rows, int cap) {
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t nck = (size_t)(cap + AT - 1) / AT;
    AttnLayout L;
    L.cnt_off = 0;
    L.s_off = al((size_t)rows * 2 * 4);
    L.st_off = L.s_off + al((size_t)rows * QB_QH * cap * 4);
    L.part_off = L.st_off + al((size_t)rows * QB_QH * nck * 8);
    L.total = L.part_off + al((size_t)rows * QB_QH * nck * 64 * 4);
    return L;
}

size_t attention_workspace(int rows, int cap) { return attn_layout(rows, cap).total; }

__global__ void __launch_bounds__(AT) attn_score_kernel(AttnArgs a) {
    const int c = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
    const int L = (int)a.positions[r] + 1;
    const int t0 = c * AT;
    if (t0 >= L) return;
    const int slot = (int)a.slots[r];
    // q of the group's heads as int8 limbs: ql[h][word][limb] holds dims
    // 4*word .. 4*word+3 of limb l of Q = rint(q * 2^(26-E_h))
    __shared__ __align__(16) uint32_t ql[7][16][4];
    __shared__ int qe[7];
    __shared__ float red[AT / 32][7];
    {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int h = warp; h < 7; h += AT / 32) {
            const uint16_t *qh = a.q + (size_t)r * QB_HID + (g * 7 + h) * QB_HD;
            const float q0 = bf2f(qh[lane]), q1 = bf2f(qh[lane + 32]);
            const float amax = warp_max(fmaxf(fabsf(q0), fabsf(q1)));
            const int e = row_exponent(amax);
            const float qv[2] = {q0, q1};
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int d = lane + 32 * k;
                const int qi = align28_int(qv[k], e);
                const int l0 = ((qi + 64) & 127) - 64;
                const int r1 = (qi - l0) >> 7;
                const int l1 = ((r1 + 64) & 127) - 64;
                const int r2 = (r1 - l1) >> 7;
                const int l2 = ((r2 + 64) & 127) - 64;
                const int l3 = (r2 - l2) >> 7;
                const int limb[4] = {l0, l1, l2, l3};
#pragma unroll
                for (int l = 0; l < 4; ++l)
                    reinterpret_cast<int8_t *>(&ql[h][d >> 2][l])[d & 3] = (int8_t)limb[l];
            }
            if (lane == 0) qe[h] = e;
        }
    }
    __syncthreads();
    const int t = t0 + threadIdx.x;
    const bool valid = t < L;
    float sc[7];
#pragma unroll
    for (int h = 0; h < 7; ++h) sc[h] = 0.f;
    if (valid) {
        const size_t base = ((size_t)slot * QB_KVH + g) * a.cap + t;
        const float s = a.ks[base];
        const uint4 *kp = reinterpret_cast<const uint4 *>(a.kc + base * QB_HD);
        int acc[7][4];
#pragma unroll
        for (int h = 0; h < 7; ++h)
#pragma unroll
            for (int l = 0; l < 4; ++l) acc[h][l] = 0;
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
            const uint4 kw = kp[v4];
            const int words[4] = {(int)kw.x, (int)kw.y, (int)kw.z, (int)kw.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                for (int h = 0; h < 7; ++h) {
                    const uint4 lq = *reinterpret_cast<const uint4 *>(&ql[h][v4 * 4 + wi][0]);
                    acc[h][0] = __dp4a(words[wi], (int)lq.x, acc[h][0]);
                    acc[h][1] = __dp4a(words[wi], (int)lq.y, acc[h][1]);
                    acc[h][2] = __dp4a(words[wi], (int)lq.z, acc[h][2]);
                    acc[h][3] = __dp4a(words[wi], (int)lq.w, acc[h][3]);
                }
        }
#pragma unroll
        for (int h = 0; h < 7; ++h) {
            const long long dot = (long long)acc[h][0] + ((long long)acc[h][1] << 7) + ((long long)acc[h][2] << 14) +
                                  ((long long)acc[h][3] << 21);
            sc[h] = rbf(__fmul_rn(unalign28(dot, qe[h]), s) * 0.125f);
            a.S[((size_t)r * QB_QH + g * 7 + h) * a.cap + t] = sc[h];
        }
    } else {
#pragma unroll
        for (int h = 0; h < 7; ++h) sc[h] = -INFINITY;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float mc[7];
#pragma unroll
    for (int h = 0; h < 7; ++h) {
        const float m = warp_max(sc[h]);
        if (lane == 0) red[warp][h] = m;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 7; ++h) {
        float m = red[0][h];
        for (int w = 1; w < AT / 32; ++w) m = fmaxf(m, red[w][h]);
        mc[h] = m;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 7; ++h) {
        const float e = valid ? expf(sc[h] - mc[h]) : 0.f;
        const float l = warp_sum(e);
        if (lane == 0) red[warp][h] = l;
    }
    __syncthreads();
    if (threadIdx.x < 7) {
        const int h = threadIdx.x;
        float l = 0.f;
        for (int w = 0; w < AT / 32; ++w) l += red[w][h];
        a.stats[((size_t)r * QB_QH + g * 7 + h) * a.nck + c] = make_float2(mc[h], l);
    }
}

__global__ void __launch_bounds__(7 * QB_HD) attn_pv_kernel(AttnArgs a) {
    const int c = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
    const int L = (int)a.positions[r] + 1;
    const int t0 = c * AT;
    if (t0 >= L) return;
    // Chunks actually launched for this row: a caller bound below positions+1
    // truncates the context instead of leaving the combine waiting for chunks.
    const int nch = min((L + AT - 1) / AT, (int)gridDim.x);
    const int slot = (int)a.slots[r];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ float Ms[7], Is[7];
    __shared__ float P[7][AT];
    __shared__ __align__(16) float V[AT][QB_HD];  // written with float4 stores
    __shared__ unsigned ticket;
    if (warp < 7) {
        const float2 *st = a.stats + ((size_t)r * QB_QH + g * 7 + warp) * a.nck;
        float mx = -INFINITY;
        for (int i = lane; i < nch; i += 32) mx = fmaxf(mx, st[i].x);
        mx = warp_max(mx);
        float z = 0.f;
        for (int i = lane; i < nch; i += 32) {
            const float2 s = st[i];
            z += s.y * expf(s.x - mx);
        }
        z = warp_sum(z);
        if (lane == 0) {
            Ms[warp] = mx;
            Is[warp] = 1.0f / z;
        }
    }
    // V chunk, dequantised to fp32: V[t][d] = code * scale.
    for (int i = tid; i < AT * 16; i += 7 * QB_HD) {
        const int tt = i >> 4, q4 = i & 15, t = t0 + tt;
        float f[4] = {0.f, 0.f, 0.f, 0.f};
        if (t < L) {
            const size_t base = ((size_t)slot * QB_KVH + g) * a.cap + t;
            const uint32_t w = *reinterpret_cast<const uint32_t *>(a.vc + base * QB_HD + q4 * 4);
            const float s = a.vs[base];
            i8x4_to_f32(w, f[0], f[1], f[2], f[3]);
#pragma unroll
            for (int j = 0; j < 4; ++j) f[j] = __fmul_rn(f[j], s);
        }
        *reinterpret_cast<float4 *>(&V[tt][q4 * 4]) = make_float4(f[0], f[1], f[2], f[3]);
    }
    __syncthreads();
    for (int i = tid; i < 7 * AT; i += 7 * QB_HD) {
        const int h = i / AT, tt = i % AT, t = t0 + tt;
        float p = 0.f;
        if (t < L) p = rbf(expf(a.S[((size_t)r * QB_QH + g * 7 + h) * a.cap + t] - Ms[h]) * Is[h]);
        P[h][tt] = p;
    }
    __syncthreads();
    const int h = tid >> 6, d = tid & 63;
    const int nt = min(AT, L - t0);
    float acc = 0.f;
    for (int tt = 0; tt < nt; ++tt) acc = fmaf(P[h][tt], V[tt][d], acc);
    float *pp = a.part + ((size_t)r * QB_QH + g * 7 + h) * a.nck * QB_HD;
    pp[(size_t)c * QB_HD + d] = acc;
    // The last CTA of this (row, kv head) combines the partials in chunk order.
    __threadfence();
    __syncthreads();
    if (tid == 0) ticket = atomicAdd(&a.counters[r * 2 + g], 1u);
    __syncthreads();
    if (ticket != (unsigned)(nch - 1)) return;
    __threadfence();
    float sum = 0.f;
    for (int cc = 0; cc < nch; ++cc) sum += __ldcg(pp + (size_t)cc * QB_HD + d);
    a.ctx[(size_t)r * QB_HID + (g * 7 + h) * QB_HD + d] = f2bf(sum);
    if (tid == 0) a.counters[r * 2 + g] = 0u;  // ready for the next launch
}

int launch_attention(const uint16_t *q, int rows, const uint32_t *slots, const uint32_t *positions, int max_len,
                     const int8_t *kc, const float *ks, const int8_t *vc, const float *vs, int cap, uint16_t *ctx,
                     void *ws, size_t ws_bytes, int ws_rows, bool clear_counters, cudaStream_t st) {
    if (rows <= 0 || rows > ws_rows || max_len <= 0 || max_len > cap) return -1;
    const AttnLayout L = attn_layout(ws_rows, cap);
    if (ws_bytes < L.total) return -1;
    char *base = reinterpret_cast<char *>(ws);
    AttnArgs a;
    a.q = q;
    a.slots = slots;
    a.positions = positions;
    a.kc = kc;
    a.vc = vc;
    a.ks = ks;
    a.vs = vs;
    a.cap = cap;
    a.ctx = ctx;
    a.S = reinterpret_cast<float *>(base + L.s_off);
    a.stats = reinterpret_cast<float2 *>(base + L.st_off);
    a.part = reinterpret_cast<float *>(base + L.part_off);
    a.counters = reinterpret_cast<unsigned *>(base + L.cnt_off);
    a.nck = (cap + AT - 1) / AT;
    if (clear_counters && cudaMemsetAsync(a.counters, 0, (size_t)rows * 2 * 4, st) != cudaSuccess) return -3;
    dim3 grid((max_len + AT - 1) / AT, QB_KVH, rows);
    attn_score_kernel<<<grid, AT, 0, st>>>(a);
    attn_pv_kernel<<<grid, 7 * QB_HD, 0, st>>>(a);
    return QB_LAUNCH_CHECK();
}

}  // namespace qb

namespace qb {

// ------------------------------------------------------- no-allocation variant
// Attention scratch for callers that cannot allocate device memory: one
// fixed array per GPU, part of the library image, held from the time the
// library is loaded on a device until the process exits.
static __device__ __align__(256) uint8_t g_attn_scratch[QWEN_B200_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
// per device: the address and the unique id of the context it belongs to
void *g_scratch_addr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long *);

// Unique id (cuCtxGetId: never reused within the process) of the context
// current on this thread; 0 when it cannot be read.
unsigned long long current_context_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static bool resolved = false;
    if (!resolved) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
        resolved = true;
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}
}  // namespace

// Device address of g_attn_scratch in the current context. Host code only
// sees a host-side stand-in under that name, so the address is looked up with
// the device current, once per device and context: after cudaDeviceReset, or
// when the caller makes another driver context current on the same device,
// the context id changes and the address is looked up again.
static int noalloc_scratch(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QWEN_B200_EDEVICE;
    unsigned long long ctx = current_context_id();  // 0 before the runtime has bound a context
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!ctx || !g_scratch_addr[dev] || g_scratch_ctx[dev] != ctx) {
        void *p = nullptr;
        // (binds the device's primary context first when none is current)
        if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return QWEN_B200_EDEVICE;
        }
        ctx = current_context_id();
        if (!ctx) return QWEN_B200_EDEVICE;
        g_scratch_addr[dev] = p;
        g_scratch_ctx[dev] = ctx;
    }
    *out = g_scratch_addr[dev];
    return QWEN_B200_OK;
}

}  // namespace qb

extern "C" int qwen_b200_op_attention_noalloc(const uint16_t *q, uint32_t rows, const uint32_t *slots,
                                              const uint32_t *positions, uint32_t max_len, const int8_t *kcodes,
                                              const float *kscales, const int8_t *vcodes, const float *vscales,
                                              uint32_t capacity, uint16_t *ctx, void *stream) {
    using namespace qb;
    if (!q || !slots || !positions || !kcodes || !kscales || !vcodes || !vscales || !ctx) return QWEN_B200_EINVAL;
    if (rows == 0 || capacity == 0) return QWEN_B200_EINVAL;
    // the request must fit the fixed scratch (checked before touching the GPU)
    if (attention_workspace((int)rows, (int)capacity) > (size_t)QWEN_B200_NOALLOC_SCRATCH_BYTES)
        return QWEN_B200_ESCRATCH;
    void *scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // the completion counters are zeroed at the start of every call; the rest
    // of the scratch is overwritten before it is read
    return launch_attention(q, (int)rows, slots, positions, (int)max_len, kcodes, kscales, vcodes, vscales,
                            (int)capacity, ctx, scratch, QWEN_B200_NOALLOC_SCRATCH_BYTES, (int)rows, true,
                            (cudaStream_t)stream);
}
