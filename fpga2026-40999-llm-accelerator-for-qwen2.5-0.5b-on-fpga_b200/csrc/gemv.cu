// W8A16 GEMV-family kernels for small row counts (decode): int8 weights are
// streamed from HBM with 16-byte non-allocating loads, dequantised in registers
// and multiplied with a bf16 activation tile held in shared memory; fp32
// accumulation, per-output-channel scale in the epilogue.
//
// Arithmetic contract (legacy_100mhz_closed/src/PC/model_backend.py:62-67):
//   y = bf16(bf16(sum_k x[k] * code[n][k]) * scale[n])   (+ bias / residual)
// Every product bf16 x int8 is exact in fp32; only the summation order differs
// from a sequential sum (per lane in k order, then a fixed butterfly).
#include "common.cuh"
#include "kernels.h"
#include "qkv_epi.cuh"

namespace qb {

// Loads rows [m0, m0+mrows) of x [rows][K] (bf16) into xs [MT][K] (zero rows
// beyond mrows); with gamma != nullptr applies RMSNorm in place:
// bf16(bf16(x * 1/sqrt(mean(x^2) + eps)) * gamma) (model_backend.py:69-71).
template <int K, int MT, int NT>
__device__ __forceinline__ void load_x_tile(const uint16_t *__restrict__ x, int m0, int mrows,
                                            const uint16_t *__restrict__ gamma, float eps, uint32_t *xs) {
    constexpr int V = K / 8;
    for (int i = threadIdx.x; i < MT * V; i += NT) {
        const int m = i / V, c = i - m * V;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (m < mrows) v = *reinterpret_cast<const uint4 *>(x + (size_t)(m0 + m) * K + c * 8);
        reinterpret_cast<uint4 *>(xs)[i] = v;
    }
    __syncthreads();
    if (gamma != nullptr) {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int m = warp; m < mrows; m += NT / 32) {
            uint32_t *row = xs + m * (K / 2);
            float ss = 0.f;
            for (int i = lane; i < K / 2; i += 32) {
                const uint32_t w = row[i];
                const float a = bflo(w), b = bfhi(w);
                ss += a * a;
                ss += b * b;
            }
            ss = warp_sum(ss);
            const float rs = 1.0f / sqrtf(ss / (float)K + eps);
            for (int i = lane; i < K / 2; i += 32) {
                const uint32_t w = row[i];
                const uint32_t gw = reinterpret_cast<const uint32_t *>(gamma)[i];
                const float a = rbf(rbf(bflo(w) * rs) * bflo(gw));
                const float b = rbf(rbf(bfhi(w) * rs) * bfhi(gw));
                row[i] = (uint32_t)f2bf(a) | ((uint32_t)f2bf(b) << 16);
            }
        }
        __syncthreads();
    }
}

// One warp: acc[r][m] = sum_k xs[m][k] * W[n0 + r][k] for RW rows, MT tile rows.
// Lane l owns 16-byte chunks l, l+32, ... of each weight row. gemv_load
// requests every chunk of the warp's rows (deep loads in flight; weights are
// constant, so this may precede pdl_wait), gemv_dot does the arithmetic.
template <int K, int RW>
struct GemvRows {
    static constexpr int NCH = K / 16, CPL = (NCH + 31) / 32;
    uint4 wr[CPL][RW];
};

template <int K, int RW>
__device__ __forceinline__ void gemv_load(const int8_t *__restrict__ w, int n0, bool active, GemvRows<K, RW> &g) {
    constexpr int NCH = GemvRows<K, RW>::NCH, CPL = GemvRows<K, RW>::CPL;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        const int ch = lane + 32 * c;
#pragma unroll
        for (int r = 0; r < RW; ++r)
            g.wr[c][r] = (active && ch < NCH) ? ldg_stream(w + (size_t)(n0 + r) * K + ch * 16)
                                             : make_uint4(0u, 0u, 0u, 0u);
    }
}

template <int K, int RW, int MT>
__device__ __forceinline__ void gemv_dot(const GemvRows<K, RW> &g, const uint32_t *xs, float (&acc)[RW][MT]) {
    constexpr int NCH = GemvRows<K, RW>::NCH, CPL = GemvRows<K, RW>::CPL;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[r][m] = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        const int ch = lane + 32 * c;
        if (ch < NCH) {
            float wf[RW][16];
#pragma unroll
            for (int r = 0; r < RW; ++r) {
                i8x4_to_f32(g.wr[c][r].x, wf[r][0], wf[r][1], wf[r][2], wf[r][3]);
                i8x4_to_f32(g.wr[c][r].y, wf[r][4], wf[r][5], wf[r][6], wf[r][7]);
                i8x4_to_f32(g.wr[c][r].z, wf[r][8], wf[r][9], wf[r][10], wf[r][11]);
                i8x4_to_f32(g.wr[c][r].w, wf[r][12], wf[r][13], wf[r][14], wf[r][15]);
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const uint4 *xp = reinterpret_cast<const uint4 *>(xs + m * (K / 2) + ch * 8);
                const uint4 a0 = xp[0], a1 = xp[1];
                const float xf[16] = {bflo(a0.x), bfhi(a0.x), bflo(a0.y), bfhi(a0.y), bflo(a0.z), bfhi(a0.z),
                                      bflo(a0.w), bfhi(a0.w), bflo(a1.x), bfhi(a1.x), bflo(a1.y), bfhi(a1.y),
                                      bflo(a1.z), bfhi(a1.z), bflo(a1.w), bfhi(a1.w)};
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[r][m] = fmaf(xf[j], wf[r][j], acc[r][m]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[r][m] = warp_sum(acc[r][m]);
}

template <int K, int RW, int NW, int MT, int EPI>
__global__ void __launch_bounds__(NW * 32) gemv_kernel(const uint16_t *__restrict__ x, int rows,
                                                       const uint16_t *__restrict__ gamma, float eps,
                                                       const int8_t *__restrict__ w, const float *__restrict__ scale,
                                                       const uint16_t *__restrict__ bias, int n, uint16_t *y) {
    extern __shared__ __align__(16) uint32_t xs[];
    const int m0 = blockIdx.y * MT;
    const int mrows = min(MT, rows - m0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = (blockIdx.x * NW + warp) * RW;
    GemvRows<K, RW> g;
    gemv_load<K, RW>(w, n0, n0 < n, g);
    pdl_wait();
    pdl_trigger();
    load_x_tile<K, MT, NW * 32>(x, m0, mrows, gamma, eps, xs);
    if (n0 >= n) return;
    float acc[RW][MT];
    gemv_dot<K, RW, MT>(g, xs, acc);
    if constexpr (EPI == EPI_SWIGLU) {
        // rows n0+2p (gate j) and n0+2p+1 (up j): model_backend.py:105-106
        const int nh = n >> 1;
#pragma unroll
        for (int p = 0; p < RW / 2; ++p)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (((p * MT + m) & 31) != lane || m >= mrows) continue;
                const int ng = n0 + 2 * p;
                const float g = rbf(rbf(acc[2 * p][m]) * scale[ng]);
                const float u = rbf(rbf(acc[2 * p + 1][m]) * scale[ng + 1]);
                const float sl = g / (1.0f + expf(-g));
                y[(size_t)(m0 + m) * nh + (ng >> 1)] = f2bf(rbf(sl) * u);
            }
    } else {
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (((r * MT + m) & 31) != lane || m >= mrows) continue;
                const int nn = n0 + r;
                float v = rbf(rbf(acc[r][m]) * scale[nn]);
                uint16_t *yp = y + (size_t)(m0 + m) * n + nn;
                if (EPI == EPI_BIAS) v = rbf(v + bf2f(bias[nn]));
                if (EPI == EPI_RESIDUAL) v = rbf(bf2f(*yp) + v);
                *yp = f2bf(v);
            }
    }
}

template <int K, int RW, int NW, int MT, int EPI>
static int run_gemv(const uint16_t *x, int rows, const uint16_t *gamma, float eps, const int8_t *w,
                    const float *scale, const uint16_t *bias, int n, uint16_t *y, cudaStream_t st) {
    const size_t smem = (size_t)MT * K * 2;
    if (smem > 48 * 1024) {
        // The opt-in is per device; remember it per device ordinal.
        static unsigned configured = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        if (!(configured & (1u << (dev & 31)))) {
            if (cudaFuncSetAttribute(gemv_kernel<K, RW, NW, MT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem) != cudaSuccess)
                return -3;
            configured |= 1u << (dev & 31);
        }
    }
    dim3 grid((n + RW * NW - 1) / (RW * NW), (rows + MT - 1) / MT);
    return launch_pdl(gemv_kernel<K, RW, NW, MT, EPI>, grid, dim3(NW * 32), smem, st, 1, x, rows, gamma, eps, w, scale,
                      bias, n, y);
}

template <int K, int RW, int EPI>
static int dispatch_mt(const uint16_t *x, int rows, const uint16_t *gamma, float eps, const int8_t *w,
                       const float *scale, const uint16_t *bias, int n, uint16_t *y, cudaStream_t st) {
    if (rows <= 1) return run_gemv<K, RW, 8, 1, EPI>(x, rows, gamma, eps, w, scale, bias, n, y, st);
    if (rows <= 2) return run_gemv<K, RW, 8, 2, EPI>(x, rows, gamma, eps, w, scale, bias, n, y, st);
    if (rows <= 4) return run_gemv<K, RW, 8, 4, EPI>(x, rows, gamma, eps, w, scale, bias, n, y, st);
    return run_gemv<K, RW, 8, 8, EPI>(x, rows, gamma, eps, w, scale, bias, n, y, st);
}

int launch_gemv(int epi, const uint16_t *x, int rows, int k, const uint16_t *gamma, float eps, const int8_t *w,
                const float *scale, const uint16_t *bias, int n, uint16_t *y, cudaStream_t st) {
    if (rows <= 0 || n <= 0 || n % 4) return -1;
    if (gamma && k != QB_HID) return -1;
    if (k == QB_HID) {
        switch (epi) {
            case EPI_PLAIN: return dispatch_mt<QB_HID, 4, EPI_PLAIN>(x, rows, gamma, eps, w, scale, bias, n, y, st);
            case EPI_BIAS: return dispatch_mt<QB_HID, 4, EPI_BIAS>(x, rows, gamma, eps, w, scale, bias, n, y, st);
            case EPI_RESIDUAL:
                return dispatch_mt<QB_HID, 4, EPI_RESIDUAL>(x, rows, gamma, eps, w, scale, bias, n, y, st);
            case EPI_SWIGLU:
                return dispatch_mt<QB_HID, 4, EPI_SWIGLU>(x, rows, gamma, eps, w, scale, bias, n, y, st);
        }
        return -1;
    }
    if (k == QB_FFN) {
        switch (epi) {
            case EPI_PLAIN: return dispatch_mt<QB_FFN, 1, EPI_PLAIN>(x, rows, gamma, eps, w, scale, bias, n, y, st);
            case EPI_BIAS: return dispatch_mt<QB_FFN, 1, EPI_BIAS>(x, rows, gamma, eps, w, scale, bias, n, y, st);
            case EPI_RESIDUAL:
                return dispatch_mt<QB_FFN, 1, EPI_RESIDUAL>(x, rows, gamma, eps, w, scale, bias, n, y, st);
        }
        return -1;
    }
    return -1;
}

// ---------------------------------------------------------------- QKV block
// One CTA per 64-row head block hb (q: 0..13, k: 14..15, v: 16..17) so that
// RoPE (pairs i, i+32) and the KV8 amax (64 dims) stay inside the CTA.
template <int MT>
__global__ void __launch_bounds__(256) qkv_kernel(QkvArgs a) {
    constexpr int K = QB_HID;
    extern __shared__ __align__(16) uint32_t xs[];
    __shared__ float outs[MT][64];
    const int m0 = blockIdx.y * MT;
    const int mrows = min(MT, a.rows - m0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hb = blockIdx.x;
    GemvRows<K, 4> g[2];
#pragma unroll
    for (int half = 0; half < 2; ++half) gemv_load<K, 4>(a.w, hb * 64 + warp * 8 + half * 4, true, g[half]);
    pdl_wait();
    pdl_trigger();
    load_x_tile<K, MT, 256>(a.x, m0, mrows, a.gamma, a.eps, xs);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int local = warp * 8 + half * 4;
        const int n0 = hb * 64 + local;
        float acc[4][MT];
        gemv_dot<K, 4, MT>(g[half], xs, acc);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (((r * MT + m) & 31) != lane || m >= mrows) continue;
                const int nn = n0 + r;
                // model_backend.py:66-67: bf16(bf16(bf16(acc) * scale) + bias)
                float v = rbf(rbf(acc[r][m]) * a.scale[nn]);
                outs[m][local + r] = rbf(v + bf2f(a.bias[nn]));
            }
    }
    __syncthreads();
    if (warp >= mrows) return;
    const int row = m0 + warp;
    qkv_head_epilogue(outs[warp][lane], outs[warp][lane + 32], row, hb, a.slots[row], a.positions[row], a.table,
                      a.q_out, a.kc, a.ks, a.vc, a.vs, a.cap, a.kv_out);
}

template <int MT>
static int run_qkv(const QkvArgs &a, cudaStream_t st) {
    const size_t smem = (size_t)MT * QB_HID * 2;
    dim3 grid(QB_QH + 2 * QB_KVH, (a.rows + MT - 1) / MT);
    return launch_pdl(qkv_kernel<MT>, grid, dim3(256), smem, st, 1, a);
}

int launch_qkv(const QkvArgs &a, cudaStream_t st) {
    if (a.rows <= 0) return -1;
    if (a.rows <= 1) return run_qkv<1>(a, st);
    if (a.rows <= 2) return run_qkv<2>(a, st);
    if (a.rows <= 4) return run_qkv<4>(a, st);
    return run_qkv<8>(a, st);
}

// ------------------------------------------------------------- LM head + argmax
// logits = bf16(bf16(acc) * scale) (model_backend.py:109); each CTA reduces
// its 32 rows to a (value, index) candidate per tile row; argmax_reduce picks
// the best per row with the highest index on ties (model_backend.py:113-114).
template <int MT>
__global__ void __launch_bounds__(256) lm_head_kernel(const uint16_t *__restrict__ x, int rows,
                                                      const uint16_t *__restrict__ gamma, float eps,
                                                      const int8_t *__restrict__ w, const float *__restrict__ scale,
                                                      int vocab, uint16_t *logits, float *pv, uint32_t *pi,
                                                      int nblk) {
    constexpr int K = QB_HID, RW = 4, NW = 8;
    extern __shared__ __align__(16) uint32_t xs[];
    __shared__ float bv[NW][MT];
    __shared__ uint32_t bi[NW][MT];
    const int m0 = blockIdx.y * MT;
    const int mrows = min(MT, rows - m0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = (blockIdx.x * NW + warp) * RW;
    GemvRows<K, RW> g;
    gemv_load<K, RW>(w, n0, n0 < vocab, g);
    pdl_wait();
    pdl_trigger();
    load_x_tile<K, MT, NW * 32>(x, m0, mrows, gamma, eps, xs);
    float best_v[MT];
    uint32_t best_i[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        best_v[m] = -INFINITY;
        best_i[m] = 0;
    }
    if (n0 < vocab) {
        float acc[RW][MT];
        gemv_dot<K, RW, MT>(g, xs, acc);
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const float v = rbf(rbf(acc[r][m]) * scale[n0 + r]);
                if (better(v, (uint32_t)(n0 + r), best_v[m], best_i[m])) {
                    best_v[m] = v;
                    best_i[m] = (uint32_t)(n0 + r);
                }
                if (logits && ((r * MT + m) & 31) == lane && m < mrows)
                    logits[(size_t)(m0 + m) * vocab + n0 + r] = f2bf(v);
            }
    }
    if (lane == 0)
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            bv[warp][m] = best_v[m];
            bi[warp][m] = best_i[m];
        }
    __syncthreads();
    if (threadIdx.x < mrows) {
        const int m = threadIdx.x;
        float v = bv[0][m];
        uint32_t i = bi[0][m];
        for (int k = 1; k < NW; ++k)
            if (better(bv[k][m], bi[k][m], v, i)) {
                v = bv[k][m];
                i = bi[k][m];
            }
        pv[(size_t)(m0 + m) * nblk + blockIdx.x] = v;
        pi[(size_t)(m0 + m) * nblk + blockIdx.x] = i;
    }
}

__global__ void __launch_bounds__(256) argmax_reduce_kernel(const float *pv, const uint32_t *pi, int nblk,
                                                            uint32_t *tokens) {
    __shared__ float sv[256];
    __shared__ uint32_t si[256];
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x;
    float v = -INFINITY;
    uint32_t i = 0;
    for (int k = threadIdx.x; k < nblk; k += 256) {
        const float cv = pv[(size_t)row * nblk + k];
        const uint32_t ci = pi[(size_t)row * nblk + k];
        if (better(cv, ci, v, i)) {
            v = cv;
            i = ci;
        }
    }
    sv[threadIdx.x] = v;
    si[threadIdx.x] = i;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (threadIdx.x < s && better(sv[threadIdx.x + s], si[threadIdx.x + s], sv[threadIdx.x], si[threadIdx.x])) {
            sv[threadIdx.x] = sv[threadIdx.x + s];
            si[threadIdx.x] = si[threadIdx.x + s];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) tokens[row] = si[0];
}

int launch_argmax_reduce(const float *pv, const uint32_t *pi, int rows, int nblk, uint32_t *tokens, cudaStream_t st) {
    return launch_pdl(argmax_reduce_kernel, dim3(rows), dim3(256), 0, st, 1, pv, pi, nblk, tokens);
}

size_t lm_head_workspace(int rows, int vocab) {
    const size_t nblk = (size_t)(vocab + 31) / 32;
    return (size_t)rows * nblk * 8 + 256;
}

template <int MT>
static int run_lm(const uint16_t *x, int rows, const uint16_t *gamma, float eps, const int8_t *w, const float *scale,
                  int vocab, uint16_t *logits, float *pv, uint32_t *pi, int nblk, cudaStream_t st) {
    const size_t smem = (size_t)MT * QB_HID * 2;
    dim3 grid(nblk, (rows + MT - 1) / MT);
    return launch_pdl(lm_head_kernel<MT>, grid, dim3(256), smem, st, 1, x, rows, gamma, eps, w, scale, vocab, logits,
                      pv, pi, nblk);
}

int launch_lm_head(const uint16_t *x, int rows, const uint16_t *gamma, float eps, const int8_t *w,
                   const float *scale, int vocab, uint16_t *logits, uint32_t *tokens, void *ws, size_t ws_bytes,
                   cudaStream_t st) {
    if (rows <= 0 || vocab <= 0 || vocab % 4) return -1;
    if (ws_bytes < lm_head_workspace(rows, vocab)) return -1;
    const int nblk = (vocab + 31) / 32;
    float *pv = reinterpret_cast<float *>(ws);
    uint32_t *pi = reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(ws) + (size_t)rows * nblk * 4);
    int rc;
    if (rows <= 1)
        rc = run_lm<1>(x, rows, gamma, eps, w, scale, vocab, logits, pv, pi, nblk, st);
    else if (rows <= 2)
        rc = run_lm<2>(x, rows, gamma, eps, w, scale, vocab, logits, pv, pi, nblk, st);
    else if (rows <= 4)
        rc = run_lm<4>(x, rows, gamma, eps, w, scale, vocab, logits, pv, pi, nblk, st);
    else
        rc = run_lm<8>(x, rows, gamma, eps, w, scale, vocab, logits, pv, pi, nblk, st);
    if (rc) return rc;
    return launch_pdl(argmax_reduce_kernel, dim3(rows), dim3(256), 0, st, 1, pv, pi, nblk, tokens);
}

}  // namespace qb
