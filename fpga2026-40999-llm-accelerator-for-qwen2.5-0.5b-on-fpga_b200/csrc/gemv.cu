// W8A16 GEMV-family kernels for small row counts (decode): int8 weights are
// streamed from HBM with 16-byte non-allocating loads and multiplied, as
// integers, with the activation rows held in shared memory as int8 limbs.
//
// Arithmetic contract (legacy_100mhz_closed/src/PC/model_backend.py:62-67,
// with the projection sums in the accelerator's order, oracle REF_EXACT):
//   E   = exponent of max|x[m][:]|, X[k] = rint(x[m][k] * 2^(26-E))
//   acc = RN32(sum_k X[k] * code[n][k]) * 2^(E-26)   (exact integer sum)
//   y   = bf16(bf16(acc) * scale[n])   (+ bias / residual / SiLU*mul)
// X is held as four signed 7-bit limbs (X = L0 + 2^7 L1 + 2^14 L2 + 2^21 L3);
// dp4a multiplies four codes by four limb bytes at a time, the limb sums fold
// in int64 and the lanes' partial sums are added exactly, so the result does
// not depend on how the sum is split.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "qkv_epi.cuh"
#include "xlimbs.cuh"

namespace qb {

// One warp: the dot products of RW weight rows with MT activation rows.
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

// acc[r][m] = RN32(sum_k X_m[k] * W[n0 + r][k]) * 2^(ex[m] - 26), exact sum.
template <int K, int RW, int MT>
__device__ __forceinline__ void gemv_dot(const GemvRows<K, RW> &g, const int8_t *xl, const int *ex,
                                         float (&acc)[RW][MT]) {
    constexpr int NCH = GemvRows<K, RW>::NCH, CPL = GemvRows<K, RW>::CPL;
    const int lane = threadIdx.x & 31;
    int d[RW][MT][4];
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int l = 0; l < 4; ++l) d[r][m][l] = 0;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        const int ch = lane + 32 * c;
        if (ch < NCH) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    const uint4 xw = *reinterpret_cast<const uint4 *>(xl + (size_t)(m * 4 + l) * K + ch * 16);
#pragma unroll
                    for (int r = 0; r < RW; ++r) {
                        int t = d[r][m][l];
                        t = __dp4a((int)g.wr[c][r].x, (int)xw.x, t);
                        t = __dp4a((int)g.wr[c][r].y, (int)xw.y, t);
                        t = __dp4a((int)g.wr[c][r].z, (int)xw.z, t);
                        t = __dp4a((int)g.wr[c][r].w, (int)xw.w, t);
                        d[r][m][l] = t;
                    }
                }
        }
    }
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            long long v = (long long)d[r][m][0] + ((long long)d[r][m][1] << 7) + ((long long)d[r][m][2] << 14) +
                          ((long long)d[r][m][3] << 21);
            v = warp_sum_ll(v);
            acc[r][m] = unalign28(v, ex[m]);
        }
}

template <int K, int RW, int NW, int MT, int EPI>
__global__ void __launch_bounds__(NW * 32) gemv_kernel(const uint16_t *__restrict__ x, int rows,
                                                       const uint16_t *__restrict__ gamma, float eps,
                                                       const int8_t *__restrict__ w, const float *__restrict__ scale,
                                                       const uint16_t *__restrict__ bias, int n, uint16_t *y) {
    extern __shared__ __align__(16) uint8_t gsm[];
    int8_t *xl = reinterpret_cast<int8_t *>(gsm);
    int *ex = reinterpret_cast<int *>(gsm + MT * 4 * K);
    const int m0 = blockIdx.y * MT;
    const int mrows = min(MT, rows - m0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = (blockIdx.x * NW + warp) * RW;
    GemvRows<K, RW> g;
    gemv_load<K, RW>(w, n0, n0 < n, g);
    pdl_wait();
    pdl_trigger();
    load_x_limbs<K, MT, NW * 32>(x, m0, mrows, gamma, eps, xl, ex);
    if (n0 >= n) return;
    float acc[RW][MT];
    gemv_dot<K, RW, MT>(g, xl, ex, acc);
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
                const float sl = silu_q(g);
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
    const size_t smem = (size_t)MT * (4 * K + 4);
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
    return run_gemv<K, RW, 8, 4, EPI>(x, rows, gamma, eps, w, scale, bias, n, y, st);  // 4-row tiles
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
    extern __shared__ __align__(16) uint8_t gsm[];
    int8_t *xl = reinterpret_cast<int8_t *>(gsm);
    int *ex = reinterpret_cast<int *>(gsm + MT * 4 * K);
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
    load_x_limbs<K, MT, 256>(a.x, m0, mrows, a.gamma, a.eps, xl, ex);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int local = warp * 8 + half * 4;
        const int n0 = hb * 64 + local;
        float acc[4][MT];
        gemv_dot<K, 4, MT>(g[half], xl, ex, acc);
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
    const size_t smem = (size_t)MT * (4 * QB_HID + 4);
    dim3 grid(QB_QH + 2 * QB_KVH, (a.rows + MT - 1) / MT);
    return launch_pdl(qkv_kernel<MT>, grid, dim3(256), smem, st, 1, a);
}

int launch_qkv(const QkvArgs &a, cudaStream_t st) {
    if (a.rows <= 0) return -1;
    if (a.rows <= 1) return run_qkv<1>(a, st);
    if (a.rows <= 2) return run_qkv<2>(a, st);
    return run_qkv<4>(a, st);  // 4-row tiles
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
                                                      int nblk, int n_base) {
    constexpr int K = QB_HID, RW = 4, NW = 8;
    extern __shared__ __align__(16) uint8_t gsm[];
    int8_t *xl = reinterpret_cast<int8_t *>(gsm);
    int *ex = reinterpret_cast<int *>(gsm + MT * 4 * K);
    __shared__ float bv[NW][MT];
    __shared__ uint32_t bi[NW][MT];
    const int m0 = blockIdx.y * MT;
    const int mrows = min(MT, rows - m0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the CTA walks 32-row blocks blockIdx.x, + gridDim.x, ...: the tile rows'
    // RMSNorm and limb planes once, the next block's weight rows in flight
    // while the current one is reduced
    int blk = blockIdx.x;
    GemvRows<K, RW> g;
    {
        const int n0 = (blk * NW + warp) * RW;
        gemv_load<K, RW>(w, n0, n0 < vocab, g);
    }
    pdl_wait();
    pdl_trigger();
    load_x_limbs<K, MT, NW * 32>(x, m0, mrows, gamma, eps, xl, ex);
    for (; blk < nblk; blk += gridDim.x) {
        const int n0 = (blk * NW + warp) * RW;
        GemvRows<K, RW> gn;
        const int nb = blk + (int)gridDim.x, n1 = (nb * NW + warp) * RW;
        if (nb < nblk) gemv_load<K, RW>(w, n1, n1 < vocab, gn);
        float best_v[MT];
        uint32_t best_i[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            best_v[m] = -INFINITY;
            best_i[m] = 0;
        }
        if (n0 < vocab) {
            float acc[RW][MT];
            gemv_dot<K, RW, MT>(g, xl, ex, acc);
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    const float v = rbf(rbf(acc[r][m]) * scale[n0 + r]);
                    if (better(v, (uint32_t)(n_base + n0 + r), best_v[m], best_i[m])) {
                        best_v[m] = v;
                        best_i[m] = (uint32_t)(n_base + n0 + r);
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
            pv[(size_t)(m0 + m) * nblk + blk] = v;
            pi[(size_t)(m0 + m) * nblk + blk] = i;
        }
        __syncthreads();  // bv / bi are written again by the next block
        if (nb < nblk) g = gn;
    }
}

__global__ void __launch_bounds__(256) argmax_reduce_kernel(const float *pv, const uint32_t *pi, int nblk,
                                                            uint32_t *tokens, float *values) {
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
    if (threadIdx.x == 0) {
        tokens[row] = si[0];
        if (values) values[row] = sv[0];
    }
}

int launch_argmax_reduce(const float *pv, const uint32_t *pi, int rows, int nblk, uint32_t *tokens, cudaStream_t st,
                         float *values) {
    return launch_pdl(argmax_reduce_kernel, dim3(rows), dim3(256), 0, st, 1, pv, pi, nblk, tokens, values);
}

size_t lm_head_workspace(int rows, int vocab) {
    const size_t nblk = (size_t)(vocab + 31) / 32;
    return (size_t)rows * nblk * 8 + 256;
}

template <int MT>
static int run_lm(const uint16_t *x, int rows, const uint16_t *gamma, float eps, const int8_t *w, const float *scale,
                  int vocab, uint16_t *logits, float *pv, uint32_t *pi, int nblk, int n_base, cudaStream_t st) {
    const size_t smem = (size_t)MT * (4 * QB_HID + 4);
    // as many CTAs per row tile as fit on the GPU at once (each then walks
    // several 32-row blocks): one RMSNorm per CTA instead of one per block
    static int resident = 0;
    if (!resident) {
        int dev = 0, sms = 0, per_sm = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lm_head_kernel<MT>, 256, smem) != cudaSuccess ||
            per_sm < 1)
            return -3;
        resident = sms * per_sm;
    }
    const int tiles = (rows + MT - 1) / MT;
    const int per_tile = std::max(1, std::min(nblk, resident / tiles));
    dim3 grid(per_tile, tiles);
    return launch_pdl(lm_head_kernel<MT>, grid, dim3(256), smem, st, 1, x, rows, gamma, eps, w, scale, vocab, logits,
                      pv, pi, nblk, n_base);
}

int launch_lm_head(const uint16_t *x, int rows, const uint16_t *gamma, float eps, const int8_t *w,
                   const float *scale, int vocab, uint16_t *logits, uint32_t *tokens, void *ws, size_t ws_bytes,
                   cudaStream_t st, int n_base, float *values) {
    if (rows <= 0 || vocab <= 0 || vocab % 4) return -1;
    if (ws_bytes < lm_head_workspace(rows, vocab)) return -1;
    const int nblk = (vocab + 31) / 32;
    float *pv = reinterpret_cast<float *>(ws);
    uint32_t *pi = reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(ws) + (size_t)rows * nblk * 4);
    int rc;
    if (rows <= 1)
        rc = run_lm<1>(x, rows, gamma, eps, w, scale, vocab, logits, pv, pi, nblk, n_base, st);
    else if (rows <= 2)
        rc = run_lm<2>(x, rows, gamma, eps, w, scale, vocab, logits, pv, pi, nblk, n_base, st);
    else
        rc = run_lm<4>(x, rows, gamma, eps, w, scale, vocab, logits, pv, pi, nblk, n_base, st);  // 4-row tiles
    if (rc) return rc;
    return launch_pdl(argmax_reduce_kernel, dim3(rows), dim3(256), 0, st, 1, pv, pi, nblk, tokens, values);
}

}  // namespace qb
