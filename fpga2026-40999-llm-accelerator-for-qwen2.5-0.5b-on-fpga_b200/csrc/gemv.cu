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
#include "tc05.cuh"
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

// One activation row: the LM head as one CTA per SM, each streaming its share
// of the vocabulary rows through a shared-memory ring of 32-row pieces (with
// their scales) filled by bulk copies from a producer warp, the row's RMSNorm
// and limb planes formed once per CTA. Warps 2 (p % 4) and 2 (p % 4) + 1 take
// the two 16-row halves of piece p on m16n8k32 int8 MMAs (weight rows as A,
// the four limb planes as the N columns; every per-limb sum exact in int32).
// The CTA's best (value, index) goes to pv / pi[blockIdx.x] for
// argmax_reduce. Every mbarrier wait is bounded (codes 48, 49 in *err).
constexpr int L1_ROWS = 32, L1_SLOTS = 6, L1_CW = 8, L1_THREADS = 32 * (L1_CW + 1);
constexpr int L1_WBYTES = L1_ROWS * QB_HID;     // weight rows of a piece
constexpr int L1_SLOT = L1_WBYTES + 160;        // + the piece's scales (16-byte aligned superset)
constexpr int L1_XL = L1_SLOTS * L1_SLOT;       // limb planes [4][896]
constexpr int L1_EX = L1_XL + 4 * QB_HID;       // row exponent (16 bytes)
constexpr int L1_BARS = L1_EX + 16;             // full [SLOTS], empty [SLOTS]
constexpr int L1_RED = L1_BARS + 2 * L1_SLOTS * 8;  // best value [8], index [8]
constexpr int L1_SMEM = L1_RED + L1_CW * 8;
static_assert(L1_SLOT % 16 == 0 && L1_XL % 16 == 0 && L1_BARS % 8 == 0, "aligned shared-memory areas");

// m16n8k32 int8 MMA (s8 x s8 -> s32), accumulating into d
__device__ __forceinline__ void l1_mma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// 16 weight rows [m0, m0 + 16) of a piece (rows >= nr read as 0) against the
// four limb planes (N columns 0..3), K = 896: thread (gid, tig) loads 16 bytes
// of rows gid and gid + 8 at k = 64 kb + 16 tig and the limb words at the same
// k; c = the accumulator fragment (rows gid | gid + 8, limbs 2 tig, 2 tig + 1).
__device__ __forceinline__ void l1_tile(const int8_t *w, int nr, int m0, const int8_t *xl, int (&c)[4]) {
    const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int ra = m0 + gid, rb = ra + 8;
    const int8_t *pa = w + ra * QB_HID + 16 * tig, *pb = w + rb * QB_HID + 16 * tig;
    const int8_t *px = xl + (gid & 3) * QB_HID + 16 * tig;
    c[0] = c[1] = c[2] = c[3] = 0;
#pragma unroll 2
    for (int kb = 0; kb < QB_HID / 64; ++kb) {
        const uint4 u = ra < nr ? *reinterpret_cast<const uint4 *>(pa + 64 * kb) : make_uint4(0u, 0u, 0u, 0u);
        const uint4 v = rb < nr ? *reinterpret_cast<const uint4 *>(pb + 64 * kb) : make_uint4(0u, 0u, 0u, 0u);
        const uint4 x = gid < 4 ? *reinterpret_cast<const uint4 *>(px + 64 * kb) : make_uint4(0u, 0u, 0u, 0u);
        l1_mma(c, u.x, v.x, u.y, v.y, x.x, x.y);
        l1_mma(c, u.z, v.z, u.w, v.w, x.z, x.w);
    }
}
__device__ __forceinline__ void l1_sync() { asm volatile("bar.sync 1, %0;" ::"n"(L1_CW * 32) : "memory"); }

__global__ void __launch_bounds__(L1_THREADS, 1)
    lm_head1_kernel(const uint16_t *__restrict__ x, const uint16_t *__restrict__ gamma, float eps,
                    const int8_t *__restrict__ w, const float *__restrict__ scale, int vocab, uint16_t *logits,
                    float *pv, uint32_t *pi, int n_base, unsigned *err) {
    extern __shared__ __align__(128) uint8_t sm[];
    int8_t *xl = reinterpret_cast<int8_t *>(sm + L1_XL);
    int *ex = reinterpret_cast<int *>(sm + L1_EX);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + L1_BARS), *empty = full + L1_SLOTS;
    float *bv = reinterpret_cast<float *>(sm + L1_RED);
    uint32_t *bi = reinterpret_cast<uint32_t *>(sm + L1_RED + L1_CW * 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = (int)((long long)vocab * blockIdx.x / gridDim.x);
    const int e = (int)((long long)vocab * (blockIdx.x + 1) / gridDim.x);
    const int np = (e - b + L1_ROWS - 1) / L1_ROWS;
    if (tid == 0) {
        for (int s = 0; s < L1_SLOTS; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], L1_CW);
        }
        tc::mbar_fence_init();
    }
    __syncthreads();
    if (warp == L1_CW) {
        // producer: the weights are constant, so they stream before the wait
        // for the kernel that writes x
        if (lane == 0)
            for (int p = 0; p < np; ++p) {
                const int s = p % L1_SLOTS;
                if (p >= L1_SLOTS && !tc::mbar_wait(&empty[s], (uint32_t)((p / L1_SLOTS) - 1) & 1u, err, 48)) break;
                const int r0 = b + p * L1_ROWS, nr = min(L1_ROWS, e - r0);
                const uintptr_t sa = reinterpret_cast<uintptr_t>(scale + r0), sal = sa & ~(uintptr_t)15,
                                send = (sa + 4 * (uintptr_t)nr + 15) & ~(uintptr_t)15;
                tc::mbar_arrive_expect_tx(&full[s], (uint32_t)(nr * QB_HID) + (uint32_t)(send - sal));
                tc::bulk_load(sm + s * L1_SLOT, w + (size_t)r0 * QB_HID, (uint32_t)(nr * QB_HID), &full[s]);
                tc::bulk_load(sm + s * L1_SLOT + L1_WBYTES, reinterpret_cast<const void *>(sal),
                              (uint32_t)(send - sal), &full[s]);
            }
        return;
    }
    pdl_wait();
    pdl_trigger();
    // (no CTA-wide barrier: the producer warp never joins one)
    load_x_limbs<QB_HID, 1, L1_CW * 32, false, false>(x, 0, 1, gamma, eps, xl, ex);
    l1_sync();
    const int e0 = ex[0];
    const int gid = lane >> 2, tig = lane & 3;
    float best = -INFINITY;
    uint32_t bidx = 0;
    bool ok = true;
    // piece p: warps 2 (p % 4) and 2 (p % 4) + 1 (one 16-row m-tile each);
    // every warp waits for every piece and releases it
    for (int p = 0; p < np; ++p) {
        const int s = p % L1_SLOTS;
        if (ok) ok = tc::mbar_wait(&full[s], (uint32_t)(p / L1_SLOTS) & 1u, err, 49);
        if ((p & 3) == (warp >> 1)) {
            const int r0 = b + p * L1_ROWS, nr = min(L1_ROWS, e - r0), m0 = 16 * (warp & 1);
            const int8_t *wp = reinterpret_cast<const int8_t *>(sm + s * L1_SLOT);
            const float *sp = reinterpret_cast<const float *>(sm + s * L1_SLOT + L1_WBYTES +
                                                              (reinterpret_cast<uintptr_t>(scale + r0) & 15));
            int cf[4];
            l1_tile(wp, nr, m0, xl, cf);
            // exact sums of rows m0 + gid and m0 + gid + 8 on the tig == 0 lanes
            // (limbs 2 and 3 from the tig == 1 lane)
            const int c0 = __shfl_down_sync(0xffffffffu, cf[0], 1), c1 = __shfl_down_sync(0xffffffffu, cf[1], 1);
            const int c2 = __shfl_down_sync(0xffffffffu, cf[2], 1), c3 = __shfl_down_sync(0xffffffffu, cf[3], 1);
            if (tig == 0) {
                const long long sum[2] = {
                    (long long)cf[0] + (long long)cf[1] * 128ll + (long long)c0 * 16384ll + (long long)c1 * 2097152ll,
                    (long long)cf[2] + (long long)cf[3] * 128ll + (long long)c2 * 16384ll + (long long)c3 * 2097152ll};
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int rr = m0 + gid + 8 * half;
                    if (rr < nr) {
                        const int row = r0 + rr;
                        const float val = rbf(rbf(unalign28(sum[half], e0)) * sp[rr]);
                        if (logits) logits[row] = f2bf(val);
                        if (better(val, (uint32_t)(n_base + row), best, bidx)) {
                            best = val;
                            bidx = (uint32_t)(n_base + row);
                        }
                    }
                }
            }
        }
        // this warp is done with the piece's shared memory
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
    // best of the warp (the tig == 0 lanes hold candidates)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (better(ov, oi, best, bidx)) {
            best = ov;
            bidx = oi;
        }
    }
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = bidx;
    }
    l1_sync();
    if (tid == 0) {
        float v = bv[0];
        uint32_t i = bi[0];
        for (int k = 1; k < L1_CW; ++k)
            if (better(bv[k], bi[k], v, i)) {
                v = bv[k];
                i = bi[k];
            }
        pv[blockIdx.x] = v;
        pi[blockIdx.x] = i;
    }
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
                   cudaStream_t st, int n_base, float *values, unsigned *err) {
    if (rows <= 0 || vocab <= 0 || vocab % 4) return -1;
    if (ws_bytes < lm_head_workspace(rows, vocab)) return -1;
    const int nblk = (vocab + 31) / 32;
    float *pv = reinterpret_cast<float *>(ws);
    uint32_t *pi = reinterpret_cast<uint32_t *>(reinterpret_cast<char *>(ws) + (size_t)rows * nblk * 4);
    int rc;
    if (rows == 1 && ((reinterpret_cast<uintptr_t>(w) & 15) == 0)) {
        static int sms = 0;
        if (!sms) {
            int dev = 0;
            if (cudaGetDevice(&dev) != cudaSuccess ||
                cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
                cudaFuncSetAttribute(lm_head1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L1_SMEM) !=
                    cudaSuccess)
                return -3;
        }
        // one CTA per SM, at least 32 rows each; bounded-wait codes go to err,
        // else to the word after pv / pi in the workspace
        const int grid = std::max(1, std::min(sms, (vocab + L1_ROWS - 1) / L1_ROWS));
        unsigned *flag = err ? err : reinterpret_cast<unsigned *>(reinterpret_cast<char *>(ws) + (size_t)rows * nblk * 8);
        rc = launch_pdl(lm_head1_kernel, dim3(grid), dim3(L1_THREADS), (size_t)L1_SMEM, st, 1, x, gamma, eps, w, scale,
                        vocab, logits, pv, pi, n_base, flag);
        if (rc) return rc;
        return launch_pdl(argmax_reduce_kernel, dim3(1), dim3(256), 0, st, 1, pv, pi, grid, tokens, values);
    }
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
