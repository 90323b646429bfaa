// W8A16 GEMM on the 5th-generation tensor cores (tcgen05) for batched decode
// and prefill. Swap-AB formulation: D^T[n][m] = W[n][:] . X[m][:], so the
// 128 output channels of a CTA tile fill the UMMA M dimension and the batch
// rows (BN of them) the N dimension.
//
//   warp 0      TMA producer: the int8 weight tile [128][64] (8 KB, contiguous
//               in the tiled layout [N/128][K/64][128][64]) by bulk copy into
//               an 8-deep ring, and the activation tile [BN rows][64 k] bf16 by
//               a 2D tensor-map load with 128-byte swizzle (zero fill past the
//               last row)
//   warp 1      owns TMEM (BN fp32 columns) and issues tcgen05.mma (one thread)
//   warps 2..9  dequantise each weight tile (exact int8 -> bf16) from the ring
//               into the 128-byte-swizzled K-major A stage; then the epilogue
//               (tcgen05.ld of the accumulator, per-channel scale, bf16
//               rounding points of model_backend.py:62-67, bias / residual /
//               SiLU*mul / LM-head argmax)
// Split-K: the CTAs of one output tile form a thread-block cluster. Each
// writes its fp32 partial tile to its own shared memory; after a cluster
// barrier every CTA reduces its share of the tile (32x32 units) by reading the
// partials of all CTAs over distributed shared memory in rank order and runs
// the epilogue on it. No global scratch, no atomics, deterministic.
// Every mbarrier wait is bounded: on timeout the kernel records an error code
// in a device flag, skips its remaining work and still frees its TMEM.
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace qb {

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;
constexpr int TC_STAGES = 4;   // bf16 A / B stages consumed by the MMA
constexpr int TC_WSTAGES = 8;  // int8 weight tiles in flight
constexpr int TC_CONV = 256;                 // dequant / epilogue threads (warps 2..9)
constexpr int TC_THREADS = 64 + TC_CONV;
constexpr int TC_MAX_SPLITS = 8;

template <int BN>
struct TcSmem {
    static constexpr int W_BYTES = TC_BM * TC_BK;      // 8 KB int8 tile
    static constexpr int A_BYTES = TC_BM * TC_BK * 2;  // 16 KB bf16 tile
    static constexpr int B_BYTES = BN * TC_BK * 2;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + TC_STAGES * A_BYTES;
    static constexpr int W_OFF = B_OFF + TC_STAGES * B_BYTES;
    static constexpr int BAR_OFF = W_OFF + TC_WSTAGES * W_BYTES;
    static constexpr int NBARS = 3 * TC_STAGES + 2 * TC_WSTAGES + 2;
    static constexpr int SLOT_OFF = BAR_OFF + NBARS * 8;
    static constexpr int RED_OFF = SLOT_OFF + 16;
    static constexpr int RED_BYTES = 4 * BN * 8;
    static constexpr int TOTAL = RED_OFF + RED_BYTES;
    static constexpr int ALLOC = TOTAL + 1024;  // slack for 1024-byte alignment of the stages
    static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Epilogue of 32 accumulators of output channel n: columns c0..c0+31 of the
// tile (batch rows m0 + c0 + j). Residual rows are read before any write.
template <int BN, int EPI>
__device__ __forceinline__ void tc_epilogue32(const TcArgs &a, const float (&v)[32], int n, int m0, int c0, int q,
                                              int lane, uint8_t *red) {
    const float sc = a.scale[n];
    float res[32];
    if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int m = m0 + c0 + j;
            res[j] = m < a.M ? bf2f(a.y[(size_t)m * a.N + n]) : 0.f;
        }
    }
    float bias = 0.f;
    if constexpr (EPI == EPI_BIAS) bias = bf2f(a.bias[n]);
    float *red_v = reinterpret_cast<float *>(red);
    uint32_t *red_i = reinterpret_cast<uint32_t *>(red + 4 * BN * 4);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const int cj = c0 + j, m = m0 + cj;
        const bool valid = m < a.M;
        float val = rbf(rbf(v[j]) * sc);
        if constexpr (EPI == EPI_SWIGLU) {
            // rows 2j (gate) and 2j+1 (up) sit in adjacent lanes
            const float other = __shfl_xor_sync(0xffffffffu, val, 1);
            if (valid && !(lane & 1)) {
                const float sl = val / (1.0f + expf(-val));
                a.y[(size_t)m * (a.N >> 1) + (n >> 1)] = f2bf(rbf(sl) * other);
            }
        } else if constexpr (EPI == EPI_ARGMAX) {
            if (valid && a.logits) a.logits[(size_t)m * a.N + n] = f2bf(val);
            float bv = valid ? val : -INFINITY;
            uint32_t bi = (uint32_t)n;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) {
                red_v[q * BN + cj] = bv;
                red_i[q * BN + cj] = bi;
            }
        } else if (valid) {
            if (EPI == EPI_BIAS) val = rbf(val + bias);
            if (EPI == EPI_RESIDUAL) val = rbf(res[j] + val);
            a.y[(size_t)m * a.N + n] = f2bf(val);
        }
    }
}

// Best (value, index) per batch row over the tile's four lane quarters.
template <int BN>
__device__ __forceinline__ void tc_argmax_flush(const TcArgs &a, const uint8_t *red, int m0, int n_tile, int ct) {
    const float *red_v = reinterpret_cast<const float *>(red);
    const uint32_t *red_i = reinterpret_cast<const uint32_t *>(red + 4 * BN * 4);
    for (int m = ct; m < BN; m += TC_CONV) {
        if (m0 + m >= a.M) continue;
        float bv = red_v[m];
        uint32_t bi = red_i[m];
        for (int qq = 1; qq < 4; ++qq)
            if (better(red_v[qq * BN + m], red_i[qq * BN + m], bv, bi)) {
                bv = red_v[qq * BN + m];
                bi = red_i[qq * BN + m];
            }
        a.pv[(size_t)(m0 + m) * a.nblk + n_tile] = bv;
        a.pi[(size_t)(m0 + m) * a.nblk + n_tile] = bi;
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap xmap, TcArgs a) {
    using L = TcSmem<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *full_a = bars, *full_b = bars + TC_STAGES, *empty = bars + 2 * TC_STAGES;
    uint64_t *w_full = bars + 3 * TC_STAGES, *w_empty = w_full + TC_WSTAGES;
    uint64_t *accum = w_empty + TC_WSTAGES, *done = accum + 1;
    uint32_t *slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = a.splits > 1 ? (int)tc::cluster_rank() : 0;
    const int n_tile = blockIdx.x / a.splits, m_tile = blockIdx.z;
    const int n0 = n_tile * TC_BM, m0 = m_tile * BN;
    const int KC = a.K / TC_BK;
    const int kc0 = split * a.kc_per_split;
    const int nk = min(KC, kc0 + a.kc_per_split) - kc0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; ++s) {
            tc::mbar_init(&full_a[s], TC_CONV);
            tc::mbar_init(&full_b[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < TC_WSTAGES; ++s) {
            tc::mbar_init(&w_full[s], 1);
            tc::mbar_init(&w_empty[s], TC_CONV);
        }
        tc::mbar_init(accum, 1);
        tc::mbar_init(done, 1);
        tc::mbar_fence_init();
        tc::tma_prefetch_desc(&xmap);
    }
    if (warp == 1) tc::tmem_alloc(slot, L::TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *slot;
    bool ok = nk > 0;

    if (warp == 0) {
        if (lane == 0 && ok) {
            // weight tiles run up to TC_WSTAGES ahead; activation tiles follow
            // the MMA's stage ring
            const int8_t *wsrc = a.w + ((size_t)n_tile * KC + kc0) * L::W_BYTES;
            int iw = 0, ib = 0;
            while (ok && ib < nk) {
                if (iw < nk && iw < ib + TC_WSTAGES) {
                    const int s = iw % TC_WSTAGES, ph = (iw / TC_WSTAGES) & 1;
                    if (tc::mbar_try_wait(&w_empty[s], ph ^ 1)) {
                        tc::mbar_arrive_expect_tx(&w_full[s], (uint32_t)L::W_BYTES);
                        tc::bulk_load(smem + L::W_OFF + s * L::W_BYTES, wsrc + (size_t)iw * L::W_BYTES,
                                      (uint32_t)L::W_BYTES, &w_full[s]);
                        ++iw;
                        continue;
                    }
                }
                const int s = ib % TC_STAGES, ph = (ib / TC_STAGES) & 1;
                if (ib < iw || iw == nk) {
                    if (!tc::mbar_wait(&empty[s], ph ^ 1, a.err, 1)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&full_b[s], (uint32_t)L::B_BYTES);
                    tc::tma_load_2d(smem + L::B_OFF + s * L::B_BYTES, &xmap, &full_b[s], (kc0 + ib) * TC_BK, m0);
                    ++ib;
                } else if (!tc::mbar_wait(&w_empty[iw % TC_WSTAGES], ((iw / TC_WSTAGES) & 1) ^ 1, a.err, 7)) {
                    ok = false;
                    break;
                }
            }
            while (ok && iw < nk) {
                const int s = iw % TC_WSTAGES, ph = (iw / TC_WSTAGES) & 1;
                if (!tc::mbar_wait(&w_empty[s], ph ^ 1, a.err, 7)) break;
                tc::mbar_arrive_expect_tx(&w_full[s], (uint32_t)L::W_BYTES);
                tc::bulk_load(smem + L::W_OFF + s * L::W_BYTES, wsrc + (size_t)iw * L::W_BYTES,
                              (uint32_t)L::W_BYTES, &w_full[s]);
                ++iw;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_bf16_f32(TC_BM, BN);
            int i = 0;
            for (; ok && i < nk; ++i) {
                const int s = i % TC_STAGES, ph = (i / TC_STAGES) & 1;
                if (!tc::mbar_wait(&full_a[s], ph, a.err, 2) || !tc::mbar_wait(&full_b[s], ph, a.err, 3)) break;
                tc::tc_fence_after();
                const uint32_t ab = tc::smem_u32(smem + L::A_OFF + s * L::A_BYTES);
                const uint32_t bb = tc::smem_u32(smem + L::B_OFF + s * L::B_BYTES);
#pragma unroll
                for (int j = 0; j < TC_BK / 16; ++j)
                    tc::mma_bf16(tmem, tc::smem_desc_sw128(ab + 32 * j), tc::smem_desc_sw128(bb + 32 * j), idesc,
                                 i > 0 || j > 0);
                tc::mma_commit(&empty[s]);
            }
            if (i == nk && ok) tc::mma_commit(accum);
            // all MMAs issued by this thread have finished before TMEM is freed
            tc::mma_commit(done);
            tc::mbar_wait(done, 0, a.err, 4);
        }
        __syncwarp();
    } else {
        // ---------------- weight dequantisation (TC_CONV threads)
        const int ct = threadIdx.x - 64;
        constexpr int ITEMS = TC_BM * TC_BK / 16 / TC_CONV;  // 16-byte pieces per thread per tile
        for (int i = 0; ok && i < nk; ++i) {
            const int s = i % TC_STAGES, ph = (i / TC_STAGES) & 1;
            const int sw = i % TC_WSTAGES, phw = (i / TC_WSTAGES) & 1;
            if (!tc::mbar_wait(&w_full[sw], phw, a.err, 8) || !tc::mbar_wait(&empty[s], ph ^ 1, a.err, 5)) {
                ok = false;
                break;
            }
            const uint4 *src = reinterpret_cast<const uint4 *>(smem + L::W_OFF + sw * L::W_BYTES);
            uint4 wv[ITEMS];
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) wv[j] = src[ct + TC_CONV * j];
            tc::mbar_arrive(&w_empty[sw]);  // the int8 slot may be refilled
            uint8_t *dst = smem + L::A_OFF + s * L::A_BYTES;
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) {
                const int item = ct + TC_CONV * j, row = item >> 2, piece = item & 3;
                const int c0 = (2 * piece) ^ (row & 7), c1 = (2 * piece + 1) ^ (row & 7);
                uint4 lo, hi;
                codes4_to_bf16(wv[j].x, lo.x, lo.y);
                codes4_to_bf16(wv[j].y, lo.z, lo.w);
                codes4_to_bf16(wv[j].z, hi.x, hi.y);
                codes4_to_bf16(wv[j].w, hi.z, hi.w);
                *reinterpret_cast<uint4 *>(dst + row * 128 + c0 * 16) = lo;
                *reinterpret_cast<uint4 *>(dst + row * 128 + c1 * 16) = hi;
            }
            tc::fence_proxy_async_smem();
            tc::mbar_arrive(&full_a[s]);
        }
        // ---------------- epilogue: this thread owns output channel n and
        // half of the tile's columns (two warps per TMEM lane quarter)
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        constexpr int HALF = BN / 2;
        const int cbeg = ((warp - 2) >> 2) * HALF;
        ok = ok && tc::mbar_wait(accum, 0, a.err, 6);
        tc::tc_fence_after();
        if (a.splits > 1) {
            // this warp's 32 x HALF block of the fp32 partial tile -> own shared
            // memory (the A stages are free once the accumulator is complete),
            // 16-byte groups rotated by lane to spread shared-memory banks
            float *part = reinterpret_cast<float *>(smem + L::A_OFF);
            const int unit = ((warp - 2) >> 2) * 4 + q;  // half * 4 + lane quarter
#pragma unroll 1
            for (int c = 0; c < HALF; c += 32) {
                float v[32];
                if (ok) {
                    tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cbeg + c), v);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0.f;
                }
                float *row = part + ((size_t)(unit * 32 + lane) * HALF + c);
#pragma unroll
                for (int g = 0; g < 8; ++g)
                    *reinterpret_cast<float4 *>(row + 4 * ((g + lane) & 7)) =
                        make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
            }
        } else {
            const int n = n0 + q * 32 + lane;
#pragma unroll 1
            for (int c = cbeg; c < cbeg + HALF; c += 32) {
                float v[32];
                if (ok) {
                    tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0.f;
                }
                tc_epilogue32<BN, EPI>(a, v, n, m0, c, q, lane, smem + L::RED_OFF);
            }
            if constexpr (EPI == EPI_ARGMAX) {
                epi_bar();
                tc_argmax_flush<BN>(a, smem + L::RED_OFF, m0, n_tile, ct);
            }
        }
    }
    if (EPI != EPI_ARGMAX && a.splits > 1) {  // the LM head (argmax) never splits K
        tc::cluster_sync();  // every partial tile of the cluster is in shared memory
        if (warp >= 2) {
            // unit u = (half, quarter) of the tile is reduced by CTA u % splits,
            // warp 2 + u / splits; sources are added in rank order
            const int j = warp - 2;
            const int u = j * a.splits + split;
            if (u < 8) {
                const int uq = u & 3, uhalf = u >> 2;
                const int n = n0 + uq * 32 + lane;
                constexpr int HALF = BN / 2;
                const float *part = reinterpret_cast<const float *>(smem + L::A_OFF);
#pragma unroll 1
                for (int c = 0; c < HALF; c += 32) {
                    const uint32_t row =
                        tc::smem_u32(part + ((size_t)(u * 32 + lane) * HALF + c));
                    float v[32];
#pragma unroll
                    for (int k = 0; k < 32; ++k) v[k] = 0.f;
                    for (int sr = 0; sr < a.splits; ++sr) {
#pragma unroll
                        for (int h = 0; h < 8; h += 4) {
                            float4 g4[4];
#pragma unroll
                            for (int g = 0; g < 4; ++g)
                                g4[g] = tc::ld_dsmem_f4(row + 16u * ((h + g + lane) & 7), sr);
#pragma unroll
                            for (int g = 0; g < 4; ++g) {
                                v[4 * (h + g)] += g4[g].x;
                                v[4 * (h + g) + 1] += g4[g].y;
                                v[4 * (h + g) + 2] += g4[g].z;
                                v[4 * (h + g) + 3] += g4[g].w;
                            }
                        }
                    }
                    tc_epilogue32<BN, EPI>(a, v, n, m0, uhalf * HALF + c, uq, lane, smem + L::RED_OFF);
                }
            }
        }
        tc::cluster_sync();  // no CTA leaves while another may still read its shared memory
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

// ------------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// Activation map: [rows][K] bf16 row-major, box [BN rows][64 k], 128-byte swizzle.
int make_act_map(CUtensorMap *map, const uint16_t *x, int rows, int K, int BN) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -3;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || K % TC_BK || rows <= 0) return -1;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)BN};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -3;
}

int tc_bn_for_rows(int rows) { return rows <= 64 ? 64 : 128; }

// Workspace: the 4-byte error flag of the bounded waits (256 bytes reserved).
size_t tc_gemm_workspace(int rows, int n, int splits) {
    (void)rows;
    (void)n;
    (void)splits;
    return 256;
}

int tc_pick_splits(int rows, int n, int k) {
    const int bn = tc_bn_for_rows(rows);
    const int tiles = (n / TC_BM) * ((rows + bn - 1) / bn);
    const int kc = k / TC_BK;
    int s = (148 + tiles - 1) / tiles;
    s = s < 1 ? 1 : s;
    s = s > TC_MAX_SPLITS ? TC_MAX_SPLITS : s;
    s = s > kc / 2 ? kc / 2 : s;  // at least two k chunks per split
    if (s < 1) s = 1;
    while (s > 1 && (s - 1) * ((kc + s - 1) / s) >= kc) --s;  // no empty split
    return s;
}

template <int BN, int EPI>
static int run_tc(const CUtensorMap &map, TcArgs &a, int splits, cudaStream_t st) {
    using L = TcSmem<BN>;
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << (dev & 31)))) {
        if (cudaFuncSetAttribute(tc_gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) !=
            cudaSuccess)
            return -3;
        configured |= 1u << (dev & 31);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.N / TC_BM) * splits, 1, (a.M + BN - 1) / BN);
    cfg.blockDim = dim3(TC_THREADS, 1, 1);
    cfg.dynamicSmemBytes = L::ALLOC;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)splits;  // the split CTAs of a tile share one cluster
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, EPI>, map, a) != cudaSuccess) return -3;
    return QB_LAUNCH_CHECK();
}

template <int BN>
static int dispatch_epi(int epi, const CUtensorMap &map, TcArgs &a, int splits, cudaStream_t st) {
    switch (epi) {
        case EPI_PLAIN: return run_tc<BN, EPI_PLAIN>(map, a, splits, st);
        case EPI_BIAS: return run_tc<BN, EPI_BIAS>(map, a, splits, st);
        case EPI_RESIDUAL: return run_tc<BN, EPI_RESIDUAL>(map, a, splits, st);
        case EPI_SWIGLU: return run_tc<BN, EPI_SWIGLU>(map, a, splits, st);
        case EPI_ARGMAX: return run_tc<BN, EPI_ARGMAX>(map, a, splits, st);
    }
    return -1;
}

int launch_gemm_tc(int epi, const CUtensorMap &xmap, int rows, int k, const int8_t *w_tiled, const float *scale,
                   const uint16_t *bias, int n, uint16_t *y, int splits, void *ws, size_t ws_bytes, bool clear,
                   const TcArgmax *am, cudaStream_t st) {
    if (rows <= 0 || n % TC_BM || k % TC_BK || splits < 1 || splits > k / TC_BK || splits > TC_MAX_SPLITS) return -1;
    if (epi == EPI_ARGMAX && (!am || splits != 1)) return -1;
    if (ws_bytes < tc_gemm_workspace(rows, n, splits)) return -1;
    const int bn = tc_bn_for_rows(rows);
    const int kc = k / TC_BK;
    const int kcps = (kc + splits - 1) / splits;
    if ((splits - 1) * kcps >= kc) return -1;  // every split owns at least one k chunk
    TcArgs a;
    a.w = w_tiled;
    a.scale = scale;
    a.bias = bias;
    a.y = y;
    a.M = rows;
    a.N = n;
    a.K = k;
    a.Mpad = ((rows + bn - 1) / bn) * bn;
    a.kc_per_split = kcps;
    a.splits = splits;
    a.err = reinterpret_cast<unsigned *>(ws);
    a.counters = nullptr;
    a.part = nullptr;
    a.pv = am ? am->pv : nullptr;
    a.pi = am ? am->pi : nullptr;
    a.nblk = am ? am->nblk : 0;
    a.logits = am ? am->logits : nullptr;
    if (clear) {
        if (cudaMemsetAsync(ws, 0, 256, st) != cudaSuccess) return -3;
        pdl_break();
    }
    return bn == 64 ? dispatch_epi<64>(epi, xmap, a, splits, st) : dispatch_epi<128>(epi, xmap, a, splits, st);
}

}  // namespace qb
