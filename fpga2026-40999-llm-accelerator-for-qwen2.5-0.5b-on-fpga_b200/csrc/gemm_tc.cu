// W8A16 GEMM on the 5th-generation tensor cores (tcgen05) for batched decode
// and prefill. Swap-AB formulation: D^T[n][m] = W[n][:] . X[m][:], so the
// 128 output channels of a CTA tile fill the UMMA M dimension and the batch
// rows (BN of them) the N dimension.
//
//   warp 0      producer: the int8 weight tile [128][64] (8 KB, contiguous in
//               the tiled layout [N/128][K/64][128][64]) by bulk copy into its
//               ring, and the activation tile [BN rows][64 k] bf16 by a 2D
//               tensor-map load with 128-byte swizzle (zero fill past the last
//               row) into a separate ring. Weights are constant, so the weight
//               ring is filled before the programmatic-launch wait for the
//               preceding kernel; activations are loaded after it.
//   warp 1      owns TMEM (BN fp32 columns) and issues tcgen05.mma (one thread)
//   warps 2..9  dequantise each weight tile (exact int8 -> bf16) into the
//               128-byte-swizzled K-major A stage; then the epilogue
// Epilogue: the fp32 accumulator tile is written transposed ([BN][128]) into
// the CTA's own shared memory (over the drained A/B stages). Split-K: the CTAs
// of one output tile form a thread-block cluster, and after a cluster barrier
// the 256 x splits epilogue threads of the cluster each take 4-channel items
// of the tile, load that item from every CTA's shared memory at once over
// distributed shared memory, add them in rank order and apply the epilogue
// (per-channel scale and the bf16 rounding points of model_backend.py:62-67,
// bias / residual / SiLU*mul) with vector loads and stores. The LM head
// (argmax epilogue) never splits K and reduces (value, index) per row in the
// CTA. No global scratch, no atomics, deterministic.
// Every mbarrier wait is bounded: on timeout the kernel records an error code
// in a device flag, skips its remaining work and still frees its TMEM.
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace qb {

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;
constexpr int TC_CONV = 256;                 // dequant / epilogue threads (warps 2..9)
constexpr int TC_THREADS = 64 + TC_CONV;
constexpr int TC_MAX_SPLITS = 8;
// One CTA per SM. With two co-resident CTAs per SM (smaller rings) a stress
// test of the 200-row SwiGLU shape returned a wrong 8-channel group (one
// dequantising warp's rows of one tile) in about 1 run in 10; with one CTA
// per SM it never did, whatever the ring depths.
// Split planning counts 2 x 148 CTA slots (a second wave for the largest
// tile counts).
constexpr int TC_SLOTS = 2 * 148;

// Shared memory: A (bf16 weights) | B (bf16 activations) | W (int8 weights)
// rings | mbarriers | TMEM address | argmax partials (about 195 KB). The
// accumulator tile [BN][128] fp32 of the epilogue reuses the A and B stages
// once every MMA has completed.
template <int BN>
struct TcSmem {
    static constexpr int A_STAGES = 4;
    static constexpr int B_STAGES = BN == 64 ? 8 : 4;
    static constexpr int W_STAGES = 8;
    static constexpr int W_BYTES = TC_BM * TC_BK;      // 8 KB int8 tile
    static constexpr int A_BYTES = TC_BM * TC_BK * 2;  // 16 KB bf16 tile
    static constexpr int B_BYTES = BN * TC_BK * 2;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + A_STAGES * A_BYTES;
    static constexpr int W_OFF = B_OFF + B_STAGES * B_BYTES;
    static constexpr int TILE_BYTES = BN * TC_BM * 4;
    static_assert(TILE_BYTES <= W_OFF, "accumulator tile must fit over the A and B stages");
    static constexpr int BAR_OFF = W_OFF + W_STAGES * W_BYTES;
    static constexpr int NBARS = 2 * A_STAGES + 2 * B_STAGES + 2 * W_STAGES + 2;
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

// Item i of the transposed accumulator tile: batch row m = i / 32 of the
// tile, channels 4*(i % 32) .. +3. The partial tiles of all `splits` CTAs of
// the cluster are read at once and added in rank order, then the epilogue of
// model_backend.py:62-67 runs on the four channels.
template <int BN, int EPI>
__device__ __forceinline__ void tc_epilogue4(const TcArgs &a, int i, int m0, int n0, uint32_t tile_saddr,
                                             const float *tile) {
    const int m = i >> 5, nl = 4 * (i & 31), n = n0 + nl, mg = m0 + m;
    const bool valid = mg < a.M;
    uint2 res = make_uint2(0u, 0u);
    if (EPI == EPI_RESIDUAL && valid) res = *reinterpret_cast<const uint2 *>(a.y + (size_t)mg * a.N + n);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.splits > 1) {
        const uint32_t addr = tile_saddr + (uint32_t)(m * TC_BM + nl) * 4u;
        float4 part[TC_MAX_SPLITS];
#pragma unroll
        for (int sr = 0; sr < TC_MAX_SPLITS; ++sr)
            if (sr < a.splits) part[sr] = tc::ld_dsmem_f4(addr, (uint32_t)sr);
#pragma unroll
        for (int sr = 0; sr < TC_MAX_SPLITS; ++sr)
            if (sr < a.splits) {
                v.x += part[sr].x;
                v.y += part[sr].y;
                v.z += part[sr].z;
                v.w += part[sr].w;
            }
    } else {
        const float4 p = *reinterpret_cast<const float4 *>(tile + m * TC_BM + nl);
        v.x += p.x;
        v.y += p.y;
        v.z += p.z;
        v.w += p.w;
    }
    if (!valid) return;
    const float4 sc = *reinterpret_cast<const float4 *>(a.scale + n);
    float o[4] = {rbf(rbf(v.x) * sc.x), rbf(rbf(v.y) * sc.y), rbf(rbf(v.z) * sc.z), rbf(rbf(v.w) * sc.w)};
    if constexpr (EPI == EPI_SWIGLU) {
        // channels 2j (gate j) and 2j+1 (up j): model_backend.py:105-106
        const float s0 = o[0] / (1.0f + expf(-o[0])), s1 = o[2] / (1.0f + expf(-o[2]));
        const uint32_t w = (uint32_t)f2bf(rbf(s0) * o[1]) | ((uint32_t)f2bf(rbf(s1) * o[3]) << 16);
        *reinterpret_cast<uint32_t *>(a.y + (size_t)mg * (a.N >> 1) + (n >> 1)) = w;
    } else {
        if constexpr (EPI == EPI_BIAS) {
            const uint2 b = *reinterpret_cast<const uint2 *>(a.bias + n);
            o[0] = rbf(o[0] + bflo(b.x));
            o[1] = rbf(o[1] + bfhi(b.x));
            o[2] = rbf(o[2] + bflo(b.y));
            o[3] = rbf(o[3] + bfhi(b.y));
        }
        if constexpr (EPI == EPI_RESIDUAL) {
            o[0] = rbf(bflo(res.x) + o[0]);
            o[1] = rbf(bfhi(res.x) + o[1]);
            o[2] = rbf(bflo(res.y) + o[2]);
            o[3] = rbf(bfhi(res.y) + o[3]);
        }
        uint2 w;
        w.x = (uint32_t)f2bf(o[0]) | ((uint32_t)f2bf(o[1]) << 16);
        w.y = (uint32_t)f2bf(o[2]) | ((uint32_t)f2bf(o[3]) << 16);
        *reinterpret_cast<uint2 *>(a.y + (size_t)mg * a.N + n) = w;
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap xmap, TcArgs a) {
    using L = TcSmem<BN>;
    constexpr int AS = L::A_STAGES, BS = L::B_STAGES, WS = L::W_STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *full_a = bars, *empty_a = full_a + AS, *full_b = empty_a + AS, *empty_b = full_b + BS;
    uint64_t *w_full = empty_b + BS, *w_empty = w_full + WS;
    uint64_t *accum = w_empty + WS, *done = accum + 1;
    uint32_t *slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = a.splits > 1 ? (int)tc::cluster_rank() : 0;
    const int n_tile = blockIdx.x / a.splits, m_tile = blockIdx.z;
    const int n0 = n_tile * TC_BM, m0 = m_tile * BN;
    const int KC = a.K / TC_BK;
    const int kc0 = split * a.kc_per_split;
    const int nk = min(KC, kc0 + a.kc_per_split) - kc0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < AS; ++s) {
            tc::mbar_init(&full_a[s], TC_CONV);
            tc::mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < BS; ++s) {
            tc::mbar_init(&full_b[s], 1);
            tc::mbar_init(&empty_b[s], 1);
        }
        for (int s = 0; s < WS; ++s) {
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
    pdl_trigger();
    bool ok = nk > 0;

    if (warp == 0) {
        if (lane == 0) {
            const int8_t *wsrc = a.w + ((size_t)n_tile * KC + kc0) * L::W_BYTES;
            int iw = 0, ib = 0;
            // weights are constant: fill the weight ring before waiting for the
            // kernel that produces the activations
            for (; ok && iw < min(nk, WS); ++iw) {
                tc::mbar_arrive_expect_tx(&w_full[iw], (uint32_t)L::W_BYTES);
                tc::bulk_load(smem + L::W_OFF + iw * L::W_BYTES, wsrc + (size_t)iw * L::W_BYTES, (uint32_t)L::W_BYTES,
                              &w_full[iw]);
            }
            pdl_wait();
            uint32_t idle = 0;
            while (ok && (ib < nk || iw < nk)) {
                bool progress = false;
                if (ib < nk) {
                    const int s = ib % BS, ph = (ib / BS) & 1;
                    if (tc::mbar_try_wait(&empty_b[s], ph ^ 1)) {
                        tc::mbar_arrive_expect_tx(&full_b[s], (uint32_t)L::B_BYTES);
                        tc::tma_load_2d(smem + L::B_OFF + s * L::B_BYTES, &xmap, &full_b[s], (kc0 + ib) * TC_BK, m0);
                        ++ib;
                        progress = true;
                    }
                }
                if (iw < nk) {
                    const int s = iw % WS, ph = (iw / WS) & 1;
                    if (tc::mbar_try_wait(&w_empty[s], ph ^ 1)) {
                        tc::mbar_arrive_expect_tx(&w_full[s], (uint32_t)L::W_BYTES);
                        tc::bulk_load(smem + L::W_OFF + s * L::W_BYTES, wsrc + (size_t)iw * L::W_BYTES,
                                      (uint32_t)L::W_BYTES, &w_full[s]);
                        ++iw;
                        progress = true;
                    }
                }
                if (progress) {
                    idle = 0;
                } else if (++idle > (1u << 21)) {
                    atomicExch(a.err, 1u);
                    ok = false;
                }
            }
        } else {
            pdl_wait();
        }
    } else if (warp == 1) {
        pdl_wait();
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_bf16_f32(TC_BM, BN);
            int i = 0;
            for (; ok && i < nk; ++i) {
                const int sa = i % AS, pa = (i / AS) & 1;
                const int sb = i % BS, pb = (i / BS) & 1;
                if (!tc::mbar_wait(&full_a[sa], pa, a.err, 2) || !tc::mbar_wait(&full_b[sb], pb, a.err, 3)) break;
                tc::tc_fence_after();
                const uint32_t ab = tc::smem_u32(smem + L::A_OFF + sa * L::A_BYTES);
                const uint32_t bb = tc::smem_u32(smem + L::B_OFF + sb * L::B_BYTES);
#pragma unroll
                for (int j = 0; j < TC_BK / 16; ++j)
                    tc::mma_bf16(tmem, tc::smem_desc_sw128(ab + 32 * j), tc::smem_desc_sw128(bb + 32 * j), idesc,
                                 i > 0 || j > 0);
                tc::mma_commit(&empty_a[sa]);
                tc::mma_commit(&empty_b[sb]);
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
            const int s = i % AS, ph = (i / AS) & 1;
            const int sw = i % WS, phw = (i / WS) & 1;
            if (!tc::mbar_wait(&w_full[sw], phw, a.err, 8) || !tc::mbar_wait(&empty_a[s], ph ^ 1, a.err, 5)) {
                ok = false;
                break;
            }
            // the tensor core's reads of this A stage (async proxy) are ordered
            // before the generic-proxy stores that refill it
            tc::fence_proxy_async_smem();
            const uint4 *src = reinterpret_cast<const uint4 *>(smem + L::W_OFF + sw * L::W_BYTES);
            uint4 wv[ITEMS];
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) wv[j] = src[ct + TC_CONV * j];
            tc::mbar_arrive(&w_empty[sw]);  // the int8 slot may be refilled
            uint8_t *dst = smem + L::A_OFF + s * L::A_BYTES;
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) {
                // the tiled layout stores codes in the byte order (k0, k2, k1,
                // k3), which codes4_to_bf16 unpacks to (k0, k1), (k2, k3)
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
        pdl_wait();  // residual rows and outputs of the preceding kernel
        // ---------------- epilogue: this thread owns output channel n (TMEM
        // lane) and half of the tile's columns (two warps per lane quarter)
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        constexpr int HALF = BN / 2;
        const int cbeg = ((warp - 2) >> 2) * HALF;
        ok = ok && tc::mbar_wait(accum, 0, a.err, 6);
        tc::tc_fence_after();
        tc::fence_proxy_async_smem();  // A/B stages (async-proxy traffic) become the generic accumulator tile
        if constexpr (EPI == EPI_ARGMAX) {
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
            epi_bar();
            tc_argmax_flush<BN>(a, smem + L::RED_OFF, m0, n_tile, ct);
        } else {
            // accumulator -> tile[m][n] (fp32), lanes on consecutive channels
            float *tile = reinterpret_cast<float *>(smem + L::A_OFF);
#pragma unroll 1
            for (int c = 0; c < HALF; c += 32) {
                float v[32];
                if (ok) {
                    tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cbeg + c), v);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0.f;
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) tile[(cbeg + c + j) * TC_BM + q * 32 + lane] = v[j];
            }
        }
    }
    if constexpr (EPI != EPI_ARGMAX) {
        // every partial tile of the cluster is complete in shared memory
        if (a.splits > 1)
            tc::cluster_sync();
        else
            __syncthreads();
        if (warp >= 2) {
            const float *tile = reinterpret_cast<const float *>(smem + L::A_OFF);
            const uint32_t tsa = tc::smem_u32(tile);
            for (int i = split * TC_CONV + (threadIdx.x - 64); i < BN * (TC_BM / 4); i += a.splits * TC_CONV)
                tc_epilogue4<BN, EPI>(a, i, m0, n0, tsa, tile);
        }
        if (a.splits > 1) tc::cluster_sync();  // no CTA leaves while another may still read its tile
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

// Splits of K so that the tiles fill TC_SLOTS CTA slots, with at least two k
// chunks per split and no empty split.
int tc_pick_splits(int rows, int n, int k) {
    const int bn = tc_bn_for_rows(rows);
    const int tiles = (n / TC_BM) * ((rows + bn - 1) / bn);
    const int kc = k / TC_BK;
    int s = TC_SLOTS / tiles;
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
    // the split CTAs of a tile share one cluster
    return launch_pdl(tc_gemm_kernel<BN, EPI>, dim3((a.N / TC_BM) * splits, 1, (a.M + BN - 1) / BN),
                      dim3(TC_THREADS), (size_t)L::ALLOC, st, (unsigned)splits, map, a);
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
    // vector loads and stores of the epilogue: 4 scales, 4 bias / output values
    if ((reinterpret_cast<uintptr_t>(scale) & 15) || (reinterpret_cast<uintptr_t>(bias) & 7) ||
        (reinterpret_cast<uintptr_t>(y) & 7))
        return -1;
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
