// Exact W8A16 projections on the 5th-generation tensor cores (tcgen05,
// kind::i8) for batched decode and prefill. The arithmetic is the oracle's
// REF_EXACT order (the RTL array's block-aligned integer sums,
// src/rtl/qwen_gemm_array_i.sv, with one 28-bit alignment per activation row):
//   X[m][k] = L0 + 2^7 L1 + 2^14 L2 + 2^21 L3   (int8 limbs, made by
//             rmsnorm_kernel / act_quant_kernel, row exponent ex[m])
//   dot[n][m] = sum_k W[n][k] * X[m][k]          (exact: int32 per limb, int64)
//   acc = RN32(dot) * 2^(ex[m] - 26), then the bf16 rounding points of
//   model_backend.py:62-67 (scale, bias / residual / SiLU*mul / argmax)
// so every CTA shape and split-K plan gives the same bits.
//
// Swap-AB: 128 output channels fill UMMA M; the B operand is the four limb
// planes of 64 batch rows, 256 rows of 128 bytes (UMMA N = 256), so one
// tcgen05.mma.kind::i8 (K = 32) covers all limbs; TMEM holds D[128][256]
// int32 (column l*64 + m).
//   warp 0     producer: the weight tiles [128 n][128 k] (row-major int8, 2D
//              tensor map) into a 4-deep ring, the CTA's first 4 k chunks
//              (all of them for the split projections) issued before the
//              programmatic-launch wait, so they load while the preceding
//              kernel runs; the limb tiles
//              [4][64][128] (3D tensor map, from L2) into a 3-deep ring after
//              it; 128-byte swizzle
//   warp 1     owns TMEM (256 columns), issues the MMAs (one thread)
//   warps 2..9 epilogue: the four limb column groups of 16 rows are read from
//              TMEM together and fold into int64. Unsplit, the int64 tile
//              [64 rows][128 channels] is staged in the CTA's shared memory
//              (over the drained weight ring). Split-K CTAs of a tile form a
//              thread-block cluster and write their partial tiles straight
//              to an L2-resident workspace; after the cluster barrier each of
//              the 256 x splits epilogue threads takes 4-channel items, reads
//              the item's partials of every split at once and adds them
//              exactly (pulling the partials over distributed shared memory
//              instead measured ~4 us per tile). Per-channel scales and biases
//              are staged in shared memory before the launch wait, every
//              residual row a thread adds is requested before any is used.
// The LM head (argmax epilogue) is tc_lmhead_kernel below: the same roles in a
// persistent loop over tiles.
// No atomics; every TMA load fills this CTA's own shared memory. Every mbarrier wait is bounded: on timeout
// the kernel records an error code in a device flag, skips its remaining work
// and still frees its TMEM.
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace qb {

constexpr int TC_BM = 128;           // output channels per tile
constexpr int TC_BN = 64;            // batch rows per tile
constexpr int TC_BK = 128;           // k per stage (bytes of int8)
constexpr int TC_NL = 4;             // activation limbs
constexpr int TC_MN = TC_NL * TC_BN; // UMMA N
constexpr int TC_CONV = 512;         // epilogue threads (warps 2..17): four warps per TMEM lane quarter
constexpr int TC_THREADS = 64 + TC_CONV;
constexpr int TP_CONV = TC_CONV;     // the persistent kernels' epilogue threads
constexpr int TP_THREADS = 64 + TP_CONV;
constexpr int TC_MAX_SPLITS = 8;
constexpr int TC_SLOTS = 148;        // one CTA per SM

struct TcSmem {
    // 4 + 3 stages: measured against 7 + 3, 6 + 3, 5 + 3 and 6 + 2 (bs64 decode
    // 1.748 ms per step against 1.767, 1.752, 1.749 and 1.766); the smaller
    // footprint lets more of the neighbouring kernels overlap
    static constexpr int A_STAGES = 4, B_STAGES = 3;
    static constexpr int A_BYTES = TC_BM * TC_BK;  // 16 KB weight tile
    static constexpr int B_BYTES = TC_MN * TC_BK;  // 32 KB limb tile
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + A_STAGES * A_BYTES;
    static constexpr int TILE_BYTES = TC_BN * TC_BM * 8;  // int64 tile
    static_assert(TILE_BYTES <= B_OFF, "the int64 tile must fit over the weight ring");
    static constexpr int BAR_OFF = B_OFF + B_STAGES * B_BYTES;
    static constexpr int NBARS = 2 * A_STAGES + 2 * B_STAGES + 2;
    static constexpr int SLOT_OFF = BAR_OFF + NBARS * 8;
    static constexpr int SC_OFF = SLOT_OFF + 16;  // the tile's 128 scales, 128 biases (bf16), 64 row exponents
    static constexpr int SC_BYTES = TC_BM * 4 + TC_BM * 2 + TC_BN * 4;
    static constexpr int TOTAL = SC_OFF + SC_BYTES;
    static constexpr int ALLOC = TOTAL + 1024;  // slack for 1024-byte alignment of the stages
    static constexpr uint32_t TMEM_COLS = TC_MN;
};

// kind::i8 instruction descriptor: D s32, A and B signed int8, both K-major.
__host__ __device__ constexpr uint32_t idesc_s8_s32(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_s8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate));
}
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(tc::smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(tc::smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
// 16 columns of this warp's TMEM lane quarter; tmem_ld_wait() completes them
__device__ __forceinline__ void tmem_ld16i_nowait(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
// 8 columns of this warp's TMEM lane quarter; tmem_ld_wait() completes them
__device__ __forceinline__ void tmem_ld8i_nowait(uint32_t taddr, int (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ float exact_acc(long long dot, int e) { return unalign28(dot, e); }


// LM head: NR accumulators of output channel n (rows m0 + c0 + j), logits
// bf16(bf16(acc) * scale) (model_backend.py:109), best (value, index) per
// row over this warp's 32 channels into red (highest index on ties). The
// cross-lane reduction is a butterfly that halves the rows at each level
// (lanes exchange the half they do not keep), so a warp does NR - 1 + the
// remaining levels' exchanges instead of 5 per row; (value, index) order is
// a total order, so the result does not depend on the reduction order.
template <int NR>
__device__ __forceinline__ void tc_argmax_rows(const TcArgs &a, const float (&v)[NR], int n, int m0, int c0, int q,
                                               int lane, uint8_t *red) {
    static_assert(NR == 8 || NR == 16 || NR == 32, "rows per call");
    const float sc = a.scale[n];
    float *red_v = reinterpret_cast<float *>(red);
    uint32_t *red_i = reinterpret_cast<uint32_t *>(red + 4 * TC_BN * 4);
    float bv[NR];
    uint32_t bi[NR];
#pragma unroll
    for (int j = 0; j < NR; ++j) {
        const int m = m0 + c0 + j;
        const bool valid = m < a.M;
        const float val = rbf(rbf(v[j]) * sc);
        if (valid && a.logits) a.logits[(size_t)m * a.N + n] = f2bf(val);
        bv[j] = valid ? val : -INFINITY;
        bi[j] = (uint32_t)(a.n_base + n);
    }
    int row = 0;  // first row (of the NR) this lane holds after the halvings
#pragma unroll
    for (int lv = 0; lv < 5; ++lv) {
        const int o = 16 >> lv, cnt = NR >> lv;
        if (cnt > 1) {
            const int half = cnt >> 1;
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int k = 0; k < half; ++k) {
                const float sv = up ? bv[k] : bv[k + half];
                const uint32_t si = up ? bi[k] : bi[k + half];
                float kv = up ? bv[k + half] : bv[k];
                uint32_t ki = up ? bi[k + half] : bi[k];
                const float rv = __shfl_xor_sync(0xffffffffu, sv, o);
                const uint32_t ri = __shfl_xor_sync(0xffffffffu, si, o);
                if (better(rv, ri, kv, ki)) {
                    kv = rv;
                    ki = ri;
                }
                bv[k] = kv;
                bi[k] = ki;
            }
            if (up) row += half;
        } else {
            const float rv = __shfl_xor_sync(0xffffffffu, bv[0], o);
            const uint32_t ri = __shfl_xor_sync(0xffffffffu, bi[0], o);
            if (better(rv, ri, bv[0], bi[0])) {
                bv[0] = rv;
                bi[0] = ri;
            }
        }
    }
    // NR = 32: lane l holds row l; NR = 16: lanes 2r and 2r + 1 both hold row
    // r; NR = 8: lanes 4r .. 4r + 3
    if ((lane & (32 / NR - 1)) == 0) {
        red_v[q * TC_BN + c0 + row] = bv[0];
        red_i[q * TC_BN + c0 + row] = bi[0];
    }
}

// Best (value, index) per batch row over the tile's four lane quarters.
__device__ __forceinline__ void tc_argmax_flush(const TcArgs &a, const uint8_t *red, int m0, int n_tile, int ct) {
    const float *red_v = reinterpret_cast<const float *>(red);
    const uint32_t *red_i = reinterpret_cast<const uint32_t *>(red + 4 * TC_BN * 4);
    for (int m = ct; m < TC_BN; m += TC_CONV) {
        if (m0 + m >= a.M) continue;
        float bv = red_v[m];
        uint32_t bi = red_i[m];
        for (int qq = 1; qq < 4; ++qq)
            if (better(red_v[qq * TC_BN + m], red_i[qq * TC_BN + m], bv, bi)) {
                bv = red_v[qq * TC_BN + m];
                bi = red_i[qq * TC_BN + m];
            }
        a.pv[(size_t)(m0 + m) * a.nblk + n_tile] = bv;
        a.pi[(size_t)(m0 + m) * a.nblk + n_tile] = bi;
    }
}

// Item i of the int64 tile: batch row m = i / 32, channels 4*(i % 32) .. +3.
// The exact partials of all `splits` CTAs of the cluster are read at once and
// added, then the epilogue of model_backend.py:62-67 runs on the four channels.
template <int EPI>
__device__ __forceinline__ void tc_epilogue4(const TcArgs &a, int i, int m0, int n0, int tile_lin,
                                             const long long *tile, const uint8_t *sc_smem, uint2 res) {
    const int m = i >> 5, nl = 4 * (i & 31), n = n0 + nl, mg = m0 + m;
    const bool valid = mg < a.M;
    long long t[4] = {0, 0, 0, 0};
    if (a.splits > 1) {
        // the split CTAs' partials of these four channels, all requested at once
        const longlong2 *pp = reinterpret_cast<const longlong2 *>(
            a.part + (size_t)tile_lin * a.splits * (TC_BN * TC_BM) + m * TC_BM + nl);
        longlong2 p[TC_MAX_SPLITS][2];
#pragma unroll
        for (int sr = 0; sr < TC_MAX_SPLITS; ++sr)
            if (sr < a.splits) {
                p[sr][0] = __ldcg(pp + (size_t)sr * (TC_BN * TC_BM / 2));
                p[sr][1] = __ldcg(pp + (size_t)sr * (TC_BN * TC_BM / 2) + 1);
            }
#pragma unroll
        for (int sr = 0; sr < TC_MAX_SPLITS; ++sr)
            if (sr < a.splits) {
                t[0] += p[sr][0].x;
                t[1] += p[sr][0].y;
                t[2] += p[sr][1].x;
                t[3] += p[sr][1].y;
            }
    } else {
        const longlong2 u = *reinterpret_cast<const longlong2 *>(tile + m * TC_BM + nl);
        const longlong2 w = *reinterpret_cast<const longlong2 *>(tile + m * TC_BM + nl + 2);
        t[0] = u.x;
        t[1] = u.y;
        t[2] = w.x;
        t[3] = w.y;
    }
    if (!valid) return;
    const int e = reinterpret_cast<const int *>(sc_smem + TC_BM * 6)[m];
    const float4 sc = reinterpret_cast<const float4 *>(sc_smem)[nl >> 2];
    float o[4] = {rbf(rbf(exact_acc(t[0], e)) * sc.x), rbf(rbf(exact_acc(t[1], e)) * sc.y),
                  rbf(rbf(exact_acc(t[2], e)) * sc.z), rbf(rbf(exact_acc(t[3], e)) * sc.w)};
    if constexpr (EPI == EPI_SWIGLU) {
        // channels 2j (gate j) and 2j+1 (up j): model_backend.py:105-106
        const float s0 = silu_q(o[0]), s1 = silu_q(o[2]);
        const uint32_t w = (uint32_t)f2bf(rbf(s0) * o[1]) | ((uint32_t)f2bf(rbf(s1) * o[3]) << 16);
        *reinterpret_cast<uint32_t *>(a.y + (size_t)mg * (a.N >> 1) + (n >> 1)) = w;
    } else {
        if constexpr (EPI == EPI_BIAS) {
            const uint2 b = *reinterpret_cast<const uint2 *>(sc_smem + TC_BM * 4 + nl * 2);
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

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap lmap, TcArgs a) {
    using L = TcSmem;
    constexpr int AS = L::A_STAGES, BS = L::B_STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *full_a = bars, *empty_a = full_a + AS, *full_b = empty_a + AS, *empty_b = full_b + BS;
    uint64_t *accum = empty_b + BS, *done = accum + 1;
    uint32_t *slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = a.splits > 1 ? (int)tc::cluster_rank() : 0;
    const int n_tile = blockIdx.x / a.splits, m_tile = blockIdx.z;
    const int n0 = n_tile * TC_BM, m0 = m_tile * TC_BN;
    const int KC = a.K / TC_BK;
    const int kc0 = split * a.kc_per_split;
    const int nk = min(KC, kc0 + a.kc_per_split) - kc0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < AS; ++s) {
            tc::mbar_init(&full_a[s], 1);
            tc::mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < BS; ++s) {
            tc::mbar_init(&full_b[s], 1);
            tc::mbar_init(&empty_b[s], 1);
        }
        tc::mbar_init(accum, 1);
        tc::mbar_init(done, 1);
        tc::mbar_fence_init();
        tc::tma_prefetch_desc(&wmap);
        tc::tma_prefetch_desc(&lmap);
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
            int ia = 0, ib = 0;
            // weights are constant: fill the weight ring before waiting for the
            // kernel that produces the activation limbs
            for (; ok && ia < min(nk, AS); ++ia) {
                tc::mbar_arrive_expect_tx(&full_a[ia], (uint32_t)L::A_BYTES);
                tc::tma_load_2d(smem + L::A_OFF + ia * L::A_BYTES, &wmap, &full_a[ia], (kc0 + ia) * TC_BK, n0);
            }
            pdl_wait();
            uint32_t idle = 0;
            while (ok && (ib < nk || ia < nk)) {
                bool progress = false;
                if (ib < nk) {
                    const int s = ib % BS, ph = (ib / BS) & 1;
                    if (tc::mbar_try_wait(&empty_b[s], ph ^ 1)) {
                        tc::mbar_arrive_expect_tx(&full_b[s], (uint32_t)L::B_BYTES);
                        tma_load_3d(smem + L::B_OFF + s * L::B_BYTES, &lmap, &full_b[s], (kc0 + ib) * TC_BK, m0, 0);
                        ++ib;
                        progress = true;
                    }
                }
                if (ia < nk) {
                    const int s = ia % AS, ph = (ia / AS) & 1;
                    if (tc::mbar_try_wait(&empty_a[s], ph ^ 1)) {
                        tc::mbar_arrive_expect_tx(&full_a[s], (uint32_t)L::A_BYTES);
                        tc::tma_load_2d(smem + L::A_OFF + s * L::A_BYTES, &wmap, &full_a[s], (kc0 + ia) * TC_BK, n0);
                        ++ia;
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
            constexpr uint32_t idesc = idesc_s8_s32(TC_BM, TC_MN);
            int i = 0;
            for (; ok && i < nk; ++i) {
                const int sa = i % AS, pa = (i / AS) & 1;
                const int sb = i % BS, pb = (i / BS) & 1;
                if (!tc::mbar_wait(&full_a[sa], pa, a.err, 2) || !tc::mbar_wait(&full_b[sb], pb, a.err, 3)) break;
                tc::tc_fence_after();
                const uint32_t ab = tc::smem_u32(smem + L::A_OFF + sa * L::A_BYTES);
                const uint32_t bb = tc::smem_u32(smem + L::B_OFF + sb * L::B_BYTES);
#pragma unroll
                for (int j = 0; j < TC_BK / 32; ++j)
                    mma_s8(tmem, tc::smem_desc_sw128(ab + 32 * j), tc::smem_desc_sw128(bb + 32 * j), idesc,
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
        // this warp: TMEM lane quarter q (channels 32q..32q+31), rows 16h..16h+15
        const int q = warp & 3, h = (warp - 2) >> 2, ct = threadIdx.x - 64;
        // per-channel scales and biases are constants: staged before the wait
        float *scs = reinterpret_cast<float *>(smem + L::SC_OFF);
        uint16_t *bss = reinterpret_cast<uint16_t *>(smem + L::SC_OFF + TC_BM * 4);
        int *exs = reinterpret_cast<int *>(smem + L::SC_OFF + TC_BM * 6);
        if (ct < TC_BM) {
            scs[ct] = a.scale[n0 + ct];
            if (EPI == EPI_BIAS) bss[ct] = a.bias[n0 + ct];
        }
        pdl_wait();  // row exponents, residual rows and outputs of earlier kernels
        if (ct < TC_BN) exs[ct] = m0 + ct < a.M ? a.ex[m0 + ct] : 0;
        ok = ok && tc::mbar_wait(accum, 0, a.err, 6);
        tc::tc_fence_after();
        tc::fence_proxy_async_smem();  // the weight ring (async-proxy writes) becomes the generic int64 tile
        // the limbs of 16 rows at a time fold into int64 (keeps the fold in registers)
        long long *tile = reinterpret_cast<long long *>(smem + L::A_OFF);
        long long *pt = a.part + ((size_t)(m_tile * (a.N / TC_BM) + n_tile) * a.splits + split) * (TC_BN * TC_BM);
        {
            long long v[16];
            int d[TC_NL][16];
            // the four limb column groups in flight together, one wait
#pragma unroll
            for (int l = 0; l < TC_NL; ++l) {
                if (ok) {
                    tmem_ld16i_nowait(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(l * TC_BN + 16 * h), d[l]);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) d[l][j] = 0;
                }
            }
            if (ok) tmem_ld_wait();
            if (nk <= 14) {
                // |limb sum| <= 64 * 128 * 128 * nk < 2^24: limb pairs fold in
                // int32 (|l0 + 128 l1| < 2^31), then one int64 step
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int lo = d[0][j] + d[1][j] * 128, hi = d[2][j] + d[3][j] * 128;
                    v[j] = (long long)lo + (long long)hi * 16384ll;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    v[j] = (long long)d[0][j] + (long long)d[1][j] * 128ll + (long long)d[2][j] * 16384ll +
                           (long long)d[3][j] * 2097152ll;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int r = 16 * h + j;
                if (a.splits > 1)
                    pt[r * TC_BM + q * 32 + lane] = v[j];  // 256 contiguous bytes per warp and row
                else
                    tile[r * TC_BM + q * 32 + lane] = v[j];
            }
        }
    }
    {
        // every partial tile of the cluster is complete (in L2 when split,
        // cluster release/acquire orders the global writes; else in this CTA)
        if (a.splits > 1)
            tc::cluster_sync();
        else
            __syncthreads();
        if (warp >= 2) {
            const long long *tile = reinterpret_cast<const long long *>(smem + L::A_OFF);
            const int tile_lin = m_tile * (a.N / TC_BM) + n_tile;
            const uint8_t *sc = smem + L::SC_OFF;
            constexpr int ITEMS = TC_BN * (TC_BM / 4);  // 4-channel items of the tile
            constexpr int MAXK = ITEMS / TC_CONV;       // items per thread when the tile is not split
            const int i0 = split * TC_CONV + (threadIdx.x - 64), di = a.splits * TC_CONV;
            // every residual row this thread adds is requested before any is used
            uint2 res[MAXK];
#pragma unroll
            for (int k = 0; k < MAXK; ++k) {
                const int i = i0 + k * di, mg = m0 + (i >> 5);
                res[k] = make_uint2(0u, 0u);
                if (EPI == EPI_RESIDUAL && i < ITEMS && mg < a.M)
                    res[k] = *reinterpret_cast<const uint2 *>(a.y + (size_t)mg * a.N + n0 + 4 * (i & 31));
            }
#pragma unroll
            for (int k = 0; k < MAXK; ++k) {
                const int i = i0 + k * di;
                if (i < ITEMS) tc_epilogue4<EPI>(a, i, m0, n0, tile_lin, tile, sc, res[k]);
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

// ---------------------------------------------------------- LM head (argmax)
// The vocabulary projection as a persistent kernel: one CTA per SM walks the
// (row tile, 128-channel tile) list with a stride of the grid, so weight and
// limb tiles stream without a gap between tiles. The accumulator is double
// buffered in TMEM (2 x 256 columns): the MMA warp fills one buffer while the
// epilogue warps fold, scale and reduce the other to per-row (value, index)
// candidates. Same roles and arithmetic as tc_gemm_kernel.
struct LhSmem {
    static constexpr int A_STAGES = 4, B_STAGES = 4;
    static constexpr int A_BYTES = TC_BM * TC_BK;
    static constexpr int B_BYTES = TC_MN * TC_BK;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + A_STAGES * A_BYTES;
    static constexpr int BAR_OFF = B_OFF + B_STAGES * B_BYTES;
    static constexpr int NBARS = 2 * A_STAGES + 2 * B_STAGES + 4 + 1;
    static constexpr int SLOT_OFF = BAR_OFF + ((NBARS * 8 + 15) / 16) * 16;
    static constexpr int RED_OFF = SLOT_OFF + 16;
    static constexpr int RED_BYTES = 4 * TC_BN * 8;  // per buffer: best value and index per (quarter, row)
    static constexpr int TOTAL = RED_OFF + 2 * RED_BYTES;
    static constexpr int ALLOC = TOTAL + 1024;
    static constexpr uint32_t TMEM_COLS = 2 * TC_MN;
    static_assert(ALLOC <= 227 * 1024, "shared memory of one CTA");
};

// Barrier 1 over the N epilogue threads, returning the AND of v over them
// (every epilogue thread leaves a tile loop at the same iteration).
template <int N>
__device__ __forceinline__ bool epi_bar_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(N)
        : "memory");
    return r != 0;
}

__global__ void __launch_bounds__(TP_THREADS, 1)
    tc_lmhead_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap lmap, TcArgs a) {
    using L = LhSmem;
    constexpr int AS = L::A_STAGES, BS = L::B_STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *full_a = bars, *empty_a = full_a + AS, *full_b = empty_a + AS, *empty_b = full_b + BS;
    uint64_t *acc_full = empty_b + BS, *acc_empty = acc_full + 2, *done = acc_empty + 2;
    uint32_t *slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntn = a.N / TC_BM;                               // channel tiles
    const int total = ntn * ((a.M + TC_BN - 1) / TC_BN);       // (row tile, channel tile) pairs
    const int G = (int)gridDim.x;
    const int nt = total > (int)blockIdx.x ? (total - (int)blockIdx.x + G - 1) / G : 0;  // this CTA's tiles
    const int KC = a.K / TC_BK;
    const int nchunks = nt * KC;

    if (threadIdx.x == 0) {
        for (int s = 0; s < AS; ++s) {
            tc::mbar_init(&full_a[s], 1);
            tc::mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < BS; ++s) {
            tc::mbar_init(&full_b[s], 1);
            tc::mbar_init(&empty_b[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], TP_CONV / 32);  // one arrival per epilogue warp
        }
        tc::mbar_init(done, 1);
        tc::mbar_fence_init();
        tc::tma_prefetch_desc(&wmap);
        tc::tma_prefetch_desc(&lmap);
    }
    if (warp == 1) tc::tmem_alloc(slot, L::TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *slot;
    pdl_trigger();
    bool ok = nt > 0;

    if (warp == 0) {
        if (lane == 0) {
            auto tile_of = [&](int g, int &n0, int &m0) {
                const int t = (int)blockIdx.x + (g / KC) * G;
                n0 = (t % ntn) * TC_BM;
                m0 = (t / ntn) * TC_BN;
            };
            auto issue_a = [&](int g) {
                int n0, m0;
                tile_of(g, n0, m0);
                const int s = g % AS;
                tc::mbar_arrive_expect_tx(&full_a[s], (uint32_t)L::A_BYTES);
                tc::tma_load_2d(smem + L::A_OFF + s * L::A_BYTES, &wmap, &full_a[s], (g % KC) * TC_BK, a.n_base + n0);
            };
            int ia = 0, ib = 0;
            // weights are constant: the first stages load before the wait for
            // the kernel that writes the limb planes
            for (; ok && ia < min(nchunks, AS); ++ia) issue_a(ia);
            pdl_wait();
            uint32_t idle = 0;
            while (ok && (ib < nchunks || ia < nchunks)) {
                bool progress = false;
                if (ib < nchunks) {
                    const int s = ib % BS, ph = (ib / BS) & 1;
                    if (tc::mbar_try_wait(&empty_b[s], ph ^ 1)) {
                        int n0, m0;
                        tile_of(ib, n0, m0);
                        tc::mbar_arrive_expect_tx(&full_b[s], (uint32_t)L::B_BYTES);
                        tma_load_3d(smem + L::B_OFF + s * L::B_BYTES, &lmap, &full_b[s], (ib % KC) * TC_BK, m0, 0);
                        ++ib;
                        progress = true;
                    }
                }
                if (ia < nchunks) {
                    const int s = ia % AS, ph = (ia / AS) & 1;
                    if (tc::mbar_try_wait(&empty_a[s], ph ^ 1)) {
                        issue_a(ia);
                        ++ia;
                        progress = true;
                    }
                }
                if (progress) {
                    idle = 0;
                } else if (++idle > (1u << 22)) {
                    atomicExch(a.err, 21u);
                    ok = false;
                }
            }
        } else {
            pdl_wait();
        }
    } else if (warp == 1) {
        pdl_wait();
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_s8_s32(TC_BM, TC_MN);
            for (int j = 0; ok && j < nt; ++j) {
                const int buf = j & 1;
                // the epilogue has read this buffer's previous tile
                if (j >= 2 && !tc::mbar_wait(&acc_empty[buf], ((j >> 1) - 1) & 1, a.err, 22)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * TC_MN);
                for (int kc = 0; kc < KC; ++kc) {
                    const int g = j * KC + kc;
                    const int sa = g % AS, sb = g % BS;
                    if (!tc::mbar_wait(&full_a[sa], (g / AS) & 1, a.err, 23) ||
                        !tc::mbar_wait(&full_b[sb], (g / BS) & 1, a.err, 24)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t ab = tc::smem_u32(smem + L::A_OFF + sa * L::A_BYTES);
                    const uint32_t bb = tc::smem_u32(smem + L::B_OFF + sb * L::B_BYTES);
#pragma unroll
                    for (int k = 0; k < TC_BK / 32; ++k)
                        mma_s8(d, tc::smem_desc_sw128(ab + 32 * k), tc::smem_desc_sw128(bb + 32 * k), idesc,
                               kc > 0 || k > 0);
                    tc::mma_commit(&empty_a[sa]);
                    tc::mma_commit(&empty_b[sb]);
                }
                if (ok) tc::mma_commit(&acc_full[buf]);
            }
            // every MMA issued by this thread has finished before TMEM is freed
            tc::mma_commit(done);
            tc::mbar_wait(done, 0, a.err, 25);
        }
        __syncwarp();
    } else {
        // lane quarter q (channels 32q..32q+31 of a tile), rows 16h..16h+15
        // (16 epilogue warps: four per quarter), in two sub-passes of 8 rows
        const int q = warp & 3, h = (warp - 2) >> 2, ct = threadIdx.x - 64;
        pdl_wait();  // row exponents come from the preceding kernel
        for (int j = 0; j < nt; ++j) {
            const int buf = j & 1;
            const int t = (int)blockIdx.x + j * G;
            const int n_tile = t % ntn, n0 = n_tile * TC_BM, m0 = (t / ntn) * TC_BN;
            ok = ok && tc::mbar_wait(&acc_full[buf], (j >> 1) & 1, a.err, 26);
            tc::tc_fence_after();
            uint8_t *red = smem + L::RED_OFF + buf * L::RED_BYTES;
#pragma unroll 1
            for (int sp = 0; sp < 2; ++sp) {
                const int c0 = 16 * h + 8 * sp;  // first of this sub-pass's 8 rows in the tile
                float f[8];
                int d[TC_NL][8];
#pragma unroll
                for (int l = 0; l < TC_NL; ++l) {
                    if (ok) {
                        tmem_ld8i_nowait(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * TC_MN + l * TC_BN + c0),
                                         d[l]);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) d[l][jj] = 0;
                    }
                }
                int exr[8];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) exr[jj] = m0 + c0 + jj < a.M ? __ldg(a.ex + m0 + c0 + jj) : 0;
                if (ok) tmem_ld_wait();
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    // K = 896: limb pairs fold in int32 as in tc_gemm_kernel
                    const long long v = KC <= 14 ? (long long)(d[0][jj] + d[1][jj] * 128) +
                                                       (long long)(d[2][jj] + d[3][jj] * 128) * 16384ll
                                                 : (long long)d[0][jj] + (long long)d[1][jj] * 128ll +
                                                       (long long)d[2][jj] * 16384ll + (long long)d[3][jj] * 2097152ll;
                    f[jj] = m0 + c0 + jj < a.M ? exact_acc(v, exr[jj]) : 0.f;
                }
                if (sp == 1) {
                    // this warp's TMEM reads are complete: the buffer may be refilled
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&acc_empty[buf]);
                }
                tc_argmax_rows<8>(a, f, n0 + q * 32 + lane, m0, c0, q, lane, red);
            }
            if (!epi_bar_and<TP_CONV>(ok)) break;
            tc_argmax_flush(a, red, m0, n_tile, ct);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

// ------------------------------------------------- persistent projections
// The projections at prefill sizes (enough (row tile, channel tile) pairs to
// fill the GPU twice) as a persistent kernel with the LM head's roles: one
// CTA per SM walks the tile list with a stride of the grid, the weight and
// limb tiles stream without a gap between tiles, and the accumulator is double
// buffered in TMEM so the epilogue warps fold, scale and write one tile while
// the MMA warp computes the next. The epilogue works from registers: TMEM lane
// = output channel, so for each row the 32 lanes of a warp write 32
// consecutive channels; SiLU(gate) * up pairs the channels of neighbouring
// lanes. Same arithmetic as tc_gemm_kernel (bit-identical outputs).
template <int EPI>
__global__ void __launch_bounds__(TP_THREADS, 1)
    tc_persist_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap lmap, TcArgs a) {
    using L = LhSmem;
    constexpr int AS = L::A_STAGES, BS = L::B_STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *full_a = bars, *empty_a = full_a + AS, *full_b = empty_a + AS, *empty_b = full_b + BS;
    uint64_t *acc_full = empty_b + BS, *acc_empty = acc_full + 2, *done = acc_empty + 2;
    uint32_t *slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntn = a.N / TC_BM;                          // channel tiles
    const int total = ntn * ((a.M + TC_BN - 1) / TC_BN);  // (row tile, channel tile) pairs
    const int G = (int)gridDim.x;
    const int nt = total > (int)blockIdx.x ? (total - (int)blockIdx.x + G - 1) / G : 0;  // this CTA's tiles
    const int KC = a.K / TC_BK;
    const int nchunks = nt * KC;

    if (threadIdx.x == 0) {
        for (int s = 0; s < AS; ++s) {
            tc::mbar_init(&full_a[s], 1);
            tc::mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < BS; ++s) {
            tc::mbar_init(&full_b[s], 1);
            tc::mbar_init(&empty_b[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], TP_CONV / 32);  // one arrival per epilogue warp
        }
        tc::mbar_init(done, 1);
        tc::mbar_fence_init();
        tc::tma_prefetch_desc(&wmap);
        tc::tma_prefetch_desc(&lmap);
    }
    if (warp == 1) tc::tmem_alloc(slot, L::TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *slot;
    pdl_trigger();
    bool ok = nt > 0;

    if (warp == 0) {
        if (lane == 0) {
            auto tile_of = [&](int g, int &n0, int &m0) {
                const int t = (int)blockIdx.x + (g / KC) * G;
                n0 = (t % ntn) * TC_BM;
                m0 = (t / ntn) * TC_BN;
            };
            auto issue_a = [&](int g) {
                int n0, m0;
                tile_of(g, n0, m0);
                const int s = g % AS;
                tc::mbar_arrive_expect_tx(&full_a[s], (uint32_t)L::A_BYTES);
                tc::tma_load_2d(smem + L::A_OFF + s * L::A_BYTES, &wmap, &full_a[s], (g % KC) * TC_BK, n0);
            };
            int ia = 0, ib = 0;
            // weights are constant: the first stages load before the wait for
            // the kernel that writes the limb planes
            for (; ok && ia < min(nchunks, AS); ++ia) issue_a(ia);
            pdl_wait();
            uint32_t idle = 0;
            while (ok && (ib < nchunks || ia < nchunks)) {
                bool progress = false;
                if (ib < nchunks) {
                    const int s = ib % BS, ph = (ib / BS) & 1;
                    if (tc::mbar_try_wait(&empty_b[s], ph ^ 1)) {
                        int n0, m0;
                        tile_of(ib, n0, m0);
                        tc::mbar_arrive_expect_tx(&full_b[s], (uint32_t)L::B_BYTES);
                        tma_load_3d(smem + L::B_OFF + s * L::B_BYTES, &lmap, &full_b[s], (ib % KC) * TC_BK, m0, 0);
                        ++ib;
                        progress = true;
                    }
                }
                if (ia < nchunks) {
                    const int s = ia % AS, ph = (ia / AS) & 1;
                    if (tc::mbar_try_wait(&empty_a[s], ph ^ 1)) {
                        issue_a(ia);
                        ++ia;
                        progress = true;
                    }
                }
                if (progress) {
                    idle = 0;
                } else if (++idle > (1u << 22)) {
                    atomicExch(a.err, 27u);
                    ok = false;
                }
            }
        } else {
            pdl_wait();
        }
    } else if (warp == 1) {
        pdl_wait();
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_s8_s32(TC_BM, TC_MN);
            for (int j = 0; ok && j < nt; ++j) {
                const int buf = j & 1;
                // the epilogue has read this buffer's previous tile
                if (j >= 2 && !tc::mbar_wait(&acc_empty[buf], ((j >> 1) - 1) & 1, a.err, 28)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * TC_MN);
                for (int kc = 0; kc < KC; ++kc) {
                    const int g = j * KC + kc;
                    const int sa = g % AS, sb = g % BS;
                    if (!tc::mbar_wait(&full_a[sa], (g / AS) & 1, a.err, 29) ||
                        !tc::mbar_wait(&full_b[sb], (g / BS) & 1, a.err, 30)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t ab = tc::smem_u32(smem + L::A_OFF + sa * L::A_BYTES);
                    const uint32_t bb = tc::smem_u32(smem + L::B_OFF + sb * L::B_BYTES);
#pragma unroll
                    for (int k = 0; k < TC_BK / 32; ++k)
                        mma_s8(d, tc::smem_desc_sw128(ab + 32 * k), tc::smem_desc_sw128(bb + 32 * k), idesc,
                               kc > 0 || k > 0);
                    tc::mma_commit(&empty_a[sa]);
                    tc::mma_commit(&empty_b[sb]);
                }
                if (ok) tc::mma_commit(&acc_full[buf]);
            }
            // every MMA issued by this thread has finished before TMEM is freed
            tc::mma_commit(done);
            tc::mbar_wait(done, 0, a.err, 31);
        }
        __syncwarp();
    } else {
        // lane quarter q: channels 32q..32q+31 of a tile (this thread: one
        // channel), rows 16h..16h+15 (16 epilogue warps: four per quarter)
        const int q = warp & 3, h = (warp - 2) >> 2;
        pdl_wait();  // row exponents and residual rows come from preceding kernels
        for (int j = 0; j < nt; ++j) {
            const int buf = j & 1;
            const int t = (int)blockIdx.x + j * G;
            const int n = (t % ntn) * TC_BM + q * 32 + lane, m0 = (t / ntn) * TC_BN;
            const float scn = __ldg(a.scale + n);
            const float bn = EPI == EPI_BIAS ? bf2f(a.bias[n]) : 0.f;
            ok = ok && tc::mbar_wait(&acc_full[buf], (j >> 1) & 1, a.err, 26);
            tc::tc_fence_after();
#pragma unroll 1
            for (int sp = 0; sp < 2; ++sp) {
                // rows r0 .. r0 + 7 of this warp's 16 (fewer live registers
                // than one pass of 16 with 16 epilogue warps)
                const int r0 = m0 + 16 * h + 8 * sp;
                int d[TC_NL][8];
#pragma unroll
                for (int l = 0; l < TC_NL; ++l) {
                    if (ok) {
                        tmem_ld8i_nowait(tmem + ((uint32_t)(q * 32) << 16) +
                                             (uint32_t)(buf * TC_MN + l * TC_BN + 16 * h + 8 * sp),
                                         d[l]);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) d[l][jj] = 0;
                    }
                }
                // residual rows and row exponents, requested before the TMEM
                // data is used
                float res[8];
                if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj)
                        res[jj] = r0 + jj < a.M ? bf2f(a.y[(size_t)(r0 + jj) * a.N + n]) : 0.f;
                }
                int exr[8];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) exr[jj] = r0 + jj < a.M ? __ldg(a.ex + r0 + jj) : 0;
                if (ok) tmem_ld_wait();
                if (sp == 1) {
                    // this warp's TMEM reads are complete: the buffer may be refilled
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&acc_empty[buf]);
                }
                float o[8];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    // K = 896: limb pairs fold in int32 as in tc_gemm_kernel
                    const long long v = KC <= 14 ? (long long)(d[0][jj] + d[1][jj] * 128) +
                                                       (long long)(d[2][jj] + d[3][jj] * 128) * 16384ll
                                                 : (long long)d[0][jj] + (long long)d[1][jj] * 128ll +
                                                       (long long)d[2][jj] * 16384ll + (long long)d[3][jj] * 2097152ll;
                    o[jj] = r0 + jj < a.M ? rbf(rbf(exact_acc(v, exr[jj])) * scn) : 0.f;
                }
                if constexpr (EPI == EPI_SWIGLU) {
                    // channels 2i (gate i) and 2i+1 (up i), model_backend.py:105-106;
                    // rows in pairs so that both lanes of a channel pair work: the
                    // gate lane takes the first row, the up lane the second
#pragma unroll
                    for (int jj = 0; jj < 8; jj += 2) {
                        const bool odd = lane & 1;
                        const float other = __shfl_xor_sync(0xffffffffu, odd ? o[jj] : o[jj + 1], 1);
                        const float gt = odd ? other : o[jj], up = odd ? o[jj + 1] : other;
                        const int m = r0 + jj + (odd ? 1 : 0);
                        if (m < a.M) a.y[(size_t)m * (a.N >> 1) + (n >> 1)] = f2bf(rbf(silu_q(gt)) * up);
                    }
                } else {
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const int m = r0 + jj;
                        if (m < a.M) {  // the same for every lane of the warp
                            float w = o[jj];
                            if constexpr (EPI == EPI_BIAS) w = rbf(o[jj] + bn);
                            if constexpr (EPI == EPI_RESIDUAL) w = rbf(res[jj] + o[jj]);
                            a.y[(size_t)m * a.N + n] = f2bf(w);
                        }
                    }
                }
            }
        }
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

// Weight map: W [n][k] int8 row-major, box [128 n][128 k], 128-byte swizzle.
int make_weight_map(CUtensorMap *map, const int8_t *w, int n, int k) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -3;
    if ((reinterpret_cast<uintptr_t>(w) & 15) || k % TC_BK || n % TC_BM || n <= 0) return -1;
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)k};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BM};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(w), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -3;
}

// K-cache map: rows of 64 int8 codes (one key of one KV head), box 128 rows,
// 64-byte swizzle (the score operand of attention_tile.cu); rows past the end
// read as zero.
int make_kcache_map(CUtensorMap *map, const int8_t *kc, long long rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -3;
    if ((reinterpret_cast<uintptr_t>(kc) & 15) || rows <= 0) return -1;
    cuuint64_t dims[2] = {64, (cuuint64_t)rows};
    cuuint64_t strides[1] = {64};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(kc), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -3;
}

// Limb map: limbs[l][row][k] int8 (plane bytes apart, rows ld bytes apart,
// rows_alloc rows), box [4][64 rows][128 k], 128-byte swizzle; rows past
// rows_alloc read as zero.
int make_limb_map(CUtensorMap *map, const int8_t *limbs, int rows_alloc, int ld, size_t plane, int k) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -3;
    if ((reinterpret_cast<uintptr_t>(limbs) & 15) || (ld & 15) || (plane & 15) || k % TC_BK || k > ld ||
        rows_alloc <= 0)
        return -1;
    cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows_alloc, (cuuint64_t)TC_NL};
    cuuint64_t strides[2] = {(cuuint64_t)ld, (cuuint64_t)plane};
    cuuint32_t box[3] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BN, (cuuint32_t)TC_NL};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(limbs), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -3;
}

// Workspace: the 4-byte error flag of the bounded waits (256 bytes reserved).
// 256-byte error word, then (split K only) the partial tiles: the split CTAs
// of a tile write their exact int64 partials to L2 and each reduces its own
// share of the tile after the cluster barrier.
size_t tc_gemm_workspace(int rows, int n, int splits) {
    const size_t tiles = (size_t)(n / TC_BM) * ((rows + TC_BN - 1) / TC_BN);
    return 256 + (splits > 1 ? tiles * splits * (size_t)TC_BN * TC_BM * 8 : 0);
}

// Splits of K so that the tiles fill the GPU once (one CTA per SM), each
// split owning at least one k chunk; any split gives the same (exact) result.
int tc_pick_splits(int rows, int n, int k) {
    const int tiles = (n / TC_BM) * ((rows + TC_BN - 1) / TC_BN);
    const int kc = k / TC_BK;
    int s = TC_SLOTS / tiles;
    s = s < 1 ? 1 : s;
    s = s > TC_MAX_SPLITS ? TC_MAX_SPLITS : s;
    s = s > kc ? kc : s;
    while (s > 1 && (s - 1) * ((kc + s - 1) / s) >= kc) --s;  // no empty split
    return s;
}

template <int EPI>
static int run_tc(const CUtensorMap &wmap, const CUtensorMap &lmap, TcArgs &a, int splits, cudaStream_t st) {
    using L = TcSmem;
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << (dev & 31)))) {
        if (cudaFuncSetAttribute(tc_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) !=
            cudaSuccess)
            return -3;
        configured |= 1u << (dev & 31);
    }
    // the split CTAs of a tile share one cluster
    return launch_pdl(tc_gemm_kernel<EPI>, dim3((a.N / TC_BM) * splits, 1, (a.M + TC_BN - 1) / TC_BN),
                      dim3(TC_THREADS), (size_t)L::ALLOC, st, (unsigned)splits, wmap, lmap, a);
}

// The persistent LM head: one CTA per SM at most, each walking its share of
// the tile list.
static int run_lmhead(const CUtensorMap &wmap, const CUtensorMap &lmap, TcArgs &a, cudaStream_t st) {
    using L = LhSmem;
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << (dev & 31)))) {
        if (cudaFuncSetAttribute(tc_lmhead_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) !=
            cudaSuccess)
            return -3;
        configured |= 1u << (dev & 31);
    }
    const int tiles = (a.N / TC_BM) * ((a.M + TC_BN - 1) / TC_BN);
    return launch_pdl(tc_lmhead_kernel, dim3(tiles < TC_SLOTS ? tiles : TC_SLOTS), dim3(TP_THREADS), (size_t)L::ALLOC,
                      st, 1u, wmap, lmap, a);
}

template <int EPI>
static int run_persist(const CUtensorMap &wmap, const CUtensorMap &lmap, TcArgs &a, cudaStream_t st) {
    using L = LhSmem;
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << (dev & 31)))) {
        if (cudaFuncSetAttribute(tc_persist_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) !=
            cudaSuccess)
            return -3;
        configured |= 1u << (dev & 31);
    }
    const int tiles = (a.N / TC_BM) * ((a.M + TC_BN - 1) / TC_BN);
    return launch_pdl(tc_persist_kernel<EPI>, dim3(tiles < TC_SLOTS ? tiles : TC_SLOTS), dim3(TP_THREADS),
                      (size_t)L::ALLOC, st, 1u, wmap, lmap, a);
}

int launch_gemm_tc(int epi, const CUtensorMap &wmap, const CUtensorMap &lmap, const int *ex, int rows, int k,
                   const float *scale, const uint16_t *bias, int n, uint16_t *y, int splits, void *ws,
                   size_t ws_bytes, bool clear, const TcArgmax *am, cudaStream_t st) {
    if (rows <= 0 || n % TC_BM || k % TC_BK || splits < 1 || splits > k / TC_BK || splits > TC_MAX_SPLITS || !ex)
        return -1;
    if (epi == EPI_ARGMAX && (!am || splits != 1)) return -1;
    // vector loads and stores of the epilogue: 4 scales, 4 bias / output values
    if ((reinterpret_cast<uintptr_t>(scale) & 15) || (reinterpret_cast<uintptr_t>(bias) & 7) ||
        (reinterpret_cast<uintptr_t>(y) & 7))
        return -1;
    if (ws_bytes < tc_gemm_workspace(rows, n, splits)) return -1;
    const int kc = k / TC_BK;
    const int kcps = (kc + splits - 1) / splits;
    if ((splits - 1) * kcps >= kc) return -1;  // every split owns at least one k chunk
    TcArgs a;
    a.scale = scale;
    a.bias = bias;
    a.y = y;
    a.ex = ex;
    a.M = rows;
    a.N = n;
    a.K = k;
    a.kc_per_split = kcps;
    a.splits = splits;
    a.err = reinterpret_cast<unsigned *>(ws);
    a.part = reinterpret_cast<long long *>(reinterpret_cast<char *>(ws) + 256);
    a.pv = am ? am->pv : nullptr;
    a.pi = am ? am->pi : nullptr;
    a.nblk = am ? am->nblk : 0;
    a.logits = am ? am->logits : nullptr;
    a.n_base = am ? am->n_base : 0;
    if (clear) {
        if (cudaMemsetAsync(ws, 0, 256, st) != cudaSuccess) return -3;
        pdl_break();
    }
    // prefill sizes (the tiles fill the GPU at least twice, no split): the
    // persistent form overlaps each tile's epilogue with the next tile's MMAs
    const int tiles = (n / TC_BM) * ((rows + TC_BN - 1) / TC_BN);
    if (splits == 1 && tiles >= 2 * TC_SLOTS && epi != EPI_ARGMAX) {
        switch (epi) {
            case EPI_PLAIN: return run_persist<EPI_PLAIN>(wmap, lmap, a, st);
            case EPI_BIAS: return run_persist<EPI_BIAS>(wmap, lmap, a, st);
            case EPI_RESIDUAL: return run_persist<EPI_RESIDUAL>(wmap, lmap, a, st);
            case EPI_SWIGLU: return run_persist<EPI_SWIGLU>(wmap, lmap, a, st);
        }
    }
    switch (epi) {
        case EPI_PLAIN: return run_tc<EPI_PLAIN>(wmap, lmap, a, splits, st);
        case EPI_BIAS: return run_tc<EPI_BIAS>(wmap, lmap, a, splits, st);
        case EPI_RESIDUAL: return run_tc<EPI_RESIDUAL>(wmap, lmap, a, splits, st);
        case EPI_SWIGLU: return run_tc<EPI_SWIGLU>(wmap, lmap, a, splits, st);
        case EPI_ARGMAX: return run_lmhead(wmap, lmap, a, st);
    }
    return -1;
}

}  // namespace qb
