// GQA decode/prefill attention over the KV8 cache with the scores held in
// registers: one CTA (or a thread-block cluster of up to 8 CTAs splitting the
// context) per (query row, KV head), 12 warps.
// Arithmetic: the oracle's REF_KV8 | REF_EXACT attention, the same as
// attention_cluster.cu (legacy_100mhz_closed/src/PC/model_backend.py:97-102 in
// the accelerator's order, src/rtl/kv8_score_scale8.sv:6-12 for the K scale,
// src/rtl/kv8_v_pscale.sv:1-20 for the V scale), every sum exact:
//   S[h][t] = bf16(RN32(RN32(Q_h . kcode[t]) * 2^(E_h-26) * kscale[t]) / 8)
//   E[h][t] = qexp(S[h][t] - max_t S[h]),  Z_h = RN32(sum_t rint(E * 2^40)) 2^-40
//   W[h][t] = rint(RN32(bf16(E / Z_h) * vscale[t]) * 2^(26-F_h))
//   ctx[h]  = bf16(RN32(sum_t W[h][t] * vcode[t]) * 2^(F_h-26))
// so the context is bit-identical to the oracle's whatever the split.
//
// Layout of the work. A chunk is 192 keys, one 16-key block per warp; warp w
// owns block w of every chunk of its CTA's key range (at most 12 chunks, 2304
// keys, per CTA).
//   scores   computed transposed on the tensor cores, D[16][8 keys] =
//            Qlimb[16][64] . Kcode^T (m16n8k32, s8): rows 0-7 of m-tile 0
//            are limb 0 of heads 0-6 (row 7 unused), rows 8-15 limb 1; m-tile
//            1 holds limbs 2 and 3. Lane (g, i) then holds all four limbs of
//            head g for keys 2i, 2i+1 of each 8-key n-tile and folds them in
//            registers; its four keys of a block, {2i, 2i+1, 8+2i, 9+2i}, are
//            exactly the k slots it supplies to the P.V product below, so a
//            lane only ever reads back its own scores: they are kept in shared
//            memory as one float4 per lane and chunk (lane-private,
//            conflict-free, no exchange between warps).
//   softmax  per-head max and exact sum: lanes -> warp (shuffles) -> CTA
//            (shared memory) -> cluster (distributed shared memory)
//   context  D[16 dims][8 heads] += Vcode^T[16][16 keys] . Wbyte[16][8]
//            (m16n8k16, s8 x u8): W >= 0 split into four byte planes, the V
//            codes transposed 4 x 4 bytes with byte permutes; int32 per plane,
//            folded to int64 at the end, warps then cluster ranks added.
// Memory: the K chunks and then the V chunks stream through one 10-slot ring
// of bulk copies completing on mbarriers; a K chunk's item also copies the
// chunk's K and V scales into shared memory (when the cache rows are 16-byte
// aligned; otherwise every thread stages them with plain loads first). There is no producer warp and no
// CTA-wide barrier in the loops: each warp counts its release of a slot on an
// acquire-release shared-memory counter and the warp that releases it last
// refills it ten items ahead. The chunk loops are not unrolled: a kernel
// that kept the scores in registers (unrolling every chunk) measured 33 us
// at 64 rows x 2049 keys, its warps stalled on instruction fetch. Every wait
// is bounded (error codes 32-33).
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace qb {

// The kernel's shape: 12 warps and one CTA per SM, up to 12 chunks (2304
// keys) per CTA. (Measured against two 8-warp CTAs per SM of up to 1152 keys
// each, at 64 rows x 2049 keys: 22.6 against 26.6 us.)
template <int NW>
struct ArCfg {
    static constexpr int WARPS = NW;
    static constexpr int THREADS = 32 * NW;
    static constexpr int NB = 12;                         // chunks (blocks per warp) per CTA at most
    static constexpr int CHUNK = 16 * NW;                 // keys per chunk
    static constexpr int CHUNK_BYTES = CHUNK * QB_HD;
    static constexpr int MAX_KPC = CHUNK * NB;            // keys per CTA
    static constexpr int RING = 10;                       // ring slots (K chunks, then V chunks)
    static constexpr int STAGE_LOADS = (MAX_KPC + THREADS - 1) / THREADS;  // scale loads per thread
    static constexpr int RED_BYTES = NW * 8 * 4 + NW * 8 * 8 + NW * 4 + RING * 4;
    static_assert(NW * 8 * QB_HD * 8 <= RING * CHUNK_BYTES, "context partials fit in the ring");
    static_assert(RED_BYTES % 8 == 0, "aligned sub-areas");
};
constexpr int AR_NW = 12;
constexpr int AR_MAX_SPLITS = 16;  // 9-16: non-portable clusters, when the GPU can place one
constexpr int AR_SMS = 148;

struct ArArgs {
    const uint16_t *q;
    const uint32_t *slots, *positions;
    const int8_t *kc, *vc;
    const float *ks, *vs;
    int cap;
    uint16_t *ctx;
    int kpc;  // keys per CTA (multiple of the chunk)
    unsigned *err;
};

// ring [RING][CHUNK][64] int8 (reused for the per-warp context partials
// [WARPS][8][64] int64) | S [WARPS][NB chunks][32 lanes] float4 | K scales
// [kpc] | V scales [kpc] | stat: max[8] (slot 7: largest V scale) | Z[8]
// int64 | inv, s1, s2, F [4][8] | context partial [7][64] int64 | per-warp
// max [WARPS][8], Z [WARPS][8] int64, V-scale max [WARPS] | slot release
// counters [RING] | mbarriers [RING]
struct ArSmem {
    int ring, s, kss, vss, stat, red, bars, total;
};
constexpr int AR_ST_Z = 32, AR_ST_HV = 96, AR_ST_CTX = 224;
constexpr int AR_STAT_BYTES = AR_ST_CTX + 7 * QB_HD * 8;
static_assert(AR_STAT_BYTES % 16 == 0, "aligned sub-areas");
template <int NW>
__host__ __device__ inline ArSmem ar_smem(int kpc) {
    using C = ArCfg<NW>;
    ArSmem L;
    L.ring = 0;
    L.s = L.ring + C::RING * C::CHUNK_BYTES;
    L.kss = L.s + C::WARPS * C::NB * 32 * 16;
    L.vss = L.kss + kpc * 4;
    L.stat = L.vss + kpc * 4;
    L.red = L.stat + AR_STAT_BYTES;
    L.bars = (L.red + C::RED_BYTES + 7) & ~7;
    L.total = L.bars + C::RING * 8;
    return L;
}

__device__ __forceinline__ void ar_mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ar_mma_s8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.u8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ uint32_t ar_prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
// 4 x 4 byte transpose: o[j] byte i = r[i] byte j.
__device__ __forceinline__ void ar_transpose4(const uint32_t (&r)[4], uint32_t (&o)[4]) {
    const uint32_t t0 = ar_prmt(r[0], r[1], 0x5140u), t1 = ar_prmt(r[0], r[1], 0x7362u);
    const uint32_t t2 = ar_prmt(r[2], r[3], 0x5140u), t3 = ar_prmt(r[2], r[3], 0x7362u);
    o[0] = ar_prmt(t0, t2, 0x5410u);
    o[1] = ar_prmt(t0, t2, 0x7632u);
    o[2] = ar_prmt(t1, t3, 0x5410u);
    o[3] = ar_prmt(t1, t3, 0x7632u);
}
// One fp32 of CTA `rank`'s shared memory at this CTA's address of it.
__device__ __forceinline__ float ar_ld_dsmem(uint32_t local_saddr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}
// *p += 1 with acquire-release order at CTA scope; returns the old value.
__device__ __forceinline__ unsigned ar_release_count(unsigned *p) {
    unsigned old;
    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;" : "=r"(old) : "r"(tc::smem_u32(p)) : "memory");
    return old;
}

template <int NW, bool CLUSTER>
__global__ void __launch_bounds__(32 * NW, 1) attn_rs_kernel(ArArgs a) {
    using C = ArCfg<NW>;
    extern __shared__ __align__(128) uint8_t sm[];
    const int kpc = a.kpc;
    const ArSmem L = ar_smem<NW>(kpc);
    uint8_t *ring = sm + L.ring;
    float4 *S = reinterpret_cast<float4 *>(sm + L.s);
    float *kss = reinterpret_cast<float *>(sm + L.kss);
    float *vss = reinterpret_cast<float *>(sm + L.vss);
    float *stat = reinterpret_cast<float *>(sm + L.stat);
    long long *statz = reinterpret_cast<long long *>(sm + L.stat + AR_ST_Z);
    float *hv = reinterpret_cast<float *>(sm + L.stat + AR_ST_HV);
    long long *ctxp = reinterpret_cast<long long *>(sm + L.stat + AR_ST_CTX);
    float *red_m = reinterpret_cast<float *>(sm + L.red);
    long long *red_z = reinterpret_cast<long long *>(sm + L.red + C::WARPS * 8 * 4);
    float *red_v = reinterpret_cast<float *>(sm + L.red + C::WARPS * 8 * 12);
    unsigned *released = reinterpret_cast<unsigned *>(sm + L.red + C::WARPS * 8 * 12 + C::WARPS * 4);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + L.bars);
    long long *part = reinterpret_cast<long long *>(sm + L.ring);  // after the last chunk

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int kvh = blockIdx.y, r = blockIdx.z;
    const int rank = CLUSTER ? (int)tc::cluster_rank() : 0;
    const int nranks = CLUSTER ? (int)gridDim.x : 1;
    float4 *Sl = S + warp * C::NB * 32 + lane;  // this lane's scores, one float4 per chunk (stride 32)

    if (tid == 0) {
        for (int i = 0; i < C::RING; ++i) {
            tc::mbar_init(&full[i], 1);
            released[i] = 0;
        }
        tc::mbar_fence_init();
    }
    pdl_wait();  // q, positions and the newest cache entries come from earlier kernels
    pdl_trigger();
    // q of head g = gid, dims 16 tig .. 16 tig + 15 (requested first: it does
    // not depend on the row's position)
    uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
    if (gid < 7) {
        const uint4 *qp = reinterpret_cast<const uint4 *>(a.q + (size_t)r * QB_HID + (kvh * 7 + gid) * QB_HD + 16 * tig);
        q0 = qp[0];
        q1 = qp[1];
    }
    const int L_row = (int)a.positions[r] + 1;
    const int slot = (int)a.slots[r];
    const int t_begin = rank * kpc;
    const int nkeys = max(0, min(L_row, t_begin + kpc) - t_begin);
    const int nchunks = (nkeys + C::CHUNK - 1) / C::CHUNK;
    const int items = 2 * nchunks;  // ring items: K chunks 0..n-1, then V chunks
    const size_t kvbase = ((size_t)slot * QB_KVH + kvh) * a.cap + t_begin;  // first key of this CTA
    __syncthreads();  // barriers and counters initialised
    const int8_t *kg = a.kc + kvbase * QB_HD;
    const int8_t *vg = a.vc + kvbase * QB_HD;
    // scales come with the K chunks when their rows start on 16 bytes (the
    // copied rows are rounded up to 4 keys, which stay inside a row whose
    // capacity is a multiple of 4)
    const bool bulk_scales = ((a.cap & 3) == 0) &&
                             ((reinterpret_cast<uintptr_t>(a.ks) | reinterpret_cast<uintptr_t>(a.vs)) & 15) == 0;
    auto issue = [&](int i) {
        const int c = i < nchunks ? i : i - nchunks, sl = i % C::RING;
        const int n = min(C::CHUNK, nkeys - c * C::CHUNK);
        const uint32_t bytes = (uint32_t)(n * QB_HD), sbytes = (uint32_t)(((n + 3) & ~3) * 4);
        const bool with_scales = bulk_scales && i < nchunks;
        tc::mbar_arrive_expect_tx(&full[sl], bytes + (with_scales ? 2 * sbytes : 0u));
        tc::bulk_load(ring + sl * C::CHUNK_BYTES, (i < nchunks ? kg : vg) + (size_t)c * C::CHUNK_BYTES, bytes,
                      &full[sl]);
        if (with_scales) {
            tc::bulk_load(kss + c * C::CHUNK, a.ks + kvbase + c * C::CHUNK, sbytes, &full[sl]);
            tc::bulk_load(vss + c * C::CHUNK, a.vs + kvbase + c * C::CHUNK, sbytes, &full[sl]);
        }
    };
    // this warp is done reading item i's slot; the last warp to say so
    // refills it with item i + C::RING
    auto release = [&](int i) {
        __syncwarp();
        if (lane == 0 && ar_release_count(&released[i % C::RING]) == C::WARPS - 1) {
            atomicExch(&released[i % C::RING], 0u);
            tc::fence_proxy_async_smem();  // generic reads of the slot before the bulk copy's writes
            if (i + C::RING < items) issue(i + C::RING);
        }
    };
    if (tid == 0)
        for (int i = 0; i < min(C::RING, items); ++i) issue(i);

    // ---------------- q as int8 limbs; the scales staged here unless they come with the K chunks
    float vmax = 0.f;
    if (!bulk_scales) {
        float kv[C::STAGE_LOADS], vv[C::STAGE_LOADS];
#pragma unroll
        for (int j = 0; j < C::STAGE_LOADS; ++j) {
            const int t = tid + j * C::THREADS;
            kv[j] = t < nkeys ? __ldg(a.ks + kvbase + t) : 0.f;
            vv[j] = t < nkeys ? __ldg(a.vs + kvbase + t) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < C::STAGE_LOADS; ++j) {
            const int t = tid + j * C::THREADS;
            if (t < nkeys) {
                kss[t] = kv[j];
                vss[t] = vv[j];
            }
        }
    }
    // q aligned to the head's largest exponent E as 28-bit integers split into four signed 7-bit limbs;
    // word i of limb plane l holds dims 16 tig + 4i .. +3 (the same dims the
    // lane's K words cover, so q and K share one k-slot permutation)
    uint32_t qa[2][2][4];  // [m-tile: limbs 0,1 | 2,3][k step][a0..a3]
    int e_g;
    {
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        float qf[16];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qf[2 * i] = bflo(w[i]);
            qf[2 * i + 1] = bfhi(w[i]);
            amax = fmaxf(amax, fmaxf(fabsf(qf[2 * i]), fabsf(qf[2 * i + 1])));
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        e_g = row_exponent(amax);
        uint32_t lb[4][4] = {};  // [limb][word of 4 dims]
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            int l4[4];
            limbs4(align28_int(qf[i], e_g), l4);
#pragma unroll
            for (int l = 0; l < 4; ++l) lb[l][i >> 2] |= ((uint32_t)l4[l] & 0xffu) << (8 * (i & 3));
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                qa[mt][s][0] = lb[2 * mt][2 * s];
                qa[mt][s][1] = lb[2 * mt + 1][2 * s];
                qa[mt][s][2] = lb[2 * mt][2 * s + 1];
                qa[mt][s][3] = lb[2 * mt + 1][2 * s + 1];
            }
    }
    __syncthreads();  // staged scales visible to every warp
    bool ok = true;
    // unalign28(., e_g) = (RN32(.) * 2^s1) * 2^(s - s1): the two factors once
    const int ush = e_g - 26, ush1 = max(ush, -126);
    const float uc1 = pow2i(ush1), uc2 = pow2i(ush - ush1);

    // ---------------- phase 1: scores of this warp's blocks -> Sl[c]
    // Sl[c] = head gid, keys 192 c + 16 warp + {2tig, 2tig+1, 8+2tig, 9+2tig}
    float mrun = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
        const int sl = c % C::RING;
        if (ok) ok = tc::mbar_wait(&full[sl], (uint32_t)(c / C::RING) & 1u, a.err, 32);
        const int kb = c * C::CHUNK + 16 * warp;  // first key of this warp's block
        float sc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (ok && lane < 16 && kb + lane < nkeys) vmax = fmaxf(vmax, vss[kb + lane]);
        if (ok && kb < nkeys) {
            const int8_t *blk = reinterpret_cast<const int8_t *>(ring + sl * C::CHUNK_BYTES) + 16 * warp * QB_HD;
            int d[2][2][4];  // [n-tile][m-tile][fragment]
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                const uint4 u = *reinterpret_cast<const uint4 *>(blk + (8 * nt + gid) * QB_HD + 16 * tig);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    d[nt][mt][0] = d[nt][mt][1] = d[nt][mt][2] = d[nt][mt][3] = 0;
                    ar_mma_s8(d[nt][mt], qa[mt][0][0], qa[mt][0][1], qa[mt][0][2], qa[mt][0][3], u.x, u.y);
                    ar_mma_s8(d[nt][mt], qa[mt][1][0], qa[mt][1][1], qa[mt][1][2], qa[mt][1][3], u.z, u.w);
                }
            }
            const float2 k01 = *reinterpret_cast<const float2 *>(kss + kb + 2 * tig);
            const float2 k23 = *reinterpret_cast<const float2 *>(kss + kb + 8 + 2 * tig);
            const float kk[4] = {k01.x, k01.y, k23.x, k23.y};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int nt = i >> 1, cc = i & 1;
                const int key = kb + 8 * nt + 2 * tig + cc;
                // per-limb sums over 64 dims are below 2^20: pairs add in int32
                const long long dot = (long long)(d[nt][0][cc] + d[nt][0][cc + 2] * 128) +
                                      (long long)(d[nt][1][cc] + d[nt][1][cc + 2] * 128) * 16384ll;
                const float v = rbf(__fmul_rn((__ll2float_rn(dot) * uc1) * uc2, kk[i]) * 0.125f);
                sc[i] = key < nkeys ? v : -INFINITY;
                mrun = fmaxf(mrun, sc[i]);
            }
        }
        Sl[c * 32] = make_float4(sc[0], sc[1], sc[2], sc[3]);
        release(c);
    }
    // per-head max: the four lanes of a group hold the same head
    mrun = fmaxf(mrun, __shfl_xor_sync(0xffffffffu, mrun, 1));
    mrun = fmaxf(mrun, __shfl_xor_sync(0xffffffffu, mrun, 2));
    vmax = warp_max(vmax);
    if (tig == 0) red_m[warp * 8 + gid] = mrun;
    if (lane == 0) red_v[warp] = vmax;
    __syncthreads();
    if (tid < 8) {
        float m = -INFINITY;
        if (tid < 7) {
            for (int w = 0; w < C::WARPS; ++w) m = fmaxf(m, red_m[w * 8 + tid]);
        } else {
            m = 0.f;
            for (int w = 0; w < C::WARPS; ++w) m = fmaxf(m, red_v[w]);
        }
        stat[tid] = m;
    }
    float Mg, Mv;  // the row's max of head gid; its largest V scale
    if constexpr (CLUSTER) {
        tc::cluster_sync();  // (1)
        const uint32_t sa = tc::smem_u32(stat);
        Mg = -INFINITY;
        Mv = 0.f;
        for (int sr = 0; sr < nranks; ++sr) {
            Mg = fmaxf(Mg, ar_ld_dsmem(sa + 4u * (uint32_t)gid, sr));
            Mv = fmaxf(Mv, ar_ld_dsmem(sa + 28u, sr));
        }
    } else {
        __syncthreads();
        Mg = stat[gid];
        Mv = stat[7];
    }

    // ---------------- phase 2: E = qexp(S - max) in place, exact sums
    long long z = 0;
#pragma unroll 2
    for (int c = 0; c < nchunks; ++c) {
        const float4 s4 = Sl[c * 32];
        float e0, e1, e2, e3;
        qexp2(__fsub_rn(s4.x, Mg), __fsub_rn(s4.y, Mg), e0, e1);
        qexp2(__fsub_rn(s4.z, Mg), __fsub_rn(s4.w, Mg), e2, e3);
        // rint(e * 2^40) (0 <= e <= 1, the product exact): the conversion
        // rounds to nearest even, as rint does
        z += __float2ll_rn(__fmul_rn(e0, 0x1p40f)) + __float2ll_rn(__fmul_rn(e1, 0x1p40f)) +
             __float2ll_rn(__fmul_rn(e2, 0x1p40f)) + __float2ll_rn(__fmul_rn(e3, 0x1p40f));
        Sl[c * 32] = make_float4(e0, e1, e2, e3);
    }
    z += __shfl_xor_sync(0xffffffffu, z, 1);
    z += __shfl_xor_sync(0xffffffffu, z, 2);
    if (tig == 0) red_z[warp * 8 + gid] = z;
    __syncthreads();
    if (tid < 8) {
        long long zz = 0;
        for (int w = 0; w < C::WARPS; ++w) zz += red_z[w * 8 + tid];
        statz[tid] = zz;
    }
    if constexpr (CLUSTER) {
        tc::cluster_sync();  // (2)
    } else {
        __syncthreads();
    }
    // per-head 1/Z, the bound of w and its alignment factors (every CTA of
    // the cluster forms the same values from the same totals)
    if (tid < 8) {
        long long zt = 0;
        if constexpr (CLUSTER) {
            const uint32_t za = tc::smem_u32(statz) + 8u * (uint32_t)(tid & ~1);
            for (int sr = 0; sr < nranks; ++sr) {
                const float4 v = tc::ld_dsmem_f4(za, sr);
                const longlong2 zz = *reinterpret_cast<const longlong2 *>(&v);
                zt += (tid & 1) ? zz.y : zz.x;
            }
        } else {
            zt = statz[tid];
        }
        float inv = 0.f, s1 = 0.f, s2 = 0.f;
        int f = 0;
        if (tid < 7 && zt > 0) {
            inv = __fdiv_rn(1.0f, __fmul_rn(__ll2float_rn(zt), 0x1p-40f));
            f = row_exponent(__fmul_rn(rbf(inv), Mv));
            const int sh = 26 - f, sh1 = min(sh, 127);
            s1 = pow2i(sh1);
            s2 = pow2i(sh - sh1);
        }
        hv[tid] = inv;
        hv[8 + tid] = s1;
        hv[16 + tid] = s2;
        hv[24 + tid] = __int_as_float(f);
    }
    __syncthreads();

    // ---------------- phase 3: context on the tensor cores, V from the ring
    const float inv_g = hv[gid], s1_g = hv[8 + gid], s2_g = hv[16 + gid];
    const bool gv = gid < 7;
    int acc[4][4][4];  // [m-tile j: dims 4gid+j | 32+4gid+j][byte plane l][fragment]
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int l = 0; l < 4; ++l) acc[j][l][0] = acc[j][l][1] = acc[j][l][2] = acc[j][l][3] = 0;
#pragma unroll 1
    for (int c = 0; c < nchunks; ++c) {
        const int item = nchunks + c, sl = item % C::RING;
        if (ok) ok = tc::mbar_wait(&full[sl], (uint32_t)(item / C::RING) & 1u, a.err, 33);
        const int kb = c * C::CHUNK + 16 * warp;
        if (ok && kb < nkeys) {
            const float4 e4 = Sl[c * 32];
            const float2 v01 = *reinterpret_cast<const float2 *>(vss + kb + 2 * tig);
            const float2 v23 = *reinterpret_cast<const float2 *>(vss + kb + 8 + 2 * tig);
            const float ev[4] = {e4.x, e4.y, e4.z, e4.w}, vv[4] = {v01.x, v01.y, v23.x, v23.y};
            const int koff[4] = {2 * tig, 2 * tig + 1, 8 + 2 * tig, 9 + 2 * tig};
            // w = rint(RN32(bf16(E * inv) * vscale) * s1 * s2), two keys per
            // packed fp32 operation (each half one IEEE operation)
            uint32_t wq[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i += 2) {
                float p0, p1;
                unpk2(mul2(pk2(ev[i], ev[i + 1]), dup2(inv_g)), p0, p1);
                const __nv_bfloat162 bb = __floats2bfloat162_rn(p0, p1);
                float w0, w1;
                unpk2(mul2(mul2(mul2(pk2(__low2float(bb), __high2float(bb)), pk2(vv[i], vv[i + 1])), dup2(s1_g)),
                           dup2(s2_g)),
                      w0, w1);
                wq[i] = (gv && kb + koff[i] < nkeys) ? __float2uint_rn(w0) : 0u;
                wq[i + 1] = (gv && kb + koff[i + 1] < nkeys) ? __float2uint_rn(w1) : 0u;
            }
            ar_transpose4(wq, b);
            const uint32_t *vb =
                reinterpret_cast<const uint32_t *>(ring + sl * C::CHUNK_BYTES) + 16 * warp * (QB_HD / 4);
            uint32_t rl[4], rh[4], alo[4], ahi[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                rl[i] = vb[koff[i] * (QB_HD / 4) + gid];
                rh[i] = vb[koff[i] * (QB_HD / 4) + gid + 8];
            }
            ar_transpose4(rl, alo);
            ar_transpose4(rh, ahi);
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int l = 0; l < 4; ++l) ar_mma_s8u8(acc[j][l], alo[j], ahi[j], b[l]);
        }
        release(item);
    }

    // ---------------- phase 4: byte planes -> int64, warps -> CTA -> rank 0
    tc::fence_proxy_async_smem();  // the ring (bulk-copy writes) becomes generic int64 partials
    __syncthreads();               // every warp is past its last read of the ring
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            const long long v = (long long)acc[j][0][cc] + (long long)acc[j][1][cc] * 256ll +
                                (long long)acc[j][2][cc] * 65536ll + (long long)acc[j][3][cc] * 16777216ll;
            const int h = 2 * tig + (cc & 1), d = 4 * gid + 32 * (cc >> 1) + j;
            part[(warp * 8 + h) * QB_HD + d] = v;
        }
    __syncthreads();
    for (int i = tid; i < 7 * QB_HD; i += C::THREADS) {
        const int h = i >> 6, d = i & 63;
        long long sum = 0;
#pragma unroll
        for (int w = 0; w < C::WARPS; ++w) sum += part[(w * 8 + h) * QB_HD + d];
        ctxp[i] = sum;
    }
    if constexpr (CLUSTER) {
        tc::cluster_sync();  // (3)
        if (rank == 0) {
            const uint32_t ca = tc::smem_u32(ctxp);
            for (int i2 = tid; i2 < 7 * QB_HD / 2; i2 += C::THREADS) {
                long long s0 = 0, s1 = 0;
                for (int sr = 0; sr < nranks; ++sr) {
                    const float4 v = tc::ld_dsmem_f4(ca + 16u * i2, sr);
                    const longlong2 pp = *reinterpret_cast<const longlong2 *>(&v);
                    s0 += pp.x;
                    s1 += pp.y;
                }
                const int i = 2 * i2, h = i >> 6, d = i & 63;
                const int f = __float_as_int(hv[24 + h]);
                *reinterpret_cast<uint32_t *>(a.ctx + (size_t)r * QB_HID + (kvh * 7 + h) * QB_HD + d) =
                    (uint32_t)f2bf(unalign28(s0, f)) | ((uint32_t)f2bf(unalign28(s1, f)) << 16);
            }
        }
        tc::cluster_sync();  // (4) peers' shared memory stays alive until rank 0 has read it
    } else {
        __syncthreads();
        for (int i2 = tid; i2 < 7 * QB_HD / 2; i2 += C::THREADS) {
            const int i = 2 * i2, h = i >> 6, d = i & 63;
            const int f = __float_as_int(hv[24 + h]);
            *reinterpret_cast<uint32_t *>(a.ctx + (size_t)r * QB_HID + (kvh * 7 + h) * QB_HD + d) =
                (uint32_t)f2bf(unalign28(ctxp[i], f)) | ((uint32_t)f2bf(unalign28(ctxp[i + 1], f)) << 16);
        }
    }
}

// Split plan: as many CTAs per row as fill the GPU once at one CTA per SM
// (contexts split up to max_splits ways), at least enough to keep each within
// the key limit. -1 when a row needs more than max_splits CTAs.
template <int NW>
int attention_rs_plan(int rows, int max_len, int *splits, int *kpc, int max_splits = 8) {
    using C = ArCfg<NW>;
    if (max_len <= 0 || rows <= 0) return -1;
    const int chunks = (max_len + C::CHUNK - 1) / C::CHUNK;
    int s = AR_SMS / (2 * rows);
    s = s < 1 ? 1 : (s > max_splits ? max_splits : s);
    s = s > chunks ? chunks : s;
    const int need = (chunks + C::NB - 1) / C::NB;
    s = s < need ? need : s;
    if (s > max_splits) return -1;
    // beyond 8 splits only while the CTAs fill at most four waves: larger
    // batches of such rows run faster on the two-CTAs-per-SM kernel (64 rows
    // x 32768 keys: 469 against 434 us; 16 rows: 129 against 148 us)
    if (s > 8 && rows * QB_KVH * s > 4 * AR_SMS) return -1;
    const int cpc = (chunks + s - 1) / s;  // chunks per CTA
    *kpc = cpc * C::CHUNK;
    *splits = (chunks + cpc - 1) / cpc;
    return 0;
}

template <int NW, bool CLUSTER>
static int configure_ar() {
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << (dev & 31)))) {
        if (cudaFuncSetAttribute(attn_rs_kernel<NW, CLUSTER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 ar_smem<NW>(ArCfg<NW>::MAX_KPC).total) != cudaSuccess)
            return -3;
        if (CLUSTER &&
            cudaFuncSetAttribute(attn_rs_kernel<NW, CLUSTER>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
                cudaSuccess)
            return -3;
        configured |= 1u << (dev & 31);
    }
    return 0;
}

// Largest split this device can place as one cluster of full-size CTAs (one
// per SM): 16 when a 16-CTA cluster fits in a GPC, else the portable 8;
// decided once per device.
template <int NW>
static int ar_max_splits() {
    static int cached[32] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int &m = cached[dev & 31];
    if (m) return m;
    m = 8;
    if (configure_ar<NW, true>()) return m;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(AR_MAX_SPLITS, QB_KVH, 1);
    cfg.blockDim = dim3(32 * NW);
    cfg.dynamicSmemBytes = (size_t)ar_smem<NW>(ArCfg<NW>::MAX_KPC).total;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = AR_MAX_SPLITS;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, attn_rs_kernel<NW, true>, &cfg) == cudaSuccess && clusters >= 2)
        m = AR_MAX_SPLITS;
    cudaGetLastError();
    return m;
}

template <int NW, bool CLUSTER>
static int run_ar(const ArArgs &a, int rows, int splits, cudaStream_t st) {
    if (configure_ar<NW, CLUSTER>()) return -3;
    return launch_pdl(attn_rs_kernel<NW, CLUSTER>, dim3(splits, QB_KVH, rows), dim3(32 * NW),
                      (size_t)ar_smem<NW>(a.kpc).total, st, CLUSTER ? (unsigned)splits : 1u, a);
}

int launch_attention_rs(const uint16_t *q, int rows, const uint32_t *slots, const uint32_t *positions, int max_len,
                        const int8_t *kc, const float *ks, const int8_t *vc, const float *vs, int cap, uint16_t *ctx,
                        unsigned *err, cudaStream_t st) {
    int splits, kpc;
    if (attention_rs_plan<AR_NW>(rows, max_len, &splits, &kpc, ar_max_splits<AR_NW>())) return 1;
    ArArgs a;
    a.q = q;
    a.slots = slots;
    a.positions = positions;
    a.kc = kc;
    a.vc = vc;
    a.ks = ks;
    a.vs = vs;
    a.cap = cap;
    a.ctx = ctx;
    a.kpc = kpc;
    a.err = err;
    return splits > 1 ? run_ar<AR_NW, true>(a, rows, splits, st) : run_ar<AR_NW, false>(a, rows, 1, st);
}

}  // namespace qb
