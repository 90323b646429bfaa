// GQA decode/prefill attention over the KV8 cache in one launch: one
// thread-block cluster per (query row, KV head), its CTAs splitting the row's
// context. Arithmetic of legacy_100mhz_closed/src/PC/model_backend.py:97-102
// over the KV8 cache in the accelerator's order, every sum exact (the
// oracle's REF_KV8 | REF_EXACT mode):
//   S[h][t] = bf16(RN32(RN32(Q_h . kcode[t]) * 2^(E_h-26) * kscale[t]) / 8)
//             with q_h aligned to its largest exponent E_h as 28-bit integers
//             Q_h[d] = rint(q_h[d] * 2^(26-E_h)) and an exact integer dot
//   E[h][t] = qexp(S[h][t] - max_t S[h]),  Z_h = RN32(sum_t rint(E * 2^40)) 2^-40
//   P[h][t] = bf16(E[h][t] / Z_h),  w[h][t] = RN32(P[h][t] * vscale[t])
//   ctx[h]  = bf16(RN32(sum_t W[h][t] * vcode[t]) * 2^(F_h-26)),
//             W = rint(w * 2^(26-F_h)), F_h = exponent of
//             RN32(bf16(1/Z_h) * max_t vscale[t]) (a bound of every w)
// (the V scale enters the reduction with the probability, as in
// src/rtl/kv8_v_pscale.sv:1-20). Both products run on the tensor cores
// (mma.sync, register fragments), int8 x int8 -> int32:
//   scores   D[16 keys][8 heads] = Kcode[16][64] . Q^T[64][8] (m16n8k32): Q
//            is split into four signed 7-bit limbs, the raw codes are the A
//            operand as they sit in shared memory, the limb sums fold in int64
//   context  D[16 dims][8 heads] += Vcode^T[16][16 keys] . W[16 keys][8]
//            (m16n8k16, s8 x u8): W >= 0 is split into its four bytes (one
//            n-tile each), the V codes are transposed 4 x 4 bytes at a time
//            with byte permutes into the A fragment; a warp covers all 64
//            dims of its 16 keys, accumulating int32 per byte plane
// so the context is bit-identical to the oracle's whatever the split.
// K and then V stream through one 4-slot shared-memory ring in 128-key chunks
// (8 KB of codes) by bulk copy, completing on mbarriers (bounded waits); the
// per-key scales are staged in shared memory once.
//   phase 1  scores of this CTA's keys -> shared memory, per-head CTA max and
//            the CTA's largest V scale; the cluster forms the global values
//   phase 2  E = qexp(S - max) in place, exact per-head sums; the cluster
//            adds them; per-head 1/Z and context alignment F_h
//   phase 3  per chunk: W from E, the products on the tensor cores
//   phase 4  byte planes fold to int64, the warps' partials are added, CTA
//            rank 0 adds the ranks' partials and writes ctx (bf16)
// No global scratch, no atomics; results do not depend on scheduling.
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace qb {

constexpr int AM_THREADS = 256;
constexpr int AM_WARPS = AM_THREADS / 32;
constexpr int AM_CHUNK = 16 * AM_WARPS;  // keys per ring stage: a 16-key block per warp
constexpr int AM_STAGE_BYTES = AM_CHUNK * QB_HD;
constexpr int AM_SLOTS_RING = 4;  // ring slots (K chunks, then V chunks)
constexpr int AM_MAX_SPLITS = 8;
constexpr int AM_MAX_KPC = 4096;  // keys per CTA (shared-memory score budget)
constexpr int AM_SLOTS = 2 * 148;  // resident CTAs the split plan aims at (2 per SM)

struct AcArgs {
    const uint16_t *q;
    const uint32_t *slots, *positions;
    const int8_t *kc, *vc;
    const int8_t *klo;  // nullable: low planes of 16-bit K codes (256 * kc + klo), same layout as kc
    const float *ks, *vs;
    int cap;
    uint16_t *ctx;
    int kpc;  // keys per CTA (multiple of AM_CHUNK)
    unsigned *err;
};

struct AcSmem {
    int ring, s, sld, kss, vss, stat, red, bars, total;
};

// ring [4][128][64] int8 | S [7][kpc + 4] fp32 | K scales [kpc] | V scales
// [kpc] | stat | per-warp reductions | mbarriers [4]. stat: max[8] (head 7:
// largest V scale) | Z[8] int64 | per-head inv, align factors, F [4][8] |
// context partial [7][64] int64. Per-warp reductions: max [8][8] fp32, Z
// [8][8] int64. The per-warp context partials [8][8][64] int64 reuse the ring
// once the last chunk is consumed.
constexpr int AC_ST_Z = 32, AC_ST_HV = 96, AC_ST_CTX = 224;
constexpr int AC_STAT_BYTES = AC_ST_CTX + 7 * QB_HD * 8;
__host__ __device__ inline AcSmem ac_smem(int kpc) {
    AcSmem L;
    L.ring = 0;
    L.s = L.ring + AM_SLOTS_RING * AM_STAGE_BYTES;
    L.sld = kpc + 4;  // row stride: the 4 head rows a warp writes fall in distinct banks
    L.kss = L.s + 7 * L.sld * 4;
    L.vss = L.kss + kpc * 4;
    L.stat = L.vss + kpc * 4;
    L.red = L.stat + AC_STAT_BYTES;
    L.bars = L.red + AM_WARPS * 8 * 4 + AM_WARPS * 8 * 8;
    L.total = L.bars + AM_SLOTS_RING * 8;
    return L;
}
static_assert(AM_WARPS * 8 * QB_HD * 8 <= AM_SLOTS_RING * AM_STAGE_BYTES, "context partials fit in the ring");

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8u8_16816(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.u8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// 4 x 4 byte transpose: o[j] byte i = r[i] byte j.
__device__ __forceinline__ void transpose4(const uint32_t (&r)[4], uint32_t (&o)[4]) {
    const uint32_t t0 = prmt(r[0], r[1], 0x5140u), t1 = prmt(r[0], r[1], 0x7362u);
    const uint32_t t2 = prmt(r[2], r[3], 0x5140u), t3 = prmt(r[2], r[3], 0x7362u);
    o[0] = prmt(t0, t2, 0x5410u);
    o[1] = prmt(t0, t2, 0x7632u);
    o[2] = prmt(t1, t3, 0x5410u);
    o[3] = prmt(t1, t3, 0x7632u);
}

template <bool CLUSTER>
__global__ void __launch_bounds__(AM_THREADS, 2) attn_cluster_kernel(AcArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int kpc = a.kpc;
    const AcSmem L = ac_smem(kpc);
    const int8_t *ring = reinterpret_cast<const int8_t *>(sm + L.ring);
    float *S = reinterpret_cast<float *>(sm + L.s);
    float *kss = reinterpret_cast<float *>(sm + L.kss);
    float *vss = reinterpret_cast<float *>(sm + L.vss);
    long long *part = reinterpret_cast<long long *>(sm + L.ring);  // phase 4, after the last chunk
    float *stat = reinterpret_cast<float *>(sm + L.stat);             // max[8]
    long long *statz = reinterpret_cast<long long *>(sm + L.stat + AC_ST_Z);
    float *hv = reinterpret_cast<float *>(sm + L.stat + AC_ST_HV);    // inv[8] s1[8] s2[8] F[8]
    long long *ctxp = reinterpret_cast<long long *>(sm + L.stat + AC_ST_CTX);
    float *red = reinterpret_cast<float *>(sm + L.red);
    long long *redz = reinterpret_cast<long long *>(sm + L.red + AM_WARPS * 8 * 4);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + L.bars);
    const int sld = L.sld;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gid = lane >> 2, tig = lane & 3;  // fragment row group / thread in group
    const int kvh = blockIdx.y, r = blockIdx.z;
    const int rank = CLUSTER ? (int)tc::cluster_rank() : 0;
    const int nranks = CLUSTER ? (int)gridDim.x : 1;
    const int L_row = (int)a.positions[r] + 1;
    const int slot = (int)a.slots[r];
    const int t_begin = rank * kpc;
    const int nkeys = max(0, min(L_row, t_begin + kpc) - t_begin);
    const int nchunks = (nkeys + AM_CHUNK - 1) / AM_CHUNK;
    const size_t kvbase = ((size_t)slot * QB_KVH + kvh) * a.cap + t_begin;  // first key of this CTA
    const int8_t *kg = a.kc + kvbase * QB_HD;
    const int8_t *vg = a.vc + kvbase * QB_HD;

    // ring item i: K chunk i (i < nchunks), then V chunk i - nchunks; slot i % 8
    const int items = 2 * nchunks;
    auto issue = [&](int i) {
        const bool isv = i >= nchunks;
        const int c = isv ? i - nchunks : i;
        const int n = min(AM_CHUNK, nkeys - c * AM_CHUNK);
        const int sl = i % AM_SLOTS_RING;
        tc::mbar_arrive_expect_tx(&full[sl], (uint32_t)(n * QB_HD));
        tc::bulk_load(sm + L.ring + sl * AM_STAGE_BYTES, (isv ? vg : kg) + (size_t)c * AM_STAGE_BYTES,
                      (uint32_t)(n * QB_HD), &full[sl]);
    };
    if (tid == 0) {
        for (int sl = 0; sl < AM_SLOTS_RING; ++sl) tc::mbar_init(&full[sl], 1);
        tc::mbar_fence_init();
    }
    pdl_wait();  // q and the newest cache entries come from the preceding kernel
    pdl_trigger();
    if (tid == 0)
        for (int i = 0; i < min(items, AM_SLOTS_RING); ++i) issue(i);
    float vmax = 0.f;  // largest V scale of this CTA's keys
#pragma unroll 4
    for (int t = tid; t < nkeys; t += AM_THREADS) {
        const float kv = __ldg(a.ks + kvbase + t), vv = __ldg(a.vs + kvbase + t);
        kss[t] = kv;
        vss[t] = vv;
        vmax = fmaxf(vmax, vv);
    }
    bool ok = true;

    // q as int8 limbs (B operand of the score product): head gid, dims
    // 16*tig .. 16*tig+15. E = exponent of max|q| over the head's 64 dims;
    // Q = rint(q * 2^(26-E)) = L0 + 2^7 L1 + 2^14 L2 + 2^21 L3 with L0..L2 in
    // [-64, 63]. In k step s the fragment's k = 4tig..4tig+3 | 16+4tig..
    // 16+4tig+3 map to dims 16tig + 8s + 0..3 | 16tig + 8s + 4..7, so both
    // operands are plain 32-bit words of consecutive dims.
    uint32_t qb[4][2][2];  // [limb][k step][register]
    int e_h0, e_h1;        // exponents of heads 2tig, 2tig+1 (the C fragment's columns)
    {
        uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
        if (gid < 7) {
            const uint4 *qp =
                reinterpret_cast<const uint4 *>(a.q + (size_t)r * QB_HID + (kvh * 7 + gid) * QB_HD + 16 * tig);
            q0 = qp[0];
            q1 = qp[1];
        }
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
        const int e = row_exponent(amax);
        uint32_t lb[4][4] = {};  // [limb][word of 4 dims]
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int qi = align28_int(qf[i], e);
            const int l0 = ((qi + 64) & 127) - 64;
            const int r1 = (qi - l0) >> 7;
            const int l1 = ((r1 + 64) & 127) - 64;
            const int r2 = (r1 - l1) >> 7;
            const int l2 = ((r2 + 64) & 127) - 64;
            const int l3 = (r2 - l2) >> 7;
            const int limb[4] = {l0, l1, l2, l3};
#pragma unroll
            for (int l = 0; l < 4; ++l) lb[l][i >> 2] |= ((uint32_t)limb[l] & 0xffu) << (8 * (i & 3));
        }
#pragma unroll
        for (int l = 0; l < 4; ++l)
#pragma unroll
            for (int st = 0; st < 2; ++st) {
                qb[l][st][0] = lb[l][2 * st];
                qb[l][st][1] = lb[l][2 * st + 1];
            }
        e_h0 = __shfl_sync(0xffffffffu, e, 4 * (2 * tig));
        e_h1 = __shfl_sync(0xffffffffu, e, 4 * (2 * tig + 1));
    }
    __syncthreads();  // staged scales visible; barriers initialised

    // ---------------- phase 1: scores
    float m0 = -INFINITY, m1 = -INFINITY;  // heads 2tig, 2tig+1
    const int h0 = 2 * tig, h1 = 2 * tig + 1;
    for (int c = 0; c < nchunks; ++c) {
        const int sl = c % AM_SLOTS_RING;
        const int kb = c * AM_CHUNK + 16 * warp;  // this warp's 16-key block
        const int k0 = kb + gid, k1 = kb + gid + 8;
        if (ok) ok = tc::mbar_wait(&full[sl], (c / AM_SLOTS_RING) & 1, a.err, 11);
        if (ok && kb < nkeys) {
            const int8_t *blk = ring + sl * AM_STAGE_BYTES + 16 * warp * QB_HD;
            const uint4 u = *reinterpret_cast<const uint4 *>(blk + gid * QB_HD + 16 * tig);
            const uint4 v = *reinterpret_cast<const uint4 *>(blk + (gid + 8) * QB_HD + 16 * tig);
            int d[4][4];  // [limb][fragment]
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                d[l][0] = d[l][1] = d[l][2] = d[l][3] = 0;
                mma_s8_16832(d[l], u.x, v.x, u.y, v.y, qb[l][0][0], qb[l][0][1]);
                mma_s8_16832(d[l], u.z, v.z, u.w, v.w, qb[l][1][0], qb[l][1][1]);
            }
            long long dot[4];
#pragma unroll
            for (int f = 0; f < 4; ++f)  // per-limb sums over 64 dims are below 2^20: pairs add in int32
                dot[f] = (long long)(d[0][f] + d[1][f] * 128) + (long long)(d[2][f] + d[3][f] * 128) * 16384ll;
            if (a.klo) {
                // 16-bit codes: dot = 256 * (Q . high) + Q . low, the low plane
                // read straight from the cache (keys past the end read as 0)
                const int8_t *lg = a.klo + (kvbase + kb) * QB_HD;
                const uint4 z4 = make_uint4(0, 0, 0, 0);
                const uint4 ul = k0 < nkeys ? *reinterpret_cast<const uint4 *>(lg + gid * QB_HD + 16 * tig) : z4;
                const uint4 vl =
                    k1 < nkeys ? *reinterpret_cast<const uint4 *>(lg + (gid + 8) * QB_HD + 16 * tig) : z4;
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    int e[4] = {0, 0, 0, 0};
                    mma_s8_16832(e, ul.x, vl.x, ul.y, vl.y, qb[l][0][0], qb[l][0][1]);
                    mma_s8_16832(e, ul.z, vl.z, ul.w, vl.w, qb[l][1][0], qb[l][1][1]);
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        const long long wl = 1ll << (7 * l);
                        dot[f] += (long long)d[l][f] * 255ll * wl + (long long)e[f] * wl;
                    }
                }
            }
            float sc[4];
#pragma unroll
            for (int f = 0; f < 4; ++f) {
                const float ks = kss[f < 2 ? k0 : k1];
                sc[f] = rbf(__fmul_rn(unalign28(dot[f], (f & 1) ? e_h1 : e_h0), ks) * 0.125f);
            }
            if (k0 < nkeys) {
                S[h0 * sld + k0] = sc[0];
                m0 = fmaxf(m0, sc[0]);
                if (h1 < 7) {
                    S[h1 * sld + k0] = sc[1];
                    m1 = fmaxf(m1, sc[1]);
                }
            }
            if (k1 < nkeys) {
                S[h0 * sld + k1] = sc[2];
                m0 = fmaxf(m0, sc[2]);
                if (h1 < 7) {
                    S[h1 * sld + k1] = sc[3];
                    m1 = fmaxf(m1, sc[3]);
                }
            }
        }
        __syncthreads();  // every warp is done with this slot
        if (tid == 0 && ok && c + AM_SLOTS_RING < items) issue(c + AM_SLOTS_RING);
    }
    // per-head max: lanes of equal tig hold the same two heads
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    vmax = warp_max(vmax);
    if (gid == 0) {
        red[warp * 8 + h0] = m0;
        if (h1 < 7) red[warp * 8 + h1] = m1;
    }
    if (lane == 0) red[warp * 8 + 7] = vmax;
    __syncthreads();
    if (tid < 8) {
        float m = red[tid];
        for (int w = 1; w < AM_WARPS; ++w) m = fmaxf(m, red[w * 8 + tid]);
        stat[tid] = m;
    }
    __syncthreads();
    float M[8];  // per-head max; M[7] = largest V scale of the row's keys
    if constexpr (CLUSTER) {
        tc::cluster_sync();
        const uint32_t sa = tc::smem_u32(stat);
#pragma unroll
        for (int h = 0; h < 8; ++h) M[h] = -INFINITY;
        for (int sr = 0; sr < nranks; ++sr) {
            const float4 m03 = tc::ld_dsmem_f4(sa, sr), m47 = tc::ld_dsmem_f4(sa + 16, sr);
            const float mv[8] = {m03.x, m03.y, m03.z, m03.w, m47.x, m47.y, m47.z, m47.w};
#pragma unroll
            for (int h = 0; h < 8; ++h) M[h] = fmaxf(M[h], mv[h]);
        }
    } else {
#pragma unroll
        for (int h = 0; h < 8; ++h) M[h] = stat[h];
    }

    // ---------------- phase 2: E = qexp(S - max) in place, exact per-head sums
    long long zl[7];
#pragma unroll
    for (int h = 0; h < 7; ++h) {
        long long z = 0;
        for (int t = tid; t < nkeys; t += AM_THREADS) {
            const float e = qexp(__fsub_rn(S[h * sld + t], M[h]));
            S[h * sld + t] = e;
            z += rint_2p40(e);
        }
        zl[h] = z;
    }
#pragma unroll
    for (int h = 0; h < 7; ++h) {
        const long long z = warp_sum_ll(zl[h]);
        if (lane == 0) redz[warp * 8 + h] = z;
    }
    __syncthreads();
    if (tid < 8) {
        long long z = 0;
        if (tid < 7)
            for (int w = 0; w < AM_WARPS; ++w) z += redz[w * 8 + tid];
        statz[tid] = z;
    }
    if constexpr (CLUSTER) {
        tc::cluster_sync();
    } else {
        __syncthreads();
    }
    // per-head 1/Z, the bound of w and its alignment factors (every CTA of the
    // cluster forms the same values from the same totals)
    if (tid < 8) {
        long long z = 0;
        if constexpr (CLUSTER) {
            const uint32_t za = tc::smem_u32(statz) + 8u * (uint32_t)(tid & ~1);
            for (int sr = 0; sr < nranks; ++sr) {
                const float4 v = tc::ld_dsmem_f4(za, sr);
                const longlong2 zz = *reinterpret_cast<const longlong2 *>(&v);
                z += (tid & 1) ? zz.y : zz.x;
            }
        } else {
            z = statz[tid];
        }
        float inv = 0.f, s1 = 0.f, s2 = 0.f;
        int f = 0;
        if (tid < 7 && z > 0) {
            inv = __fdiv_rn(1.0f, __fmul_rn(__ll2float_rn(z), 0x1p-40f));
            f = row_exponent(__fmul_rn(rbf(inv), M[7]));
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

    // ---------------- phase 3: context on the tensor cores. Warp w takes keys
    // 16w..16w+15 of each chunk; lane (gid, tig) supplies k slots 4tig..4tig+3
    // = keys 16w+4tig+i: the W bytes of head gid (B) and, transposed, the V
    // codes of dims 4gid..4gid+3 and 4gid+32..4gid+35 (A rows gid and gid+8
    // of m-tile j hold dims 4gid+j and 4gid+32+j).
    const bool gv = gid < 7;
    const float inv_g = hv[gid], s1_g = hv[8 + gid], s2_g = hv[16 + gid];
    int acc[4][4][4];  // [m-tile j][byte plane l][fragment]
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int l = 0; l < 4; ++l) acc[j][l][0] = acc[j][l][1] = acc[j][l][2] = acc[j][l][3] = 0;
    for (int c = 0; c < nchunks; ++c) {
        const int item = nchunks + c;
        const int sl = item % AM_SLOTS_RING;
        const int c0 = c * AM_CHUNK, kb = 16 * warp;
        if (ok) ok = tc::mbar_wait(&full[sl], (item / AM_SLOTS_RING) & 1, a.err, 12);
        if (ok && c0 + kb < nkeys) {
            const int tb = c0 + kb + 4 * tig;  // first of this lane's keys (CTA-relative)
            float4 e4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (gv) e4 = *reinterpret_cast<const float4 *>(S + gid * sld + tb);
            const float4 v4 = *reinterpret_cast<const float4 *>(vss + tb);
            const float ev[4] = {e4.x, e4.y, e4.z, e4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w};
            uint32_t wq[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float w = (gv && tb + i < nkeys) ? __fmul_rn(rbf(__fmul_rn(ev[i], inv_g)), vv[i]) : 0.f;
                wq[i] = __float2uint_rn(__fmul_rn(__fmul_rn(w, s1_g), s2_g));
            }
            transpose4(wq, b);
            const uint32_t *vrow =
                reinterpret_cast<const uint32_t *>(ring + sl * AM_STAGE_BYTES) + (kb + 4 * tig) * (QB_HD / 4);
            uint32_t rl[4], rh[4], alo[4], ahi[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                rl[i] = vrow[i * (QB_HD / 4) + gid];
                rh[i] = vrow[i * (QB_HD / 4) + gid + 8];
            }
            transpose4(rl, alo);
            transpose4(rh, ahi);
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int l = 0; l < 4; ++l) mma_s8u8_16816(acc[j][l], alo[j], ahi[j], b[l]);
        }
        __syncthreads();  // every warp is done with this slot
        if (tid == 0 && ok && item + AM_SLOTS_RING < items) issue(item + AM_SLOTS_RING);
    }

    // ---------------- phase 4: byte planes -> int64, warps -> CTA -> rank 0
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
    for (int i = tid; i < 7 * QB_HD; i += AM_THREADS) {
        const int h = i >> 6, d = i & 63;
        long long sum = 0;
#pragma unroll
        for (int w = 0; w < AM_WARPS; ++w) sum += part[(w * 8 + h) * QB_HD + d];
        ctxp[i] = sum;
    }
    if constexpr (CLUSTER) {
        tc::cluster_sync();
        if (rank == 0) {
            const uint32_t ca = tc::smem_u32(ctxp);
            for (int i2 = tid; i2 < 7 * QB_HD / 2; i2 += AM_THREADS) {
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
        tc::cluster_sync();  // peers' shared memory stays alive until rank 0 has read it
    } else {
        __syncthreads();
        for (int i = tid; i < 7 * QB_HD; i += AM_THREADS) {
            const int h = i >> 6, d = i & 63;
            a.ctx[(size_t)r * QB_HID + (kvh * 7 + h) * QB_HD + d] =
                f2bf(unalign28(ctxp[i], __float_as_int(hv[24 + h])));
        }
    }
}

// Splits: enough CTAs to fill the GPU once at two per SM, at least enough to
// keep every CTA within AM_MAX_KPC keys, at most one 128-key chunk per CTA
// and AM_MAX_SPLITS; no empty rank for the longest row.
int attention_cluster_plan(int rows, int max_len, int *splits, int *kpc) {
    if (max_len <= 0 || rows <= 0) return -1;
    const int chunks = (max_len + AM_CHUNK - 1) / AM_CHUNK;
    int s = AM_SLOTS / (2 * rows);
    s = s < 1 ? 1 : (s > AM_MAX_SPLITS ? AM_MAX_SPLITS : s);
    s = s > chunks ? chunks : s;
    const int need = (max_len + AM_MAX_KPC - 1) / AM_MAX_KPC;
    s = s < need ? need : s;
    if (s > AM_MAX_SPLITS) return -1;
    const int cpc = (chunks + s - 1) / s;  // chunks per CTA
    *kpc = cpc * AM_CHUNK;
    *splits = (chunks + cpc - 1) / cpc;
    return 0;
}

template <bool CLUSTER>
static int run_ac(const AcArgs &a, int rows, int splits, cudaStream_t st) {
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << (dev & 31)))) {
        if (cudaFuncSetAttribute(attn_cluster_kernel<CLUSTER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 ac_smem(AM_MAX_KPC).total) != cudaSuccess)
            return -3;
        configured |= 1u << (dev & 31);
    }
    return launch_pdl(attn_cluster_kernel<CLUSTER>, dim3(splits, QB_KVH, rows), dim3(AM_THREADS),
                      (size_t)ac_smem(a.kpc).total, st, CLUSTER ? (unsigned)splits : 1u, a);
}

static __device__ unsigned g_attn_op_err;  // wait-timeout flag of calls that pass none

int launch_attention_cluster(const uint16_t *q, int rows, const uint32_t *slots, const uint32_t *positions,
                             int max_len, const int8_t *kc, const float *ks, const int8_t *vc, const float *vs, int cap,
                             uint16_t *ctx, unsigned *err, cudaStream_t st, const int8_t *klo) {
    if (rows <= 0 || max_len > cap || rows > 65535) return -1;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc) |
         reinterpret_cast<uintptr_t>(klo)) & 15)
        return -1;  // 16-byte q loads and bulk copies of the code rows
    if (reinterpret_cast<uintptr_t>(ctx) & 7) return -1;
    if (!err && cudaGetSymbolAddress(reinterpret_cast<void **>(&err), g_attn_op_err) != cudaSuccess) return -3;
    // contexts up to 8 x 2304 keys with 8-bit K codes: scores in registers
    // (attention_rs.cu)
    if (!klo) {
        const int rc = launch_attention_rs(q, rows, slots, positions, max_len, kc, ks, vc, vs, cap, ctx, err, st);
        if (rc != 1) return rc;
    }
    int splits, kpc;
    if (attention_cluster_plan(rows, max_len, &splits, &kpc)) return -1;
    AcArgs a;
    a.q = q;
    a.slots = slots;
    a.positions = positions;
    a.kc = kc;
    a.vc = vc;
    a.klo = klo;
    a.ks = ks;
    a.vs = vs;
    a.cap = cap;
    a.ctx = ctx;
    a.kpc = kpc;
    a.err = err;
    return splits > 1 ? run_ac<true>(a, rows, splits, st) : run_ac<false>(a, rows, 1, st);
}

}  // namespace qb
