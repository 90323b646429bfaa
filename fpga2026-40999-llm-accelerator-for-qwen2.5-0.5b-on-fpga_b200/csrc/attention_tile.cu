// Query-tiled GQA attention over the KV8 cache for prefill rows, both
// products on the 5th-generation tensor cores (tcgen05.mma kind::i8, TMEM
// accumulators). A tile is up to 4 consecutive positions of one slot; a CTA
// takes one tile and one KV head over a range of at most 1024 keys, and a
// thread-block cluster of up to 8 CTAs splits a longer prefix.
//
// Arithmetic: the exact attention of attention_rs.cu / attention_cluster.cu
// (the oracle's REF_KV8 | REF_EXACT order, model_backend.py:97-102 in the
// accelerator's order), row by row, with each row's causal prefix (keys
// 0..pos):
//   S[t] = bf16(RN32(RN32(Q . kcode[t]) * 2^(E-26) * kscale[t]) / 8)
//   E[t] = qexp(S[t] - max S), Z = RN32(sum_t rint(E[t] * 2^40)) * 2^-40
//   W[t] = rint(RN32(bf16(E[t] / Z) * vscale[t]) * 2^(26-F))
//   ctx  = bf16(RN32(sum_t W[t] * vcode[t]) * 2^(F-26))
// All sums are exact integers, so the result is bit-identical to the
// oracle's whatever the tiling and the split.
//
// Products:
//   scores  D1[128 keys][128] = Kchunk[128][64] . B1[128][64]^T, B1 row
//           l*32 + q*8 + h = limb l of query row q, head h (h = 7 and rows
//           beyond the tile are zero), K = 64 dims; D1 in TMEM columns 0-127 /
//           128-255 for even / odd chunks, one thread per key folds the four
//           limb columns into int64
//   context D2[128][64 dims] += A2[128][128 keys] . B2[64][128 keys]^T with
//           A2 row p*32 + q*8 + h = byte p of W (unsigned), B2 = the V chunk
//           transposed (signed); D2 in TMEM columns 0-63, int32 per byte
//           plane (at most 1024 x 255 x 127 < 2^31), folded to int64 at the end
// Operands: K chunks by TMA (64-byte swizzle), V chunks by bulk copy through
// the same 4-slot ring; B1, A2 and B2 written by the compute warps in the
// swizzled K-major layouts the MMA descriptors name.
// Warps: 0 producer, 1 TMEM owner and MMA issuer (one thread), 2-17 compute.
// Every wait is bounded (error codes 40-47); a CTA that gives up keeps
// taking part in the cluster barriers and still frees its TMEM.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace qb {

constexpr int AT_QT = 4;                  // query rows per tile
constexpr int AT_QH = AT_QT * 7;          // (query, head) pairs of a tile
constexpr int AT_CH = 128;                // keys per chunk
constexpr int AT_MAXC = 8;                // chunks per CTA
constexpr int AT_KPC = AT_CH * AT_MAXC;   // keys per CTA at most
constexpr int AT_SLD = AT_KPC + 1;        // score row stride (floats, odd: rows fall on distinct banks)
constexpr int AT_RING = 4;
constexpr int AT_CW = 16;                 // compute warps: 4 per TMEM lane quarter
constexpr int AT_CT = 32 * AT_CW;         // compute threads
constexpr int AT_THREADS = 64 + AT_CT;
constexpr int AT_MAX_SPLITS = 8;
constexpr uint32_t AT_TMEM_COLS = 256;    // D1 double-buffered: 0-127 / 128-255; D2 over the first (cols 0-63)

struct AtSmem {
    static constexpr int B1 = 0;                          // [128][64] sw64
    static constexpr int RING = B1 + 128 * 64;            // [4][128][64]
    static constexpr int A2 = RING + AT_RING * AT_CH * 64;  // [2][128][128] sw128
    static constexpr int B2 = A2 + 2 * 128 * 128;         // [2][64][128] sw128
    static constexpr int S = B2 + 2 * 64 * 128;           // [28][AT_SLD] fp32
    static constexpr int KSS = S + AT_QH * AT_SLD * 4;    // [1024] fp32
    static constexpr int VSS = KSS + AT_KPC * 4;
    static constexpr int QE = VSS + AT_KPC * 4;           // [28] int: query row exponents
    static constexpr int WMAX = QE + 32 * 4;              // [8 warps][28] fp32
    static constexpr int WV = WMAX + AT_CW * 32 * 4;      // [8 warps][4] fp32: V-scale maxima
    static constexpr int WZ = WV + AT_CW * 4 * 4;         // [8 warps][32] int64: partial exact sums
    static constexpr int ST = WZ + AT_CW * 32 * 8;        // statistics (below)
    // words: max [28], largest V scale per query row [4], Z [28] int64, 1/Z,
    // the two alignment factors and F [28] each
    static constexpr int ST_M = 0, ST_V = 28, ST_Z = 32, ST_INV = 88, ST_S1 = 120, ST_S2 = 152, ST_F = 184;
    static constexpr int ST_WORDS = 216;
    static constexpr int BARS = ST + ST_WORDS * 4;
    static constexpr int NBARS = 2 * AT_RING + 12;  // ring full / empty, d1 full / empty x 2, ops full / empty x 2, d2, done, b1, scales
    static constexpr int SLOT = BARS + NBARS * 8;
    static constexpr int TOTAL = SLOT + 16;
    static constexpr int ALLOC = TOTAL + 1024;            // 1024-byte alignment of the base
};
static_assert(AtSmem::ST_Z * 4 % 8 == 0 && AtSmem::ST_Z + 2 * AT_QH <= AtSmem::ST_INV, "stat layout");
static_assert(AtSmem::ST % 8 == 0 && AtSmem::BARS % 8 == 0 && AtSmem::WZ % 8 == 0, "aligned sub-areas");
static_assert(4 * 64 * 32 * 4 <= 2 * 128 * 128 && 64 * 33 * 8 <= AT_RING * AT_CH * 64, "context staging fits over A2 / the ring");
static_assert(AtSmem::ALLOC <= 232448, "shared memory per CTA");

struct AtArgs {
    const uint16_t *q;     // [rows][896] post-RoPE queries
    const AtTile *tiles;   // this launch's tiles
    const int8_t *vc;      // V codes [slot][2][cap][64] (this layer)
    const float *ks, *vs;  // [slot][2][cap]
    long long krow0;       // K tensor-map row of (slot 0, KV head 0, key 0) of this layer
    int cap, kpc;
    uint16_t *ctx;         // [rows][896]
    unsigned *err;
};

// kind::i8, D s32, K-major A and B; a_signed / b_signed select s8 or u8.
__host__ __device__ constexpr uint32_t at_idesc(int m, int n, bool a_signed, bool b_signed) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void at_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)acc));
}
// Shared-memory descriptor of a K-major operand in the 64-byte swizzle layout:
// rows of 64 bytes, 8-row groups 512 bytes apart.
__device__ __forceinline__ uint64_t at_desc_sw64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(512u >> 4) << 32;   // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;             // descriptor version for sm_100
    d |= (uint64_t)4 << 61;             // SWIZZLE_64B
    return d;
}
__device__ __forceinline__ void at_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void at_ld8(uint32_t taddr, int (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void at_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Barrier of the compute warps only (named barrier 1).
__device__ __forceinline__ void at_csync() { asm volatile("bar.sync 1, %0;" ::"n"(AT_CT) : "memory"); }
__device__ __forceinline__ long long at_ld_dsmem_ll(uint32_t local_saddr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
    long long v;
    asm volatile("ld.shared::cluster.s64 %0, [%1];" : "=l"(v) : "r"(remote) : "memory");
    return v;
}
__device__ __forceinline__ float at_ld_dsmem_f(uint32_t local_saddr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}
// Byte offset of 16-byte chunk c of row r in a swizzled K-major tile.
__device__ __forceinline__ uint32_t at_sw64(int r, int c) { return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4)); }
__device__ __forceinline__ uint32_t at_sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }
__device__ __forceinline__ uint32_t at_prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
// 4 x 4 byte transpose: o[j] byte i = w[i] byte j.
__device__ __forceinline__ void at_transpose4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t (&o)[4]) {
    const uint32_t t0 = at_prmt(w0, w1, 0x5140u), t1 = at_prmt(w0, w1, 0x7362u);
    const uint32_t t2 = at_prmt(w2, w3, 0x5140u), t3 = at_prmt(w2, w3, 0x7362u);
    o[0] = at_prmt(t0, t2, 0x5410u);
    o[1] = at_prmt(t0, t2, 0x7632u);
    o[2] = at_prmt(t1, t3, 0x5410u);
    o[3] = at_prmt(t1, t3, 0x7632u);
}

template <bool CLUSTER>
__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_tile_kernel(const __grid_constant__ CUtensorMap kmap, AtArgs a) {
    using L = AtSmem;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + L::BARS);
    uint64_t *full = bars, *empty = bars + AT_RING;
    uint64_t *d1full = bars + 2 * AT_RING, *d1empty = d1full + 1, *opsfull = d1full + 2, *opsempty = d1full + 4;
    uint32_t *slot_p = reinterpret_cast<uint32_t *>(sm + L::SLOT);
    float *S = reinterpret_cast<float *>(sm + L::S);
    float *kss = reinterpret_cast<float *>(sm + L::KSS), *vss = reinterpret_cast<float *>(sm + L::VSS);
    int *qe = reinterpret_cast<int *>(sm + L::QE);
    float *wmax = reinterpret_cast<float *>(sm + L::WMAX), *wv = reinterpret_cast<float *>(sm + L::WV);
    long long *wz = reinterpret_cast<long long *>(sm + L::WZ);
    float *st = reinterpret_cast<float *>(sm + L::ST);
    float *stM = st + L::ST_M, *stV = st + L::ST_V, *stInv = st + L::ST_INV, *stS1 = st + L::ST_S1,
          *stS2 = st + L::ST_S2;
    int *stF = reinterpret_cast<int *>(st + L::ST_F);
    long long *stZ = reinterpret_cast<long long *>(st + L::ST_Z);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = blockIdx.y;
    const AtTile tile = a.tiles[blockIdx.z];
    const int rank = CLUSTER ? (int)tc::cluster_rank() : 0;
    const int nranks = CLUSTER ? (int)gridDim.x : 1;
    const int keys = tile.pos0 + tile.nq;  // the tile's prefix: keys 0 .. last position
    // the prefix split evenly over the cluster, in whole chunks (at most 1024 keys a CTA)
    const int kpc = min(AT_KPC, ((keys + nranks - 1) / nranks + AT_CH - 1) / AT_CH * AT_CH);
    const int k_begin = rank * kpc;
    const int nkeys = max(0, min(kpc, keys - k_begin));
    const int nch = (nkeys + AT_CH - 1) / AT_CH;
    const size_t kvrow = ((size_t)tile.slot * QB_KVH + g) * a.cap + k_begin;  // this CTA's first key

    if (tid == 0) {
        for (int s = 0; s < AT_RING; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(d1full, 1);
        tc::mbar_init(d1empty, AT_CW);  // one arrival per compute warp
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&opsfull[b], AT_CW);
            tc::mbar_init(&opsempty[b], 1);
        }
        tc::mbar_init(d1full + 6, 1);  // D2 complete
        tc::mbar_init(d1full + 7, 1);  // every MMA complete (TMEM may be freed)
        tc::mbar_init(d1full + 8, 1);  // B1 written
        tc::mbar_init(d1full + 9, 1);  // the CTA's key and V scales copied
        tc::mbar_init(d1full + 10, 1);  // second D1 buffer full
        tc::mbar_init(d1full + 11, AT_CW);  // second D1 buffer read
        tc::mbar_fence_init();
        tc::tma_prefetch_desc(&kmap);
    }
    uint64_t *d2full = d1full + 6, *mdone = d1full + 7, *b1ready = d1full + 8, *sbar = d1full + 9;
    uint64_t *d1f[2] = {d1full, d1full + 10}, *d1e[2] = {d1empty, d1full + 11};
    // scales by bulk copy when both rows are 16-byte aligned and whole 16-byte runs stay inside the slot's row
    const int nk4 = (nkeys + 3) & ~3;
    const bool bulk_scales = nkeys > 0 && ((kvrow & 3) == 0) && k_begin + nk4 <= a.cap &&
                             ((reinterpret_cast<uintptr_t>(a.ks) | reinterpret_cast<uintptr_t>(a.vs)) & 15) == 0;
    if (warp == 1) tc::tmem_alloc(slot_p, AT_TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *slot_p;
    pdl_wait();  // q and the newest cache entries come from the preceding kernels
    pdl_trigger();
    bool ok = true;

    if (warp == 0) {
        // ---------------- producer: the scales, K chunks (TMA, swizzled), then V chunks
        if (lane == 0) {
            if (bulk_scales) {
                tc::mbar_arrive_expect_tx(sbar, (uint32_t)(2 * nk4 * 4));
                tc::bulk_load(kss, a.ks + kvrow, (uint32_t)(nk4 * 4), sbar);
                tc::bulk_load(vss, a.vs + kvrow, (uint32_t)(nk4 * 4), sbar);
            }
            for (int c = 0; c < nch; ++c) {
                const int s = c % AT_RING;
                if (ok) ok = tc::mbar_wait(&empty[s], ((c / AT_RING) & 1) ^ 1, a.err, 40);
                if (!ok) break;
                tc::mbar_arrive_expect_tx(&full[s], (uint32_t)(AT_CH * 64));
                tc::tma_load_2d(sm + L::RING + s * AT_CH * 64, &kmap, &full[s], 0,
                                (int)(a.krow0 + (long long)kvrow + c * AT_CH));
            }
        }
        __syncwarp();
        if constexpr (CLUSTER) {
            tc::cluster_sync();  // (1) maxima
            tc::cluster_sync();  // (2) sums
        }
        if (lane == 0) {
            for (int c = 0; c < nch; ++c) {
                const int i = nch + c, s = i % AT_RING;
                if (ok) ok = tc::mbar_wait(&empty[s], ((i / AT_RING) & 1) ^ 1, a.err, 41);
                if (!ok) break;
                const int n = min(AT_CH, nkeys - c * AT_CH);
                tc::mbar_arrive_expect_tx(&full[s], (uint32_t)(n * 64));
                tc::bulk_load(sm + L::RING + s * AT_CH * 64, a.vc + (kvrow + (size_t)c * AT_CH) * 64, (uint32_t)(n * 64),
                              &full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t id1 = at_idesc(128, 128, true, true);
            if (nch > 0) ok = tc::mbar_wait(b1ready, 0, a.err, 42);
            for (int c = 0; c < nch && ok; ++c) {
                const int s = c % AT_RING;
                if (!tc::mbar_wait(&full[s], (c / AT_RING) & 1, a.err, 42)) { ok = false; break; }
                const int b = c & 1, use = c >> 1;  // D1 buffer and its use
                if (use > 0 && !tc::mbar_wait(d1e[b], (use - 1) & 1, a.err, 43)) { ok = false; break; }
                tc::tc_fence_after();
                const uint32_t ka = tc::smem_u32(sm + L::RING + s * AT_CH * 64), qb = tc::smem_u32(sm + L::B1);
#pragma unroll
                for (int j = 0; j < 2; ++j)
                    at_mma(tmem + 128 * b, at_desc_sw64(ka + 32 * j), at_desc_sw64(qb + 32 * j), id1, j > 0);
                tc::mma_commit(d1f[b]);
                tc::mma_commit(&empty[s]);
            }
        }
        __syncwarp();
        if constexpr (CLUSTER) {
            tc::cluster_sync();  // (1)
            tc::cluster_sync();  // (2)
        }
        if (lane == 0) {
            constexpr uint32_t id2 = at_idesc(128, 64, false, true);
            // phase-1 MMAs are complete once the compute warps have read the last D1
            for (int c = 0; c < nch && ok; ++c) {
                const int b = c & 1;
                if (!tc::mbar_wait(&opsfull[b], (c >> 1) & 1, a.err, 44)) { ok = false; break; }
                tc::tc_fence_after();
                const uint32_t aa = tc::smem_u32(sm + L::A2 + b * 128 * 128), bb = tc::smem_u32(sm + L::B2 + b * 64 * 128);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    at_mma(tmem, tc::smem_desc_sw128(aa + 32 * j), tc::smem_desc_sw128(bb + 32 * j), id2,
                           c > 0 || j > 0);
                tc::mma_commit(&opsempty[b]);
                tc::mma_commit(&empty[(nch + c) % AT_RING]);  // the compute warps read that V chunk before opsfull
            }
            if (ok && nch > 0) tc::mma_commit(d2full);
            tc::mma_commit(mdone);
            tc::mbar_wait(mdone, 0, a.err, 45);
        }
        __syncwarp();
    } else {
        // ---------------- compute warps
        const int ct = tid - 64, cw = warp - 2;
        const int quarter = warp & 3, part = cw >> 2;  // TMEM lane quarter; query row (phase 1), dims 16 part.. (phase 4)
        // B1: the tile's query limbs; thread: (q, h8) = ct / 8, dims 8 (ct % 8) .. + 7
        if (ct < 256) {
            const int r8 = ct >> 3, dg = ct & 7, q = r8 >> 3, h8 = r8 & 7;
            const bool live = h8 < 7 && q < tile.nq;
            float v[8];
            float amax = 0.f;
            if (live) {
                const uint4 w = *reinterpret_cast<const uint4 *>(a.q + (size_t)(tile.row0 + q) * QB_HID +
                                                                 (g * 7 + h8) * QB_HD + 8 * dg);
                const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    v[2 * i] = bflo(ww[i]);
                    v[2 * i + 1] = bfhi(ww[i]);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const int e = row_exponent(amax);
            uint32_t lb[4][2] = {};
            if (live) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    int l4[4];
                    limbs4(align28_int(v[i], e), l4);
#pragma unroll
                    for (int l = 0; l < 4; ++l) lb[l][i >> 2] |= ((uint32_t)l4[l] & 0xffu) << (8 * (i & 3));
                }
                if (dg == 0) qe[q * 7 + h8] = e;
            }
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const int n = l * 32 + r8;
                *reinterpret_cast<uint2 *>(sm + L::B1 + at_sw64(n, dg >> 1) + 8 * (dg & 1)) = make_uint2(lb[l][0], lb[l][1]);
            }
        }
        // scales of this CTA's keys (bulk copies of the producer, or plain
        // loads); largest V scale of each query row's keys
        if (!bulk_scales)
            for (int t = ct; t < nkeys; t += AT_CT) {
                kss[t] = __ldg(a.ks + kvrow + t);
                vss[t] = __ldg(a.vs + kvrow + t);
            }
        tc::fence_proxy_async_smem();  // B1 (generic writes) is read by the MMAs
        at_csync();
        if (ct == 0) tc::mbar_arrive(b1ready);
        if (bulk_scales && ok) ok = tc::mbar_wait(sbar, 0, a.err, 46);
        float vm[AT_QT] = {0.f, 0.f, 0.f, 0.f};
        for (int t = ct; t < nkeys; t += AT_CT) {
            const float vv = vss[t];
#pragma unroll
            for (int q = 0; q < AT_QT; ++q)
                if (k_begin + t <= tile.pos0 + q) vm[q] = fmaxf(vm[q], vv);
        }
#pragma unroll
        for (int q = 0; q < AT_QT; ++q) {
            const float m = warp_max(vm[q]);
            if (lane == 0) wv[cw * 4 + q] = m;
        }
        // ---------------- phase 1: scores (thread: one key, query row `part`, 7 heads)
        // the two power-of-two factors of unalign28 for this row's heads
        float uc1[7], uc2[7];
#pragma unroll
        for (int h8 = 0; h8 < 7; ++h8) {
            const int e = part < tile.nq ? qe[part * 7 + h8] : 0;
            const int sh = e - 26, sh1 = max(sh, -126);
            uc1[h8] = pow2i(sh1);
            uc2[h8] = pow2i(sh - sh1);
        }
        float mx[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) mx[j] = -INFINITY;
        for (int c = 0; c < nch; ++c) {
            int d[4][8];
            const int b = c & 1;
            if (ok) ok = tc::mbar_wait(d1f[b], (c >> 1) & 1, a.err, 46);
            tc::tc_fence_after();
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                if (ok) {
                    at_ld8(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(128 * b + l * 32 + part * 8), d[l]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) d[l][j] = 0;
                }
            }
            if (ok) at_ld_wait();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(d1e[b]);  // this warp's part of the D1 buffer may be overwritten
            const int kk = c * AT_CH + quarter * 32 + lane;  // CTA-local key
            const int q = part;
            const bool in = kk < nkeys && q < tile.nq;
            const bool vis = in && k_begin + kk <= tile.pos0 + q;
            const float ksc = in ? kss[kk] : 0.f;
#pragma unroll
            for (int h8 = 0; h8 < 7; ++h8) {
                const long long dot =
                    (long long)(d[0][h8] + d[1][h8] * 128) + (long long)(d[2][h8] + d[3][h8] * 128) * 16384ll;
                // unalign28(dot, e): (RN32(dot) * 2^s1) * 2^(s - s1)
                const float u = (__ll2float_rn(dot) * uc1[h8]) * uc2[h8];
                const float s = vis ? rbf(__fmul_rn(u, ksc) * 0.125f) : -INFINITY;
                if (in) S[(q * 7 + h8) * AT_SLD + kk] = s;
                mx[h8] = fmaxf(mx[h8], s);
            }
        }
        // per (q, h) maxima: lanes, then the four warps of a query row
#pragma unroll
        for (int j = 0; j < 7; ++j) {
            float m = mx[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            mx[j] = m;
        }
        if (lane == 0)
#pragma unroll
            for (int j = 0; j < 7; ++j) wmax[cw * 32 + part * 7 + j] = mx[j];
        at_csync();
        if (ct < AT_QH) {
            const int q = ct / 7;  // the part that computed this pair
            float m = -INFINITY;
            for (int w = 0; w < 4; ++w) m = fmaxf(m, wmax[(q * 4 + w) * 32 + ct]);
            stM[ct] = m;
        } else if (ct >= 32 && ct < 32 + AT_QT) {
            const int q = ct - 32;
            float m = 0.f;
            for (int w = 0; w < AT_CW; ++w) m = fmaxf(m, wv[w * 4 + q]);
            stV[q] = m;
        }
        at_csync();
        if constexpr (CLUSTER) tc::cluster_sync();  // (1)
        float Mrow = -INFINITY;  // this lane's pair in phase 2: (q, h) = lane
        if (lane < AT_QH) {
            if constexpr (CLUSTER) {
                const uint32_t sa = tc::smem_u32(stM + lane);
                for (int r = 0; r < nranks; ++r) Mrow = fmaxf(Mrow, at_ld_dsmem_f(sa, (uint32_t)r));
            } else {
                Mrow = stM[lane];
            }
        }
        // ---------------- phase 2: E = qexp(S - max) in place, exact sums;
        // lane = (q, h), warp w takes keys w, w + 16, ... four at a time
        {
            const int qh = lane;
            long long z = 0;
            if (qh < AT_QH) {
                const int q = qh / 7;
                const int lim = min(nkeys, tile.pos0 + q + 1 - k_begin);  // visible keys of this row
                float *row = S + qh * AT_SLD;
                int t = cw;
                for (; t + 3 * AT_CW < lim; t += 4 * AT_CW) {
                    float e0, e1, e2, e3;
                    qexp2(__fsub_rn(row[t], Mrow), __fsub_rn(row[t + AT_CW], Mrow), e0, e1);
                    qexp2(__fsub_rn(row[t + 2 * AT_CW], Mrow), __fsub_rn(row[t + 3 * AT_CW], Mrow), e2, e3);
                    row[t] = e0;
                    row[t + AT_CW] = e1;
                    row[t + 2 * AT_CW] = e2;
                    row[t + 3 * AT_CW] = e3;
                    // rint(e * 2^40): the scaling is exact, one conversion rounds to nearest even
                    z += (__float2ll_rn(__fmul_rn(e0, 0x1p40f)) + __float2ll_rn(__fmul_rn(e1, 0x1p40f))) +
                         (__float2ll_rn(__fmul_rn(e2, 0x1p40f)) + __float2ll_rn(__fmul_rn(e3, 0x1p40f)));
                }
                for (; t < lim; t += AT_CW) {
                    const float e = qexp(__fsub_rn(row[t], Mrow));
                    row[t] = e;
                    z += __float2ll_rn(__fmul_rn(e, 0x1p40f));
                }
            }
            wz[cw * 32 + lane] = z;
            at_csync();
            if (ct < AT_QH) {
                long long zz = 0;
                for (int w = 0; w < AT_CW; ++w) zz += wz[w * 32 + ct];
                stZ[ct] = zz;
            }
        }
        at_csync();
        if constexpr (CLUSTER) tc::cluster_sync();  // (2)
        if (ct < AT_QH) {
            long long z = 0;
            float vmax = 0.f;
            const int q = ct / 7;
            if constexpr (CLUSTER) {
                const uint32_t za = tc::smem_u32(stZ + ct), va = tc::smem_u32(stV + q);
                for (int r = 0; r < nranks; ++r) {
                    z += at_ld_dsmem_ll(za, (uint32_t)r);
                    vmax = fmaxf(vmax, at_ld_dsmem_f(va, (uint32_t)r));
                }
            } else {
                z = stZ[ct];
                vmax = stV[q];
            }
            float inv = 0.f, s1 = 0.f, s2 = 0.f;
            int f = 0;
            if (z > 0) {
                inv = __fdiv_rn(1.0f, __fmul_rn(__ll2float_rn(z), 0x1p-40f));
                f = row_exponent(__fmul_rn(rbf(inv), vmax));
                const int sh = 26 - f, sh1 = min(sh, 127);
                s1 = pow2i(sh1);
                s2 = pow2i(sh - sh1);
            }
            stInv[ct] = inv;
            stS1[ct] = s1;
            stS2[ct] = s2;
            stF[ct] = f;
        }
        at_csync();
        // ---------------- phase 3: context on the tensor cores
        for (int c = 0; c < nch; ++c) {
            const int i = nch + c, s = i % AT_RING, b = c & 1;
            if (ok) ok = tc::mbar_wait(&full[s], (i / AT_RING) & 1, a.err, 47);
            if (ok) ok = tc::mbar_wait(&opsempty[b], ((c >> 1) & 1) ^ 1, a.err, 47);
            const uint8_t *ring = sm + L::RING + s * AT_CH * 64;
            uint8_t *A2 = sm + L::A2 + b * 128 * 128, *B2 = sm + L::B2 + b * 64 * 128;
            if (ok && cw < 4) {
                // V^T: dims 4 dg .. 4 dg + 3 of keys 16 kgrp .. 16 kgrp + 15
                const int dg = lane & 15, kgrp = 2 * cw + (lane >> 4);
                uint32_t o[4][4];
#pragma unroll
                for (int i4 = 0; i4 < 4; ++i4) {
                    const uint32_t *src = reinterpret_cast<const uint32_t *>(ring + (16 * kgrp + 4 * i4) * 64) + dg;
                    at_transpose4(src[0], src[16], src[32], src[48], o[i4]);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<uint4 *>(B2 + at_sw128(4 * dg + j, kgrp)) =
                        make_uint4(o[0][j], o[1][j], o[2][j], o[3][j]);
            }
            if (ok) {
                // W bytes: lane = row (q, h8), warp = keys 8 cw .. 8 cw + 7
                const int q = lane >> 3, h8 = lane & 7;
                uint32_t pw[4][2] = {};
                if (h8 < 7 && q < tile.nq) {
                    const int qh = q * 7 + h8;
                    const float inv = stInv[qh], s1 = stS1[qh], s2 = stS2[qh];
                    const float *row = S + qh * AT_SLD;
                    const int k0 = c * AT_CH + 8 * cw;
                    const int vis = min(nkeys, tile.pos0 + q + 1 - k_begin) - k0;  // keys of this group it sees
                    // w = rint(RN32(bf16(E * inv) * vscale) * s1 * s2), two keys per
                    // packed fp32 operation (each half one IEEE operation)
                    const float4 v0 = *reinterpret_cast<const float4 *>(vss + k0);
                    const float4 v1 = *reinterpret_cast<const float4 *>(vss + k0 + 4);
                    const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                    uint32_t wq[8];
#pragma unroll
                    for (int t = 0; t < 8; t += 2) {
                        const unsigned long long e = mul2(pk2(row[k0 + t], row[k0 + t + 1]), dup2(inv));
                        float e0, e1;
                        unpk2(e, e0, e1);
                        const __nv_bfloat162 bb = __floats2bfloat162_rn(e0, e1);
                        const unsigned long long w =
                            mul2(mul2(mul2(pk2(__low2float(bb), __high2float(bb)), pk2(vv[t], vv[t + 1])), dup2(s1)),
                                 dup2(s2));
                        float w0, w1;
                        unpk2(w, w0, w1);
                        wq[t] = t < vis ? __float2uint_rn(w0) : 0u;
                        wq[t + 1] = t + 1 < vis ? __float2uint_rn(w1) : 0u;
                    }
#pragma unroll
                    for (int i4 = 0; i4 < 2; ++i4) {
                        uint32_t pl[4];
                        // pl[p] byte k = byte p of key 4 i4 + k
                        at_transpose4(wq[4 * i4], wq[4 * i4 + 1], wq[4 * i4 + 2], wq[4 * i4 + 3], pl);
#pragma unroll
                        for (int pp = 0; pp < 4; ++pp) pw[pp][i4] = pl[pp];
                    }
                }
#pragma unroll
                for (int pp = 0; pp < 4; ++pp)
                    *reinterpret_cast<uint2 *>(A2 + at_sw128(pp * 32 + lane, cw >> 1) + 8 * (cw & 1)) =
                        make_uint2(pw[pp][0], pw[pp][1]);
            }
            tc::fence_proxy_async_smem();
            tc::tc_fence_before();  // D1 reads of phase 1 precede the D2 MMAs over the same columns
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&opsfull[b]);
        }
        // ---------------- phase 4: byte planes -> int64, CTA -> cluster rank 0
        int32_t *planes = reinterpret_cast<int32_t *>(sm + L::A2);    // [4][64 dims][32 rows]
        long long *ctxp = reinterpret_cast<long long *>(sm + L::RING);  // [64 dims][33] (row (q, h8))
        if (ok && nch > 0) ok = tc::mbar_wait(d2full, 0, a.err, 47);
        tc::tc_fence_after();
        at_csync();  // every operand read by the MMAs is over once D2 is complete
        {
            // lane quarter p = byte plane, lane = row (q, h8); columns: dims 16 part .. + 15
            int v[16];
            if (ok && nch > 0) {
                at_ld16(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(16 * part), v);
                at_ld_wait();
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) planes[(quarter * 64 + 16 * part + j) * 32 + lane] = v[j];
        }
        at_csync();
        for (int i = ct; i < 64 * 32; i += AT_CT) {
            const int d = i >> 5, r8 = i & 31;
            const long long sum = (long long)planes[(0 * 64 + d) * 32 + r8] + ((long long)planes[(1 * 64 + d) * 32 + r8] << 8) +
                                  ((long long)planes[(2 * 64 + d) * 32 + r8] << 16) +
                                  ((long long)planes[(3 * 64 + d) * 32 + r8] << 24);
            ctxp[d * 33 + r8] = sum;
        }
        tc::tc_fence_before();
        at_csync();
    }
    // ---------------- cluster combine and the context rows
    if constexpr (CLUSTER) tc::cluster_sync();  // (3)
    if (warp >= 2 && rank == 0) {
        const long long *ctxp = reinterpret_cast<const long long *>(sm + L::RING);
        for (int i = tid - 64; i < AT_QH * 64; i += AT_CT) {
            const int qh = i >> 6, d = i & 63, q = qh / 7, h = qh % 7, r8 = q * 8 + h;
            if (q >= tile.nq) continue;
            long long sum = 0;
            if constexpr (CLUSTER) {
                const uint32_t ca = tc::smem_u32(ctxp + d * 33 + r8);
                for (int r = 0; r < nranks; ++r) sum += at_ld_dsmem_ll(ca, (uint32_t)r);
            } else {
                sum = ctxp[d * 33 + r8];
            }
            a.ctx[(size_t)(tile.row0 + q) * QB_HID + (g * 7 + h) * QB_HD + d] = f2bf(unalign28(sum, stF[qh]));
        }
    }
    if constexpr (CLUSTER) tc::cluster_sync();  // (4) peers' shared memory stays alive until rank 0 has read it
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, AT_TMEM_COLS);
}

// Tiles of up to 4 consecutive positions of one slot over rows whose
// (slot, position) are given; grouped by the number of 1024-key CTAs their
// prefix needs (1..8). -1 when a row's prefix needs more than 8 (the caller
// then uses the per-row kernels).
int attention_tile_plan(int rows, const uint32_t *slots, const uint32_t *positions, AtTile *tiles,
                        std::vector<AtGroup> &groups) {
    groups.clear();
    std::vector<AtTile> by[AT_MAX_SPLITS + 1];
    for (int r = 0; r < rows;) {
        AtTile t{r, 1, (int)slots[r], (int)positions[r]};
        while (t.nq < AT_QT && r + t.nq < rows && slots[r + t.nq] == slots[r] &&
               positions[r + t.nq] == positions[r] + (uint32_t)t.nq)
            ++t.nq;
        const int keys = t.pos0 + t.nq, splits = (keys + AT_KPC - 1) / AT_KPC;
        if (splits > AT_MAX_SPLITS) return -1;
        by[splits].push_back(t);
        r += t.nq;
    }
    int n = 0;
    for (int sp = 1; sp <= AT_MAX_SPLITS; ++sp) {
        if (by[sp].empty()) continue;
        int maxkeys = 0;
        for (const AtTile &t : by[sp]) maxkeys = std::max(maxkeys, t.pos0 + t.nq);
        const int per = (maxkeys + sp - 1) / sp, kpc = (per + AT_CH - 1) / AT_CH * AT_CH;
        groups.push_back(AtGroup{sp, kpc, n, (int)by[sp].size()});
        for (const AtTile &t : by[sp]) tiles[n++] = t;
    }
    return 0;
}

template <bool CLUSTER>
static int run_at(const CUtensorMap &kmap, const AtArgs &a, int ntiles, int splits, cudaStream_t st) {
    static unsigned configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1u << (dev & 31)))) {
        if (cudaFuncSetAttribute(attn_tile_kernel<CLUSTER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 AtSmem::ALLOC) != cudaSuccess)
            return -3;
        configured |= 1u << (dev & 31);
    }
    return launch_pdl(attn_tile_kernel<CLUSTER>, dim3(splits, QB_KVH, ntiles), dim3(AT_THREADS), (size_t)AtSmem::ALLOC,
                      st, CLUSTER ? (unsigned)splits : 1u, kmap, a);
}

int launch_attention_tiles(const CUtensorMap &kmap, long long krow0, const AtTile *d_tiles, const AtGroup &grp,
                           const uint16_t *q, const int8_t *vc, const float *ks, const float *vs, int cap,
                           uint16_t *ctx, unsigned *err, cudaStream_t st) {
    if (grp.count <= 0 || grp.splits < 1 || grp.splits > AT_MAX_SPLITS || grp.kpc <= 0 || grp.kpc > AT_KPC ||
        grp.count > 65535)
        return -1;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(vc)) & 15) return -1;
    AtArgs a;
    a.q = q;
    a.tiles = d_tiles + grp.first;
    a.vc = vc;
    a.ks = ks;
    a.vs = vs;
    a.krow0 = krow0;
    a.cap = cap;
    a.kpc = grp.kpc;
    a.ctx = ctx;
    a.err = err;
    return grp.splits > 1 ? run_at<true>(kmap, a, grp.count, grp.splits, st) : run_at<false>(kmap, a, grp.count, 1, st);
}

}  // namespace qb
