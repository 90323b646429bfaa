// One batch-1 decode step (all 24 layers, final RMSNorm, LM head and greedy
// argmax of legacy_100mhz_closed/src/PC/model_backend.py:57-115) in a single
// persistent cooperative launch of one CTA per SM, in the same exact
// arithmetic as the multi-kernel path (the oracle's REF_KV8 | REF_EXACT mode),
// so both give the same bits.
//
// Weights stream continuously: every CTA owns a fixed slice of rows of each
// projection (QKV, O, gate/up pairs, down, then its share of the LM head in
// 32-row pieces). One thread keeps a 172 KB shared-memory ring filled with the
// upcoming slices by bulk copies, each slice together with everything its
// phase reads besides the activations (the slice's per-channel scales and
// biases, the RMSNorm gains), completing on one mbarrier per slice; slices are
// issued as soon as ring space frees, so the next layers' weights arrive while
// the current phase computes or waits. Phases are separated by grid barriers
// (an arrival counter in global memory, bounded spin):
//   A  every CTA: RMSNorm of x (exact sum of squares) -> limb planes in shared
//      memory; its QKV rows + bias -> qkv (pre-RoPE, bf16). Meanwhile warp 7
//      starts the bulk copies of this layer's KV8 history (short contexts)
//   B+C short contexts (<= 64 keys): every CTA computes the attention of all
//      14 heads itself from the prefetched history and the new key/value (RoPE,
//      KV8 quantise; CTA 0 appends them to the cache), then its O rows +
//      residual -> x. Longer contexts: B on CTAs 0 and 1 (one KV head each,
//      history read from the cache), a grid barrier, then C on every CTA
//   D  RMSNorm of x -> limbs; its gate/up pairs + SiLU*mul -> mid
//   E  mid -> limbs; its down rows + residual -> x
//   LM final RMSNorm -> limbs; its LM-head rows -> logits and its best (value,
//      index); after a last barrier CTA 0 picks the token (highest index on
//      ties, model_backend.py:113-114)
// Activations written by other CTAs of the launch are read through L2 only.
// Every wait is bounded: on timeout a code goes to the error flag and the CTA
// stops waiting (its results are then garbage, and the host reports the flag).
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"
#include "xlimbs.cuh"

namespace qb {

constexpr int D1_THREADS = 256;                  // compute threads (warps 0..7)
constexpr int D1_WARPS = D1_THREADS / 32;
constexpr int D1_BLOCK = D1_THREADS + 32;        // + warp 8: the ring producer
constexpr int D1_RING = 172 * 1024;
constexpr int D1_SEGS = 16;      // slices in flight at most (one mbarrier each)
constexpr int D1_LM_ROWS = 32;   // LM-head rows per slice
constexpr int D1_MAXROWS = 72;   // largest projection slice of one CTA (gate/up pairs)
constexpr int D1_SHORT = 64;     // contexts up to this many keys use the fused B+C phase
constexpr unsigned D1_BAR_STRIDE = 128;  // grid barriers per launch at most (97 short, 121 long)

constexpr int D1S_QLS = 4 * 64 + 16;  // q limb planes per head: 16-byte aligned, padded against bank conflicts

// long-context attention scratch (phase B on CTAs 0 and 1), inside the work area
constexpr int D1A_QF = 0;                              // float [7][64] q after RoPE
constexpr int D1A_QL = D1A_QF + 7 * 64 * 4;            // int8 [7][260] q limb planes (padded rows)
constexpr int D1A_NEW = D1A_QL + 7 * D1S_QLS;          // int8 [2][64] new k / v codes
constexpr int D1A_MISC = D1A_NEW + 128;                // qe[8] int, M[8], inv[8], s1[8], s2[8], F[8], new scales[2], vmax
constexpr int D1A_RED = D1A_MISC + 64 * 4;             // (unused: reductions use the shared red area)
constexpr int D1A_KS = D1A_RED + D1_WARPS * 8 * 8;     // float [maxkeys] K scales, V scales, S [7][maxkeys + 1]
constexpr int D1A_SS = QB_D1_MAX_KEYS + 1;             // score row stride (padded against bank conflicts)
constexpr int D1_LONG_BYTES = D1A_KS + 4 * (2 * QB_D1_MAX_KEYS + 7 * D1A_SS);

// short-context area (after the limb planes): prefetched history and scratch;
// every region starts on a 16-byte boundary (vector and bulk-copy accesses)
__host__ __device__ constexpr int d1_al16(int x) { return (x + 15) & ~15; }
constexpr int D1S_KC = 0;                                            // int8 [2][64 keys][64] K codes
constexpr int D1S_VC = d1_al16(D1S_KC + 2 * D1_SHORT * 64);          // int8 [2][64][64] V codes
constexpr int D1S_KS = d1_al16(D1S_VC + 2 * D1_SHORT * 64);          // float [2][64 + 8] K scales (16-byte aligned superset)
constexpr int D1S_VS = d1_al16(D1S_KS + 2 * (D1_SHORT + 8) * 4);     // float [2][64 + 8] V scales
constexpr int D1S_QL = d1_al16(D1S_VS + 2 * (D1_SHORT + 8) * 4);     // int8 [14][272] q limb planes
constexpr int D1S_WS = D1_SHORT + 2;                                  // softmax weights per head (+1 zero), 8-byte rows
constexpr int D1S_W = d1_al16(D1S_QL + 14 * D1S_QLS);                // u32 [14][66] softmax weights W
constexpr int D1S_CTX = d1_al16(D1S_W + 14 * D1S_WS * 4);            // bf16 [896] context
constexpr int D1S_MISC = d1_al16(D1S_CTX + QB_HID * 2);              // qe[16], nsc[4]
constexpr int D1_SHORT_BYTES = d1_al16(D1S_MISC + 32 * 4);
constexpr int D1_LIMB_BYTES = d1_al16(4 * QB_FFN + 16);
static_assert(D1S_QLS % 16 == 0 && D1_RING % 16 == 0, "16-byte aligned rows");

struct D1Smem {
    int ring, work, shortw, bars, segs, layers, red, accs, part, total;
};
__host__ __device__ constexpr D1Smem d1_smem() {
    D1Smem L{};
    L.ring = 0;
    L.work = L.ring + D1_RING;
    L.shortw = L.work + D1_LIMB_BYTES;
    const int work = D1_LIMB_BYTES + D1_SHORT_BYTES > D1_LONG_BYTES ? D1_LIMB_BYTES + D1_SHORT_BYTES : D1_LONG_BYTES;
    L.bars = d1_al16(L.work + work);
    L.segs = L.bars + (2 * D1_SEGS + 2) * 8;  // full / empty mbarriers per slot, then the KV-history one
    L.layers = L.segs + 512;                  // per slot: ring offset, side offsets
    L.red = d1_al16(L.layers + QB_NL * (int)sizeof(D1Layer));
    L.accs = L.red + D1_WARPS * 16 * 8;
    L.part = L.accs + D1_MAXROWS * 4;  // split-K partial sums [8 slices][16 rows][4 limbs] int32
    L.total = L.part + D1_WARPS * 16 * 4 * 4;
    return L;
}
// 227 KB per CTA, less 256 bytes for the static shared variables (128 used)
static_assert(d1_smem().total <= 232448 - 256, "shared memory of the persistent decode CTA");
static_assert(d1_smem().shortw % 16 == 0 && d1_smem().work % 16 == 0 && d1_smem().red % 16 == 0 &&
                  d1_smem().part % 16 == 0,
              "16-byte aligned regions");

// Barrier of the 256 compute threads (the producer warp never joins).
__device__ __forceinline__ void d1_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Two-way dot products of two unsigned 16-bit halves of a with two signed
// bytes of b (bytes 0, 1 for lo, bytes 2, 3 for hi), plus c.
__device__ __forceinline__ int dp2a_lo_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// [begin, end) of part c of n items split over g parts
__device__ __forceinline__ void d1_part(int n, int c, int g, int &b, int &e) {
    b = (int)((unsigned)(n * c) / (unsigned)g);  // n * (c + 1) < 2^31 for every n here
    e = (int)((unsigned)(n * (c + 1)) / (unsigned)g);
}

// One ring slice: up to four contiguous pieces placed back to back (each a
// multiple of 16 bytes); side data is copied as the 16-byte-aligned superset
// of its range and found at rel[i] + delta[i].
struct D1Seg {
    const uint8_t *src[4];
    uint32_t bytes[4], rel[4], delta[4];
    int n;
    uint32_t total;
};
__device__ __forceinline__ void d1_piece(D1Seg &g, const void *p, uint32_t len) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p), al = a & ~(uintptr_t)15;
    const uintptr_t end = (a + len + 15) & ~(uintptr_t)15;
    g.src[g.n] = reinterpret_cast<const uint8_t *>(al);
    g.bytes[g.n] = (uint32_t)(end - al);
    g.rel[g.n] = g.total;
    g.delta[g.n] = (uint32_t)(a - al);
    g.total += g.bytes[g.n];
    ++g.n;
}

// Slice s of this CTA: layer s / 4, phase s % 4 (QKV, O, gate/up, down), then
// the LM-head pieces. Piece 0 is always the weight rows, piece 1 their scales.
__device__ __forceinline__ bool d1_seg(const D1Args &a, const D1Layer *layers, int s, D1Seg &g) {
    const int c = blockIdx.x, G = gridDim.x;
    int b, e;
    g.n = 0;
    g.total = 0;
    if (s < 4 * QB_NL) {
        const D1Layer &W = layers[s >> 2];
        switch (s & 3) {
            case 0:
                d1_part(QB_QKV, c, G, b, e);
                d1_piece(g, W.qkv + (size_t)b * QB_HID, (e - b) * QB_HID);
                d1_piece(g, W.s_qkv + b, (e - b) * 4);
                d1_piece(g, W.bias + b, (e - b) * 2);
                d1_piece(g, W.g_attn, QB_HID * 2);
                break;
            case 1:
                d1_part(QB_HID, c, G, b, e);
                d1_piece(g, W.o + (size_t)b * QB_HID, (e - b) * QB_HID);
                d1_piece(g, W.s_o + b, (e - b) * 4);
                break;
            case 2:
                d1_part(QB_FFN, c, G, b, e);
                d1_piece(g, W.gu + (size_t)2 * b * QB_HID, 2 * (e - b) * QB_HID);
                d1_piece(g, W.s_gu + 2 * b, 2 * (e - b) * 4);
                d1_piece(g, W.g_ffn, QB_HID * 2);
                break;
            default:
                d1_part(QB_HID, c, G, b, e);
                d1_piece(g, W.d + (size_t)b * QB_FFN, (e - b) * QB_FFN);
                d1_piece(g, W.s_d + b, (e - b) * 4);
                break;
        }
        return true;
    }
    d1_part(QB_VOCAB, c, G, b, e);
    const int p = s - 4 * QB_NL, r0 = b + p * D1_LM_ROWS;
    if (r0 >= e) return false;
    const int nr = min(D1_LM_ROWS, e - r0);
    d1_piece(g, a.lmw + (size_t)r0 * QB_HID, nr * QB_HID);
    d1_piece(g, a.s_lm + r0, nr * 4);
    if (p == 0) d1_piece(g, a.g_final, QB_HID * 2);
    return true;
}

struct D1Ring {
    uint8_t *ring;
    uint64_t *full, *empty;  // per slot: data landed / all 8 compute warps done with it
    uint32_t *off;           // per slot: ring offset of the slice
    uint32_t *side;          // per slot: byte offsets (from the slice base) of pieces 1..3' data
    const D1Layer *layers;   // shared-memory copy
};

// The producer (lane 0 of warp 8): issues every slice of the launch in order,
// each as soon as its mbarrier slot and enough ring space are free, i.e. once
// the compute warps have released the older slices. Slices never wrap: one
// that does not fit before the end of the ring starts at offset 0.
__device__ void d1_produce(const D1Args &a, D1Ring &R) {
    uint32_t head = 0, tail = 0, vend[D1_SEGS];
    int oldest = 0;  // first slice not yet known to be released
    for (int s = 0;; ++s) {
        D1Seg g;
        if (!d1_seg(a, R.layers, s, g)) break;
        uint32_t v = head;
        if ((v % D1_RING) + g.total > (uint32_t)D1_RING) v += D1_RING - (v % D1_RING);
        while (oldest < s && (oldest <= s - D1_SEGS || v + g.total - tail > (uint32_t)D1_RING)) {
            if (!tc::mbar_wait(&R.empty[oldest % D1_SEGS], (uint32_t)(oldest / D1_SEGS) & 1u, a.err, 23, 1u << 24))
                return;
            tail = vend[oldest % D1_SEGS];
            ++oldest;
        }
        const int slot = s % D1_SEGS;
        R.off[slot] = v % D1_RING;
        for (int i = 1; i < 4; ++i) R.side[slot * 4 + i] = i < g.n ? g.rel[i] + g.delta[i] : 0u;
        vend[slot] = v + g.total;
        tc::mbar_arrive_expect_tx(&R.full[slot], g.total);
        for (int i = 0; i < g.n; ++i) tc::bulk_load(R.ring + v % D1_RING + g.rel[i], g.src[i], g.bytes[i], &R.full[slot]);
        head = v + g.total;
    }
}

// Slice s is complete in the ring (compute threads); returns its base, and in
// side[1..3] the offsets of its side pieces. The producer wrote the slot's
// offsets before its arrive on the slot's mbarrier (release), so they are
// visible once the wait has observed the phase (acquire).
__device__ __forceinline__ const uint8_t *d1_wait(const D1Args &a, D1Ring &R, int s, uint32_t (&side)[4], bool &ok) {
    const int slot = s % D1_SEGS;
    if (ok) ok = tc::mbar_wait(&R.full[slot], (uint32_t)(s / D1_SEGS) & 1u, a.err, 21);
#pragma unroll
    for (int i = 0; i < 4; ++i) side[i] = R.side[slot * 4 + i];
    return R.ring + R.off[slot];
}

// This warp is done with slice s (every warp calls it once per slice).
__device__ __forceinline__ void d1_done(D1Ring &R, int s) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) tc::mbar_arrive(&R.empty[s % D1_SEGS]);
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier number k (1-based) of the launch: one release arrival per CTA
// (its writes become visible first), thread 0 polls the counter with acquire
// loads, the CTA proceeds together. After `limit` polls the wait gives up
// with code 20 in the error flag; `extra` raises the target (a host-set test
// switch makes the last barrier unreachable that way, see D1Args).
__device__ __forceinline__ void d1_grid_sync(const D1Args &a, unsigned base, unsigned k, bool &ok, unsigned extra = 0,
                                             uint32_t limit = 1u << 24) {
    __shared__ int s_ok;
    d1_sync();
    if (threadIdx.x == 0) {
        // release: the CTA's writes (ordered before this thread by the CTA barrier) become visible first
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
        bool good = ok;
        if (good) {
            const unsigned target = base + k * gridDim.x + extra;
            uint32_t spins = 0;
            while ((int)(ld_acquire_gpu(a.bar) - target) < 0) {  // wrap-safe
                if (++spins > limit) {
                    atomicExch(a.err, 20u);
                    good = false;
                    break;
                }
            }
        }
        s_ok = good;
    }
    d1_sync();
    ok = s_ok != 0;
}

// The four int8 limb planes xl[4][896] of one 896-wide row and its exponent,
// with the CTA's 256 threads at once (thread t < 224 owns values 4t..4t+3);
// with NORM the row is RMSNormed first (exact sum of squares on the 21-bit
// grid, model_backend.py:69-71). The same values as load_x_limbs, with three
// CTA-wide reductions instead of one warp's serial chain. CG: x was written by
// other CTAs of this launch (read through L2); otherwise x may be shared memory.
template <bool NORM, bool CG>
__device__ void d1_row896(const uint16_t *x, const uint16_t *gamma, float eps, int8_t *xl, int *ex, uint8_t *red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float *r0 = reinterpret_cast<float *>(red), *r2 = r0 + 16;
    long long *r1 = reinterpret_cast<long long *>(red + 128);
    const bool act = tid < QB_HID / 4;
    uint2 xv = make_uint2(0u, 0u);
    if (act) {
        const uint2 *p = reinterpret_cast<const uint2 *>(x) + tid;
        if constexpr (CG)
            xv = __ldcg(p);
        else
            xv = *p;
    }
    float v[4] = {bflo(xv.x), bfhi(xv.x), bflo(xv.y), bfhi(xv.y)};
    if constexpr (NORM) {
        float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        m = warp_max(m);
        if (lane == 0) r0[warp] = m;
        d1_sync();
        m = r0[0];
#pragma unroll
        for (int w = 1; w < D1_WARPS; ++w) m = fmaxf(m, r0[w]);
        const int e0 = row_exponent(m);
        long long s2 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const long long q = __float2int_rn(align21(v[i], e0));
            s2 += q * q;
        }
        s2 = warp_sum_ll(s2);
        if (lane == 0) r1[warp] = s2;
        d1_sync();
        s2 = r1[0];
#pragma unroll
        for (int w = 1; w < D1_WARPS; ++w) s2 += r1[w];
        const float ss = ldexpf(__ll2float_rn(s2), 2 * e0 - 40);
        const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)QB_HID), eps)));
        uint2 gv = make_uint2(0u, 0u);
        if (act) gv = reinterpret_cast<const uint2 *>(gamma)[tid];
        const float gg[4] = {bflo(gv.x), bfhi(gv.x), bflo(gv.y), bfhi(gv.y)};
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = rbf(rbf(v[i] * rs) * gg[i]);
    }
    float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    m = warp_max(m);
    if (lane == 0) r2[warp] = m;
    d1_sync();
    m = r2[0];
#pragma unroll
    for (int w = 1; w < D1_WARPS; ++w) m = fmaxf(m, r2[w]);
    const int e = row_exponent(m);
    if (act) {
        int lv[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) limbs4(align28_int(v[i], e), lv[i]);
#pragma unroll
        for (int l = 0; l < 4; ++l)
            reinterpret_cast<uint32_t *>(xl + l * QB_HID)[tid] = ((uint32_t)lv[0][l] & 0xffu) |
                                                                  (((uint32_t)lv[1][l] & 0xffu) << 8) |
                                                                  (((uint32_t)lv[2][l] & 0xffu) << 16) |
                                                                  ((uint32_t)lv[3][l] << 24);
    }
    if (tid == 0) ex[0] = e;
    d1_sync();
}

// acc[r] = RN32(sum_k X[k] * W[r][k]) * 2^(ex - 26) for the nrows rows of a
// ring slice (row-major, K bytes each): warp w takes rows w*RW .. w*RW+RW-1
// (one pass), lanes split the rows into 16-byte chunks, dp4a against the four
// limb planes; lane 0 of the warp then runs epi(r0, nr, acc) on its rows.
template <int K, int RW, class Epi>
__device__ __forceinline__ void d1_dot(const int8_t *w, int nrows, const int8_t *xl, int ex, Epi epi) {
    constexpr int NCH = K / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = warp * RW, nr = min(RW, nrows - r0);
    if (nr <= 0) return;
    int d[RW][4];
#pragma unroll
    for (int r = 0; r < RW; ++r) d[r][0] = d[r][1] = d[r][2] = d[r][3] = 0;
    for (int ch = lane; ch < NCH; ch += 32) {
        uint4 xw[4];
#pragma unroll
        for (int l = 0; l < 4; ++l) xw[l] = *reinterpret_cast<const uint4 *>(xl + l * K + ch * 16);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            if (r >= nr) break;
            const uint4 wv = *reinterpret_cast<const uint4 *>(w + (size_t)(r0 + r) * K + ch * 16);
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                int t = d[r][l];
                t = __dp4a((int)wv.x, (int)xw[l].x, t);
                t = __dp4a((int)wv.y, (int)xw[l].y, t);
                t = __dp4a((int)wv.z, (int)xw[l].z, t);
                t = __dp4a((int)wv.w, (int)xw[l].w, t);
                d[r][l] = t;
            }
        }
    }
    float acc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        long long v = (long long)d[r][0] + (long long)d[r][1] * 128ll + (long long)d[r][2] * 16384ll +
                      (long long)d[r][3] * 2097152ll;
        acc[r] = unalign28(warp_sum_ll(v), ex);
    }
    if (lane == 0) epi(r0, nr, acc);
}

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Tensor-core form of the exact projection dot products: one m-tile of 16
// weight rows [row0, row0 + 16) (rows >= nrows read as 0) against the four
// limb planes (the N columns 0..3 of m16n8k32, s8 x s8 -> s32) over the 64-k
// blocks [kb0, kb1). Thread (gid, tig) loads 16 bytes of rows gid and gid + 8
// at k = 64 kb + 16 tig; MMA step s uses bytes 8s..8s+7 of them, and the limb
// words at the same k, so both operands are plain words of consecutive k.
// c[0..3] = the m16n8 accumulator fragment (rows gid | gid + 8, limbs 2 tig,
// 2 tig + 1; tig >= 2 holds the unused columns).
template <int K>
__device__ __forceinline__ void d1_mma_tile(const int8_t *w, int nrows, int row0, int kb0, int kb1, const int8_t *xl,
                                            int (&c)[4]) {
    const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int ra = row0 + gid, rb = ra + 8;
    const int8_t *pa = w + (size_t)ra * K + 16 * tig, *pb = w + (size_t)rb * K + 16 * tig;
    const int8_t *px = xl + (size_t)(gid & 3) * K + 16 * tig;
    c[0] = c[1] = c[2] = c[3] = 0;
    for (int kb = kb0; kb < kb1; ++kb) {
        const uint4 u = ra < nrows ? *reinterpret_cast<const uint4 *>(pa + 64 * kb) : make_uint4(0u, 0u, 0u, 0u);
        const uint4 v = rb < nrows ? *reinterpret_cast<const uint4 *>(pb + 64 * kb) : make_uint4(0u, 0u, 0u, 0u);
        const uint4 x = gid < 4 ? *reinterpret_cast<const uint4 *>(px + 64 * kb) : make_uint4(0u, 0u, 0u, 0u);
        mma_s8_16832(c, u.x, v.x, u.y, v.y, x.x, x.y);
        mma_s8_16832(c, u.z, v.z, u.w, v.w, x.z, x.w);
    }
}

// Exact sums of rows gid and gid + 8 of a fragment, on the lanes with tig == 0
// (limbs 2 and 3 come from the tig == 1 lane).
__device__ __forceinline__ void d1_fold(const int (&c)[4], long long &lo, long long &hi) {
    const int c0 = __shfl_down_sync(0xffffffffu, c[0], 1), c1 = __shfl_down_sync(0xffffffffu, c[1], 1);
    const int c2 = __shfl_down_sync(0xffffffffu, c[2], 1), c3 = __shfl_down_sync(0xffffffffu, c[3], 1);
    lo = (long long)c[0] + (long long)c[1] * 128ll + (long long)c0 * 16384ll + (long long)c1 * 2097152ll;
    hi = (long long)c[2] + (long long)c[3] * 128ll + (long long)c2 * 16384ll + (long long)c3 * 2097152ll;
}

// Rows [0, nrows) (nrows <= 16) of a slice, K split over the 8 compute warps
// into `part`; after the compute barrier, thread r < nrows runs epi(r, acc).
template <int K, class Epi>
__device__ __forceinline__ void d1_mma_rows16(const int8_t *w, int nrows, const int8_t *xl, int ex, int *part, Epi epi) {
    constexpr int NB = K / 64;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int kb0 = NB * warp / D1_WARPS, kb1 = NB * (warp + 1) / D1_WARPS;
    int c[4];
    d1_mma_tile<K>(w, nrows, 0, kb0, kb1, xl, c);
    if (tig < 2) {
        int *p = part + warp * 64;
        p[gid * 4 + 2 * tig] = c[0];
        p[gid * 4 + 2 * tig + 1] = c[1];
        p[(gid + 8) * 4 + 2 * tig] = c[2];
        p[(gid + 8) * 4 + 2 * tig + 1] = c[3];
    }
    d1_sync();
    if (threadIdx.x < nrows) {
        const int r = threadIdx.x;
        int l4[4] = {0, 0, 0, 0};
#pragma unroll
        for (int sl = 0; sl < D1_WARPS; ++sl)
#pragma unroll
            for (int l = 0; l < 4; ++l) l4[l] += part[sl * 64 + r * 4 + l];
        const long long v = (long long)l4[0] + (long long)l4[1] * 128ll + (long long)l4[2] * 16384ll +
                            (long long)l4[3] * 2097152ll;
        epi(r, unalign28(v, ex));
    }
}

// The four int8 limb planes of one 4864-wide row (plain conversion), every
// compute thread on 16-byte pieces; the maximum meets in shared memory.
__device__ void d1_row4864(const uint16_t *x, int8_t *xl, int *ex, uint8_t *red) {
    constexpr int K = QB_FFN, NPC = K / 8, NP = (NPC + D1_THREADS - 1) / D1_THREADS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float *r0 = reinterpret_cast<float *>(red);
    uint4 xv[NP];
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        const int p = tid + D1_THREADS * j;
        xv[j] = p < NPC ? __ldcg(reinterpret_cast<const uint4 *>(x) + p) : make_uint4(0u, 0u, 0u, 0u);
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        const uint32_t w[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
#pragma unroll
        for (int t = 0; t < 4; ++t) amax = fmaxf(amax, fmaxf(fabsf(bflo(w[t])), fabsf(bfhi(w[t]))));
    }
    amax = warp_max(amax);
    if (lane == 0) r0[warp] = amax;
    d1_sync();
    amax = r0[0];
#pragma unroll
    for (int w2 = 1; w2 < D1_WARPS; ++w2) amax = fmaxf(amax, r0[w2]);
    const int e = row_exponent(amax);
#pragma unroll
    for (int j = 0; j < NP; ++j) {
        const int p = tid + D1_THREADS * j;
        if (p >= NPC) continue;
        const uint32_t w[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
        uint32_t pk[4][2];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            int la[4], lb[4];
            limbs4(align28_int(bflo(w[t]), e), la);
            limbs4(align28_int(bfhi(w[t]), e), lb);
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const uint32_t two = limb_bytes(la, lb, l);
                if (t & 1)
                    pk[l][t >> 1] |= two << 16;
                else
                    pk[l][t >> 1] = two;
            }
        }
#pragma unroll
        for (int l = 0; l < 4; ++l)
            *reinterpret_cast<uint2 *>(xl + l * K + 8 * p) = make_uint2(pk[l][0], pk[l][1]);
    }
    if (tid == 0) ex[0] = e;
    d1_sync();
}

// Phase B for KV head g: see the file comment. L = pos + 1 keys.
__device__ void d1_attention(const D1Args &a, int layer, int g, uint32_t slot, uint32_t pos, uint8_t *work,
                             uint8_t *red8) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int L = (int)pos + 1;
    float *qf = reinterpret_cast<float *>(work + D1A_QF);
    int8_t *ql = reinterpret_cast<int8_t *>(work + D1A_QL);
    int8_t *knew = reinterpret_cast<int8_t *>(work + D1A_NEW), *vnew = knew + 64;
    int *qe = reinterpret_cast<int *>(work + D1A_MISC);
    float *M = reinterpret_cast<float *>(work + D1A_MISC) + 8, *inv = M + 8, *s1 = M + 16, *s2 = M + 24;
    int *F = reinterpret_cast<int *>(M + 32);
    float *nsc = M + 40;  // new k, v scales, [2] = vmax
    long long *red = reinterpret_cast<long long *>(red8);
    float *kss = reinterpret_cast<float *>(work + D1A_KS);
    float *vss = kss + QB_D1_MAX_KEYS;
    float *S = vss + QB_D1_MAX_KEYS;  // [7][maxkeys]: scores, then E, then W (as u32)
    const size_t lc = (size_t)a.codes_per_layer * layer, ls = (size_t)a.scales_per_layer * layer;
    const size_t base = ((size_t)slot * 2 + g) * a.cap;  // key 0 of this (slot, head)
    const int8_t *kc = a.kc + lc + base * 64, *vc = a.vc + lc + base * 64;
    const float *ks = a.ks + ls + base, *vs = a.vs + ls + base;
    const uint16_t *qkv = a.qkv;

    // RoPE (model_backend.py:73-78) of q heads 7g..7g+6 (warps 0..6) and of
    // k; KV8 quantise-append of k and v (warp 7)
    const float *cs = a.rope + (size_t)pos * 64;
    const float c = cs[lane & 31], sn = cs[32 + (lane & 31)];
    if (warp < 7) {
        const uint16_t *qp = qkv + (size_t)(7 * g + warp) * 64;
        const float lo = bf2f(__ldcg(qp + lane)), hi = bf2f(__ldcg(qp + lane + 32));
        const float nlo = rbf(__fadd_rn(__fmul_rn(lo, c), __fmul_rn(-hi, sn)));
        const float nhi = rbf(__fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, sn)));
        qf[warp * 64 + lane] = nlo;
        qf[warp * 64 + lane + 32] = nhi;
        // 28-bit alignment of the head, four limb planes
        const int e = row_exponent(warp_max(fmaxf(fabsf(nlo), fabsf(nhi))));
        int l0[4], l1[4];
        limbs4(align28_int(nlo, e), l0);
        limbs4(align28_int(nhi, e), l1);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            ql[warp * D1S_QLS + l * 64 + lane] = (int8_t)l0[l];
            ql[warp * D1S_QLS + l * 64 + lane + 32] = (int8_t)l1[l];
        }
        if (lane == 0) qe[warp] = e;
    } else {
#pragma unroll
        for (int isv = 0; isv < 2; ++isv) {
            const uint16_t *p = qkv + QB_HID + isv * 128 + g * 64;
            float lo = bf2f(__ldcg(p + lane)), hi = bf2f(__ldcg(p + lane + 32));
            if (!isv) {
                const float nlo = rbf(__fadd_rn(__fmul_rn(lo, c), __fmul_rn(-hi, sn)));
                const float nhi = rbf(__fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, sn)));
                lo = nlo;
                hi = nhi;
            }
            const float amax = warp_max(fmaxf(fabsf(lo), fabsf(hi)));
            const float s = __fdiv_rn(amax, 127.0f);
            int clo = 0, chi = 0;
            if (s > 0.f) {
                clo = (int)fminf(fmaxf(rintf(__fdiv_rn(lo, s)), -127.f), 127.f);
                chi = (int)fminf(fmaxf(rintf(__fdiv_rn(hi, s)), -127.f), 127.f);
            }
            int8_t *gc = const_cast<int8_t *>(isv ? vc : kc) + (size_t)pos * 64;
            int8_t *nc = isv ? vnew : knew;
            gc[lane] = (int8_t)clo;
            gc[lane + 32] = (int8_t)chi;
            nc[lane] = (int8_t)clo;
            nc[lane + 32] = (int8_t)chi;
            if (lane == 0) {
                const_cast<float *>(isv ? vs : ks)[pos] = s;
                nsc[isv] = s;
            }
        }
    }
    for (int t = tid; t < L - 1; t += D1_THREADS) {
        kss[t] = __ldg(ks + t);
        vss[t] = __ldg(vs + t);
    }
    d1_sync();
    if (tid == 0) {
        kss[L - 1] = nsc[0];
        vss[L - 1] = nsc[1];
    }
    d1_sync();

    // scores: thread (key t = tid/8 + 32 i, head h = tid % 8)
    const int h = tid & 7, tl = tid >> 3;
    float mloc = -INFINITY, vloc = 0.f;
    for (int t = tl; t < L; t += D1_THREADS / 8) {
        vloc = fmaxf(vloc, vss[t]);
        if (h == 7) continue;
        const uint32_t *kr = reinterpret_cast<const uint32_t *>(t == L - 1 ? knew : kc + (size_t)t * 64);
        const uint32_t *qr = reinterpret_cast<const uint32_t *>(ql + h * D1S_QLS);
        int d4[4] = {0, 0, 0, 0};
#pragma unroll
        for (int wi = 0; wi < 16; ++wi) {
            const int kw = (int)(t == L - 1 ? kr[wi] : __ldg(kr + wi));
#pragma unroll
            for (int l = 0; l < 4; ++l) d4[l] = __dp4a(kw, (int)qr[l * 16 + wi], d4[l]);
        }
        const long long dot = (long long)d4[0] + (long long)d4[1] * 128ll + (long long)d4[2] * 16384ll +
                              (long long)d4[3] * 2097152ll;
        const float sc = rbf(__fmul_rn(unalign28(dot, qe[h]), kss[t]) * 0.125f);
        S[h * D1A_SS + t] = sc;
        mloc = fmaxf(mloc, sc);
    }
    // per-head max and the largest V scale
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 8));
    mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 16));
    vloc = warp_max(vloc);
    float *redf = reinterpret_cast<float *>(red);
    if (lane < 8) redf[warp * 8 + lane] = (lane == 7) ? vloc : mloc;
    d1_sync();
    if (tid < 8) {
        float m = redf[tid];
        for (int w = 1; w < D1_WARPS; ++w) m = fmaxf(m, redf[w * 8 + tid]);
        if (tid < 7)
            M[tid] = m;
        else
            nsc[2] = m;
    }
    d1_sync();
    // E = qexp(S - max) in place, exact sums
    long long z = 0;
    if (h < 7)
        for (int t = tl; t < L; t += D1_THREADS / 8) {
            const float e = qexp(__fsub_rn(S[h * D1A_SS + t], M[h]));
            S[h * D1A_SS + t] = e;
            z += rint_2p40(e);
        }
    z += __shfl_xor_sync(0xffffffffu, z, 8);
    z += __shfl_xor_sync(0xffffffffu, z, 16);
    if (lane < 8) red[warp * 8 + lane] = z;
    d1_sync();
    if (tid < 7) {
        long long zt = 0;
        for (int w = 0; w < D1_WARPS; ++w) zt += red[w * 8 + tid];
        const float iv = __fdiv_rn(1.0f, __fmul_rn(__ll2float_rn(zt), 0x1p-40f));
        const int f = row_exponent(__fmul_rn(rbf(iv), nsc[2]));
        const int sh = 26 - f, sh1 = min(sh, 127);
        inv[tid] = iv;
        F[tid] = f;
        s1[tid] = pow2i(sh1);
        s2[tid] = pow2i(sh - sh1);
    }
    d1_sync();
    // W = rint(RN32(P * vscale) * 2^(26-F)), P = bf16(E / Z)
    if (h < 7)
        for (int t = tl; t < L; t += D1_THREADS / 8) {
            const float w = __fmul_rn(rbf(__fmul_rn(S[h * D1A_SS + t], inv[h])), vss[t]);
            reinterpret_cast<uint32_t *>(S)[h * D1A_SS + t] =
                __float2uint_rn(__fmul_rn(__fmul_rn(w, s1[h]), s2[h]));
        }
    d1_sync();
    // context: thread (half, head, 4 dims), keys t = half, half + 2, ...
    long long acc[4] = {0, 0, 0, 0};
    const int half = tid / 112, rem = tid % 112, hh = rem >> 4, d4 = rem & 15;
    if (tid < 224) {
        const uint32_t *W = reinterpret_cast<const uint32_t *>(S) + hh * D1A_SS;
        for (int t = half; t < L; t += 2) {
            const uint32_t cw = t == L - 1 ? reinterpret_cast<const uint32_t *>(vnew)[d4]
                                           : __ldg(reinterpret_cast<const uint32_t *>(vc + (size_t)t * 64) + d4);
            const long long wt = (long long)W[t];
            acc[0] += wt * (int)(int8_t)(cw & 0xffu);
            acc[1] += wt * (int)(int8_t)((cw >> 8) & 0xffu);
            acc[2] += wt * (int)(int8_t)((cw >> 16) & 0xffu);
            acc[3] += wt * (int)(int8_t)(cw >> 24);
        }
    }
    long long *part = reinterpret_cast<long long *>(kss);  // kss/vss are no longer needed
    d1_sync();
    if (tid >= 112 && tid < 224)
#pragma unroll
        for (int i = 0; i < 4; ++i) part[rem * 4 + i] = acc[i];
    d1_sync();
    if (tid < 112) {
        uint16_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = f2bf(unalign28(acc[i] + part[rem * 4 + i], F[hh]));
        uint2 pk;
        pk.x = (uint32_t)o[0] | ((uint32_t)o[1] << 16);
        pk.y = (uint32_t)o[2] | ((uint32_t)o[3] << 16);
        *reinterpret_cast<uint2 *>(a.ctx + (size_t)(7 * g + hh) * 64 + 4 * d4) = pk;
    }
}


// KV8 history of this layer for the fused short-context phase: K and V codes
// of keys [0, pos) of both KV heads and their scales, into the short area
// (one thread; completes on kvbar).
__device__ void d1_issue_history(const D1Args &a, int layer, uint32_t slot, uint32_t pos, uint8_t *sw,
                                 uint64_t *kvbar) {
    uint32_t total = 0;
    const uint8_t *src[8];
    uint32_t bytes[8], dst[8];
    int n = 0;
    const size_t lc = (size_t)a.codes_per_layer * layer, ls = (size_t)a.scales_per_layer * layer;
    for (int g = 0; g < QB_KVH && pos > 0; ++g) {
        const size_t base = ((size_t)slot * 2 + g) * a.cap;
        src[n] = reinterpret_cast<const uint8_t *>(a.kc + lc + base * 64);
        bytes[n] = pos * 64;
        dst[n++] = D1S_KC + g * D1_SHORT * 64;
        src[n] = reinterpret_cast<const uint8_t *>(a.vc + lc + base * 64);
        bytes[n] = pos * 64;
        dst[n++] = D1S_VC + g * D1_SHORT * 64;
        for (int isv = 0; isv < 2; ++isv) {
            const uintptr_t p = reinterpret_cast<uintptr_t>((isv ? a.vs : a.ks) + ls + base);
            const uintptr_t al = p & ~(uintptr_t)15, end = (p + 4 * pos + 15) & ~(uintptr_t)15;
            src[n] = reinterpret_cast<const uint8_t *>(al);
            bytes[n] = (uint32_t)(end - al);
            dst[n++] = (isv ? D1S_VS : D1S_KS) + g * (D1_SHORT + 8) * 4;
        }
    }
    for (int i = 0; i < n; ++i) total += bytes[i];
    tc::mbar_arrive_expect_tx(kvbar, total);
    for (int i = 0; i < n; ++i) tc::bulk_load(sw + dst[i], src[i], bytes[i], kvbar);
}

// Fused short-context attention (every CTA, all 14 heads): see the file
// comment; leaves ctx (bf16 [896]) in shared memory. Every step runs on
// half-warps (16 lanes): the 18 head vectors of this step's q | k | v, then
// one half-warp per query head for the scores, the softmax and the context,
// with one CTA barrier between the two and one at the end. The new key and
// value go into row pos of the history area, next to the bulk-copied rows
// [0, pos), so the loops over the keys read one layout.
__device__ void d1_attention_short(const D1Args &a, int layer, uint32_t slot, uint32_t pos, uint8_t *sw,
                                   uint64_t *kvbar, bool &ok) {
    const int tid = threadIdx.x, warp = tid >> 5, hl = tid & 15;
    const int L = (int)pos + 1;
    int8_t *ql = reinterpret_cast<int8_t *>(sw + D1S_QL);
    int8_t *kc = reinterpret_cast<int8_t *>(sw + D1S_KC), *vc = reinterpret_cast<int8_t *>(sw + D1S_VC);
    uint16_t *ctx = reinterpret_cast<uint16_t *>(sw + D1S_CTX);
    int *qe = reinterpret_cast<int *>(sw + D1S_MISC);
    float *nsc = reinterpret_cast<float *>(qe + 16);  // new scales [k|v][g]
    // 18 head vectors: q heads 0..13, k heads (14, 15), v heads (16, 17); lane
    // hl of a half-warp holds dims 2 hl, 2 hl + 1 and their RoPE partners
    // 2 hl + 32, 2 hl + 33 (model_backend.py:73-78)
    const float2 cs = reinterpret_cast<const float2 *>(a.rope + (size_t)pos * 64)[hl];
    const float2 sn = reinterpret_cast<const float2 *>(a.rope + (size_t)pos * 64 + 32)[hl];
    for (int hv = tid >> 4; hv < 18; hv += 16) {
        const uint32_t plo = __ldcg(reinterpret_cast<const uint32_t *>(a.qkv + hv * 64) + hl);
        const uint32_t phi = __ldcg(reinterpret_cast<const uint32_t *>(a.qkv + hv * 64 + 32) + hl);
        float v[4] = {bflo(plo), bfhi(plo), bflo(phi), bfhi(phi)};  // dims 2hl, 2hl+1, 2hl+32, 2hl+33
        if (hv < 16) {
            const float c2[2] = {cs.x, cs.y}, s2[2] = {sn.x, sn.y};
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float lo = v[i], hi = v[2 + i];
                v[i] = rbf(__fadd_rn(__fmul_rn(lo, c2[i]), __fmul_rn(-hi, s2[i])));
                v[2 + i] = rbf(__fadd_rn(__fmul_rn(hi, c2[i]), __fmul_rn(lo, s2[i])));
            }
        }
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
        for (int o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (hv < QB_QH) {
            const int e = row_exponent(amax);
            int lm[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) limbs4(align28_int(v[i], e), lm[i]);
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                uint16_t *row = reinterpret_cast<uint16_t *>(ql + hv * D1S_QLS + l * 64);
                row[hl] = (uint16_t)((lm[0][l] & 0xff) | ((lm[1][l] & 0xff) << 8));
                row[16 + hl] = (uint16_t)((lm[2][l] & 0xff) | ((lm[3][l] & 0xff) << 8));
            }
            if (hl == 0) qe[hv] = e;
        } else {
            const int isv = hv >= 16, g = (hv - 14) & 1;
            const float sc = __fdiv_rn(amax, 127.0f);
            int cd[4] = {0, 0, 0, 0};
            if (sc > 0.f)
#pragma unroll
                for (int i = 0; i < 4; ++i) cd[i] = (int)fminf(fmaxf(rintf(__fdiv_rn(v[i], sc)), -127.f), 127.f);
            const uint16_t wlo = (uint16_t)((cd[0] & 0xff) | ((cd[1] & 0xff) << 8));
            const uint16_t whi = (uint16_t)((cd[2] & 0xff) | ((cd[3] & 0xff) << 8));
            uint16_t *row = reinterpret_cast<uint16_t *>((isv ? vc : kc) + (g * D1_SHORT + pos) * 64);
            row[hl] = wlo;
            row[16 + hl] = whi;
            if (hl == 0) nsc[isv * 2 + g] = sc;
            if (blockIdx.x == 0) {  // the one writer of the cache entry
                const size_t base = ((size_t)slot * 2 + g) * a.cap + pos;
                uint16_t *gc =
                    reinterpret_cast<uint16_t *>((isv ? a.vc : a.kc) + (size_t)a.codes_per_layer * layer + base * 64);
                gc[hl] = wlo;
                gc[16 + hl] = whi;
                if (hl == 0) (isv ? a.vs : a.ks)[(size_t)a.scales_per_layer * layer + base] = sc;
            }
        }
    }
    if (ok) ok = tc::mbar_wait(kvbar, (uint32_t)layer & 1u, a.err, 22);
    d1_sync();
    // scales of the history keys (inside the aligned superset copies)
    const float *ksh[2], *vsh[2];
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
        const size_t o = (size_t)a.scales_per_layer * layer + ((size_t)slot * 2 + gg) * a.cap;
        ksh[gg] = reinterpret_cast<const float *>(sw + D1S_KS + gg * (D1_SHORT + 8) * 4 +
                                                  (reinterpret_cast<uintptr_t>(a.ks + o) & 15));
        vsh[gg] = reinterpret_cast<const float *>(sw + D1S_VS + gg * (D1_SHORT + 8) * 4 +
                                                  (reinterpret_cast<uintptr_t>(a.vs + o) & 15));
    }
    // one half-warp per query head (warps 0..6): lane hl takes keys hl, hl + 16,
    // hl + 32, hl + 48 for the scores and the softmax and dims 4 hl .. 4 hl + 3
    // for the context
    if (warp < QB_QH / 2) {
        const int h = tid >> 4, g = h / 7;
        const uint4 *qr = reinterpret_cast<const uint4 *>(ql + h * D1S_QLS);
        uint32_t *W = reinterpret_cast<uint32_t *>(sw + D1S_W) + h * D1S_WS;
        const float knew = nsc[g], vnew = nsc[2 + g];
        float sc[4], vsj[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int t = hl + 16 * j;
            sc[j] = -INFINITY;
            vsj[j] = 0.f;
            if (t < L) {
                const uint4 *kr = reinterpret_cast<const uint4 *>(kc + (g * D1_SHORT + t) * 64);
                int d4[4] = {0, 0, 0, 0};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int w4 = (i + (hl >> 1)) & 3;  // 16-byte chunk order rotated by lane: no bank conflicts
                    const uint4 k4 = kr[w4];
#pragma unroll
                    for (int l = 0; l < 4; ++l) {
                        const uint4 q4 = qr[l * 4 + w4];
                        d4[l] = __dp4a((int)k4.x, (int)q4.x, d4[l]);
                        d4[l] = __dp4a((int)k4.y, (int)q4.y, d4[l]);
                        d4[l] = __dp4a((int)k4.z, (int)q4.z, d4[l]);
                        d4[l] = __dp4a((int)k4.w, (int)q4.w, d4[l]);
                    }
                }
                const long long dot = (long long)d4[0] + (long long)d4[1] * 128ll + (long long)d4[2] * 16384ll +
                                      (long long)d4[3] * 2097152ll;
                sc[j] = rbf(__fmul_rn(unalign28(dot, qe[h]), t == L - 1 ? knew : ksh[g][t]) * 0.125f);
                vsj[j] = t == L - 1 ? vnew : vsh[g][t];
            }
        }
        float M = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
        float vmax = fmaxf(fmaxf(vsj[0], vsj[1]), fmaxf(vsj[2], vsj[3]));
#pragma unroll
        for (int o = 8; o; o >>= 1) {
            M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
        }
        // E = qexp(S - max), exact sum
        float e[4];
        long long z = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            e[j] = hl + 16 * j < L ? qexp(__fsub_rn(sc[j], M)) : 0.f;
            z += rint_2p40(e[j]);
        }
#pragma unroll
        for (int o = 8; o; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        const float iv = __fdiv_rn(1.0f, __fmul_rn(__ll2float_rn(z), 0x1p-40f));
        const int f = row_exponent(__fmul_rn(rbf(iv), vmax));
        const int sh = 26 - f, sh1 = min(sh, 127);
        const float f1 = pow2i(sh1), f2 = pow2i(sh - sh1);
        // W = rint(RN32(P * vscale) * 2^(26-F)), P = bf16(E / Z) <= bf16(1 / Z), so
        // RN32(P * vscale) < 2^(F+1) and W <= 2^27
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (hl + 16 * j < L)
                W[hl + 16 * j] = __float2uint_rn(__fmul_rn(__fmul_rn(__fmul_rn(rbf(__fmul_rn(e[j], iv)), vsj[j]), f1), f2));
        if (hl == 0 && (L & 1)) W[L] = 0u;  // the odd key's partner in the pairs below
        __syncwarp();
        // context: exact sum over the keys of W times the V codes, two keys per
        // dp2a (W's 16-bit halves, unsigned, times the two keys' codes of one
        // dim, signed); every partial sum is exact in int32 (64 x 65535 x 127 < 2^30)
        int lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
        const uint32_t *vr = reinterpret_cast<const uint32_t *>(vc + g * D1_SHORT * 64) + hl;
#pragma unroll 2
        for (int t = 0; t < L; t += 2) {
            const uint2 w2 = *reinterpret_cast<const uint2 *>(W + t);
            const uint32_t wl = __byte_perm(w2.x, w2.y, 0x5410u), wh = __byte_perm(w2.x, w2.y, 0x7632u);
            const uint32_t v0 = vr[t * 16], v1 = vr[(t + 1) * 16];
            const uint32_t p01 = __byte_perm(v0, v1, 0x5140u), p23 = __byte_perm(v0, v1, 0x7362u);
            lo[0] = dp2a_lo_us(wl, p01, lo[0]);
            hi[0] = dp2a_lo_us(wh, p01, hi[0]);
            lo[1] = dp2a_hi_us(wl, p01, lo[1]);
            hi[1] = dp2a_hi_us(wh, p01, hi[1]);
            lo[2] = dp2a_lo_us(wl, p23, lo[2]);
            hi[2] = dp2a_lo_us(wh, p23, hi[2]);
            lo[3] = dp2a_hi_us(wl, p23, lo[3]);
            hi[3] = dp2a_hi_us(wh, p23, hi[3]);
        }
        long long c[4];
#pragma unroll
        for (int d = 0; d < 4; ++d) c[d] = (long long)lo[d] + (long long)hi[d] * 65536ll;
        uint2 pk;
        pk.x = (uint32_t)f2bf(unalign28(c[0], f)) | ((uint32_t)f2bf(unalign28(c[1], f)) << 16);
        pk.y = (uint32_t)f2bf(unalign28(c[2], f)) | ((uint32_t)f2bf(unalign28(c[3], f)) << 16);
        reinterpret_cast<uint2 *>(ctx + h * 64)[hl] = pk;
    }
    d1_sync();
}

__global__ void __launch_bounds__(D1_BLOCK, 1) decode1_kernel(D1Args a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const D1Smem Ls = d1_smem();
    D1Ring R;
    R.ring = sm + Ls.ring;
    R.full = reinterpret_cast<uint64_t *>(sm + Ls.bars);
    R.empty = R.full + D1_SEGS;
    uint64_t *kvbar = R.empty + D1_SEGS;
    R.off = reinterpret_cast<uint32_t *>(sm + Ls.segs);
    R.side = R.off + D1_SEGS;
    D1Layer *lay = reinterpret_cast<D1Layer *>(sm + Ls.layers);
    R.layers = lay;
    uint8_t *work = sm + Ls.work, *sw = sm + Ls.shortw;
    int8_t *xl = reinterpret_cast<int8_t *>(work);
    int *ex = reinterpret_cast<int *>(work + 4 * QB_FFN);
    uint8_t *rd = sm + Ls.red;
    int *part = reinterpret_cast<int *>(sm + Ls.part);
    const int tid = threadIdx.x, c = blockIdx.x, G = gridDim.x, warp = tid >> 5;
    for (int i = tid; i < QB_NL * (int)(sizeof(D1Layer) / 8); i += D1_BLOCK)
        reinterpret_cast<uint64_t *>(lay)[i] = reinterpret_cast<const uint64_t *>(a.layers)[i];
    if (tid == 0) {
        for (int s = 0; s < D1_SEGS; ++s) {
            tc::mbar_init(&R.full[s], 1);
            tc::mbar_init(&R.empty[s], D1_WARPS);
        }
        tc::mbar_init(kvbar, 1);
        tc::mbar_fence_init();
    }
    __syncthreads();  // the last barrier of all 288 threads
    if (warp == D1_WARPS) {
        if ((tid & 31) == 0) d1_produce(a, R);  // weights are constant: stream from the start
        return;
    }
    uint32_t id, slot, pos;
    if (a.tok_in) {  // device-resident step: the token of slot 0 at its current position
        id = __ldcg(a.tok_in);
        slot = 0;
        pos = __ldcg(a.slot_pos);
    } else {
        id = __ldcg(a.meta);
        slot = __ldcg(a.meta + 1);
        pos = __ldcg(a.meta + 2);
    }
    const uint16_t *x0 = a.embed + (size_t)id * QB_HID;  // the step's embedding row
    // barrier targets of this launch: every launch advances the arrival
    // counter by exactly D1_BAR_STRIDE arrivals per CTA (the last barrier pads it)
    const unsigned launches = __ldcg(a.bar + 1), base = launches * (D1_BAR_STRIDE * (unsigned)G);
    const bool shortctx = pos + 1 <= (uint32_t)D1_SHORT;
    // this CTA's rows of the residual stream (the O and down rows are the same
    // partition), kept here so the residual additions need no global read
    float *xo = reinterpret_cast<float *>(sm + Ls.accs);
    {
        int b, e;
        d1_part(QB_HID, c, G, b, e);
        if (tid < e - b) xo[tid] = bf2f(__ldg(x0 + b + tid));
    }
    bool ok = true;
    unsigned nbar = 0;
    int s = 0;
    uint32_t g[4];
    for (int l = 0; l < QB_NL; ++l) {
        int b, e;
        // this layer's K/V history by warp 7, which holds no values in the
        // RMSNorm below (the previous layer's reads of the area are long done)
        if (shortctx && tid == QB_HID / 4) {
            tc::fence_proxy_async_smem();
            d1_issue_history(a, l, slot, pos, sw, kvbar);
        }
        // A: RMSNorm + QKV rows + bias (pre-RoPE)
        d1_part(QB_QKV, c, G, b, e);
        {
            const uint8_t *seg = d1_wait(a, R, s, g, ok);
            d1_row896<true, true>(l == 0 ? x0 : a.x, reinterpret_cast<const uint16_t *>(seg + g[3]), a.eps, xl, ex,
                                  rd);
            const float *sc = reinterpret_cast<const float *>(seg + g[1]);
            const uint16_t *bs = reinterpret_cast<const uint16_t *>(seg + g[2]);
            d1_mma_rows16<QB_HID>(reinterpret_cast<const int8_t *>(seg), e - b, xl, ex[0], part,
                                  [&](int r, float acc) {
                                      a.qkv[b + r] = f2bf(rbf(rbf(rbf(acc) * sc[r]) + bf2f(bs[r])));
                                  });
        }
        d1_grid_sync(a, base, ++nbar, ok);
        // the slice goes back to the producer after the barrier: bulk copies
        // issued just before it were measured to delay its release fence
        d1_done(R, s++);
        // B + C: attention, then O + residual
        if (shortctx) {
            d1_attention_short(a, l, slot, pos, sw, kvbar, ok);
            d1_row896<false, false>(reinterpret_cast<const uint16_t *>(sw + D1S_CTX), nullptr, 0.f, xl, ex, rd);
        } else {
            if (c < QB_KVH) d1_attention(a, l, c, slot, pos, work, rd);
            d1_grid_sync(a, base, ++nbar, ok);
            d1_row896<false, true>(a.ctx, nullptr, 0.f, xl, ex, rd);
        }
        d1_part(QB_HID, c, G, b, e);
        {
            const uint8_t *seg = d1_wait(a, R, s, g, ok);
            const float *sc = reinterpret_cast<const float *>(seg + g[1]);
            d1_mma_rows16<QB_HID>(reinterpret_cast<const int8_t *>(seg), e - b, xl, ex[0], part,
                                  [&](int r, float acc) {
                                      const float v = rbf(xo[r] + rbf(rbf(acc) * sc[r]));
                                      xo[r] = v;
                                      a.x[b + r] = f2bf(v);
                                  });
        }
        d1_grid_sync(a, base, ++nbar, ok);
        d1_done(R, s++);
        // D: RMSNorm + gate/up pairs + SiLU*mul (rows 2j, 2j+1 stay in one warp)
        d1_part(QB_FFN, c, G, b, e);
        {
            const uint8_t *seg = d1_wait(a, R, s, g, ok);
            d1_row896<true, true>(a.x, reinterpret_cast<const uint16_t *>(seg + g[2]), a.eps, xl, ex, rd);
            const float *sc = reinterpret_cast<const float *>(seg + g[1]);
            const int nrows = 2 * (e - b), lane = tid & 31, gid = lane >> 2;
            if (16 * warp < nrows) {
                int cf[4];
                d1_mma_tile<QB_HID>(reinterpret_cast<const int8_t *>(seg), nrows, 16 * warp, 0, QB_HID / 64, xl, cf);
                long long lo, hi;
                d1_fold(cf, lo, hi);
                // rows 16w + gid (gate when gid is even) and the next row (up) of the lane 4 above
                const long long lo1 = __shfl_down_sync(0xffffffffu, lo, 4), hi1 = __shfl_down_sync(0xffffffffu, hi, 4);
                if ((lane & 3) == 0 && (gid & 1) == 0) {
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int r = 16 * warp + gid + 8 * half;
                        if (r >= nrows) break;
                        const float gt = rbf(rbf(unalign28(half ? hi : lo, ex[0])) * sc[r]);
                        const float up = rbf(rbf(unalign28(half ? hi1 : lo1, ex[0])) * sc[r + 1]);
                        a.mid[b + r / 2] = f2bf(rbf(silu_q(gt)) * up);
                    }
                }
            }
        }
        d1_grid_sync(a, base, ++nbar, ok);
        d1_done(R, s++);
        // E: down + residual
        d1_row4864(a.mid, xl, ex, rd);
        d1_part(QB_HID, c, G, b, e);
        {
            const uint8_t *seg = d1_wait(a, R, s, g, ok);
            const float *sc = reinterpret_cast<const float *>(seg + g[1]);
            d1_mma_rows16<QB_FFN>(reinterpret_cast<const int8_t *>(seg), e - b, xl, ex[0], part,
                                  [&](int r, float acc) {
                                      const float v = rbf(xo[r] + rbf(rbf(acc) * sc[r]));
                                      xo[r] = v;
                                      a.x[b + r] = f2bf(v);
                                  });
        }
        d1_grid_sync(a, base, ++nbar, ok);
        d1_done(R, s++);
    }
    // LM head: final RMSNorm (gains come with the first piece), this CTA's
    // rows in 32-row pieces (4 per warp), the warp's best (value, index)
    {
        const uint8_t *seg = d1_wait(a, R, s, g, ok);
        d1_row896<true, true>(a.x, reinterpret_cast<const uint16_t *>(seg + g[2]), a.eps, xl, ex, rd);
    }
    int lb, le;
    d1_part(QB_VOCAB, c, G, lb, le);
    float bv = -INFINITY;
    uint32_t bi = 0;
    // piece p is computed by warps 2 (p % 4) and 2 (p % 4) + 1 (one 16-row
    // m-tile each); every warp still waits for every piece before releasing
    // it, so releases stay in order per ring slot
    const int lane = tid & 31, gid = lane >> 2;
    for (int r0 = lb, p = 0; r0 < le; r0 += D1_LM_ROWS, ++p) {
        const int nr = min(D1_LM_ROWS, le - r0);
        const uint8_t *seg = d1_wait(a, R, s, g, ok);
        if ((p & 3) == (warp >> 1)) {
            const float *sc = reinterpret_cast<const float *>(seg + g[1]);
            const int m0 = 16 * (warp & 1);
            int cf[4];
            d1_mma_tile<QB_HID>(reinterpret_cast<const int8_t *>(seg), nr, m0, 0, QB_HID / 64, xl, cf);
            long long lo, hi;
            d1_fold(cf, lo, hi);
            if ((lane & 3) == 0) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int rr = m0 + gid + 8 * half;
                    if (rr < nr) {
                        const int n = r0 + rr;
                        const float v = rbf(rbf(unalign28(half ? hi : lo, ex[0])) * sc[rr]);
                        if (a.logits) a.logits[n] = f2bf(v);
                        if (better(v, (uint32_t)n, bv, bi)) {
                            bv = v;
                            bi = (uint32_t)n;
                        }
                    }
                }
            }
        }
        d1_done(R, s++);
    }
    // best of the warp (lanes 0, 4, 8, ... hold candidates)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    // best of the CTA: lane 0 of each warp holds its warp's candidate
    float *cv = reinterpret_cast<float *>(rd);
    uint32_t *ci = reinterpret_cast<uint32_t *>(rd + 64);
    if ((tid & 31) == 0) {
        cv[warp] = bv;
        ci[warp] = bi;
    }
    d1_sync();
    if (tid == 0) {
        float v = cv[0];
        uint32_t i = ci[0];
        for (int w = 1; w < D1_WARPS; ++w)
            if (better(cv[w], ci[w], v, i)) {
                v = cv[w];
                i = ci[w];
            }
        a.cand_v[c] = v;
        a.cand_i[c] = i;
    }
    // every slice has been consumed (no bulk copy is in flight) and the
    // projections run on mma.sync: nothing asynchronous is outstanding here
    d1_grid_sync(a, base, ++nbar, ok, a.expire_last_barrier ? 1u : 0u, a.expire_last_barrier ? (1u << 14) : (1u << 24));
    if (c == 0 && tid < 32) {
        float v = -INFINITY;
        uint32_t i = 0;
        for (int k = tid; k < G; k += 32) {
            const float cv2 = __ldcg(a.cand_v + k);
            const uint32_t ci2 = __ldcg(a.cand_i + k);
            if (better(cv2, ci2, v, i)) {
                v = cv2;
                i = ci2;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
            if (better(ov, oi, v, i)) {
                v = ov;
                i = oi;
            }
        }
        if (tid == 0) {
            a.tokens[0] = i;
            // every CTA has arrived at every barrier and read the counters:
            // pad the arrivals to the next launch's base, count the launch,
            // advance the slot's position (device-resident steps)
            atomicAdd(a.bar, (D1_BAR_STRIDE - nbar) * (unsigned)G);
            a.bar[1] = launches + 1;
            if (a.slot_pos) a.slot_pos[0] = pos + 1;
        }
    }
}

static int d1_grid = 0;

// The per-warp row tiling covers one CTA's slice only with at least 144 CTAs
// (QKV: 8 rows, O / down: 8 rows, gate/up: 80 rows per CTA at most).
constexpr int D1_MIN_GRID = 144;

int decode1_supported(int max_len, int limit) {
    static int sms = -1;
    if (sms < 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            sms = 0;
    }
    return sms >= D1_MIN_GRID && max_len >= 1 && max_len <= limit && max_len <= QB_D1_MAX_KEYS;
}

size_t decode1_smem_bytes() { return (size_t)d1_smem().total; }

int launch_decode1(const D1Args &a, cudaStream_t st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -3;
    static unsigned configured = 0;
    if (!(configured & (1u << (dev & 31)))) {
        if (cudaFuncSetAttribute(decode1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)decode1_smem_bytes()) != cudaSuccess)
            return -3;
        int sms = 0, per_sm = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -3;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode1_kernel, D1_BLOCK,
                                                          decode1_smem_bytes()) != cudaSuccess ||
            per_sm < 1)
            return -3;
        if (sms < D1_MIN_GRID) return -1;
        d1_grid = sms;
        configured |= 1u << (dev & 31);
    }
    pdl_break();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(d1_grid);
    cfg.blockDim = dim3(D1_BLOCK);
    cfg.dynamicSmemBytes = decode1_smem_bytes();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, decode1_kernel, a) != cudaSuccess) return -3;
    pdl_break();
    return QB_LAUNCH_CHECK();
}

}  // namespace qb
