// GQA attention over the KV8 cache in one launch: one thread-block cluster
// per (query row, KV head), its CTAs splitting the row's context. Same
// arithmetic as attention.cu (legacy_100mhz_closed/src/PC/model_backend.py:
// 97-102 with the cache dequantised as code * scale in fp32):
//   S[t] = bf16(fma-chain_d(q[d] * (kcode[t][d] * kscale[t])) / 8)   (d ascending)
//   P[t] = bf16(exp(S[t] - max S) * (1 / sum exp(S - max S)))
//   ctx  = bf16(sum_t P[t] * (vcode[t][d] * vscale[t]))
// The seven query heads of a KV head are processed together with packed
// f32x2 FMAs (each lane an IEEE fma, so S keeps the oracle's bits).
//   phase 1  S for this CTA's keys -> shared memory (bf16), per-head max
//   phase 2  per-head exp-sums; the cluster exchanges (max, sum) over
//            distributed shared memory and every CTA forms the same global
//            max and 1/sum (rank order)
//   phase 3  P for each 256-key chunk, partial P.V per CTA
//   phase 4  CTA rank 0 adds the partial contexts of all ranks in rank order
//            and writes ctx (bf16)
// No global scratch, no atomics; cluster barriers only (the hardware
// co-schedules a cluster's CTAs).
#include "common.cuh"
#include "kernels.h"
#include "tc05.cuh"

namespace qb {

constexpr int AC_THREADS = 256;
constexpr int AC_CHUNK = 256;  // keys per phase-1 pass (one per thread)
constexpr int AC_SLICES = 16;  // phase 3: 16 four-dim words x 16 key slices
constexpr int AC_MAX_SPLITS = 8;
constexpr int AC_MAX_KPC = 8192;  // keys per CTA (shared-memory S budget)

struct AcArgs {
    const uint16_t *q;
    const uint32_t *slots, *positions;
    const int8_t *kc, *vc;
    const float *ks, *vs;
    int cap;
    uint16_t *ctx;
    int kpc;  // keys per CTA (multiple of AC_CHUNK)
};

struct AcSmem {
    int s_off, p_off, q_off, part_off, stat_off, ctxp_off, red_off, v_off, vs_off, total;
};

__host__ __device__ inline AcSmem ac_smem(int kpc) {
    AcSmem L;
    L.s_off = 0;                                  // bf16 S [7][kpc]
    L.p_off = L.s_off + 7 * kpc * 2;              // float P [AC_CHUNK][8]
    L.q_off = L.p_off + AC_CHUNK * 8 * 4;         // float q [64][8]
    L.part_off = L.q_off + 64 * 8 * 4;            // float [AC_SLICES][8][64]
    L.stat_off = L.part_off + AC_SLICES * 8 * 64 * 4;  // float m[8], l[8]
    L.ctxp_off = L.stat_off + 16 * 4;             // float CTA partial [7][64]
    L.red_off = L.ctxp_off + 7 * 64 * 4;          // float [8 warps][8]
    L.v_off = L.red_off + 8 * 8 * 4 * 2;          // int8 V chunk [AC_CHUNK][64]
    L.vs_off = L.v_off + AC_CHUNK * 64;           // float V scales [AC_CHUNK]
    L.total = L.vs_off + AC_CHUNK * 4;
    return L;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

template <bool CLUSTER>
__global__ void __launch_bounds__(AC_THREADS) attn_cluster_kernel(AcArgs a) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int kpc = a.kpc;
    const AcSmem L = ac_smem(kpc);
    uint16_t *S = reinterpret_cast<uint16_t *>(sm + L.s_off);
    float *P = reinterpret_cast<float *>(sm + L.p_off);
    float *qs = reinterpret_cast<float *>(sm + L.q_off);
    float *part = reinterpret_cast<float *>(sm + L.part_off);
    float *stat = reinterpret_cast<float *>(sm + L.stat_off);
    float *ctxp = reinterpret_cast<float *>(sm + L.ctxp_off);
    float *red = reinterpret_cast<float *>(sm + L.red_off);
    uint8_t *Vc = sm + L.v_off;
    float *Vsc = reinterpret_cast<float *>(sm + L.vs_off);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = blockIdx.y, r = blockIdx.z;
    const int rank = CLUSTER ? (int)tc::cluster_rank() : 0;
    const int nranks = CLUSTER ? (int)gridDim.x : 1;
    const int L_row = (int)a.positions[r] + 1;
    const int slot = (int)a.slots[r];
    const int t_begin = rank * kpc;
    const int t_end = min(L_row, t_begin + kpc);
    const int nkeys = max(0, t_end - t_begin);
    const size_t kvbase = ((size_t)slot * QB_KVH + g) * a.cap;

    // q of the group's seven heads, [d][h] with a zero eighth head
    for (int i = tid; i < 64 * 8; i += AC_THREADS) {
        const int d = i >> 3, h = i & 7;
        qs[i] = h < 7 ? bf2f(a.q[(size_t)r * QB_HID + (g * 7 + h) * QB_HD + d]) : 0.f;
    }
    __syncthreads();

    // ---------------- phase 1: scores
    float mloc[7];
#pragma unroll
    for (int h = 0; h < 7; ++h) mloc[h] = -INFINITY;
    // each thread owns one key of every 256-key chunk; the next chunk's row
    // (64 code bytes + scale) is requested before the current one is used
    uint4 kr[4];
    float ksc = 0.f;
    auto load_krow = [&](int tl) {
        if (tl < nkeys) {
            const size_t key = kvbase + t_begin + tl;
            const uint4 *kp = reinterpret_cast<const uint4 *>(a.kc + key * QB_HD);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) kr[v4] = kp[v4];
            ksc = a.ks[key];
        }
    };
    load_krow(tid);
    for (int c0 = 0; c0 < nkeys; c0 += AC_CHUNK) {
        const int tl = c0 + tid;  // key index within this CTA
        const uint4 cur[4] = {kr[0], kr[1], kr[2], kr[3]};
        const float s = ksc;
        load_krow(tl + AC_CHUNK);
        if (tl < nkeys) {
            float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f)};
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
                const uint4 kw = cur[v4];
                const uint32_t words[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    float f[4];
                    i8x4_to_f32(words[wi], f[0], f[1], f[2], f[3]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int d = v4 * 16 + wi * 4 + j;
                        const float kd = __fmul_rn(f[j], s);
                        const float2 kk = make_float2(kd, kd);
                        const float4 q03 = *reinterpret_cast<const float4 *>(qs + d * 8);
                        const float4 q47 = *reinterpret_cast<const float4 *>(qs + d * 8 + 4);
                        acc[0] = ffma2(make_float2(q03.x, q03.y), kk, acc[0]);
                        acc[1] = ffma2(make_float2(q03.z, q03.w), kk, acc[1]);
                        acc[2] = ffma2(make_float2(q47.x, q47.y), kk, acc[2]);
                        acc[3] = ffma2(make_float2(q47.z, q47.w), kk, acc[3]);
                    }
                }
            }
            const float sc[7] = {acc[0].x, acc[0].y, acc[1].x, acc[1].y, acc[2].x, acc[2].y, acc[3].x};
#pragma unroll
            for (int h = 0; h < 7; ++h) {
                const uint16_t sb = f2bf(sc[h] * 0.125f);
                S[h * kpc + tl] = sb;
                mloc[h] = fmaxf(mloc[h], bf2f(sb));
            }
        }
    }
    // CTA max per head
#pragma unroll
    for (int h = 0; h < 7; ++h) {
        const float m = warp_max(mloc[h]);
        if (lane == 0) red[warp * 8 + h] = m;
    }
    __syncthreads();
    float mcta[7];
#pragma unroll
    for (int h = 0; h < 7; ++h) {
        float m = red[h];
        for (int w = 1; w < AC_THREADS / 32; ++w) m = fmaxf(m, red[w * 8 + h]);
        mcta[h] = m;
    }
    // ---------------- phase 2: exp-sums and the cluster-wide max / sum
    float lloc[7];
#pragma unroll
    for (int h = 0; h < 7; ++h) lloc[h] = 0.f;
    for (int tl = tid; tl < nkeys; tl += AC_THREADS)
#pragma unroll
        for (int h = 0; h < 7; ++h) lloc[h] += expf(bf2f(S[h * kpc + tl]) - mcta[h]);
    float *red2 = red + 64;
#pragma unroll
    for (int h = 0; h < 7; ++h) {
        const float l = warp_sum(lloc[h]);
        if (lane == 0) red2[warp * 8 + h] = l;
    }
    __syncthreads();
    if (tid < 7) {
        float l = 0.f;
        for (int w = 0; w < AC_THREADS / 32; ++w) l += red2[w * 8 + tid];
        stat[tid] = mcta[tid];
        stat[8 + tid] = l;
    }
    __syncthreads();
    float M[7], inv[7];
    if constexpr (CLUSTER) {
        tc::cluster_sync();
        // same order in every CTA: ranks ascending; max first, then sum
        const uint32_t sa = tc::smem_u32(stat);
#pragma unroll
        for (int h = 0; h < 7; ++h) {
            M[h] = -INFINITY;
            inv[h] = 0.f;
        }
        for (int sr = 0; sr < nranks; ++sr) {
            const float4 m03 = tc::ld_dsmem_f4(sa, sr), m47 = tc::ld_dsmem_f4(sa + 16, sr);
            const float mv[7] = {m03.x, m03.y, m03.z, m03.w, m47.x, m47.y, m47.z};
#pragma unroll
            for (int h = 0; h < 7; ++h) M[h] = fmaxf(M[h], mv[h]);
        }
        for (int sr = 0; sr < nranks; ++sr) {
            const float4 m03 = tc::ld_dsmem_f4(sa, sr), m47 = tc::ld_dsmem_f4(sa + 16, sr);
            const float4 l03 = tc::ld_dsmem_f4(sa + 32, sr), l47 = tc::ld_dsmem_f4(sa + 48, sr);
            const float mv[7] = {m03.x, m03.y, m03.z, m03.w, m47.x, m47.y, m47.z};
            const float lv[7] = {l03.x, l03.y, l03.z, l03.w, l47.x, l47.y, l47.z};
#pragma unroll
            for (int h = 0; h < 7; ++h)
                if (lv[h] > 0.f) inv[h] += lv[h] * expf(mv[h] - M[h]);  // inv holds the sum for now
        }
#pragma unroll
        for (int h = 0; h < 7; ++h) inv[h] = 1.0f / inv[h];
    } else {
#pragma unroll
        for (int h = 0; h < 7; ++h) {
            M[h] = stat[h];
            inv[h] = 1.0f / stat[8 + h];
        }
    }
    // ---------------- phase 3: P and partial P.V
    const int word = tid & 15, slice = tid >> 4;  // dims 4*word..+3, keys slice, slice+16, ...
    float2 acc[4][4];                           // [dim][head pair]
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.f, 0.f);
    // the V chunk is staged in shared memory (thread tid copies key tid's
    // row); the next chunk's rows are requested while this one is used
    uint4 vr[4];
    float vsc = 0.f;
    auto load_vrow = [&](int tl) {
        if (tl < nkeys) {
            const size_t key = kvbase + t_begin + tl;
            const uint4 *vp = reinterpret_cast<const uint4 *>(a.vc + key * QB_HD);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) vr[v4] = vp[v4];
            vsc = a.vs[key];
        }
    };
    load_vrow(tid);
    for (int c0 = 0; c0 < nkeys; c0 += AC_CHUNK) {
        const int nc = min(AC_CHUNK, nkeys - c0);
        __syncthreads();  // previous chunk's P and V fully consumed
        if (tid < nc) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) *reinterpret_cast<uint4 *>(Vc + tid * 64 + v4 * 16) = vr[v4];
            Vsc[tid] = vsc;
        }
        load_vrow(c0 + AC_CHUNK + tid);
        for (int i = tid; i < AC_CHUNK * 8; i += AC_THREADS) {
            const int tt = i >> 3, h = i & 7;
            float p = 0.f;
            if (tt < nc && h < 7) p = rbf(expf(bf2f(S[h * kpc + c0 + tt]) - M[h]) * inv[h]);
            P[i] = p;
        }
        __syncthreads();
        for (int tt = slice; tt < nc; tt += AC_SLICES) {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(Vc + tt * 64 + word * 4);
            const float s = Vsc[tt];
            float f[4];
            i8x4_to_f32(w, f[0], f[1], f[2], f[3]);
            const float4 p03 = *reinterpret_cast<const float4 *>(P + tt * 8);
            const float4 p47 = *reinterpret_cast<const float4 *>(P + tt * 8 + 4);
            const float2 pp[4] = {make_float2(p03.x, p03.y), make_float2(p03.z, p03.w), make_float2(p47.x, p47.y),
                                  make_float2(p47.z, p47.w)};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float vd = __fmul_rn(f[j], s);
                const float2 vv = make_float2(vd, vd);
#pragma unroll
                for (int hp = 0; hp < 4; ++hp) acc[j][hp] = ffma2(pp[hp], vv, acc[j][hp]);
            }
        }
    }
    // slices -> CTA partial [7][64] (slice order)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int hp = 0; hp < 4; ++hp) {
            const int d = word * 4 + j;
            part[(slice * 8 + 2 * hp) * 64 + d] = acc[j][hp].x;
            part[(slice * 8 + 2 * hp + 1) * 64 + d] = acc[j][hp].y;
        }
    __syncthreads();
    for (int i = tid; i < 7 * 64; i += AC_THREADS) {
        const int h = i >> 6, d = i & 63;
        float sum = 0.f;
        for (int sl = 0; sl < AC_SLICES; ++sl) sum += part[(sl * 8 + h) * 64 + d];
        ctxp[i] = sum;
    }
    // ---------------- phase 4: rank 0 adds the partial contexts in rank order
    if constexpr (CLUSTER) {
        tc::cluster_sync();
        if (rank == 0) {
            const uint32_t ca = tc::smem_u32(ctxp);
            for (int i4 = tid; i4 < 7 * 64 / 4; i4 += AC_THREADS) {
                float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int sr = 0; sr < nranks; ++sr) {
                    const float4 v = tc::ld_dsmem_f4(ca + 16u * i4, sr);
                    sum.x += v.x;
                    sum.y += v.y;
                    sum.z += v.z;
                    sum.w += v.w;
                }
                const int i = i4 * 4, h = i >> 6, d = i & 63;
                uint16_t *o = a.ctx + (size_t)r * QB_HID + (g * 7 + h) * QB_HD + d;
                o[0] = f2bf(sum.x);
                o[1] = f2bf(sum.y);
                o[2] = f2bf(sum.z);
                o[3] = f2bf(sum.w);
            }
        }
        tc::cluster_sync();  // peers' shared memory stays alive until rank 0 has read it
    } else {
        __syncthreads();
        for (int i = tid; i < 7 * 64; i += AC_THREADS) {
            const int h = i >> 6, d = i & 63;
            a.ctx[(size_t)r * QB_HID + (g * 7 + h) * QB_HD + d] = f2bf(ctxp[i]);
        }
    }
}

int attention_cluster_plan(int max_len, int *splits, int *kpc) {
    if (max_len <= 0) return -1;
    const int chunks = (max_len + AC_CHUNK - 1) / AC_CHUNK;
    int s = (max_len + 1023) / 1024;
    s = s < 1 ? 1 : (s > AC_MAX_SPLITS ? AC_MAX_SPLITS : s);
    const int k = ((chunks + s - 1) / s) * AC_CHUNK;
    if (k > AC_MAX_KPC) return -1;
    *splits = s;
    *kpc = k;
    return 0;
}

template <bool CLUSTER>
static int run_ac(const AcArgs &a, int rows, int splits, cudaStream_t st) {
    const int smem = ac_smem(a.kpc).total;
    if (smem > 48 * 1024) {
        static unsigned configured = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        if (!(configured & (1u << (dev & 31)))) {
            if (cudaFuncSetAttribute(attn_cluster_kernel<CLUSTER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     ac_smem(AC_MAX_KPC).total) != cudaSuccess)
                return -3;
            configured |= 1u << (dev & 31);
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, QB_KVH, rows);
    cfg.blockDim = dim3(AC_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CLUSTER ? (unsigned)splits : 1u;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, attn_cluster_kernel<CLUSTER>, a) != cudaSuccess) return -3;
    return QB_LAUNCH_CHECK();
}

int launch_attention_cluster(const uint16_t *q, int rows, const uint32_t *slots, const uint32_t *positions,
                             int max_len, const int8_t *kc, const float *ks, const int8_t *vc, const float *vs, int cap,
                             uint16_t *ctx, cudaStream_t st) {
    if (rows <= 0 || max_len > cap || rows > 65535) return -1;
    int splits, kpc;
    if (attention_cluster_plan(max_len, &splits, &kpc)) return -1;
    AcArgs a;
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
    return splits > 1 ? run_ac<true>(a, rows, splits, st) : run_ac<false>(a, rows, 1, st);
}

}  // namespace qb
