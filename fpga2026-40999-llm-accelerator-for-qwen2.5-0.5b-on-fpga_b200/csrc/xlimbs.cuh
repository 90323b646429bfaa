// Activation rows as the int8 limb planes of their 28-bit alignment, in
// shared memory: the operand of the exact projections (GEMV family and the
// persistent batch-1 decode kernel).
#pragma once
#include "common.cuh"

namespace qb {

// Activation loads: plain, or through L2 only (CG) for rows that other CTAs of
// the same persistent launch wrote.
template <bool CG>
__device__ __forceinline__ uint32_t ld_act(const uint32_t *p) {
    if constexpr (CG) return __ldcg(p);
    return *p;
}
template <bool CG>
__device__ __forceinline__ uint4 ld_act(const uint4 *p) {
    if constexpr (CG) return __ldcg(p);
    return *p;
}

// Rows [m0, m0+mrows) of x [rows][K] (bf16) as int8 limb planes
// xl[m][limb][k] of the row's 28-bit alignment and its exponent ex[m] (zero
// rows beyond mrows); with gamma != nullptr the row is RMSNormed first:
// bf16(bf16(x * 1/sqrt(mean(x^2) + eps)) * gamma) (model_backend.py:69-71),
// the sum of squares exact as in rmsnorm_kernel. All warps work on
// each row: for K = 896 every warp loads the whole row into registers (so
// every warp forms the same sum and maximum) and converts its share of the
// words; wider rows are split across the warps, the maximum meeting in
// shared memory.
// SYNC false: no CTA-wide barrier at the end (only for K = 896, whose path has
// none inside; for CTAs whose other warps never join one), the caller then
// synchronises the NT threads itself.
template <int K, int MT, int NT, bool CG = false, bool SYNC = true>
__device__ __forceinline__ void load_x_limbs(const uint16_t *__restrict__ x, int m0, int mrows,
                                             const uint16_t *__restrict__ gamma, float eps, int8_t *xl, int *ex) {
    constexpr int NWARP = NT / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float wmax[NWARP];
    for (int m = 0; m < MT; ++m) {
        int8_t *row = xl + (size_t)m * 4 * K;
        if (m >= mrows) {
            for (int i = threadIdx.x; i < K / 4; i += NT)
#pragma unroll
                for (int l = 0; l < 4; ++l) reinterpret_cast<uint32_t *>(row + l * K)[i] = 0u;
            if (threadIdx.x == 0) ex[m] = 0;
            continue;
        }
        if constexpr (K == QB_HID) {
            // 14 words (28 values) per lane: words lane + 32 j
            constexpr int NWD = K / 2 / 32;
            const uint32_t *xr = reinterpret_cast<const uint32_t *>(x + (size_t)(m0 + m) * K);
            uint32_t xv[NWD];
#pragma unroll
            for (int j = 0; j < NWD; ++j) xv[j] = ld_act<CG>(xr + lane + 32 * j);
            float a[NWD], b[NWD];
            if (gamma != nullptr) {
                const uint32_t *g32 = reinterpret_cast<const uint32_t *>(gamma);
                uint32_t gv[NWD];
#pragma unroll
                for (int j = 0; j < NWD; ++j) {
                    if constexpr (CG)
                        gv[j] = g32[lane + 32 * j];  // gains may sit in shared memory here
                    else
                        gv[j] = __ldg(g32 + lane + 32 * j);
                }
                const float rs = rms_scale_exact(xv, K, eps, row_exponent_words(xv));
#pragma unroll
                for (int j = 0; j < NWD; ++j) {
                    a[j] = rbf(rbf(bflo(xv[j]) * rs) * bflo(gv[j]));
                    b[j] = rbf(rbf(bfhi(xv[j]) * rs) * bfhi(gv[j]));
                }
            } else {
#pragma unroll
                for (int j = 0; j < NWD; ++j) {
                    a[j] = bflo(xv[j]);
                    b[j] = bfhi(xv[j]);
                }
            }
            float amax = 0.f;
#pragma unroll
            for (int j = 0; j < NWD; ++j) amax = fmaxf(amax, fmaxf(fabsf(a[j]), fabsf(b[j])));
            amax = warp_max(amax);
            const int e = row_exponent(amax);
#pragma unroll
            for (int j = 0; j < NWD; ++j) {
                if (j % NWARP != warp) continue;
                int la[4], lb[4];
                limbs4(align28_int(a[j], e), la);
                limbs4(align28_int(b[j], e), lb);
                const int i = lane + 32 * j;
#pragma unroll
                for (int l = 0; l < 4; ++l)
                    *reinterpret_cast<uint16_t *>(row + l * K + 2 * i) = (uint16_t)limb_bytes(la, lb, l);
            }
            if (threadIdx.x == 0) ex[m] = e;
        } else {
            // 16-byte pieces threadIdx.x + NT j (8 values each); no RMSNorm here
            constexpr int NPC = K / 8, NP = (NPC + NT - 1) / NT;
            const uint4 *xr = reinterpret_cast<const uint4 *>(x + (size_t)(m0 + m) * K);
            uint4 xv[NP];
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                const int p = threadIdx.x + NT * j;
                xv[j] = p < NPC ? ld_act<CG>(xr + p) : make_uint4(0u, 0u, 0u, 0u);
            }
            float amax = 0.f;
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                const uint32_t w[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
#pragma unroll
                for (int t = 0; t < 4; ++t) amax = fmaxf(amax, fmaxf(fabsf(bflo(w[t])), fabsf(bfhi(w[t]))));
            }
            amax = warp_max(amax);
            if (lane == 0) wmax[warp] = amax;
            __syncthreads();
            amax = wmax[0];
#pragma unroll
            for (int w2 = 1; w2 < NWARP; ++w2) amax = fmaxf(amax, wmax[w2]);
            __syncthreads();  // wmax is reused by the next row
            const int e = row_exponent(amax);
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                const int p = threadIdx.x + NT * j;
                if (p >= NPC) continue;
                const uint32_t w[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
                uint32_t pk[4][2];  // [limb][byte quad]
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
                    *reinterpret_cast<uint2 *>(row + l * K + 8 * p) = make_uint2(pk[l][0], pk[l][1]);
            }
            if (threadIdx.x == 0) ex[m] = e;
        }
    }
    static_assert(SYNC || K == QB_HID, "only the 896-wide path has no barrier inside");
    if constexpr (SYNC) __syncthreads();
}

}  // namespace qb
