// Device helpers shared by the sm_100a kernels: bf16 bit conversions (round to
// nearest even, matching torch's .to(bfloat16) used by model_backend.py:45),
// int8 -> fp32 unpacking, streaming loads and warp reductions.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define QB_HID 896
#define QB_FFN 4864
#define QB_QKV 1152
#define QB_VOCAB 151936
#define QB_QH 14
#define QB_KVH 2
#define QB_HD 64

namespace qb {

__device__ __forceinline__ float bf2f(uint32_t b16) { return __uint_as_float(b16 << 16); }
__device__ __forceinline__ uint16_t f2bf(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
// Round an fp32 value to the nearest bf16 value (returned as fp32).
__device__ __forceinline__ float rbf(float x) { return bf2f(f2bf(x)); }
// Low / high bf16 of a packed pair as fp32.
__device__ __forceinline__ float bflo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bfhi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Four signed bytes of w as exact fp32 values: byte j is placed into the low
// mantissa byte of 2^23 (after a +128 bias by flipping its sign bit), and the
// bias 2^23 + 128 is subtracted.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float &f0, float &f1, float &f2, float &f3) {
    const uint32_t u = w ^ 0x80808080u;
    const float bias = 8388736.0f;  // 2^23 + 128
    f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - bias;
    f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - bias;
    f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - bias;
    f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - bias;
}

// 16-byte global load that bypasses L1 allocation (weights are streamed once).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ long long warp_sum_ll(long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// (value, index) argmax with the reference's tie rule: the higher index wins
// (model_backend.py:113-114, CONFIG.JSON "greedy latest-token-index on ties").
__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i > bi);
}

// Four int8 codes, bytes (b0, b1, b2, b3) of w -> two bf16x2 words (b0, b2)
// and (b1, b3) (first element in the low half), exactly: with m = b & 0x7f and the sign
// bit s = b & 0x80 of a two's-complement code b,
//   bf16(0x4300 | m) - bf16(0x4300 | s) = (128 + m) - (128 + s) = b,
// both operands and the difference being exact bf16 values.
__device__ __forceinline__ uint32_t lop_or(uint32_t x, uint32_t mask, uint32_t bits) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(mask), "r"(bits));  // (x & mask) | bits
    return r;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ void codes4_to_bf16(uint32_t w, uint32_t &k01, uint32_t &k23) {
    const uint32_t w8 = w >> 8;
    k01 = bf16x2_sub(lop_or(w, 0x007F007Fu, 0x43004300u), lop_or(w, 0x00800080u, 0x43004300u));
    k23 = bf16x2_sub(lop_or(w8, 0x007F007Fu, 0x43004300u), lop_or(w8, 0x00800080u, 0x43004300u));
}


// ---- 28-bit row alignment of the exact projections and scores
// A row whose largest magnitude has exponent e (|x| < 2^(e+1)) is held as the
// integers rint(x * 2^(26 - e)) (|q| < 2^27); an exact integer sum d of such
// a row against int8 codes returns to fp32 as RN32(d) * 2^(e - 26).

// 2^n for -126 <= n <= 127 (exact)
__device__ __forceinline__ float pow2i(int n) { return __int_as_float((n + 127) << 23); }

// x * 2^(26 - e) with at most one rounding (only results below 2^-126 round,
// and those become 0 under rint): two power-of-two factors keep each in range
// for every bf16 exponent.
__device__ __forceinline__ float align28(float x, int e) {
    const int s = 26 - e, s1 = min(s, 127);
    return (x * pow2i(s1)) * pow2i(s - s1);
}
__device__ __forceinline__ int align28_int(float x, int e) { return __float2int_rn(align28(x, e)); }

// RN32(d) * 2^(e - 26), rounded once: the first factor keeps the product
// normal (RN32(d) >= 1 in magnitude), so only the second can round.
__device__ __forceinline__ float unalign28(long long d, int e) {
    const int s = e - 26, s1 = max(s, -126);
    return (__ll2float_rn(d) * pow2i(s1)) * pow2i(s - s1);
}

// x * 2^(bits - e) for the 21-bit grid of the RMSNorm sum of squares (same
// two-factor scaling as align28).
__device__ __forceinline__ float align21(float x, int e) {
    const int s = 20 - e, s1 = min(s, 127);
    return (x * pow2i(s1)) * pow2i(s - s1);
}

// Exponent of the largest magnitude of a row (0 for an all-zero row).
__device__ __forceinline__ int row_exponent(float amax) { return amax > 0.f ? ilogbf(amax) : 0; }

// q -> four signed 7-bit limbs, q = l0 + 2^7 l1 + 2^14 l2 + 2^21 l3 (|q| < 2^27).
__device__ __forceinline__ void limbs4(int q, int (&l)[4]) {
    l[0] = ((q + 64) & 127) - 64;
    const int r1 = (q - l[0]) >> 7;
    l[1] = ((r1 + 64) & 127) - 64;
    const int r2 = (r1 - l[1]) >> 7;
    l[2] = ((r2 + 64) & 127) - 64;
    l[3] = (r2 - l[2]) >> 7;
}
// byte l of two values' limbs, as a 16-bit pair (a low, b high)
__device__ __forceinline__ uint32_t limb_bytes(const int (&la)[4], const int (&lb)[4], int l) {
    return ((uint32_t)la[l] & 0xffu) | (((uint32_t)lb[l] & 0xffu) << 8);
}


// ---- fixed-operation exp and the exact RMSNorm scale
// exp(x) by Cody-Waite range reduction and a degree-7 Taylor polynomial
// (W. J. Cody, W. Waite, Software Manual for the Elementary Functions, 1980):
// n = rint(x log2 e), r = x - n ln2 with ln2 split into a 15-bit head and a
// tail, exp(x) = 2^n sum_{k<=7} r^k/k! by Horner's rule. Each step is one
// IEEE fp32 operation written with an explicit rounding intrinsic, so the
// result is the same bits as the oracle's ref_qexp (within 1 ulp of exp).
__device__ __forceinline__ float qexp(float x) {
    if (!(x >= -104.0f)) return 0.0f;
    if (x > 88.75f) return __int_as_float(0x7f800000);
    // rint by the 1.5 * 2^23 shift (exact round-to-nearest-even for |v| < 2^22,
    // the same value as rintf here); the integer comes from the same sum's bits
    const float sh = __fadd_rn(__fmul_rn(x, 1.44269504f), 12582912.0f);
    const float n = __fsub_rn(sh, 12582912.0f);
    float r = __fmaf_rn(-n, 0.693145751953125f, x);
    r = __fmaf_rn(-n, 1.42860677e-6f, r);
    float p = 1.98412698e-4f;
    p = __fmaf_rn(p, r, 1.38888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333e-3f);
    p = __fmaf_rn(p, r, 4.16666667e-2f);
    p = __fmaf_rn(p, r, 1.66666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = __float_as_int(sh) - 0x4B400000, n1 = min(max(ni, -126), 127);
    return __fmul_rn(__fmul_rn(p, pow2i(n1)), pow2i(ni - n1));
}

// Packed pairs of fp32 (Blackwell's f32x2 arithmetic: two IEEE fp32
// operations, each rounded to nearest even, in one instruction).
__device__ __forceinline__ unsigned long long pk2(float lo, float hi) {
    unsigned long long d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ void unpk2(unsigned long long v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b,
                                                      unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long dup2(float v) { return pk2(v, v); }

// qexp (common.cuh) of two values at once, operation for operation: the
// same IEEE fp32 operations in the same order on each half (a - b taken as
// a + (-b) and fma(-n, c, x) as fma(n, -c, x), which are the same IEEE
// results), so each half is bit-identical to qexp of that value.
__device__ __forceinline__ void qexp2(float x0, float x1, float &e0, float &e1) {
    const unsigned long long x = pk2(x0, x1);
    const unsigned long long sh = add2(mul2(x, dup2(1.44269504f)), dup2(12582912.0f));
    const unsigned long long n = add2(sh, dup2(-12582912.0f));
    unsigned long long r = fma2(n, dup2(-0.693145751953125f), x);
    r = fma2(n, dup2(-1.42860677e-6f), r);
    unsigned long long q = dup2(1.98412698e-4f);
    q = fma2(q, r, dup2(1.38888889e-3f));
    q = fma2(q, r, dup2(8.33333333e-3f));
    q = fma2(q, r, dup2(4.16666667e-2f));
    q = fma2(q, r, dup2(1.66666667e-1f));
    q = fma2(q, r, dup2(0.5f));
    q = fma2(q, r, dup2(1.0f));
    q = fma2(q, r, dup2(1.0f));
    float s0, s1;
    unpk2(sh, s0, s1);
    const int ni0 = __float_as_int(s0) - 0x4B400000, n10 = min(max(ni0, -126), 127);
    const int ni1 = __float_as_int(s1) - 0x4B400000, n11 = min(max(ni1, -126), 127);
    q = mul2(mul2(q, pk2(pow2i(n10), pow2i(n11))), pk2(pow2i(ni0 - n10), pow2i(ni1 - n11)));
    float q0, q1;
    unpk2(q, q0, q1);
    e0 = !(x0 >= -104.0f) ? 0.0f : (x0 > 88.75f ? __int_as_float(0x7f800000) : q0);
    e1 = !(x1 >= -104.0f) ? 0.0f : (x1 > 88.75f ? __int_as_float(0x7f800000) : q1);
}

// rint(e * 2^40) for 0 <= e <= 1 (the exact softmax sum's grid) without a
// conversion instruction: below 2^23 the 2^23 shift rounds to nearest even,
// above it the product is already an integer read from its bits.
__device__ __forceinline__ long long rint_2p40(float e) {
    const float v = __fmul_rn(e, 0x1p40f);
    if (v < 8388608.0f) return (long long)(__float_as_int(__fadd_rn(v, 8388608.0f)) - 0x4B000000);
    const int b = __float_as_int(v);
    return (long long)((b & 0x7FFFFF) | 0x800000) << ((b >> 23) - 150);
}

// SiLU(g) = g / (1 + exp(-g)) with qexp (model_backend.py:106)
__device__ __forceinline__ float silu_q(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, qexp(-g))); }

// RMSNorm scale 1/sqrt(mean(x^2) + eps) of a row of K values whose lane
// share is xv (two bf16 per word), the sum of squares exact on the grid of
// the row's 21-bit alignment: X = rint(x 2^(20-E)), ss = RN32(sum X^2)
// 2^(2E-40) (model_backend.py:69-71 in the oracle's exact order). e is the
// row exponent (warp-wide).
template <int NW>
__device__ __forceinline__ float rms_scale_exact(const uint32_t (&xv)[NW], int K, float eps, int e) {
    long long s2 = 0;
#pragma unroll
    for (int j = 0; j < NW; ++j) {
        const long long a = __float2int_rn(align21(bflo(xv[j]), e));
        const long long b = __float2int_rn(align21(bfhi(xv[j]), e));
        s2 += a * a + b * b;
    }
    s2 = warp_sum_ll(s2);
    const float ss = ldexpf(__ll2float_rn(s2), 2 * e - 40);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps)));
}
template <int NW>
__device__ __forceinline__ int row_exponent_words(const uint32_t (&xv)[NW]) {
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < NW; ++j) amax = fmaxf(amax, fmaxf(fabsf(bflo(xv[j])), fabsf(bfhi(xv[j]))));
    return row_exponent(warp_max(amax));
}

}  // namespace qb

// Launch error helper used by the host-side launchers.
#define QB_LAUNCH_CHECK() (cudaGetLastError() == cudaSuccess ? 0 : -3)

namespace qb {
// Programmatic dependent launch. A kernel launched with programmatic stream
// serialisation may start while the preceding kernel of its stream still
// runs; pdl_wait() returns once that kernel has completed and its memory
// operations are visible (a no-op without the launch attribute). Every
// kernel of the decode chain calls it in every CTA before it reads anything
// an earlier kernel wrote or writes anything an earlier kernel reads; only
// loads of constant data (weights) may come first. pdl_trigger() lets the
// next kernel of the stream launch (it still waits for this one to finish).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host side: a launch may overlap its predecessor only when that
// predecessor is one of this library's kernels on the same stream, launched
// inside the same PdlChain scope with nothing (copy, memset, event) enqueued
// between them. A kernel that overlapped a copy could read the copy's
// destination too early. Outside a PdlChain (the operator-level entry points)
// every launch is ordinary.
struct PdlState {
    cudaStream_t st = nullptr;
    int depth = 0;
    bool prev_ours = false;
};
inline PdlState &pdl_state() {
    static thread_local PdlState s;
    return s;
}
struct PdlChain {
    PdlChain() {
        if (pdl_state().depth++ == 0) pdl_state().prev_ours = false;
    }
    ~PdlChain() {
        if (--pdl_state().depth == 0) pdl_state().prev_ours = false;
    }
    PdlChain(const PdlChain &) = delete;
    PdlChain &operator=(const PdlChain &) = delete;
};
// Call after enqueuing anything other than one of this library's kernels.
inline void pdl_break() { pdl_state().prev_ours = false; }

// Launches kernel<<<grid, block, smem, st>>>(args...) (with a cluster shape
// when cluster_x > 1), with programmatic stream serialisation when the rules
// above allow it.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                      unsigned cluster_x, Args... args) {
    PdlState &ps = pdl_state();
    const bool overlap = ps.depth > 0 && ps.prev_ours && ps.st == st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    unsigned na = 0;
    if (overlap) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster_x > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cluster_x;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    if (cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...) != cudaSuccess) return -3;
    if (ps.depth > 0) {
        ps.prev_ours = true;
        ps.st = st;
    }
    return QB_LAUNCH_CHECK();
}
}  // namespace qb
