// The accelerator's own KV cache format (its "K16" K path; the V path and the
// engine's RTL KV mode follow), as a second cache format beside the engine's
// per-token-per-head int8 rule: the K quantiser of src/rtl/kv8_k_quant.sv with
// the K chain's parameters (MARGIN 8 as src/rtl/storage/
// qwen25_qkv_controller.v:1908 instantiates it, MTOP 65535, RSHIFT 24,
// CODE_EXTRA 8) and the block-exponent lock of
// src/rtl/kv8_k_write_chain.sv:503-600 (the first token of each 256-token
// block fixes the exponent of that (head, block); later tokens of the block
// are quantised against it):
//   maxmag = max_d (k & 0x7fff), E = maxmag >> 7, M8 = 0x80 | (maxmag & 0x7f)
//   block start: eb = E > 9 ? E - 8 : 1, m = ceil(M8 * 2^8 / 127),
//                lock = (eb > 10 ? eb - 10 : 0) + 10 (255 at the top)
//   later token: s = E - lock, n = M8 * 2^s (0x7fffff above s = 15, 0 below
//                s = -15), m = min(ceil(n / 127), 65535)
//   R = floor((2^24 + floor(m / 2)) / m), 2^24 for m = 0
//   per dim:     N = M8d * 2^(Ed - lock) (0 when Ed = 0, 0xffffff above 15),
//                q16 = min((N * R + 2^15) >> 16, 32639)
//   planes:      hi = (q16 + 128) >> 8, lo = q16 mod 256, both negated (as
//                bytes) for a negative k
// Integer arithmetic only, so the codes are the oracle's (ref_k16_quant) bit
// for bit. Two launches: the block starts among the rows publish their locks,
// then every row is quantised (a later token reads its block's lock).
#include "common.cuh"
#include "kernels.h"

namespace qb {

// Largest |k| bit pattern (sign dropped) over one head's 64 dims: thread d
// holds dim d; two warps.
__device__ __forceinline__ unsigned k16_maxmag(unsigned kk, unsigned *red) {
    unsigned m = kk & 0x7fffu;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    return max(red[0], red[1]);
}

__device__ __forceinline__ uint8_t k16_lock_of(unsigned maxmag) {
    const unsigned E = maxmag >> 7;
    const unsigned eb_r = E > 9 ? E - 8 : 1;
    const unsigned ob = eb_r > 10 ? eb_r - 10 : 0;
    return (uint8_t)(ob > 245 ? 255 : ob + 10);
}

// K16 exponent and 16-bit mantissa of one (token, head): a block's first
// token from its own maximum, a later token against its block's lock.
__device__ __forceinline__ void k16_scale(unsigned maxmag, bool first, unsigned lock, unsigned &eb, unsigned &m) {
    const unsigned E = maxmag >> 7, M8 = 0x80u | (maxmag & 0x7fu);
    if (first) {
        eb = k16_lock_of(maxmag);
        const unsigned num = M8 << 8;
        m = num / 127u + (num % 127u != 0);
    } else {
        eb = lock;
        const int s = (int)E - (int)eb;
        uint32_t n;
        if (s > 15) n = 0x7fffffu;
        else if (s < -15) n = 0;
        else if (s < 0) n = M8 >> (-s);
        else n = M8 << s;
        const uint32_t quo = n / 127u, rem = n % 127u;
        m = (quo > 65535u || (quo == 65535u && rem != 0)) ? 65535u : quo + (rem != 0);
    }
}

// The two code bytes of one dim (bf16 bits kk) at exponent eb, mantissa m.
__device__ __forceinline__ void k16_code(unsigned kk, unsigned eb, unsigned m, int8_t &hi, int8_t &lo) {
    const uint64_t R = m == 0 ? (1ull << 24) : ((1ull << 24) + (m >> 1)) / m;
    const unsigned e = (kk >> 7) & 0xffu, mm = 0x80u | (kk & 0x7fu);
    const int dd = (int)e - (int)eb;
    uint32_t nn;
    if (e == 0) nn = 0;
    else if (dd >= 0) nn = dd > 15 ? 0xffffffu : mm << dd;
    else nn = (-dd) >= 8 ? 0 : mm >> (-dd);
    const uint64_t qv = ((uint64_t)nn * R + (1ull << 15)) >> 16;
    const unsigned qmag = ((qv >> 16) != 0 || (qv & 0xffffu) > 32639u) ? 32639u : (unsigned)qv;
    const unsigned hu = ((qmag + 128u) >> 8) & 0xffu, lu = qmag & 0xffu;
    const bool neg = (kk >> 15) & 1u;
    hi = (int8_t)(uint8_t)(neg ? (0u - hu) : hu);
    lo = (int8_t)(uint8_t)(neg ? (0u - lu) : lu);
}

struct K16Args {
    const uint16_t *k;  // [rows][2][64]
    const uint32_t *slots, *positions;
    int8_t *hi, *lo;    // [slot][2][cap][64]
    uint16_t *m16;      // [slot][2][cap]
    uint8_t *lock;      // [slot][2][nblk]
    int cap, nblk;
};

// grid (2 heads, rows), 64 threads: locks of the rows that start a block
__global__ void __launch_bounds__(64) k16_lock_kernel(K16Args a) {
    __shared__ unsigned red[2];
    const int g = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
    const uint32_t pos = a.positions[r];
    if (pos % 256u) return;
    const unsigned kk = a.k[((size_t)r * 2 + g) * QB_HD + d];
    const unsigned maxmag = k16_maxmag(kk, red);
    if (d == 0) a.lock[((size_t)a.slots[r] * 2 + g) * a.nblk + pos / 256u] = k16_lock_of(maxmag);
}

// grid (2 heads, rows), 64 threads: the codes and the mantissa of every row
__global__ void __launch_bounds__(64) k16_quant_kernel(K16Args a) {
    __shared__ unsigned red[2];
    const int g = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
    const uint32_t pos = a.positions[r], slot = a.slots[r];
    const unsigned kk = a.k[((size_t)r * 2 + g) * QB_HD + d];
    const unsigned maxmag = k16_maxmag(kk, red);
    const bool first = pos % 256u == 0;
    unsigned eb, m;
    k16_scale(maxmag, first, first ? 0u : a.lock[((size_t)slot * 2 + g) * a.nblk + pos / 256u], eb, m);
    const size_t tok = ((size_t)slot * 2 + g) * a.cap + pos;
    k16_code(kk, eb, m, a.hi[tok * QB_HD + d], a.lo[tok * QB_HD + d]);
    if (d == 0) a.m16[tok] = (uint16_t)m;
}

int launch_k16_append(const uint16_t *k, int rows, const uint32_t *slots, const uint32_t *positions, int8_t *hi,
                      int8_t *lo, uint16_t *m16, uint8_t *lock, int cap, cudaStream_t st) {
    if (rows <= 0 || rows > 65535 || cap <= 0) return -1;
    K16Args a{k, slots, positions, hi, lo, m16, lock, cap, (cap + 255) / 256};
    k16_lock_kernel<<<dim3(2, rows), 64, 0, st>>>(a);
    k16_quant_kernel<<<dim3(2, rows), 64, 0, st>>>(a);
    return QB_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ V path
// The accelerator's own V cache format: the V quantiser of
// src/rtl/kv8_v_quant.sv at the V chain's margin (MARGIN 2,
// src/rtl/storage/qwen25_qkv_controller.v:1951) with the layer lock of
// src/rtl/kv8_v_write_chain.sv:387-468 (a request's first token fixes the
// exponent of each (layer, head); every token keeps its own 8-bit mantissa):
//   maxmag, E, M8 as for K
//   first token:  eb = E > 3 ? E - 2 : 1, m = ceil(M8 * 2^2 / 127),
//                 lock = max(eb, 10) (the table convention floor)
//   later token:  s = E - lock, n = M8 * 2^s (0x7fffff above 15, 0 below -15),
//                 m = ceil(n / 127), 255 when larger
//   R = floor((2^16 + floor(m / 2)) / m), 2^16 for m = 0
//   per dim:      N = (M8d * 2^(Ed - lock)) mod 2^24 (no clamp), 0 for Ed = 0,
//                 q = min((N * R + 2^15) >> 16, 127), negated for a negative v
// value = code * m * 2^(lock - 134). The lock of a slot is taken by its token
// at position 0; a later token of a slot whose lock is still 0 is quantised
// as a first token and leaves the lock unset.
struct V8Args {
    const uint16_t *v;  // [rows][2][64]
    const uint32_t *slots, *positions;
    int8_t *codes;      // [slot][2][cap][64]
    uint8_t *m8;        // [slot][2][cap]
    uint8_t *lock;      // [slot][2]
    int cap;
};

__device__ __forceinline__ unsigned v8_first_lock(unsigned maxmag) {
    const unsigned E = maxmag >> 7;
    const unsigned eb = E > 3 ? E - 2 : 1;
    return eb > 10 ? eb : 10;
}

// V exponent and 8-bit mantissa of one (token, head); lock 0 = the layer's
// first token (or no lock yet).
__device__ __forceinline__ void v8_scale(unsigned maxmag, unsigned lock, unsigned &eb, unsigned &m) {
    const unsigned E = maxmag >> 7, M8 = 0x80u | (maxmag & 0x7fu);
    if (lock == 0) {
        eb = v8_first_lock(maxmag);
        const unsigned num = M8 << 2;
        m = num / 127u + (num % 127u != 0);
    } else {
        eb = lock;
        const int s = (int)E - (int)eb;
        uint32_t n;
        if (s > 15) n = 0x7fffffu;
        else if (s < -15) n = 0;
        else if (s < 0) n = M8 >> (-s);
        else n = M8 << s;
        const uint32_t quo = n / 127u, rem = n % 127u;
        m = (quo > 255u || (quo == 255u && rem != 0)) ? 255u : quo + (rem != 0);
    }
}

// The code of one dim (bf16 bits vv) at exponent eb, mantissa m.
__device__ __forceinline__ int8_t v8_code(unsigned vv, unsigned eb, unsigned m) {
    const uint64_t R = m == 0 ? (1ull << 16) : ((1ull << 16) + (m >> 1)) / m;
    const unsigned e = (vv >> 7) & 0xffu, mm = 0x80u | (vv & 0x7fu);
    const int dd = (int)e - (int)eb;
    uint32_t nn;
    if (e == 0) nn = 0;
    else if (dd >= 0) nn = dd >= 24 ? 0 : (mm << dd) & 0xffffffu;
    else nn = (-dd) >= 8 ? 0 : mm >> (-dd);
    const uint64_t qv = ((uint64_t)nn * R + (1ull << 15)) >> 16;
    const unsigned q = qv > 127 ? 127u : (unsigned)qv;
    return (int8_t)(uint8_t)(((vv >> 15) & 1u) ? (0u - q) : q);
}

// grid (2 heads, rows), 64 threads: locks of the rows at position 0
__global__ void __launch_bounds__(64) v8_lock_kernel(V8Args a) {
    __shared__ unsigned red[2];
    const int g = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
    if (a.positions[r] != 0) return;
    const unsigned vv = a.v[((size_t)r * 2 + g) * QB_HD + d];
    const unsigned maxmag = k16_maxmag(vv, red);
    if (d == 0) a.lock[(size_t)a.slots[r] * 2 + g] = (uint8_t)v8_first_lock(maxmag);
}

// grid (2 heads, rows), 64 threads: the codes and the mantissa of every row
__global__ void __launch_bounds__(64) v8_quant_kernel(V8Args a) {
    __shared__ unsigned red[2];
    const int g = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
    const uint32_t pos = a.positions[r], slot = a.slots[r];
    const unsigned vv = a.v[((size_t)r * 2 + g) * QB_HD + d];
    const unsigned maxmag = k16_maxmag(vv, red);
    unsigned eb, m;
    v8_scale(maxmag, pos == 0 ? 0u : a.lock[(size_t)slot * 2 + g], eb, m);
    const size_t tok = ((size_t)slot * 2 + g) * a.cap + pos;
    a.codes[tok * QB_HD + d] = v8_code(vv, eb, m);
    if (d == 0) a.m8[tok] = (uint8_t)m;
}

int launch_v8_append(const uint16_t *v, int rows, const uint32_t *slots, const uint32_t *positions, int8_t *codes,
                     uint8_t *m8, uint8_t *lock, int cap, cudaStream_t st) {
    if (rows <= 0 || rows > 65535 || cap <= 0) return -1;
    V8Args a{v, slots, positions, codes, m8, lock, cap};
    v8_lock_kernel<<<dim3(2, rows), 64, 0, st>>>(a);
    v8_quant_kernel<<<dim3(2, rows), 64, 0, st>>>(a);
    return QB_LAUNCH_CHECK();
}

// ------------------------------------------------ the engine's RTL KV mode
// Both formats appended into the engine's cache arrays (one layer): K codes
// as the two planes kc (high) / klo (low) with the fp32 scale m16 *
// 2^(lock - 142), V codes with the scale m8 * 2^(lock - 134), so that the
// engine's attention reads both with its own exact arithmetic (the K code of
// a dim being 256 * high + low). kv [rows][256]: post-RoPE k of the two KV
// heads (128) | v (128), bf16.
struct RtlKvArgs {
    const uint16_t *kv;
    const uint32_t *slots, *positions;
    int8_t *kc, *klo, *vc;  // [slot][2][cap][64]
    float *ks, *vs;         // [slot][2][cap]
    uint8_t *klock;         // [slot][2][nblk]
    uint8_t *vlock;         // [slot][2]
    int cap, nblk;
};

// grid (4, rows): x = 0, 1 the K heads (block starts), 2, 3 the V heads
// (position 0); 64 threads
__global__ void __launch_bounds__(64) rtl_kv_lock_kernel(RtlKvArgs a) {
    __shared__ unsigned red[2];
    const int x = blockIdx.x, g = x & 1, r = blockIdx.y, d = threadIdx.x;
    const bool isv = x >= 2;
    const uint32_t pos = a.positions[r], slot = a.slots[r];
    if (isv ? pos != 0 : pos % 256u != 0) return;
    const unsigned bits = a.kv[(size_t)r * 256 + (isv ? 128 : 0) + g * QB_HD + d];
    const unsigned maxmag = k16_maxmag(bits, red);
    if (d != 0) return;
    if (isv) a.vlock[(size_t)slot * 2 + g] = (uint8_t)v8_first_lock(maxmag);
    else a.klock[((size_t)slot * 2 + g) * a.nblk + pos / 256u] = k16_lock_of(maxmag);
}

__global__ void __launch_bounds__(64) rtl_kv_quant_kernel(RtlKvArgs a) {
    __shared__ unsigned red[2];
    const int x = blockIdx.x, g = x & 1, r = blockIdx.y, d = threadIdx.x;
    const bool isv = x >= 2;
    const uint32_t pos = a.positions[r], slot = a.slots[r];
    const unsigned bits = a.kv[(size_t)r * 256 + (isv ? 128 : 0) + g * QB_HD + d];
    const unsigned maxmag = k16_maxmag(bits, red);
    const size_t tok = ((size_t)slot * 2 + g) * a.cap + pos;
    unsigned eb, m;
    if (isv) {
        v8_scale(maxmag, pos == 0 ? 0u : a.vlock[(size_t)slot * 2 + g], eb, m);
        a.vc[tok * QB_HD + d] = v8_code(bits, eb, m);
        if (d == 0) a.vs[tok] = scalbnf((float)m, (int)eb - 134);
    } else {
        const bool first = pos % 256u == 0;
        k16_scale(maxmag, first, first ? 0u : a.klock[((size_t)slot * 2 + g) * a.nblk + pos / 256u], eb, m);
        k16_code(bits, eb, m, a.kc[tok * QB_HD + d], a.klo[tok * QB_HD + d]);
        if (d == 0) a.ks[tok] = scalbnf((float)m, (int)eb - 142);
    }
}

int launch_rtl_kv_append(const uint16_t *kv, int rows, const uint32_t *slots, const uint32_t *positions, int8_t *kc,
                         int8_t *klo, float *ks, uint8_t *klock, int8_t *vc, float *vs, uint8_t *vlock, int cap,
                         cudaStream_t st) {
    if (rows <= 0 || rows > 65535 || cap <= 0) return -1;
    RtlKvArgs a{kv, slots, positions, kc, klo, vc, ks, vs, klock, vlock, cap, (cap + 255) / 256};
    rtl_kv_lock_kernel<<<dim3(4, rows), 64, 0, st>>>(a);
    rtl_kv_quant_kernel<<<dim3(4, rows), 64, 0, st>>>(a);
    return QB_LAUNCH_CHECK();
}

}  // namespace qb
