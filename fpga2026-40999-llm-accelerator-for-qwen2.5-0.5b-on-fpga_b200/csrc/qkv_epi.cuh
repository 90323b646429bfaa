// One (row, 64-wide head block) of the q|k|v projection after bias, held by
// one warp (lane: elements lane and lane+32): RoPE on q and k heads
// (model_backend.py:73-78, split-half rotation, no FMA contraction), then q
// is stored and k / v are KV8-quantised into the cache (scale = amax/127 in
// fp32, code = clamp(rne(x / scale), +-127); an all-zero vector gets scale 0).
#pragma once
#include "common.cuh"

namespace qb {

__device__ __forceinline__ void qkv_head_epilogue(float lo, float hi, int row, int hb, uint32_t slot, uint32_t pos,
                                                  const float *table, uint16_t *q_out, int8_t *kc, float *ks,
                                                  int8_t *vc, float *vs, int cap, uint16_t *kv_out) {
    const int lane = threadIdx.x & 31;
    if (hb < QB_QH + QB_KVH) {
        const float *cs = table + (size_t)pos * 64;
        const float c = cs[lane], s = cs[32 + lane];
        const float nlo = rbf(__fadd_rn(__fmul_rn(lo, c), __fmul_rn(-hi, s)));
        const float nhi = rbf(__fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s)));
        lo = nlo;
        hi = nhi;
    }
    if (hb < QB_QH) {
        uint16_t *q = q_out + (size_t)row * QB_HID + hb * 64;
        q[lane] = f2bf(lo);
        q[lane + 32] = f2bf(hi);
        return;
    }
    const bool isv = hb >= QB_QH + QB_KVH;
    const int g = (hb - QB_QH) & 1;
    if (kv_out) {
        uint16_t *o = kv_out + (size_t)row * 256 + (isv ? 128 : 0) + g * 64;
        o[lane] = f2bf(lo);
        o[lane + 32] = f2bf(hi);
    }
    const float amax = warp_max(fmaxf(fabsf(lo), fabsf(hi)));
    const float s = __fdiv_rn(amax, 127.0f);
    int clo = 0, chi = 0;
    if (s > 0.f) {
        clo = (int)fminf(fmaxf(rintf(__fdiv_rn(lo, s)), -127.f), 127.f);
        chi = (int)fminf(fmaxf(rintf(__fdiv_rn(hi, s)), -127.f), 127.f);
    }
    const size_t base = ((size_t)slot * 2 + g) * cap + pos;
    int8_t *codes = (isv ? vc : kc) + base * 64;
    codes[lane] = (int8_t)clo;
    codes[lane + 32] = (int8_t)chi;
    if (lane == 0) (isv ? vs : ks)[base] = s;
}

}  // namespace qb
