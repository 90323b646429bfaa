"""KV8 attention scores in the accelerator's order (the oracle's
ref_kv8_scores): q aligned to its largest exponent E as 28-bit integers
Q[d] = rint(q[d] * 2^(26-E)), an exact integer dot product with the int8 K
codes, then the per-token K scale and 1/8 (src/rtl/kv8_score_scale8.sv:6-12
applies the scale to the finished sum; src/rtl/kv8_v_pscale.sv:40-44 sums
block-aligned integers). Checked against Python integer arithmetic, including
the edge cases of the alignment: an all-zero head, components far below the
head's maximum (rounded to the 2^-26 grid), maximal codes and bf16 maxima just
below a power of two.
"""
import math

import numpy as np

from oracle import ref


def bf16(x):
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def python_scores(q, kcodes, kscales):
    q = np.asarray(q, np.float32)
    amax = float(np.abs(q).max())
    e = math.frexp(amax)[1] - 1 if amax > 0 else 0
    qi = [int(np.rint(np.float32(math.ldexp(float(v), 26 - e)))) for v in q]
    out = []
    for t in range(kcodes.shape[0]):
        dot = sum(qi[d] * int(kcodes[t, d]) for d in range(64))
        scaled = np.float32(math.ldexp(float(np.float32(dot)), e - 26))
        out.append(bf16(np.float32(np.float32(scaled * kscales[t]) / np.float32(8.0))))
    return np.array(out, np.float32)


def case(rng, t=40):
    kc = rng.integers(-127, 128, (t, 64)).astype(np.int8)
    ks = rng.uniform(0.005, 0.03, t).astype(np.float32)
    return kc, ks


def test_scores_match_integer_arithmetic():
    rng = np.random.default_rng(11)
    for trial in range(60):
        q = bf16(rng.standard_normal(64).astype(np.float32) * np.float32(10.0 ** rng.uniform(-3, 2)))
        kc, ks = case(rng)
        assert np.array_equal(ref.kv8_scores(q, kc, ks), python_scores(q, kc, ks)), trial


def test_alignment_edge_cases():
    rng = np.random.default_rng(12)
    kc, ks = case(rng)
    kc[0] = 127
    kc[1] = -127
    zero = np.zeros(64, np.float32)
    assert np.array_equal(ref.kv8_scores(zero, kc, ks), np.zeros(kc.shape[0], np.float32))
    tiny = bf16(rng.standard_normal(64).astype(np.float32))
    tiny[rng.integers(0, 64, 8)] = bf16(np.float32(3e-9))  # below the 2^-26 grid of the maximum
    near_pow2 = bf16(rng.standard_normal(64).astype(np.float32))
    near_pow2[5] = np.float32(1.9921875)  # largest bf16 below 2: |Q| reaches 255 * 2^19
    near_pow2[9] = np.float32(-1.9921875)
    for q in (tiny, near_pow2):
        assert np.array_equal(ref.kv8_scores(q, kc, ks), python_scores(q, kc, ks))
