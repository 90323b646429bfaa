"""The oracle's exact mode beyond the projections (REF_EXACT), checked against
Python integer arithmetic and float64 references:

- ref_qexp, the fixed-operation exp (Cody-Waite reduction, degree-7 Taylor):
  within 1 ulp of exp over the model's range, exactly 1 at 0, never above 1
  for x <= 0 (the KV8 context bound relies on it), 0 below -104;
- RMSNorm with the sum of squares exact on the row's 21-bit grid;
- softmax with the sum exact on the 2^-40 grid and the KV8 context with the
  V scale folded into the probability before an exact integer sum against the
  codes (src/rtl/kv8_v_pscale.sv:1-20), one 28-bit alignment per head;
- SwiGLU with ref_qexp.
"""
import math

import numpy as np
import pytest

from oracle import ref

X = ref.EXACT


def bf16(x):
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def exponent(amax):
    return math.frexp(float(amax))[1] - 1 if amax > 0 else 0


def ulp_error(got, x):
    exact = np.exp(np.float64(x))
    if exact < np.finfo(np.float32).tiny:
        return abs(float(got) - exact) / float(np.finfo(np.float32).smallest_subnormal)
    ulp = math.ldexp(1.0, math.frexp(exact)[1] - 24)
    return abs(float(got) - exact) / ulp


def test_qexp_accuracy_and_fixed_points():
    r = np.random.default_rng(11)
    xs = np.concatenate([r.uniform(-104, 88.7, 20000), r.uniform(-20, 0, 20000), r.uniform(-1e-3, 1e-3, 5000),
                         np.linspace(-30, 30, 6001)]).astype(np.float32)
    got = ref.qexp(xs)
    worst = max(ulp_error(g, x) for g, x in zip(got, xs))
    assert worst <= 1.0, worst  # measured 0.85 over 200k points
    assert ref.qexp(np.float32(0.0)) == 1.0
    assert ref.qexp(np.float32(-105.0)) == 0.0 and ref.qexp(np.float32(-np.inf)) == 0.0
    assert np.isinf(ref.qexp(np.float32(89.0)))
    neg = -np.abs(np.concatenate([xs, np.float32(2.0) ** -np.arange(1, 140, dtype=np.float32)]))
    assert (ref.qexp(neg.astype(np.float32)) <= 1.0).all()


def python_rmsnorm(x, g, eps=np.float32(1e-6)):
    out = np.empty_like(x)
    for r in range(x.shape[0]):
        e = exponent(np.abs(x[r]).max())
        s2 = sum(int(np.rint(math.ldexp(float(v), 20 - e))) ** 2 for v in x[r])
        ss = np.float32(math.ldexp(float(np.float32(float(s2))), 2 * e - 40)) if s2 < 2 ** 53 else None
        rs = np.float32(1.0) / np.sqrt(np.float32(ss / np.float32(896.0)) + eps)
        out[r] = bf16(bf16(x[r] * rs) * g)
    return out


def test_exact_rmsnorm_matches_integer_arithmetic():
    r = np.random.default_rng(4)
    x = bf16(r.standard_normal((5, 896)).astype(np.float32) * 3)
    x[1] *= np.float32(2.0) ** -60
    x[2, 5] = 1.0e4
    x[3, :7] = bf16(np.float32(1e-12))
    g = bf16(r.uniform(0.5, 1.5, 896).astype(np.float32))
    got = ref.rmsnorm(x, g, mode=X)
    assert np.array_equal(got, python_rmsnorm(x, g))
    # close to the plain fp32 version (the grid only drops bits below 2^-42 of the largest square)
    assert np.abs(got - ref.rmsnorm(x, g)).max() <= np.abs(got).max() * 2 ** -7


def python_attention(q, kc, ks, vc, vs):
    """One head: exact softmax sum and exact KV8 context (Python integers)."""
    s = ref.kv8_scores(q, kc, ks)
    m = s.max()
    e = ref.qexp((s - m).astype(np.float32))
    z_int = sum(int(np.rint(math.ldexp(float(v), 40))) for v in e)
    assert z_int < 2 ** 53
    z = np.float32(math.ldexp(float(np.float32(float(z_int))), -40))
    inv = np.float32(1.0) / z
    p = bf16(e * inv)
    bound = np.float32(bf16(inv) * vs.max())
    ex = exponent(bound)
    w = (p * vs).astype(np.float32)
    W = [int(np.rint(math.ldexp(float(v), 26 - ex))) for v in w]
    assert max(abs(v) for v in W) < 2 ** 27
    out = np.empty(64, np.float32)
    for d in range(64):
        dot = sum(W[t] * int(vc[t, d]) for t in range(len(W)))
        out[d] = bf16(np.float32(math.ldexp(float(np.float32(float(dot))), ex - 26)))
    return out


@pytest.mark.parametrize('length', [1, 5, 37, 300])
def test_exact_kv8_attention_matches_integer_arithmetic(length):
    r = np.random.default_rng(length)
    cap = 320
    q = bf16(r.standard_normal((1, 14, 64)).astype(np.float32) * 2)
    kc = r.integers(-127, 128, (2, cap, 64)).astype(np.int8)
    vc = r.integers(-127, 128, (2, cap, 64)).astype(np.int8)
    ks = r.uniform(0.005, 0.03, (2, cap)).astype(np.float32)
    vs = r.uniform(0.005, 0.03, (2, cap)).astype(np.float32)
    vs[1, length // 2] = 0.0  # an all-zero V vector
    got = ref.attention_kv8(q, [length - 1], kc, ks, vc, vs, mode=ref.KV8 | X)
    for h in (0, 6, 7, 13):
        g = h // 7
        exp = python_attention(q[0, h], kc[g, :length], ks[g, :length], vc[g, :length], vs[g, :length])
        assert np.array_equal(got[0, h * 64:(h + 1) * 64], exp), h
    # close to the float64 softmax-attention of the dequantised cache
    for h in range(14):
        g = h // 7
        s = ref.kv8_scores(q[0, h], kc[g, :length], ks[g, :length]).astype(np.float64)
        p = np.exp(s - s.max())
        p /= p.sum()
        ctx = p @ (vc[g, :length].astype(np.float64) * vs[g, :length, None])
        assert np.abs(got[0, h * 64:(h + 1) * 64] - ctx).max() <= 2 ** -7 * np.abs(ctx).max() + 1e-6


def test_exact_swiglu_uses_qexp():
    r = np.random.default_rng(9)
    g = bf16(r.standard_normal(4000).astype(np.float32) * 4)
    u = bf16(r.standard_normal(4000).astype(np.float32))
    sl = (g / (np.float32(1.0) + ref.qexp(-g))).astype(np.float32)
    assert np.array_equal(ref.swiglu(g, u, mode=X), bf16(bf16(sl) * u))
