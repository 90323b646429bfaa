"""Projections in the oracle's exact mode (REF_EXACT): each activation row is
aligned to its largest exponent E as 28-bit integers X = rint(x * 2^(26-E)),
the dot product with the int8 codes is an exact integer, then
acc = RN32(dot) * 2^(E-26) and the usual bf16 rounding points follow
(model_backend.py:62-67). This restates the RTL GEMM array's block-aligned
integer sums (src/rtl/qwen_gemm_array_i.sv) with one exponent per row.
Checked against Python integer arithmetic, including an all-zero row, entries
far below the row maximum (rounded to the 2^-26 grid), a maximum just below a
power of two and the 4864-wide down projection."""
import math

import numpy as np

from oracle import ref


def bf16(x):
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def python_linear(x, w, scale):
    out = np.empty((x.shape[0], w.shape[0]), np.float32)
    wi = w.astype(object)
    for r in range(x.shape[0]):
        amax = float(np.abs(x[r]).max())
        e = math.frexp(amax)[1] - 1 if amax > 0 else 0
        X = [int(np.rint(np.float32(math.ldexp(float(v), 26 - e)))) for v in x[r]]
        for n in range(w.shape[0]):
            dot = sum(X[k] * int(wi[n, k]) for k in range(w.shape[1]))
            acc = np.float32(math.ldexp(float(np.float32(dot)), e - 26))
            out[r, n] = bf16(np.float32(bf16(acc) * scale[n]))
    return out


def test_exact_linear_matches_integer_arithmetic():
    r = np.random.default_rng(3)
    for k, n in ((896, 24), (4864, 8)):
        x = bf16(r.standard_normal((4, k)).astype(np.float32))
        x[1] = 0.0
        x[2, r.integers(0, k, 9)] = bf16(np.float32(2e-9))
        x[3, 7] = np.float32(1.9921875)
        w = r.integers(-127, 128, size=(n, k), dtype=np.int8)
        s = bf16(r.uniform(2e-4, 4e-4, size=n).astype(np.float32))
        got = ref.linear(x, w, s, mode=ref.EXACT)
        assert np.array_equal(got, python_linear(x, w, s)), (k, n)
