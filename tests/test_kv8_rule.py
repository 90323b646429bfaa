"""KV8 quantisation rule (per token and KV head: scale = amax/127 in fp32,
code = clamp(round_half_even(x / scale), -127, 127), all-zero -> scale 0) —
the oracle's implementation against an independent numpy statement, on seeded
bf16 vectors and the edge cases (zeros, exact .5 ties, +-amax, tiny and huge
magnitudes)."""
import numpy as np

from oracle import ref


def numpy_rule(x):
    x = np.asarray(x, np.float32).reshape(-1, 64)
    amax = np.abs(x).max(axis=1).astype(np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide='ignore', invalid='ignore'):
        q = np.rint(x / s[:, None]).astype(np.float32)
    q = np.where(s[:, None] > 0, np.clip(q, -127, 127), 0).astype(np.int8)
    return q, s


def bf16_round(a):
    a = np.asarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7fff + ((u >> 16) & 1)) & 0xffff0000
    return u.astype(np.uint32).view(np.float32)


def test_random_vectors_match_rule():
    rng = np.random.default_rng(1234)
    x = bf16_round(rng.standard_normal((4096, 64)).astype(np.float32) * rng.uniform(1e-3, 30, (4096, 1)))
    codes, scales = ref.kv8_quant(x)
    ecodes, escales = numpy_rule(x)
    assert np.array_equal(scales, escales)
    assert np.array_equal(codes, ecodes)


def test_edge_cases():
    rows = np.zeros((6, 64), np.float32)
    rows[1, 0], rows[1, 1] = 127.0, -127.0           # codes +-127, scale 1
    rows[1, 2], rows[1, 3] = 2.5, 3.5                # ties -> 2, 4
    rows[2] = -np.arange(64, dtype=np.float32)       # negative ramp
    rows[3, 5] = 1e-30                               # tiny single value
    rows[4] = 3.0e38 * (np.arange(64) % 2 * 2 - 1)  # huge magnitudes
    rows[5, :] = 0.5                                 # all equal -> all 127
    codes, scales = ref.kv8_quant(bf16_round(rows))
    ecodes, escales = numpy_rule(bf16_round(rows))
    assert scales[0] == 0 and not codes[0].any()
    assert codes[1, 0] == 127 and codes[1, 1] == -127 and codes[1, 2] == 2 and codes[1, 3] == 4
    assert (codes[5] == 127).all()
    assert np.array_equal(codes, ecodes) and np.array_equal(scales, escales)
    assert np.abs(codes.astype(np.int32)).max() <= 127
