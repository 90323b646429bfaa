"""The accelerator's own V cache format (src/rtl/kv8_v_quant.sv with the V
chain's MARGIN 2 from src/rtl/storage/qwen25_qkv_controller.v:1951, layer
lock of src/rtl/kv8_v_write_chain.sv:387-468), on CPU: the C oracle
(ref_v8_quant) against an independent Python restatement written from the
RTL and from the V model of src/verification/tb_kv8_quant_pipeline.sv
(ref_recip_v, ref_mv_of_num, ref_m_lock_v, ref_lock_num, ref_q_v),
hand-derived known answers, and the edge cases the RTL has (zero head, tiny
exponents below the table floor, a later token that outgrows or underflows
the layer's exponent, the unclamped 24-bit shifter, negative zero). The
reference ships no software model of this format, so these pins come from
reading the RTL."""
import numpy as np

from oracle import ref


def py_v8(v, first, lock):
    v = [int(x) for x in v]
    maxmag = max(x & 0x7fff for x in v)
    E, M8 = maxmag >> 7, 0x80 | (maxmag & 0x7f)
    if first:
        eb_calc = E - 2 if E > 3 else 1
        q, r = divmod(M8 << 2, 127)
        m = (q + (1 if r else 0)) & 0xff
        table = eb_calc - 10 if eb_calc > 10 else 0      # o_eb, the table convention
        lock = 255 if table > 245 else table + 10          # back to the internal exponent
    else:
        s = E - lock
        n = 0x7fffff if s > 15 else 0 if s < -15 else (M8 >> -s if s < 0 else M8 << s)
        q, r = divmod(n, 127)
        m = 255 if (q > 255 or (q == 255 and r)) else q + (1 if r else 0)
    eb = lock
    R = 1 << 16 if m == 0 else ((1 << 16) + (m >> 1)) // m
    codes = []
    for x in v:
        e, mm = (x >> 7) & 0xff, 0x80 | (x & 0x7f)
        d = e - eb
        if e == 0:
            nn = 0
        elif d >= 0:
            nn = (mm << d) & 0xffffff
        else:
            nn = (mm >> -d) & 0xffffff
        qv = ((nn * R + 32768) >> 16) & 0x1ffffff
        c = 127 if qv > 127 else qv
        if x >> 15:
            c = (-c) & 0xff
        codes.append(c - 256 if c > 127 else c)
    scale = ((eb - 7) << 7) if eb > 7 else 0
    return codes, m, lock, scale, m in (0, 255)


def check(v, first, lock=0):
    got = ref.v8_quant(v, first, lock)
    exp = py_v8(v, first, lock)
    assert got[0].tolist() == exp[0], (first, lock)
    assert got[1:] == exp[1:], (got[1:], exp[1:])
    return got


def bf16_bits(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7fff + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bits_to_f32(b):
    return (np.asarray(b, np.uint32) << 16).view(np.float32)


def test_known_answer_all_ones_first_token():
    codes, m, lock, scale, clip = check(np.full(64, 0x3F80, np.uint16), True)
    # E = 127, M8 = 128: eb = 125, m = ceil(512 / 127) = 5, R = 65538 // 5 =
    # 13107, N = 128 << 2 = 512, q = (512 * 13107 + 2^15) >> 16 = 102
    assert (m, lock, clip) == (5, 125, False)
    assert scale == 0x3B00  # bf16 2^-9 = 2^(125 - 134)
    assert (codes == 102).all()
    assert abs(102 * 5 * 2.0 ** (125 - 134) - 1.0) < 5e-3


def test_known_answer_negative_and_later_tokens():
    codes, *_ = check(np.full(64, 0xBF80, np.uint16), True)
    assert (codes == -102).all()
    # same magnitude later: s = 2, n = 512, m = 5 again
    codes, m, lock, _, clip = check(np.full(64, 0x3F80, np.uint16), False, 125)
    assert (m, lock, clip) == (5, 125, False) and (codes == 102).all()
    # 32.0 (E = 132): s = 7, n = 16384 = 129 * 127 + 1 -> m = 130,
    # R = 65601 // 130 = 504, q = (16384 * 504 + 2^15) >> 16 = 126
    codes, m, _, _, clip = check(np.full(64, 0x4200, np.uint16), False, 125)
    assert (m, clip) == (130, False) and (codes == 126).all()
    # 64.0 (E = 133): n = 32768 -> quotient 258 > 255: m saturates, codes clip
    codes, m, _, _, clip = check(np.full(64, 0x4280, np.uint16), False, 125)
    assert (m, clip) == (255, True) and (codes == 127).all()


def test_underflow_and_zero_heads():
    # far below the lock: n = 0, m = 0, R = 2^16, every code 0
    codes, m, _, _, clip = check(np.full(64, bf16_bits(2.0 ** -27), np.uint16), False, 125)
    assert (m, clip) == (0, True) and (codes == 0).all()
    # zero head as a first token: E = 0 -> eb 1, table floor -> lock 10
    codes, m, lock, scale, clip = check(np.zeros(64, np.uint16), True)
    assert (m, lock, clip) == (5, 10, False) and scale == 3 << 7 and (codes == 0).all()
    # negative zeros stay 0
    codes, *_ = check(np.full(64, 0x8000, np.uint16), True)
    assert (codes == 0).all()


def test_tiny_first_token_takes_the_table_floor():
    # E = 11: eb = 9 but the lock is floored at 10 by the table convention
    v = np.full(64, (11 << 7) | 0x10, np.uint16)
    codes, m, lock, _, _ = check(v, True)
    assert lock == 10 and m == -(-(0x90 << 2) // 127)


def test_unclamped_shifter_wraps_at_24_bits():
    # a later token 17 binades above the lock: m saturates at 255 and the
    # shifter drops bit 24: mantissa 0x80 -> N = 0 -> code 0, 0xC0 -> N = 2^23
    lock = 100
    v = np.zeros(64, np.uint16)
    v[0] = ((lock + 17) << 7) | 0x00
    v[1] = ((lock + 17) << 7) | 0x40
    v[2] = 0x8000 | ((lock + 17) << 7) | 0x40
    v[3] = (lock << 7) | 0x00
    codes, m, _, _, clip = check(v, False, lock)
    assert m == 255 and clip
    assert codes[0] == 0 and codes[1] == 127 and codes[2] == -127
    assert codes[3] == ((128 * 257 + 32768) >> 16)


def test_random_heads_first_and_locked():
    r = np.random.default_rng(5)
    for i in range(300):
        scale = 2.0 ** r.integers(-20, 12)
        v = bf16_bits(r.standard_normal(64).astype(np.float32) * scale)
        if i % 7 == 0:
            v[r.integers(0, 64)] = 0x8000
        _, _, lock, _, _ = check(v, True)
        w = bf16_bits(r.standard_normal(64).astype(np.float32) * scale * 2.0 ** r.integers(-20, 20))
        check(w, False, lock)
        check(w, False, int(r.integers(1, 256)))


def test_reconstruction_of_first_tokens():
    """code * m * 2^(lock - 134) reconstructs a first token to within the
    ceil step of its mantissa (m is 5..9 at margin 2, so up to 1/5 of the
    head's largest magnitude) plus half a code."""
    r = np.random.default_rng(11)
    for _ in range(100):
        v = bf16_bits(r.standard_normal(64).astype(np.float32))
        codes, m, lock, _, _ = check(v, True)
        x = bits_to_f32(v)
        y = codes.astype(np.float64) * m * 2.0 ** (lock - 134)
        amax = np.abs(x).max()
        assert np.max(np.abs(x - y)) <= amax * (1 / 5 + 1 / 127) + 1e-12
