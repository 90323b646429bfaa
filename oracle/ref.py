"""ORACLE — test infrastructure only (tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py). ctypes wrapper of oracle/qwen_ref.c,
the plain-C restatement of legacy_100mhz_closed/src/PC/model_backend.py.
"""
import ctypes
import subprocess
from ctypes import POINTER, c_char_p, c_float, c_int, c_uint32, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / '_build' / 'libqwen_ref.so'

KV8, RND8, FUSED_BIAS, CSR_EPS, ARGMAX_F32, EXACT, RTL_KV = 1, 2, 4, 8, 16, 32, 64
VOCAB = 151936

_P8 = POINTER(ctypes.c_int8)
_PF = POINTER(c_float)
_P32 = POINTER(c_uint32)
_lib = None


def build():
    subprocess.run(['make', '-s', '-C', str(HERE)], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        sig = {
            'ref_open': (c_void_p, [c_char_p, ctypes.c_uint, c_char_p, ctypes.c_size_t]),
            'ref_close': (None, [c_void_p]),
            'ref_set_mode': (None, [c_void_p, ctypes.c_uint]),
            'ref_set_threads': (None, [c_int]),
            'ref_clear': (None, [c_void_p]),
            'ref_position': (ctypes.c_uint, [c_void_p]),
            'ref_forward': (c_int, [c_void_p, _P32, ctypes.c_uint, ctypes.c_uint, _P32, _PF]),
            'ref_set_dump': (None, [c_void_p, c_int] + [_PF] * 7),
            'ref_weight': (_P8, [c_void_p, c_int, c_int]),
            'ref_scale': (_PF, [c_void_p]),
            'ref_bias': (_PF, [c_void_p]),
            'ref_gamma': (_PF, [c_void_p]),
            'ref_lm_weight': (_P8, [c_void_p]),
            'ref_embedding': (POINTER(ctypes.c_uint16), [c_void_p]),
            'ref_kv8_state': (c_int, [c_void_p, c_int, _P8, _PF, _P8, _PF]),
            'ref_rtl_kv_state': (c_int, [c_void_p, c_int, ctypes.c_uint, ctypes.c_uint, _P8, POINTER(ctypes.c_uint8),
                                         POINTER(ctypes.c_uint8)]),
            'ref_bf': (c_float, [c_float, ctypes.c_uint]),
            'ref_qexp': (c_float, [c_float]),
            'ref_rmsnorm': (None, [_PF, ctypes.c_uint, _PF, c_float, ctypes.c_uint, _PF]),
            'ref_linear': (None, [_PF, ctypes.c_uint, ctypes.c_uint, _P8, _PF, ctypes.c_uint, ctypes.c_uint, _PF]),
            'ref_linear_bias': (None, [_PF, ctypes.c_uint, ctypes.c_uint, _P8, _PF, _PF, ctypes.c_uint,
                                       ctypes.c_uint, _PF]),
            'ref_rope_table': (None, [ctypes.c_uint, _PF]),
            'ref_rope': (None, [_PF, ctypes.c_uint, ctypes.c_uint, _P32, ctypes.c_uint, _PF]),
            'ref_kv8_quant': (None, [_PF, ctypes.c_uint, _P8, _PF]),
            'ref_attention_kv8': (None, [_PF, ctypes.c_uint, _P32, _P8, _PF, _P8, _PF, ctypes.c_uint,
                                         ctypes.c_uint, _PF]),
            'ref_attention_bf16': (None, [_PF, ctypes.c_uint, _P32, _PF, _PF, ctypes.c_uint, _PF]),
            'ref_kv8_scores': (None, [_PF, ctypes.c_uint, _P8, _PF, ctypes.c_uint, _PF]),
            'ref_swiglu': (None, [_PF, _PF, ctypes.c_uint, ctypes.c_uint, _PF]),
            'ref_lm_head': (c_uint32, [c_void_p, _PF, ctypes.c_uint, _PF]),
            'ref_fill_kv_synthetic': (c_int, [c_void_p, ctypes.c_uint, ctypes.c_uint64]),
            'ref_set_slots': (c_int, [c_void_p, ctypes.c_uint]),
            'ref_k16_quant': (None, [POINTER(ctypes.c_uint16), c_int, POINTER(ctypes.c_uint8), _P8, _P8,
                                     POINTER(ctypes.c_uint16), POINTER(ctypes.c_uint8), POINTER(c_int)]),
            'ref_v8_quant': (None, [POINTER(ctypes.c_uint16), c_int, POINTER(ctypes.c_uint8), _P8,
                                    POINTER(ctypes.c_uint8), POINTER(ctypes.c_uint16), POINTER(c_int)]),
            'ref_synth_write': (c_int, [c_char_p, ctypes.c_uint64]),
            'ref_synth_prompt': (None, [ctypes.c_uint64, ctypes.c_uint, _P32]),
            'ref_fill_kv_synthetic_slot': (c_int, [c_void_p, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint64]),
            'ref_decode_batch': (c_int, [c_void_p, ctypes.c_uint, _P32, _P32, _P32, _PF]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def pf(a):
    return a.ctypes.data_as(_PF)


def p8(a):
    return a.ctypes.data_as(_P8)


def p32(a):
    return a.ctypes.data_as(_P32)


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32)
    assert not (bits & 0xffff).any(), 'array is not bf16-valued'
    return (bits >> 16).astype(np.uint16)


def synth_write(root, seed):
    """Writes the seeded synthetic model in the reference's SD format."""
    rc = lib().ref_synth_write(str(root).encode(), seed)
    if rc:
        raise RuntimeError(f'synthetic asset writer failed ({rc})')


def synth_prompt(seed, n):
    ids = np.empty(n, np.uint32)
    lib().ref_synth_prompt(seed, n, p32(ids))
    return ids


class RefModel:
    """The oracle model over an SD-card asset folder; mirrors model_backend.Model."""

    def __init__(self, sd, capacity=256, mode=0, threads=0):
        err = ctypes.create_string_buffer(512)
        L = lib()
        if threads:
            L.ref_set_threads(threads)
        self.h = L.ref_open(str(sd).encode(), capacity, err, len(err))
        if not self.h:
            raise RuntimeError(f'oracle could not load {sd}: {err.value.decode()}')
        self.capacity = capacity
        self.set_mode(mode)
        self.last_logits = None

    def set_mode(self, mode):
        self.mode = mode
        lib().ref_set_mode(self.h, mode)

    def clear(self):
        lib().ref_clear(self.h)

    @property
    def position(self):
        return lib().ref_position(self.h)

    def forward(self, ids, position):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        tok = c_uint32()
        logits = np.empty(VOCAB, dtype=np.float32)
        rc = lib().ref_forward(self.h, p32(ids), len(ids), position, ctypes.byref(tok), pf(logits))
        if rc == -8:
            raise ValueError(f'KV position mismatch pos={position} cached={self.position} ids={len(ids)}')
        if rc:
            raise ValueError(f'oracle forward failed ({rc})')
        self.last_logits = logits
        return tok.value

    def dump(self, layer, rows):
        bufs = {k: np.zeros((rows, c), dtype=np.float32)
                for k, c in dict(q=896, k=128, v=128, context=896, h=896, m=4864, y=896).items()}
        lib().ref_set_dump(self.h, layer, *[pf(bufs[k]) for k in ['q', 'k', 'v', 'context', 'h', 'm', 'y']])
        self._dump = bufs
        return bufs

    def fill_kv_synthetic(self, length, seed):
        if lib().ref_fill_kv_synthetic(self.h, length, seed):
            raise ValueError('length exceeds capacity')

    def set_slots(self, nslots):
        """KV8 caches for nslots independent sequences (slot 0 = the forward() sequence)."""
        if lib().ref_set_slots(self.h, nslots):
            raise MemoryError(f'oracle could not hold {nslots} sequences')
        self.nslots = nslots

    def fill_kv_synthetic_slot(self, slot, length, seed):
        if lib().ref_fill_kv_synthetic_slot(self.h, slot, length, seed):
            raise ValueError('bad slot or length')

    def decode_batch(self, slots, ids, want_logits=False):
        """One decode step of distinct slots (one token each, at each slot's
        position); returns the tokens and, optionally, logits [n][151936]."""
        slots = np.ascontiguousarray(slots, dtype=np.uint32)
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        toks = np.empty(len(slots), np.uint32)
        logits = np.empty((len(slots), VOCAB), np.float32) if want_logits else None
        rc = lib().ref_decode_batch(self.h, len(slots), p32(slots), p32(ids), p32(toks),
                                    pf(logits) if want_logits else None)
        if rc:
            raise ValueError(f'oracle decode_batch failed ({rc})')
        return toks, logits

    def kv8_state(self, layer):
        n = self.position
        kc = np.empty((2, n, 64), dtype=np.int8)
        vc = np.empty((2, n, 64), dtype=np.int8)
        ks = np.empty((2, n), dtype=np.float32)
        vs = np.empty((2, n), dtype=np.float32)
        lib().ref_kv8_state(self.h, layer, p8(kc), pf(ks), p8(vc), pf(vs))
        return kc, ks, vc, vs

    def rtl_kv_state(self, layer, slot, n):
        """REF_RTL_KV: (klo [2][n][64], K block locks [2][blocks], V locks [2])."""
        klo = np.empty((2, n, 64), dtype=np.int8)
        nblk = (self.capacity + 255) // 256
        klock = np.empty((2, nblk), dtype=np.uint8)
        vlock = np.empty(2, dtype=np.uint8)
        rc = lib().ref_rtl_kv_state(self.h, layer, slot, n, p8(klo),
                                    klock.ctypes.data_as(POINTER(ctypes.c_uint8)),
                                    vlock.ctypes.data_as(POINTER(ctypes.c_uint8)))
        assert rc == 0
        return klo, klock, vlock

    def weight(self, layer, proj, shape):
        p = lib().ref_weight(self.h, layer, proj)
        return np.ctypeslib.as_array(p, shape=shape)

    def scale(self):
        return np.ctypeslib.as_array(lib().ref_scale(self.h), shape=(304128 + VOCAB,))

    def bias(self):
        return np.ctypeslib.as_array(lib().ref_bias(self.h), shape=(24 * 1152,))

    def gamma(self):
        return np.ctypeslib.as_array(lib().ref_gamma(self.h), shape=(24 * 1792 + 896,))

    def lm_weight(self):
        return np.ctypeslib.as_array(lib().ref_lm_weight(self.h), shape=(VOCAB, 896))

    def embedding(self):
        return np.ctypeslib.as_array(lib().ref_embedding(self.h), shape=(VOCAB, 896))

    def close(self):
        if self.h:
            lib().ref_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------ operator level
def qexp(x):
    """ref_qexp elementwise (the exact mode's exp)."""
    f = lib().ref_qexp
    return np.array([f(float(v)) for v in np.ravel(f32(x))], np.float32).reshape(np.shape(x))


def rmsnorm(x, gamma, eps=1e-6, mode=0):
    x = f32(x)
    out = np.empty_like(x)
    lib().ref_rmsnorm(pf(x), x.shape[0], pf(f32(gamma)), eps, mode, pf(out))
    return out


def linear(x, w, scale, bias=None, mode=0):
    x = f32(x)
    w = np.ascontiguousarray(w, dtype=np.int8)
    n, k = w.shape
    out = np.empty((x.shape[0], n), dtype=np.float32)
    if bias is None:
        lib().ref_linear(pf(x), x.shape[0], k, p8(w), pf(f32(scale)), n, mode, pf(out))
    else:
        lib().ref_linear_bias(pf(x), x.shape[0], k, p8(w), pf(f32(scale)), pf(f32(bias)), n, mode, pf(out))
    return out


def rope_table(positions):
    t = np.empty((positions, 64), dtype=np.float32)
    lib().ref_rope_table(positions, pf(t))
    return t


def rope(x, positions, mode=0):
    x = f32(x)
    rows, heads = x.shape[0], x.shape[1]
    out = np.empty_like(x)
    pos = np.ascontiguousarray(positions, dtype=np.uint32)
    lib().ref_rope(pf(x), rows, heads, p32(pos), mode, pf(out))
    return out


def kv8_quant(x):
    x = f32(x).reshape(-1, 64)
    codes = np.empty(x.shape, dtype=np.int8)
    scales = np.empty(x.shape[0], dtype=np.float32)
    lib().ref_kv8_quant(pf(x), x.shape[0], p8(codes), pf(scales))
    return codes, scales


def attention_kv8(q, positions, kcodes, kscales, vcodes, vscales, mode=0):
    """q [rows][14][64]; caches [2][cap][64] / [2][cap] of one sequence."""
    q = f32(q)
    cap = kcodes.shape[1]
    ctx = np.empty((q.shape[0], 896), dtype=np.float32)
    pos = np.ascontiguousarray(positions, dtype=np.uint32)
    lib().ref_attention_kv8(pf(q), q.shape[0], p32(pos), p8(np.ascontiguousarray(kcodes)),
                            pf(f32(kscales)), p8(np.ascontiguousarray(vcodes)), pf(f32(vscales)), cap, mode,
                            pf(ctx))
    return ctx


def kv8_scores(q, kcodes, kscales, mode=0):
    """Scores of one query head q [64] against kcodes [t][64] / kscales [t]."""
    q = f32(q).reshape(64)
    kcodes = np.ascontiguousarray(kcodes, dtype=np.int8)
    out = np.empty(kcodes.shape[0], dtype=np.float32)
    lib().ref_kv8_scores(pf(q), kcodes.shape[0], p8(kcodes), pf(f32(kscales)), mode, pf(out))
    return out


def attention_bf16(q, positions, k, v, mode=0):
    """q [rows][14][64]; k, v [t][2][64] bf16-valued (one sequence)."""
    q = f32(q)
    ctx = np.empty((q.shape[0], 896), dtype=np.float32)
    pos = np.ascontiguousarray(positions, dtype=np.uint32)
    lib().ref_attention_bf16(pf(q), q.shape[0], p32(pos), pf(f32(k)), pf(f32(v)), mode, pf(ctx))
    return ctx


def swiglu(gate, up, mode=0):
    g, u = f32(gate), f32(up)
    out = np.empty_like(g)
    lib().ref_swiglu(pf(g), pf(u), g.size, mode, pf(out))
    return out


def k16_quant(k_bits, first, lock=0):
    """RTL K16 quantiser of one head (k_bits: 64 bf16 bit patterns). Returns
    (hi, lo, m16, lock, etab, clip)."""
    k = np.ascontiguousarray(k_bits, dtype=np.uint16)
    assert k.shape == (64,)
    hi = np.empty(64, np.int8)
    lo = np.empty(64, np.int8)
    m = ctypes.c_uint16()
    lk = ctypes.c_uint8(lock)
    et = ctypes.c_uint8()
    clip = c_int()
    lib().ref_k16_quant(k.ctypes.data_as(POINTER(ctypes.c_uint16)), 1 if first else 0, ctypes.byref(lk), p8(hi),
                        p8(lo), ctypes.byref(m), ctypes.byref(et), ctypes.byref(clip))
    return hi, lo, m.value, lk.value, et.value, bool(clip.value)


def v8_quant(v_bits, first, lock=0):
    """RTL V quantiser of one head (v_bits: 64 bf16 bit patterns). Returns
    (codes, m8, lock, scale_bf16_bits, clip)."""
    v = np.ascontiguousarray(v_bits, dtype=np.uint16)
    assert v.shape == (64,)
    codes = np.empty(64, np.int8)
    m = ctypes.c_uint8()
    lk = ctypes.c_uint8(lock)
    sc = ctypes.c_uint16()
    clip = c_int()
    lib().ref_v8_quant(v.ctypes.data_as(POINTER(ctypes.c_uint16)), 1 if first else 0, ctypes.byref(lk), p8(codes),
                       ctypes.byref(m), ctypes.byref(sc), ctypes.byref(clip))
    return codes, m.value, lk.value, sc.value, bool(clip.value)
