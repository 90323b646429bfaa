"""The accelerator's own V cache format on the B200 (qwen_b200_op_v8_append)
against the oracle's restatement of src/rtl/kv8_v_quant.sv (margin 2) and
the layer lock of src/rtl/kv8_v_write_chain.sv: a request of 600 tokens in
one call (its token 0 sets the lock, the others keep their own mantissa
against it), a second call continuing it by 100 tokens, a second slot whose
token 0 arrives in its own call, and a third slot that receives a later
token before any token 0 (quantised as a first token, lock left unset).
Token magnitudes drift over six decades, so later tokens saturate (m = 255),
underflow (m = 0) and wrap the RTL's 24-bit shifter. Codes, mantissas and
locks bit-identical."""
import numpy as np
import pytest

import qwen_b200
from gpu_util import Keep, dev, host, stream, sync, vp
from oracle import ref

pytestmark = pytest.mark.gpu
L = qwen_b200.lib


def bf16_bits(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7fff + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def test_v8_append_matches_the_oracle():
    r = np.random.default_rng(8)
    cap, nslots = 1024, 3
    codes = dev(np.zeros((nslots, 2, cap, 64), np.int8))
    m8 = dev(np.zeros((nslots, 2, cap), np.uint8))
    lock = dev(np.zeros((nslots, 2), np.uint8))

    def rows_for(n):
        mag = 10.0 ** r.uniform(-3.0, 3.0, size=(n, 2, 1))
        v = bf16_bits(r.standard_normal((n, 2, 64)) * mag)
        v[r.random(v.shape) < 0.01] = 0x8000  # negative zeros
        return v
    calls = [(np.zeros(600, np.uint32), np.arange(600, dtype=np.uint32)),
             (np.concatenate([np.zeros(100, np.uint32), np.full(3, 2, np.uint32)]),
              np.concatenate([np.arange(600, 700, dtype=np.uint32), np.array([5, 6, 7], np.uint32)])),
             (np.ones(4, np.uint32), np.arange(4, dtype=np.uint32)),
             (np.ones(2, np.uint32), np.array([4, 5], np.uint32))]
    exp_codes = np.zeros((nslots, 2, cap, 64), np.int8)
    exp_m = np.zeros((nslots, 2, cap), np.uint8)
    exp_lock = np.zeros((nslots, 2), np.uint8)
    for ci, (slots, positions) in enumerate(calls):
        v = rows_for(len(slots))
        if ci == 1:
            # dims 17..20 binades above slot 0's lock: the shifter wraps
            for j in range(4):
                v[10 + j, 0, :16] = ((int(exp_lock[0, 0]) + 17 + j) << 7) | r.integers(0, 128, 16)
        keep = Keep()
        rc = L().qwen_b200_op_v8_append(keep(v.view(np.int16)), len(slots), keep(slots.view(np.int32)),
                                         keep(positions.view(np.int32)), vp(codes), vp(m8), vp(lock), cap, stream())
        assert rc == 0
        sync()
        # the call's token-0 rows set their slot's lock before any later row reads it
        for i in range(len(slots)):
            s, p = int(slots[i]), int(positions[i])
            for g in range(2):
                if p == 0:
                    exp_lock[s, g] = ref.v8_quant(v[i, g], True)[2]
        for i in range(len(slots)):
            s, p = int(slots[i]), int(positions[i])
            for g in range(2):
                first = p == 0 or exp_lock[s, g] == 0
                c, m, _, _, _ = ref.v8_quant(v[i, g], first, int(exp_lock[s, g]))
                exp_codes[s, g, p], exp_m[s, g, p] = c, m
    assert np.array_equal(host(lock), exp_lock)
    assert exp_lock[2].tolist() == [0, 0]
    assert np.array_equal(host(m8), exp_m)
    assert np.array_equal(host(codes), exp_codes)
    # the drift reaches the rule's edges
    assert (exp_m[:2] == 255).any() and (exp_m[:2, :, 1:700] == 0).any()
