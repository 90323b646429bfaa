"""The engine in the accelerator's own KV format (QWEN_B200_FLAG_RTL_KV: K16
planes with a 256-token block exponent, V8 with a per-token mantissa and a
layer exponent; src/rtl/kv8_k_quant.sv, kv8_k_write_chain.sv,
kv8_v_quant.sv, kv8_v_write_chain.sv) against the oracle in the same mode
(REF_KV8 | REF_EXACT | REF_RTL_KV) on the seeded synthetic model: a
300-token prompt (two K blocks, tensor-core prefill) and single-row decode
steps give identical tokens and logits; the caches (both K planes, scales,
V codes, K block locks, V locks) are identical; a batched step over three
slots (prompts of 300, 12 and 7 tokens: both projection paths) gives
identical tokens and logits."""
import numpy as np
import pytest

import qwen_b200
from gpu_util import from_bits
from oracle import ref

pytestmark = pytest.mark.gpu
MODE = ref.KV8 | ref.EXACT | ref.RTL_KV
CAP = 512


@pytest.fixture(scope='module')
def pair(sd_root):
    e = qwen_b200.Engine(device=0, max_seqs=3, max_context=CAP, max_rows=256,
                         flags=qwen_b200.FLAG_RTL_KV).load_assets(sd_root)
    m = ref.RefModel(sd_root, capacity=CAP, mode=MODE)
    m.set_slots(3)
    yield e, m
    m.close()
    e.close()


def test_rtl_kv_generation_caches_and_batch_match_the_oracle(pair):
    e, m = pair
    r = np.random.default_rng(300)
    prompt = [int(t) for t in r.integers(0, ref.VOCAB, 300)]
    # slot 0: prompt, then three single-row steps
    ids, pos = prompt, 0
    for step in range(4):
        t_gpu, lg = e.forward(0, ids, pos, want_logits=True)
        t_ref = m.forward(ids, pos)
        assert t_gpu == t_ref, step
        assert np.array_equal(from_bits(lg), m.last_logits), step
        pos += len(ids)
        ids = [t_gpu]
    n = pos
    for layer in (0, 11, 23):
        kc, ks, vc, vs = e.read_kv(0, layer, n)
        okc, oks, ovc, ovs = m.kv8_state(layer)
        assert np.array_equal(kc, okc) and np.array_equal(ks, oks), layer
        assert np.array_equal(vc, ovc) and np.array_equal(vs, ovs), layer
        klo, klock, vlock = e.read_kv_rtl(0, layer, n)
        oklo, oklock, ovlock = m.rtl_kv_state(layer, 0, n)
        assert np.array_equal(klo, oklo), layer
        assert np.array_equal(klock, oklock) and np.array_equal(vlock, ovlock), layer
        assert (klock[:, :2] != 0).all() and (vlock != 0).all()
    # slots 1 and 2: 12 rows (tensor-core path) and 7 rows (GEMV path)
    last = {0: ids[0]}
    for slot, length in ((1, 12), (2, 7)):
        p = [int(t) for t in r.integers(0, ref.VOCAB, length)]
        t_gpu, _ = e.forward(slot, p, 0)
        for tok in p:
            t_ref, _ = m.decode_batch([slot], [tok])
        assert t_gpu == int(t_ref[0]), slot
        last[slot] = t_gpu
    slots = [0, 1, 2]
    toks = [last[s] for s in slots]
    for step in range(2):
        out, lg = e.decode_step_logits(slots, toks)
        out_ref, lg_ref = m.decode_batch(slots, toks, want_logits=True)
        assert out.tolist() == out_ref.tolist(), step
        assert np.array_equal(from_bits(lg), lg_ref), step
        toks = out.tolist()


def test_rtl_kv_handle_refuses_the_synthetic_fill(pair):
    e, _ = pair
    with pytest.raises(qwen_b200.QwenError):
        e.fill_kv_synthetic(0, 16, 1)
