"""The benchmarked workload itself against the oracle: one batched greedy
decode step of 64 sequences at contexts 2048..2052 (the batched-serving
configuration the bench times), through the host-buffer C ABI, compared with
the oracle's batched step (KV8 + exact mode) on identical caches. The caches
are filled by the engine's seeded generator on the GPU and by the oracle's
restatement of it on the host; the first test checks that both hold the same
codes and scales. Bar: bit-identical tokens and logits for every sequence
(the reference's sign-off, compare_rtl_math.py:38, is token equality on
identical histories; a logit tolerance of max|d| <= 2e-2 x the logit range is
implied)."""
import numpy as np
import pytest

import qwen_b200
from gpu_util import from_bits
from oracle import ref

pytestmark = pytest.mark.gpu

SEQS, CONTEXT, SEED = 64, 2048, 2026


def lengths():
    return [CONTEXT + s % 5 for s in range(SEQS)]


@pytest.fixture(scope='module')
def pair(sd_root):
    cap = CONTEXT + 16
    e = qwen_b200.Engine(device=0, max_seqs=SEQS, max_context=cap, max_rows=64).load_assets(sd_root)
    m = ref.RefModel(sd_root, capacity=cap, mode=ref.KV8 | ref.EXACT)
    m.set_slots(SEQS)
    for s, n in enumerate(lengths()):
        e.fill_kv_synthetic(s, n, SEED + 17 * s)
        m.fill_kv_synthetic_slot(s, n, SEED + 17 * s)
    yield e, m
    e.close()
    m.close()


def test_oracle_fill_is_the_engine_fill(pair, sd_root):
    e, _ = pair
    m1 = ref.RefModel(sd_root, capacity=CONTEXT + 16, mode=ref.KV8)
    try:
        for s, layer in [(0, 0), (5, 23), (63, 11)]:
            n = lengths()[s]
            m1.clear()
            m1.fill_kv_synthetic(n, SEED + 17 * s)
            got = e.read_kv(s, layer, n)
            exp = m1.kv8_state(layer)
            for g, x in zip(got, exp):
                assert np.array_equal(g, x), (s, layer)
    finally:
        m1.close()


def test_batched_step_at_the_bench_shape_matches_the_oracle(pair):
    e, m = pair
    rng = np.random.default_rng(SEED)
    slots = np.arange(SEQS, dtype=np.uint32)
    toks = rng.integers(0, 151936, SEQS).astype(np.uint32)
    for step in range(2):
        got_t, got_l = e.decode_step_logits(slots, toks)
        exp_t, exp_l = m.decode_batch(slots, toks, want_logits=True)
        got_l = from_bits(got_l)
        bad = [s for s in range(SEQS) if not np.array_equal(got_l[s], exp_l[s])]
        assert not bad, f'step {step}: logits differ for slots {bad[:8]} ({len(bad)} of {SEQS})'
        assert np.array_equal(got_t, exp_t), f'step {step}: tokens differ'
        toks = got_t
    # the graph-replayed step (the one the bench times) gives the same tokens
    exp_t, _ = m.decode_batch(slots, toks)
    assert np.array_equal(e.decode_step(slots, toks), exp_t)
