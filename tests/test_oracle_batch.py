"""The oracle's batched decode step (several sequences, one row each, weights
streamed once) against its single-sequence forward: each row of a batch must
equal a one-row forward of that sequence alone, token and logits, in the
exact KV8 mode the engine computes and in the plain KV8 mode the CPU baseline
times. Also pins the synthetic KV8 fill's first codes and scales (the
engine's generator, restated)."""
import numpy as np
import pytest

from oracle import ref

SEEDS = [11, 12, 13]
LENGTHS = [40, 33, 17]


@pytest.mark.parametrize('mode', [ref.KV8 | ref.EXACT, ref.KV8])
def test_batch_rows_equal_single_sequence_forwards(sd_root, mode):
    cap = 64
    batch = ref.RefModel(sd_root, capacity=cap, mode=mode)
    single = ref.RefModel(sd_root, capacity=cap, mode=mode)
    try:
        batch.set_slots(3)
        for s in range(3):
            batch.fill_kv_synthetic_slot(s, LENGTHS[s], SEEDS[s])
        slots = np.array([2, 0, 1], np.uint32)
        ids = np.array([151935, 7, 99_000], np.uint32)
        toks, logits = batch.decode_batch(slots, ids, want_logits=True)
        for i, s in enumerate(slots):
            single.clear()
            single.fill_kv_synthetic(LENGTHS[s], SEEDS[s])
            tok = single.forward([int(ids[i])], LENGTHS[s])
            assert tok == toks[i]
            assert np.array_equal(single.last_logits, logits[i])
        # positions advanced per slot; a repeated slot is refused
        toks2, _ = batch.decode_batch(np.array([0], np.uint32), toks[1:2])
        with pytest.raises(ValueError):
            batch.decode_batch(np.array([1, 1], np.uint32), np.array([1, 2], np.uint32))
    finally:
        batch.close()
        single.close()


def test_synthetic_fill_known_values(sd_root):
    m = ref.RefModel(sd_root, capacity=8, mode=ref.KV8)
    try:
        m.fill_kv_synthetic(4, 2026)
        kc, ks, vc, vs = m.kv8_state(0)
        # SplitMix64-finaliser hash of the key seed*0x100000001B3 + (4l + 2v + g)*0x9E3779B9
        def h(x):
            x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
            x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
            x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
            return ((x ^ (x >> 31)) >> 16) & 0xFFFFFFFF
        key = (2026 * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
        assert kc[0, 0, 0] == h(key) % 255 - 127
        assert kc[0, 1, 3] == h(key + 64 + 3) % 255 - 127
        kkey = (key + 1 * 0x9E3779B9) & 0xFFFFFFFFFFFFFFFF  # head 1 of K
        assert kc[1, 2, 5] == h(kkey + 2 * 64 + 5) % 255 - 127
        hv = np.float32(h((~key + 2) & 0xFFFFFFFFFFFFFFFF) & 0xffff)
        assert ks[0, 2] == np.float32(0.01) + np.float32(0.02) * hv / np.float32(65536)
    finally:
        m.close()
