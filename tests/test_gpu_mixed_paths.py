"""Batched decode at 5 to 8 rows, where a step mixes the two projection
families: gate/up and the LM head on the tcgen05 GEMM, q|k|v, O and down on
the GEMVs. Against the oracle (KV8 + exact mode) on the seeded synthetic
model: six slots prefilled with 10-token prompts, then batched steps of 6,
then 5 and 8 slots (two slots joining late at their own positions); tokens and
logits bit-identical."""
import numpy as np
import pytest

import qwen_b200
from gpu_util import from_bits
from oracle import ref

pytestmark = pytest.mark.gpu


def test_five_to_eight_rows_match_the_oracle(sd_root):
    e = qwen_b200.Engine(device=0, max_seqs=8, max_context=256, max_rows=64).load_assets(sd_root)
    m = ref.RefModel(sd_root, capacity=256, mode=ref.KV8 | ref.EXACT)
    try:
        m.set_slots(8)
        r = np.random.default_rng(58)
        last = {}
        for slot in range(8):
            p = [int(t) for t in r.integers(0, ref.VOCAB, 10 if slot < 6 else 3)]
            t_gpu, _ = e.forward(slot, p, 0)
            for tok in p:
                t_ref, _ = m.decode_batch([slot], [tok])
            assert t_gpu == int(t_ref[0]), slot
            last[slot] = t_gpu
        for slots in ([0, 1, 2, 3, 4, 5], [0, 1, 2, 3, 4, 5], [5, 3, 1, 0, 2], list(range(8))):
            toks = [last[s] for s in slots]
            out, lg = e.decode_step_logits(slots, toks)
            out_ref, lg_ref = m.decode_batch(slots, toks, want_logits=True)
            assert out.tolist() == out_ref.tolist(), slots
            assert np.array_equal(from_bits(lg), lg_ref), slots
            for s, t in zip(slots, out.tolist()):
                last[s] = t
    finally:
        m.close()
        e.close()
