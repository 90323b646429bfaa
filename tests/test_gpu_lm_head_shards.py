"""Vocab-sharded LM head on one GPU: the LM head + argmax kernel run on two
row slices of the tied weight (the shards two ranks would own), each slice's
(value, global index) is read back and combined with the multi-rank rule
(largest value, highest index on ties, model_backend.py:113-114); the result
must equal the kernel's own full-vocabulary argmax for every row."""
import numpy as np
import pytest

import qwen_b200
import qwen_b200.distributed as D
from gpu_util import Keep, bf16_round, dev, from_bits, host, stream, sync, to_bits, vp

pytestmark = pytest.mark.gpu
L = qwen_b200.lib
VOC, HID = 151936, 896


def run_lm(x, gamma, w, s, rows):
    keep = Keep()
    vocab = w.shape[0]
    logits = dev(np.zeros((rows, vocab), np.int16))
    tokens = dev(np.zeros(rows, np.int32))
    ws_bytes = L().qwen_b200_lm_head_workspace(rows, vocab)
    ws = dev(np.zeros(ws_bytes, np.uint8))
    rc = L().qwen_b200_op_lm_head_argmax(keep(to_bits(x).view(np.int16)), rows, keep(to_bits(gamma).view(np.int16)),
                                         1e-6, keep(w), keep(s), vocab, vp(logits), vp(tokens), vp(ws), ws_bytes,
                                         stream())
    assert rc == 0
    sync()
    return host(tokens).view(np.uint32).astype(np.int64), from_bits(host(logits).view(np.uint16))


@pytest.mark.parametrize('rows', [1, 3])
def test_two_vocab_shards_combine_to_the_full_argmax(rows):
    r = np.random.default_rng(rows + 40)
    x = bf16_round(r.standard_normal((rows, HID)).astype(np.float32))
    gamma = np.ones(HID, np.float32)
    w = r.integers(-127, 128, size=(VOC, HID), dtype=np.int8)
    s = bf16_round(r.uniform(2e-4, 4e-4, size=VOC).astype(np.float32))
    full, _ = run_lm(x, gamma, w, s, rows)
    vals, idx = [], []
    for rank in range(2):
        b, e = D.vocab_shard(VOC, 2, rank)
        tok, lg = run_lm(x, gamma, np.ascontiguousarray(w[b:e]), np.ascontiguousarray(s[b:e]), rows)
        vals.append(lg[np.arange(rows), tok])
        idx.append(tok + b)
    assert D.combine_candidates(vals, idx).tolist() == full.tolist()
