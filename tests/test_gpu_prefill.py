"""Batched prefill (qwen_b200_prefill) and the vocabulary-sharded LM head
(qwen_b200_lm_head_range) on the resident weights, through the C ABI.

- Rows of several sequences go through the layers together, in chunks that
  split and mix sequences; every sequence must come out exactly as if it had
  been fed alone through qwen_b200_forward (model_backend.py:80-115): the same
  greedy token, and the same KV8 cache (checked by the next decode step's
  tokens). One sequence is also checked against the oracle.
- The LM head over vocabulary ranges [begin, end) of the resident tied head,
  combined per row by (largest value, highest index) as the multi-GPU path
  does (qwen_b200/distributed.py, model_backend.py:113-114), equals the full
  head on the GEMV path (rows <= 8) and on the tensor-core path (rows > 8),
  and the full head's index equals the prefill's own greedy token.
"""
import ctypes

import numpy as np
import pytest

import qwen_b200
import qwen_b200.distributed as D
from gpu_util import torch_cuda
from oracle import ref

pytestmark = pytest.mark.gpu
VOC = 151936


@pytest.fixture(scope='module')
def engine(sd_root):
    e = qwen_b200.Engine(device=0, max_seqs=4, max_context=256, max_rows=48).load_assets(sd_root)
    yield e
    e.close()


def prompts():
    r = np.random.default_rng(77)
    return [r.integers(0, VOC, n).astype(np.uint32) for n in (40, 17, 70)]


def test_batched_prefill_equals_single_sequence_forwards(engine, sd_root):
    ps = prompts()
    slots = [2, 0, 1]
    for s in range(4):
        engine.reset(s)
    toks, hidden = engine.prefill(slots, ps, want_hidden=True)
    nxt = engine.decode_step(slots, toks)
    for s in range(4):
        engine.reset(s)
    single = [engine.forward(s, p, 0)[0] for s, p in zip(slots, ps)]
    assert toks.tolist() == single
    assert engine.decode_step(slots, toks).tolist() == nxt.tolist()
    # the 17-token sequence against the oracle (KV8 + exact mode)
    m = ref.RefModel(sd_root, capacity=256, mode=ref.KV8 | ref.EXACT)
    try:
        assert m.forward(ps[1], 0) == toks[1]
    finally:
        m.close()


@pytest.mark.parametrize('reps', [1, 4])  # 3 rows (GEMV head) and 12 rows (tensor-core head)
def test_vocab_shards_of_the_resident_head_combine_to_the_full_argmax(engine, reps):
    torch = torch_cuda()
    ps = prompts()
    slots = [0, 1, 2]
    for s in range(4):
        engine.reset(s)
    toks, hidden = engine.prefill(slots, ps, want_hidden=True)
    rows_h = np.tile(hidden, (reps, 1))
    rows = rows_h.shape[0]
    d_hidden = torch.from_numpy(rows_h.view(np.int16)).cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def head(begin, end):
        v = torch.empty(rows, dtype=torch.float32, device='cuda')
        i = torch.empty(rows, dtype=torch.int32, device='cuda')
        engine.lm_head_range(ctypes.c_void_p(d_hidden.data_ptr()), rows, begin, end, ctypes.c_void_p(v.data_ptr()),
                             ctypes.c_void_p(i.data_ptr()), stream)
        torch.cuda.synchronize()
        return v.cpu().numpy(), i.cpu().numpy().astype(np.int64)

    fv, fi = head(0, VOC)
    assert fi.tolist() == np.tile(toks, reps).tolist()
    for world in (2, 3, 8):
        vals, idx = zip(*(head(*D.vocab_shard(VOC, world, r)) for r in range(world)))
        assert D.combine_candidates(vals, idx).tolist() == fi.tolist(), world
        # every shard's candidate is its own range's best
        for r, (v, i) in enumerate(zip(vals, idx)):
            b, e = D.vocab_shard(VOC, world, r)
            assert ((i >= b) & (i < e)).all()
    with pytest.raises(qwen_b200.QwenError):
        head(5, 128)
