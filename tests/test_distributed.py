"""Multi-rank host logic, run as two gloo ranks on the CPU: request sharding
covers every request once, max / sum over ranks, and the vocab-sharded LM
head's all-gather of per-shard (value, index) candidates reproduces the full
argmax, highest index on ties (model_backend.py:113-114), including ties that
straddle a shard boundary."""
import os
import socket

import numpy as np
import pytest

import qwen_b200.distributed as D


def test_shard_requests_cover_every_request_once():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            got = [i for r in range(world) for i in D.shard_requests(n, world, r)]
            assert got == list(range(n))
            sizes = [len(D.shard_requests(n, world, r)) for r in range(world)]
            assert max(sizes) - min(sizes) <= (1 if n else 0)
    with pytest.raises(ValueError):
        D.shard_requests(4, 2, 2)


def test_vocab_shards_tile_the_vocabulary():
    for world in (1, 2, 3, 8):
        bounds = [D.vocab_shard(151936, world, r) for r in range(world)]
        assert bounds[0][0] == 0 and bounds[-1][1] == 151936
        for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
            assert a1 == b0 and (a1 - a0) % 128 == 0


def test_combine_prefers_value_then_highest_index():
    values = [[1.0, 2.0, 5.0], [1.0, 3.0, 4.0]]
    indices = [[10, 20, 30], [70, 5, 80]]
    assert list(D.combine_candidates(values, indices)) == [70, 5, 30]


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, logits, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        rows, vocab = logits.shape
        b, e = D.vocab_shard(vocab, world, rank)
        part = logits[:, b:e]
        # local argmax over the shard, highest index on ties
        loc = part.shape[1] - 1 - np.argmax(part[:, ::-1], axis=1)
        vals = part[np.arange(rows), loc]
        tokens = D.allgather_argmax(vals, loc + b)
        mx = D.reduce_over_ranks(rank + 0.5, 'max')
        sm = D.reduce_over_ranks(rank + 1, 'sum')
        out.put((rank, tokens.tolist(), mx, sm))
    finally:
        dist.destroy_process_group()


def test_vocab_sharded_argmax_over_two_gloo_ranks():
    import torch.multiprocessing as mp
    r = np.random.default_rng(5)
    rows, vocab = 6, 1000
    # bf16-like coarse values make ties common; plant cross-shard ties
    logits = np.round(r.standard_normal((rows, vocab)).astype(np.float32) * 8) / 8
    b = D.vocab_shard(vocab, 2, 1)[0]
    logits[0, 3] = logits[0, b + 7] = 99.0    # tie across the boundary: the higher index wins
    logits[1, b - 1] = logits[1, b] = 77.0    # tie on the boundary itself
    want = vocab - 1 - np.argmax(logits[:, ::-1], axis=1)
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(k, 2, port, logits, q)) for k in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, tokens, mx, sm in res:
        assert tokens == want.tolist()
        assert tokens[0] == b + 7 and tokens[1] == b
        assert mx == 1.5 and sm == 3.0
