"""Query-tiled prefill attention on the tensor cores
(qwen_b200_op_attention_prefill, attention_tile.cu) against the oracle's
exact KV8 attention, row by row over each row's causal prefix: a prompt from
position 0 (tiles of 4 rows, one CTA per tile and KV head), a ragged
continuation from a cached prefix (partial tiles, splits of 1 and 2), and a
prefix long enough for 3-CTA clusters. Bit-identical, and the bounded-wait
flag stays clear."""
import numpy as np
import pytest

import qwen_b200
from gpu_util import Keep, dev, from_bits, host, stream, sync, to_bits, vp
from test_gpu_ops import oracle_attention, rand_bf16, random_cache, rng

pytestmark = pytest.mark.gpu
L = qwen_b200.lib


def run_prefill(q, pos0, cache, cap):
    keep = Keep()
    kc, ks, vc, vs = (dev(np.ascontiguousarray(a[0])) for a in cache)  # slot 0 of the cache
    rows = q.shape[0]
    ctx = dev(np.zeros((rows, 896), np.int16))
    ws_bytes = L().qwen_b200_attention_prefill_workspace(rows)
    ws = dev(np.zeros(ws_bytes, np.uint8))
    rc = L().qwen_b200_op_attention_prefill(keep(to_bits(q).view(np.int16)), rows, pos0, vp(kc), vp(ks), vp(vc),
                                            vp(vs), cap, vp(ctx), vp(ws), ws_bytes, stream())
    assert rc == 0
    sync()
    assert int(host(ws)[:4].view(np.uint32)[0]) == 0, 'a bounded wait expired'
    return from_bits(host(ctx).view(np.uint16))


@pytest.mark.parametrize('pos0,rows,cap', [(0, 300, 512), (700, 37, 1024), (0, 17, 64), (1500, 700, 2304)])
def test_prefill_tiles_match_the_oracle(pos0, rows, cap):
    r = rng(pos0 + rows + cap)
    cache = random_cache(r, 1, cap)
    q = rand_bf16(r, (rows, 14, 64))
    got = run_prefill(q, pos0, cache, cap)
    positions = np.arange(pos0, pos0 + rows, dtype=np.uint32)
    exp = oracle_attention(q, np.zeros(rows, np.uint32), positions, cache, exact=True)
    assert np.array_equal(got, exp), f'{np.mean(got == exp):.5f} bit-equal'
