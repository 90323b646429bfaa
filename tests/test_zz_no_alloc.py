"""The allocation-free attention entry point (qwen_b200_op_attention_noalloc),
for callers that cannot call cudaMalloc where they run attention (a host whose
own pool owns all device memory, code that must not risk the implicit device
synchronisation of cudaMalloc/cudaFree, plugins that do not own the process's
allocator). It runs the same kernels as qwen_b200_op_attention on one fixed
per-GPU scratch array built into the library instead of a caller workspace.

Checked through the C ABI on two calls in a row (the second call reuses the
scratch the first left behind): bit-identical to the workspace entry point
(the same kernels, combining the context chunks in the same order, so any
difference is a scratch-layout or reuse fault), and against the oracle's
plain KV8 attention with the bar of the other operator-level attention tests
(at least 99 % bit-equal bf16, the rest within 2 ulps); plus the size limit.
This file is collected last so that a run stopping at its first failure has
run every other test first; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import qwen_b200
from qwen_b200 import _lib
from gpu_util import Keep, assert_bf16_close, bf16_round, dev, from_bits, host, stream, sync, to_bits, vp
from oracle import ref

pytestmark = pytest.mark.gpu
L = qwen_b200.lib


def make_case(seed, positions, cap):
    r = np.random.default_rng(seed)
    n = len(positions)
    cache = (r.integers(-127, 128, size=(n, 2, cap, 64), dtype=np.int8),
             r.uniform(0.005, 0.03, size=(n, 2, cap)).astype(np.float32),
             r.integers(-127, 128, size=(n, 2, cap, 64), dtype=np.int8),
             r.uniform(0.005, 0.03, size=(n, 2, cap)).astype(np.float32))
    q = bf16_round(r.standard_normal((n, 14, 64)).astype(np.float32))
    return q, np.arange(n, dtype=np.uint32), np.array(positions, np.uint32), cache


def run(q, slots, positions, cache, cap, noalloc):
    keep = Keep()
    rows = q.shape[0]
    ctx = dev(np.zeros((rows, 896), np.int16))
    common = (keep(to_bits(q).view(np.int16)), rows, keep(slots.view(np.int32)), keep(positions.view(np.int32)),
              int(positions.max()) + 1, keep(cache[0]), keep(cache[1]), keep(cache[2]), keep(cache[3]), cap, vp(ctx))
    if noalloc:
        rc = L().qwen_b200_op_attention_noalloc(*common, stream())
    else:
        ws_bytes = L().qwen_b200_attention_workspace(rows, cap)
        ws = dev(np.zeros(ws_bytes, np.uint8))
        rc = L().qwen_b200_op_attention(*common, vp(ws), ws_bytes, stream())
    assert rc == 0
    sync()
    return host(ctx).view(np.uint16)


def oracle_plain(q, positions, cache):
    kc, ks, vc, vs = cache
    return np.concatenate([ref.attention_kv8(q[i:i + 1], positions[i:i + 1], kc[i], ks[i], vc[i], vs[i],
                                             mode=ref.KV8) for i in range(q.shape[0])])


def test_noalloc_attention_matches_workspace_entry_point_on_two_calls():
    cap = 2048
    for seed, positions in [(1, [300, 5, 2047, 129]), (2, [17, 1000, 640])]:
        q, slots, pos, cache = make_case(seed, positions, cap)
        expect = run(q, slots, pos, cache, cap, noalloc=False)
        got = run(q, slots, pos, cache, cap, noalloc=True)
        assert np.array_equal(got, expect), \
            f'noalloc attention, case {seed}: {np.mean(got == expect):.5f} of the bf16 bit patterns equal'
        assert_bf16_close(from_bits(got), oracle_plain(q, pos, cache), max_ulps=2,
                          what=f'noalloc attention vs oracle, case {seed}')


def test_noalloc_attention_rejects_requests_beyond_the_scratch():
    rows, cap = 64, 8192
    assert L().qwen_b200_attention_workspace(rows, cap) > _lib.NOALLOC_SCRATCH_BYTES
    assert L().qwen_b200_attention_workspace(64, 2048) <= _lib.NOALLOC_SCRATCH_BYTES
    keep = Keep()
    tiny = keep(np.zeros(64, np.int32))
    rc = L().qwen_b200_op_attention_noalloc(tiny, rows, tiny, tiny, 1, tiny, tiny, tiny, tiny, cap, tiny, stream())
    assert rc == _lib.ESCRATCH
