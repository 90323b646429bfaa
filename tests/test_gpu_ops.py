"""Operator-level parity of the sm_100a kernels (through the C ABI) against the
oracle on identical seeded inputs, in the style of the reference's
given-operand checks (legacy_.../tests/compare_all_layers.py:31-57).

Bars: the engine's kernels compute the oracle's exact mode (REF_EXACT: exact
integer sums for projections, RMSNorm, softmax and the KV8 context, the
fixed-operation exp), so their outputs are bit-identical to it: RMSNorm, the
projections and their epilogues, SwiGLU, fused QKV + RoPE + KV8 append, the LM
head and its argmax, and the engine's cluster attention at every context
length. The operator-level two-pass attention keeps the plain fp32 order
(expf, fp32 softmax and P.V sums) and is held to the oracle's plain KV8 mode:
>= 99 % bit-equal bf16, the rest within two ulps.
"""
import ctypes

import numpy as np
import pytest

import qwen_b200
from gpu_util import Keep, assert_bf16_close, bf16_round, dev, from_bits, host, stream, sync, to_bits, vp
from oracle import ref

pytestmark = pytest.mark.gpu

L = qwen_b200.lib


def rng(seed):
    return np.random.default_rng(seed)


def rand_bf16(r, shape, scale=1.0):
    return bf16_round(r.standard_normal(shape).astype(np.float32) * scale)


def rand_weights(r, n, k):
    w = r.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = bf16_round(r.uniform(2e-4, 4e-4, size=n).astype(np.float32))
    return w, s


def test_embed_bit_exact():
    r = rng(1)
    table = to_bits(rand_bf16(r, (1000, 896)))
    ids = r.integers(0, 1000, size=37).astype(np.uint32)
    t, i = dev(table.view(np.int16)), dev(ids.view(np.int32))
    out = dev(np.zeros((37, 896), np.int16))
    assert L().qwen_b200_op_embed(vp(t), vp(i), 37, vp(out), stream()) == 0
    sync()
    assert np.array_equal(host(out).view(np.uint16), table[ids])


@pytest.mark.parametrize('rows', [1, 7, 64])
def test_rmsnorm(rows):
    keep = Keep()
    r = rng(rows)
    x = rand_bf16(r, (rows, 896), 3.0)
    g = bf16_round(r.uniform(0.5, 1.5, 896).astype(np.float32))
    out = dev(np.zeros((rows, 896), np.int16))
    assert L().qwen_b200_op_rmsnorm(keep((to_bits(x).view(np.int16))), keep((to_bits(g).view(np.int16))), rows,
                                    ctypes.c_float(1e-6), vp(out), stream()) == 0
    sync()
    assert np.array_equal(from_bits(host(out).view(np.uint16)), ref.rmsnorm(x, g, mode=ref.EXACT))


@pytest.mark.parametrize('k,n', [(896, 1152), (896, 896), (4864, 896)])
@pytest.mark.parametrize('rows', [1, 3, 8, 13, 64])
@pytest.mark.parametrize('epi', ['plain', 'bias', 'residual'])
def test_gemm_w8a16(k, n, rows, epi):
    keep = Keep()
    r = rng(k + n + rows)
    x = rand_bf16(r, (rows, k))
    w, s = rand_weights(r, n, k)
    b = rand_bf16(r, n, 0.02)
    y0 = rand_bf16(r, (rows, n))
    yd = dev(to_bits(y0).view(np.int16))
    args = (keep((to_bits(x).view(np.int16))), rows, k, keep((w)), keep((s)), n)
    if epi == 'residual':
        assert L().qwen_b200_op_gemm_w8a16_residual(*args, vp(yd), stream()) == 0
    else:
        bias = keep((to_bits(b).view(np.int16))) if epi == 'bias' else None
        assert L().qwen_b200_op_gemm_w8a16(*args, bias, vp(yd), stream()) == 0
    sync()
    got = from_bits(host(yd).view(np.uint16))
    # projection sums are exact integers (oracle REF_EXACT): bit-identical
    if epi == 'residual':
        lin = ref.linear(x, w, s, mode=ref.EXACT)
        exp = ref.f32(np.vectorize(lambda a: ref.lib().ref_bf(a, 0))(y0 + lin))
    else:
        exp = ref.linear(x, w, s, bias=b if epi == 'bias' else None, mode=ref.EXACT)
    assert np.array_equal(got, exp), f'gemm {k}x{n} rows {rows} {epi}: {np.mean(got == exp):.5f} bit-equal'


@pytest.mark.parametrize('rows', [1, 5, 8, 16])
def test_swiglu(rows):
    keep = Keep()
    r = rng(100 + rows)
    x = rand_bf16(r, (rows, 896), 2.0)
    g = bf16_round(r.uniform(0.5, 1.5, 896).astype(np.float32))
    wg, sg = rand_weights(r, 4864, 896)
    wu, su = rand_weights(r, 4864, 896)
    wgu = np.empty((9728, 896), np.int8)
    wgu[0::2], wgu[1::2] = wg, wu
    sgu = np.empty(9728, np.float32)
    sgu[0::2], sgu[1::2] = sg, su
    mid = dev(np.zeros((rows, 4864), np.int16))
    assert L().qwen_b200_op_swiglu(keep((to_bits(x).view(np.int16))), rows, keep((to_bits(g).view(np.int16))),
                                   ctypes.c_float(1e-6), keep((wgu)), keep((sgu)), vp(mid), stream()) == 0
    sync()
    z = ref.rmsnorm(x, g, mode=ref.EXACT)
    exp = ref.swiglu(ref.linear(z, wg, sg, mode=ref.EXACT), ref.linear(z, wu, su, mode=ref.EXACT), mode=ref.EXACT)
    assert np.array_equal(from_bits(host(mid).view(np.uint16)), exp)


def rope_table(positions):
    t = np.empty((positions, 64), np.float32)
    L().qwen_b200_rope_table(positions, t.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return t


def test_rope_bit_exact():
    keep = Keep()
    r = rng(7)
    rows, heads = 23, 14
    x = rand_bf16(r, (rows, heads, 64), 2.0)
    pos = r.integers(0, 4096, rows).astype(np.uint32)
    xd = dev(to_bits(x).view(np.int16))
    assert L().qwen_b200_op_rope(vp(xd), rows, heads, keep((pos.view(np.int32))), keep(rope_table(4096)),
                                 stream()) == 0
    sync()
    assert np.array_equal(from_bits(host(xd).view(np.uint16)), ref.rope(x, pos))


def test_kv8_append_bit_exact():
    keep = Keep()
    r = rng(8)
    rows, nslots, cap = 40, 3, 64
    x = rand_bf16(r, (rows, 2, 64), 3.0)
    x[5, 1] = 0.0  # all-zero head vector -> scale 0, codes 0
    x[6, 0, :4] = [127.0, -127.0, 2.5, 3.5]
    slots = r.integers(0, nslots, rows).astype(np.uint32)
    positions = np.zeros(rows, np.uint32)
    for s in range(nslots):  # distinct positions per slot
        idx = np.nonzero(slots == s)[0]
        positions[idx] = r.permutation(cap)[:len(idx)]
    codes = dev(np.zeros((nslots, 2, cap, 64), np.int8))
    scales = dev(np.full((nslots, 2, cap), -1.0, np.float32))
    assert L().qwen_b200_op_kv8_append(keep((to_bits(x).view(np.int16))), rows, keep((slots.view(np.int32))),
                                       keep((positions.view(np.int32))), vp(codes), vp(scales), cap,
                                       stream()) == 0
    sync()
    c, s = host(codes), host(scales)
    ec, es = ref.kv8_quant(x.reshape(-1, 64))
    ec, es = ec.reshape(rows, 2, 64), es.reshape(rows, 2)
    for i in range(rows):
        for g in range(2):
            assert np.array_equal(c[slots[i], g, positions[i]], ec[i, g])
            assert s[slots[i], g, positions[i]] == es[i, g]


def random_cache(r, nslots, cap):
    kc = r.integers(-127, 128, size=(nslots, 2, cap, 64), dtype=np.int8)
    vc = r.integers(-127, 128, size=(nslots, 2, cap, 64), dtype=np.int8)
    ks = r.uniform(0.005, 0.03, size=(nslots, 2, cap)).astype(np.float32)
    vs = r.uniform(0.005, 0.03, size=(nslots, 2, cap)).astype(np.float32)
    return kc, ks, vc, vs


def run_attention(q, slots, positions, cache, cap, max_len=None, cluster=False):
    keep = Keep()
    kc, ks, vc, vs = (dev(a) for a in cache)
    rows = q.shape[0]
    ctx = dev(np.zeros((rows, 896), np.int16))
    max_len = max_len or int(positions.max()) + 1
    args = (keep((to_bits(q).view(np.int16))), rows, keep((slots.view(np.int32))), keep((positions.view(np.int32))),
            max_len, vp(kc), vp(ks), vp(vc), vp(vs), cap, vp(ctx))
    if cluster:
        rc = L().qwen_b200_op_attention_cluster(*args, stream())
    else:
        ws_bytes = L().qwen_b200_attention_workspace(rows, cap)
        ws = dev(np.zeros(ws_bytes, np.uint8))
        rc = L().qwen_b200_op_attention(*args, vp(ws), ws_bytes, stream())
    assert rc == 0
    sync()
    return from_bits(host(ctx).view(np.uint16))


def oracle_attention(q, slots, positions, cache, exact=False):
    kc, ks, vc, vs = cache
    mode = ref.KV8 | (ref.EXACT if exact else 0)
    out = np.empty((q.shape[0], 896), np.float32)
    for i in range(q.shape[0]):
        s = slots[i]
        out[i] = ref.attention_kv8(q[i:i + 1], positions[i:i + 1], kc[s], ks[s], vc[s], vs[s], mode=mode)[0]
    return out


def check_attention(got, q, slots, positions, cache, cluster, what):
    """The cluster kernel (the engine's) is bit-identical to the exact mode;
    the two-pass operator is within the plain-order bar."""
    if cluster:
        exp = oracle_attention(q, slots, positions, cache, exact=True)
        assert np.array_equal(got, exp), f'{what}: {np.mean(got == exp):.5f} bit-equal'
    else:
        assert_bf16_close(got, oracle_attention(q, slots, positions, cache), max_ulps=2, what=what)


@pytest.mark.parametrize('cluster', [False, True])
@pytest.mark.parametrize('positions', [[0], [16], [127], [128], [255], [256], [300, 5, 2047, 129]])
def test_attention_decode(positions, cluster):
    r = rng(sum(positions) + 11)
    cap = 2048
    positions = np.array(positions, np.uint32)
    slots = np.arange(len(positions), dtype=np.uint32)
    cache = random_cache(r, len(positions), cap)
    q = rand_bf16(r, (len(positions), 14, 64))
    got = run_attention(q, slots, positions, cache, cap, cluster=cluster)
    check_attention(got, q, slots, positions, cache, cluster, 'attention decode')


@pytest.mark.parametrize('cluster', [False, True])
def test_attention_prefill_rows_and_loose_bound(cluster):
    r = rng(12)
    cap = 512
    slots = np.array([1] * 40 + [0] * 3, np.uint32)  # ragged: 40 causal rows of slot 1, 3 of slot 0
    positions = np.array(list(range(200, 240)) + [0, 1, 2], np.uint32)
    cache = random_cache(r, 2, cap)
    q = rand_bf16(r, (43, 14, 64))
    got = run_attention(q, slots, positions, cache, cap, max_len=cap, cluster=cluster)  # capacity as the bound
    check_attention(got, q, slots, positions, cache, cluster, 'attention prefill')


@pytest.mark.parametrize('length', [8192, 32768])
def test_attention_cluster_long_context(length):
    """Long contexts (the attention config's 8192 / 32768): the cluster splits
    the row over up to 16 CTAs (a non-portable cluster where the GPU places
    one; 8 otherwise)."""
    r = rng(length)
    cap = length
    positions = np.array([length - 1, length // 3], np.uint32)
    slots = np.arange(2, dtype=np.uint32)
    cache = random_cache(r, 2, cap)
    q = rand_bf16(r, (2, 14, 64))
    got = run_attention(q, slots, positions, cache, cap, cluster=True)
    # every sum is exact: bit-identical at any length and split
    check_attention(got, q, slots, positions, cache, True, f'attention L={length}')


@pytest.mark.parametrize('cap', [1001, 1002])
def test_attention_cluster_unaligned_capacity(cap):
    """Capacities that are not a multiple of 4 put the per-key scale rows off
    16-byte boundaries: the kernel stages them with plain loads instead of
    bulk copies, with the same bits."""
    r = rng(cap)
    positions = np.array([cap - 1, 37, 512, 0], np.uint32)
    slots = np.array([2, 0, 1, 3], np.uint32)
    cache = random_cache(r, 4, cap)
    q = rand_bf16(r, (4, 14, 64))
    got = run_attention(q, slots, positions, cache, cap, cluster=True)
    check_attention(got, q, slots, positions, cache, True, f'attention cap={cap}')


@pytest.mark.parametrize('rows', [3, 8, 9])
def test_qkv_fused_against_oracle_chain(rows):
    keep = Keep()
    r = rng(21 + rows)
    cap = 64
    x = rand_bf16(r, (rows, 896), 2.0)
    g = bf16_round(r.uniform(0.5, 1.5, 896).astype(np.float32))
    w, s = rand_weights(r, 1152, 896)
    b = rand_bf16(r, 1152, 0.02)
    slots = np.zeros(rows, np.uint32)
    positions = np.arange(3, 3 + rows, dtype=np.uint32)
    q = dev(np.zeros((rows, 896), np.int16))
    kc, vc = dev(np.zeros((1, 2, cap, 64), np.int8)), dev(np.zeros((1, 2, cap, 64), np.int8))
    ks, vs = dev(np.zeros((1, 2, cap), np.float32)), dev(np.zeros((1, 2, cap), np.float32))
    assert L().qwen_b200_op_qkv(keep((to_bits(x).view(np.int16))), rows, keep((to_bits(g).view(np.int16))),
                                ctypes.c_float(1e-6), keep((w)), keep((s)), keep((to_bits(b).view(np.int16))),
                                keep((slots.view(np.int32))), keep((positions.view(np.int32))),
                                keep(rope_table(cap)), vp(q), vp(kc), vp(ks), vp(vc), vp(vs), cap, stream()) == 0
    sync()
    h = ref.rmsnorm(x, g, mode=ref.EXACT)
    y = ref.linear(h, w, s, bias=b, mode=ref.EXACT)
    eq = ref.rope(y[:, :896].reshape(rows, 14, 64), positions).reshape(rows, 896)
    ek = ref.rope(y[:, 896:1024].reshape(rows, 2, 64), positions)
    ev = y[:, 1024:].reshape(rows, 2, 64)
    assert np.array_equal(from_bits(host(q).view(np.uint16)), eq)
    for cache, scales, src in [(kc, ks, ek), (vc, vs, ev)]:
        codes, sc = ref.kv8_quant(src.reshape(-1, 64))
        got_c = host(cache)[0][:, positions].transpose(1, 0, 2).reshape(-1, 64)
        got_s = host(scales)[0][:, positions].T.reshape(-1)
        assert np.array_equal(got_c, codes) and np.array_equal(got_s, sc)


def lm_oracle(x, g, w, s):
    logits = ref.linear(ref.rmsnorm(x, g, mode=ref.EXACT), w, s, mode=ref.EXACT)
    toks = [int(len(row) - 1 - np.argmax(row[::-1])) for row in logits]  # highest index on ties
    return logits, toks


@pytest.mark.parametrize('rows', [1, 5, 8, 12])
def test_lm_head_argmax_with_planted_ties(rows):
    keep = Keep()
    r = rng(30 + rows)
    vocab = 8192
    x = rand_bf16(r, (rows, 896), 2.0)
    g = bf16_round(r.uniform(0.5, 1.5, 896).astype(np.float32))
    w, s = rand_weights(r, vocab, 896)
    # plant exact ties: row 0's best direction copied to a lower and a higher index
    hn = ref.rmsnorm(x, g, mode=ref.EXACT)
    best = np.sign(hn[0]).astype(np.int8) * 127
    for j in (100, 4000, 8000):
        w[j], s[j] = best, s.max()
    logits_d = dev(np.zeros((rows, vocab), np.int16))
    toks_d = dev(np.zeros(rows, np.int32))
    ws_bytes = L().qwen_b200_lm_head_workspace(rows, vocab)
    ws = dev(np.zeros(ws_bytes, np.uint8))
    assert L().qwen_b200_op_lm_head_argmax(keep((to_bits(x).view(np.int16))), rows,
                                           keep((to_bits(g).view(np.int16))), ctypes.c_float(1e-6), keep((w)),
                                           keep((s)), vocab, vp(logits_d), vp(toks_d), vp(ws), ws_bytes,
                                           stream()) == 0
    sync()
    exp_logits, exp_toks = lm_oracle(x, g, w, s)
    got_logits = from_bits(host(logits_d).view(np.uint16))
    assert np.array_equal(got_logits, exp_logits)
    got_toks = host(toks_d).view(np.uint32).tolist()
    assert got_toks[0] == 8000  # the highest of the tied indices
    assert got_toks == exp_toks


@pytest.mark.parametrize('vocab', [4, 100, 1000, 4740, 20004])
def test_one_row_lm_head_at_ragged_vocabulary_sizes(vocab):
    """The one-row LM head splits the vocabulary over one CTA per SM (fewer
    for small vocabularies) in 32-row pieces: sizes whose CTA shares end in
    partial pieces, and shares of a few rows, still give the oracle's logits
    and highest-index argmax bit for bit."""
    keep = Keep()
    r = rng(70 + vocab)
    x = rand_bf16(r, (1, 896), 2.0)
    g = bf16_round(r.uniform(0.5, 1.5, 896).astype(np.float32))
    w, s = rand_weights(r, vocab, 896)
    logits_d = dev(np.zeros((1, vocab), np.int16))
    toks_d = dev(np.zeros(1, np.int32))
    ws_bytes = L().qwen_b200_lm_head_workspace(1, vocab)
    ws = dev(np.zeros(ws_bytes, np.uint8))
    assert L().qwen_b200_op_lm_head_argmax(keep((to_bits(x).view(np.int16))), 1, keep((to_bits(g).view(np.int16))),
                                           ctypes.c_float(1e-6), keep((w)), keep((s)), vocab, vp(logits_d),
                                           vp(toks_d), vp(ws), ws_bytes, stream()) == 0
    sync()
    exp_logits, exp_toks = lm_oracle(x, g, w, s)
    assert np.array_equal(from_bits(host(logits_d).view(np.uint16)), exp_logits)
    assert host(toks_d).view(np.uint32).tolist() == exp_toks
