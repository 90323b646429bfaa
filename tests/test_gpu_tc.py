"""tcgen05 kind::i8 W8A16 projection (the batched-decode path from 2 rows)
against the oracle's exact projection order (REF_EXACT) on identical seeded
inputs, through the C ABI. The sums are exact integers and SiLU uses the
fixed-operation exp of both sides, so every epilogue's output is
bit-identical whatever the split-K plan. Also: the pipeline error flag stays
clear."""
import numpy as np
import pytest

import qwen_b200
from gpu_util import Keep, bf16_round, dev, from_bits, host, stream, sync, to_bits, vp
from oracle import ref

pytestmark = pytest.mark.gpu
L = qwen_b200.lib
X = ref.EXACT


def run_tc(x, w, s, b, y0, epi):
    keep = Keep()
    rows, k = x.shape
    n = w.shape[0]
    yd = dev(to_bits(y0).view(np.int16))
    ws_bytes = L().qwen_b200_gemm_tc_workspace(rows, n, k)
    ws = dev(np.zeros(ws_bytes, np.uint8))
    code = {'plain': 0, 'bias': 1, 'residual': 2, 'swiglu': 3}[epi]
    rc = L().qwen_b200_op_gemm_w8a16_tc(keep(to_bits(x).view(np.int16)), rows, k, keep(w), keep(s), n,
                                        keep(to_bits(b).view(np.int16)) if epi == 'bias' else None, code, vp(yd),
                                        vp(ws), ws_bytes, stream())
    assert rc == 0
    sync()
    assert int(host(ws)[:4].view(np.uint32)[0]) == 0, 'pipeline wait timed out'
    return from_bits(host(yd).view(np.uint16))


def expected(x, w, s, b, y0, epi):
    if epi == 'swiglu':
        return ref.swiglu(ref.linear(x, w[0::2], s[0::2], mode=X), ref.linear(x, w[1::2], s[1::2], mode=X), mode=X)
    if epi == 'residual':
        return ref.f32(np.vectorize(lambda a: ref.lib().ref_bf(a, 0))(y0 + ref.linear(x, w, s, mode=X)))
    return ref.linear(x, w, s, bias=b if epi == 'bias' else None, mode=X)


@pytest.mark.parametrize('k,n,epi', [(896, 896, 'plain'), (896, 1152, 'bias'), (896, 896, 'residual'),
                                     (4864, 896, 'residual'), (896, 9728, 'swiglu')])
@pytest.mark.parametrize('rows', [1, 2, 5, 9, 16, 64, 100, 200])
def test_gemm_tc(k, n, epi, rows):
    r = np.random.default_rng(k + n + rows)
    x = bf16_round(r.standard_normal((rows, k)).astype(np.float32))
    w = r.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = bf16_round(r.uniform(2e-4, 4e-4, size=n).astype(np.float32))
    b = bf16_round(r.standard_normal(n).astype(np.float32) * 0.02)
    y0 = bf16_round(r.standard_normal((rows, n // 2 if epi == 'swiglu' else n)).astype(np.float32))
    got = run_tc(x, w, s, b, y0, epi)
    exp = expected(x, w, s, b, y0, epi)
    assert np.array_equal(got, exp), f'tc gemm {k}x{n} rows {rows} {epi}: {np.mean(got == exp):.5f} bit-equal'


@pytest.mark.parametrize('rows', [12, 64])
def test_gemm_tc_extreme_rows(rows):
    """Rows with a single huge element, all-zero rows, tiny (subnormal-scale)
    rows and max-magnitude codes: the 28-bit alignment and the four limb
    planes must still give the exact sums."""
    k, n = 4864, 896
    r = np.random.default_rng(rows + 7)
    x = bf16_round(r.standard_normal((rows, k)).astype(np.float32))
    x[0] = 0.0
    x[1, 17] = 3.0e4
    x[2] *= 1e-30
    x[3] = -1.0e4
    x = bf16_round(x)
    w = r.integers(-127, 128, size=(n, k), dtype=np.int8)
    w[5] = -128
    w[6] = 127
    s = bf16_round(r.uniform(2e-4, 4e-4, size=n).astype(np.float32))
    y0 = np.zeros((rows, n), np.float32)
    got = run_tc(x, w, s, None, y0, 'plain')
    exp = expected(x, w, s, None, y0, 'plain')
    assert np.array_equal(got, exp), f'{np.mean(got == exp):.5f} bit-equal'


@pytest.mark.parametrize('k,n,epi,rows', [(896, 1152, 'bias', 256), (896, 1152, 'bias', 512),
                                          (896, 1152, 'bias', 4096), (896, 9728, 'swiglu', 256),
                                          (896, 9728, 'swiglu', 512), (896, 9728, 'swiglu', 4096),
                                          (896, 896, 'residual', 3000), (4864, 896, 'residual', 4096),
                                          (896, 896, 'plain', 4096)])
def test_gemm_tc_prefill_rows(k, n, epi, rows):
    """The microbenchmark's M = 512 / 4096 and prefill chunks on the
    projection shapes: many row tiles per channel tile (no split-K; from 296
    tiles the persistent double-buffered kernel, with a ragged last row tile
    at 3000 rows), still bit-identical to the exact projection."""
    r = np.random.default_rng(k + n + rows + 1)
    x = bf16_round(r.standard_normal((rows, k)).astype(np.float32))
    w = r.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = bf16_round(r.uniform(2e-4, 4e-4, size=n).astype(np.float32))
    b = bf16_round(r.standard_normal(n).astype(np.float32) * 0.02)
    y0 = np.zeros((rows, n // 2 if epi == 'swiglu' else n), np.float32)
    if epi == 'residual':
        y0 = bf16_round(r.standard_normal(y0.shape).astype(np.float32))
    got = run_tc(x, w, s, b, y0, epi)
    exp = expected(x, w, s, b, y0, epi)
    assert np.array_equal(got, exp), f'tc gemm {k}x{n} rows {rows} {epi}: {np.mean(got == exp):.5f} bit-equal'
