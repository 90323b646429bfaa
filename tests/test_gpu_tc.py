"""tcgen05 W8A16 GEMM (the batched-decode / prefill path for rows > 8) against
the oracle on identical seeded inputs, through the C ABI. Same bars as the
GEMV: >= 99 % bit-equal bf16, the rest within two ulps (every epilogue rounds
at least twice: bf16(bf16(acc) * scale), so a one-ulp flip of the inner value
can move the output by two). Also: the pipeline error flag stays clear."""
import ctypes

import numpy as np
import pytest

import qwen_b200
from gpu_util import Keep, assert_bf16_close, bf16_round, dev, from_bits, host, stream, sync, to_bits, vp
from oracle import ref

pytestmark = pytest.mark.gpu
L = qwen_b200.lib


def tiled(w):
    n, k = w.shape
    t = np.empty_like(w)
    assert L().qwen_b200_tile_weights(w.ctypes.data_as(ctypes.c_void_p), n, k, t.ctypes.data_as(ctypes.c_void_p)) == 0
    exp = w.reshape(n // 128, 128, k // 64, 16, 4).transpose(0, 2, 1, 3, 4)[..., [0, 2, 1, 3]]
    assert np.array_equal(t.reshape(-1), exp.reshape(-1))
    return t


@pytest.mark.parametrize('k,n,epi', [(896, 896, 'plain'), (896, 1152, 'bias'), (896, 896, 'residual'),
                                     (4864, 896, 'residual'), (896, 9728, 'swiglu')])
@pytest.mark.parametrize('rows', [9, 16, 64, 100, 200])
def test_gemm_tc(k, n, epi, rows):
    keep = Keep()
    r = np.random.default_rng(k + n + rows)
    x = bf16_round(r.standard_normal((rows, k)).astype(np.float32))
    w = r.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = bf16_round(r.uniform(2e-4, 4e-4, size=n).astype(np.float32))
    b = bf16_round(r.standard_normal(n).astype(np.float32) * 0.02)
    lin = None
    out_cols = n // 2 if epi == 'swiglu' else n
    y0 = bf16_round(r.standard_normal((rows, out_cols)).astype(np.float32))
    yd = dev(to_bits(y0).view(np.int16))
    ws_bytes = L().qwen_b200_gemm_tc_workspace(rows, n, k)
    ws = dev(np.zeros(ws_bytes, np.uint8))
    code = {'plain': 0, 'bias': 1, 'residual': 2, 'swiglu': 3}[epi]
    rc = L().qwen_b200_op_gemm_w8a16_tc(keep(to_bits(x).view(np.int16)), rows, k, keep(tiled(w)), keep(s), n,
                                        keep(to_bits(b).view(np.int16)) if epi == 'bias' else None, code, vp(yd),
                                        vp(ws), ws_bytes, stream())
    assert rc == 0
    sync()
    assert int(host(ws)[:4].view(np.uint32)[0]) == 0, 'pipeline wait timed out'
    got = from_bits(host(yd).view(np.uint16))
    if epi == 'swiglu':
        exp = ref.swiglu(ref.linear(x, w[0::2], s[0::2]), ref.linear(x, w[1::2], s[1::2]))
    elif epi == 'residual':
        lin = ref.linear(x, w, s)
        exp = ref.f32(np.vectorize(lambda a: ref.lib().ref_bf(a, 0))(y0 + lin))
    else:
        exp = ref.linear(x, w, s, bias=b if epi == 'bias' else None)
    # residual: a third rounding after a sum that may cancel -> 3 ulps of the
    # larger of the output and the added linear term
    assert_bf16_close(got, exp, max_ulps=3 if epi == 'residual' else 2, mag=lin if epi == 'residual' else None,
                      what=f'tc gemm {k}x{n} rows {rows} {epi}')
