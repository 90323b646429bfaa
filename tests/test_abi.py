"""C ABI (include/qwen_b200.h) on CPU: every declared entry point is exported
by the in-tree libqwen_b200.so, and the host logic that needs no GPU behaves
like the reference's boundary (status codes of generation.h:16, CSR map of
src/software/README.md, request checks of generation.c:8-9)."""
import ctypes
import re
from pathlib import Path

import pytest

import qwen_b200
from qwen_b200 import _lib

from qgen import EngineOps, qgen_run

HEADER = Path(__file__).resolve().parents[1] / 'include' / 'qwen_b200.h'


def declared():
    text = re.sub(r'/\*.*?\*/', '', HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r'\b(qwen_b200_\w+)\s*\(', text)))


def test_every_declared_symbol_is_exported():
    names = declared()
    assert len(names) >= 30
    so = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing


def test_every_declared_symbol_has_a_binding():
    assert set(declared()) <= set(_lib._SIGNATURES), set(declared()) - set(_lib._SIGNATURES)


@pytest.fixture
def handle():
    L = qwen_b200.lib()
    cfg = _lib.Config()
    L.qwen_b200_default_config(ctypes.byref(cfg))
    h = ctypes.c_void_p()
    assert L.qwen_b200_open(ctypes.byref(cfg), ctypes.byref(h)) == 0
    yield L, h
    assert L.qwen_b200_close(h) == 0


def test_default_config_and_bad_config():
    L = qwen_b200.lib()
    cfg = _lib.Config()
    L.qwen_b200_default_config(ctypes.byref(cfg))
    assert (cfg.device, cfg.max_seqs, cfg.max_context, cfg.max_rows) == (0, 1, 256, 256)
    assert abs(cfg.rms_eps - 1e-6) < 1e-12
    cfg.max_context = 0
    h = ctypes.c_void_p()
    assert L.qwen_b200_open(ctypes.byref(cfg), ctypes.byref(h)) == _lib.EINVAL
    assert L.qwen_b200_open(None, None) == _lib.EINVAL


def test_csr_identity_registers(handle):
    L, h = handle
    assert L.qwen_b200_csr_read(h, 0x00) == 0x515732354b563236
    assert L.qwen_b200_csr_read(h, 0x08) == 0x10000
    assert L.qwen_b200_csr_read(h, 0x18) == 0  # idle
    L.qwen_b200_csr_write(h, 0x0140, 255)      # address/config CSRs are accepted (main.c:149-161)
    assert L.qwen_b200_csr_read(h, 0x0140) == 255


def test_csr_rejects_malformed_requests(handle):
    L, h = handle
    L.qwen_b200_embedding(h, 5, 0)
    for mode, seq, ctx, pos in [(0, 0, 0, 0), (0, 1, 2, 0), (0, 1, 3, 2), (1, 1, 2, 1), (0, 300, 300, 0)]:
        L.qwen_b200_csr_write(h, 0x10, 8)  # CLEAR
        for off, v in [(0x80, mode), (0x88, seq), (0x90, ctx), (0x98, pos)]:
            L.qwen_b200_csr_write(h, off, v)
        L.qwen_b200_csr_write(h, 0x10, 1)
        assert L.qwen_b200_csr_read(h, 0x18) == 8, (mode, seq, ctx, pos)
        assert L.qwen_b200_csr_read(h, 0x30) == 1
    L.qwen_b200_embedding(h, 151936, 0)  # out-of-vocab id recorded in ACT_IN row 0
    L.qwen_b200_csr_write(h, 0x10, 8)
    for off, v in [(0x80, 0), (0x88, 1), (0x90, 1), (0x98, 0)]:
        L.qwen_b200_csr_write(h, off, v)
    L.qwen_b200_csr_write(h, 0x10, 1)
    assert L.qwen_b200_csr_read(h, 0x30) == 1


def test_generation_loop_without_model_reports_device_error(handle):
    L, h = handle
    status, res, tokens = qgen_run(EngineOps(L, h), [1, 2, 3], 4)
    assert status == -3 and res.produced == 0 and not tokens
    assert L.qwen_b200_csr_read(h, 0x30) == 3  # no model loaded


def test_sequence_calls_without_model(handle):
    L, h = handle
    tok = ctypes.c_uint32()
    ids = (ctypes.c_uint32 * 2)(1, 2)
    assert L.qwen_b200_forward(h, 0, ids, 2, 0, ctypes.byref(tok), None) == _lib.EINVAL
    assert b'no assets' in L.qwen_b200_last_error(h)
    assert L.qwen_b200_reset(h, 0) == 0
    assert L.qwen_b200_reset(h, 7) == _lib.EINVAL
    assert L.qwen_b200_load_assets(h, b'/nonexistent/sd') == _lib.EIO


def test_op_entry_points_reject_null_pointers():
    L = qwen_b200.lib()
    assert L.qwen_b200_op_embed(None, None, 1, None, None) == _lib.EINVAL
    assert L.qwen_b200_op_attention(None, 1, None, None, 1, None, None, None, None, 16, None, None, 0, None) \
        == _lib.EINVAL
    assert L.qwen_b200_attention_workspace(64, 2048) > 64 * 14 * 2048 * 4
    assert L.qwen_b200_lm_head_workspace(1, 151936) >= 4748 * 8


def test_rope_table_matches_oracle():
    import numpy as np
    from oracle import ref
    t = np.empty((300, 64), np.float32)
    qwen_b200.lib().qwen_b200_rope_table(300, t.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert np.array_equal(t, ref.rope_table(300))


def test_tensor_core_gemm_workspace_and_argument_checks():
    """Workspace = 256-byte error word + the split-K partial tiles of the
    split plan (64 x 128 int64 per tile and split) + four int8 limb planes
    [4][rows][k] + one exponent per row; malformed shapes are rejected before
    any launch."""
    L = qwen_b200.lib()
    tile = 64 * 128 * 8
    # 7 channel tiles, K = 896 (7 chunks): 7 splits; K = 4864: 8 splits
    assert L.qwen_b200_gemm_tc_workspace(64, 896, 896) == 256 + 7 * 7 * tile + 4 * 64 * 896 + 4 * 64
    assert L.qwen_b200_gemm_tc_workspace(9, 896, 4864) == 256 + 7 * 8 * tile + 4 * 9 * 4864 + 4 * 9
    # 76 gate/up tiles: one split, no partial tiles
    assert L.qwen_b200_gemm_tc_workspace(64, 9728, 896) == 256 + 4 * 64 * 896 + 4 * 64
    p = ctypes.c_void_p(16)
    ws = L.qwen_b200_gemm_tc_workspace(16, 896, 896)
    ok = dict(x=p, rows=16, k=896, w=p, scale=p, n=896, bias=None, epi=0, y=p, ws=p, ws_bytes=ws, st=None)

    def call(**kw):
        a = dict(ok, **kw)
        return L.qwen_b200_op_gemm_w8a16_tc(a['x'], a['rows'], a['k'], a['w'], a['scale'], a['n'], a['bias'],
                                            a['epi'], a['y'], a['ws'], a['ws_bytes'], a['st'])
    assert call(x=None) == _lib.EINVAL
    assert call(k=640) == _lib.EINVAL           # only the model's two projection depths
    assert call(n=200) == _lib.EINVAL           # whole 128-row weight tiles
    assert call(rows=0) == _lib.EINVAL
    assert call(epi=1) == _lib.EINVAL           # bias epilogue without a bias
    assert call(epi=7) == _lib.EINVAL
    assert call(ws_bytes=ws - 1) == _lib.EINVAL
