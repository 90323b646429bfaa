"""The persistent batch-1 decode launch (every layer, the LM head and the
argmax in one cooperative kernel) against the per-kernel path of the same
engine: both compute the oracle's exact mode, so tokens and logits must be
bit-identical, through the host forward, the host decode step and the
graph-captured device decode step, at short contexts and at contexts of
several hundred to 1024 keys (synthetic KV8 caches). The oracle comparison
of the persistent path itself is tests/test_gpu_model.py (its single-row
steps take this path)."""
import ctypes

import numpy as np
import pytest

import qwen_b200
from gpu_util import from_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def engine(sd_root):
    e = qwen_b200.Engine(device=0, max_seqs=2, max_context=1100, max_rows=64).load_assets(sd_root)
    yield e
    e.close()


def generate(engine, prompt, steps, persistent):
    engine.set_persistent(persistent)
    engine.reset(0)
    ids, pos, toks, logits = list(prompt), 0, [], []
    for _ in range(steps):
        tok, lg = engine.forward(0, ids, pos, want_logits=True)
        toks.append(tok)
        logits.append(from_bits(lg))
        pos += len(ids)
        ids = [tok]
    engine.set_persistent(True)
    return toks, logits


def test_persistent_forward_equals_per_kernel(engine, golden):
    a_toks, a_logits = generate(engine, golden['prompt'], 8, True)
    b_toks, b_logits = generate(engine, golden['prompt'], 8, False)
    assert a_toks == b_toks
    for i, (a, b) in enumerate(zip(a_logits, b_logits)):
        assert np.array_equal(a, b), f'step {i}'


@pytest.mark.parametrize('length', [90, 300, 1023])
def test_persistent_long_context_equals_per_kernel(engine, golden, length):
    """Synthetic caches of `length` keys, then single-row steps up to the
    1024-key limit of the persistent path (setting 2; the default setting
    hands contexts beyond 96 keys to the per-kernel path)."""
    out = {}
    for persistent in (2, False):
        engine.set_persistent(persistent)
        engine.reset(1)
        engine.fill_kv_synthetic(1, length, 99)
        toks, logits, tok = [], [], golden['prompt'][0]
        for i in range(2 if length == 1023 else 3):
            tok, lg = engine.forward(1, [tok], length + i, want_logits=True)
            toks.append(tok)
            logits.append(from_bits(lg))
        out[persistent] = (toks, logits)
    engine.set_persistent(True)
    assert out[2][0] == out[False][0]
    for a, b in zip(out[2][1], out[False][1]):
        assert np.array_equal(a, b)


@pytest.mark.parametrize('length', [0, 29, 61])
def test_persistent_short_context_edges_equal_per_kernel(engine, golden, length):
    """The fused short-context phase (every CTA attends over at most 64 keys,
    one warp per head, lane = keys lane and lane + 32): single-row steps from
    synthetic caches across its edges, 1..4 keys, 30..33 keys (the second key
    per lane starts at 33) and 62..65 keys (65 leaves the short phase)."""
    out = {}
    for persistent in (True, False):
        engine.set_persistent(persistent)
        engine.reset(1)
        if length:
            engine.fill_kv_synthetic(1, length, 7 + length)
        toks, logits, tok = [], [], golden['prompt'][0]
        for i in range(4):
            tok, lg = engine.forward(1, [tok], length + i, want_logits=True)
            toks.append(tok)
            logits.append(from_bits(lg))
        out[persistent] = (toks, logits)
    engine.set_persistent(True)
    assert out[True][0] == out[False][0]
    for i, (a, b) in enumerate(zip(out[True][1], out[False][1])):
        assert np.array_equal(a, b), f'step {i}'


def test_persistent_device_and_host_decode_steps(engine, golden):
    import torch
    prompt = golden['prompt']

    def run(persistent, device):
        engine.set_persistent(persistent)
        engine.reset(0)
        tok, _ = engine.forward(0, prompt, 0)
        toks = [tok]
        if device:
            bufs = [torch.tensor([tok], dtype=torch.int32, device='cuda'), torch.zeros(1, dtype=torch.int32,
                                                                                       device='cuda')]
            for i in range(5):
                engine.decode_step_device(ctypes.c_void_p(bufs[i % 2].data_ptr()), 1,
                                          ctypes.c_void_p(bufs[(i + 1) % 2].data_ptr()), None)
                torch.cuda.synchronize()
                toks.append(int(bufs[(i + 1) % 2][0].item()))
        else:
            for _ in range(5):
                toks.append(int(engine.decode_step([0], [toks[-1]])[0]))
        return toks

    ref_toks = run(False, False)
    assert run(True, False) == ref_toks
    assert run(True, True) == ref_toks
    engine.set_persistent(True)
