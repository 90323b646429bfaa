"""Continuous-batching scheduler (qwen_b200_sched_*), host logic on CPU:
argument checks and the capacity rule at submit, and that a step on a handle
without a model reports the engine's error instead of running anything (the
reference serves one request at a time, src/software/main.c:243-265; this
scheduler is beyond it)."""
import ctypes

import numpy as np
import pytest

import qwen_b200
from qwen_b200 import _lib


@pytest.fixture
def sched():
    L = qwen_b200.lib()
    cfg = _lib.Config()
    L.qwen_b200_default_config(ctypes.byref(cfg))
    cfg.max_seqs, cfg.max_context = 2, 64
    h = ctypes.c_void_p()
    assert L.qwen_b200_open(ctypes.byref(cfg), ctypes.byref(h)) == 0
    s = ctypes.c_void_p()
    assert L.qwen_b200_sched_open(h, 0, ctypes.byref(s)) == _lib.EINVAL  # a zero prefill budget
    assert L.qwen_b200_sched_open(h, 16, ctypes.byref(s)) == 0
    yield L, h, s
    assert L.qwen_b200_sched_close(s) == 0
    assert L.qwen_b200_close(h) == 0


def test_submit_checks(sched):
    L, h, s = sched
    rid = ctypes.c_uint32()
    ids = (ctypes.c_uint32 * 4)(1, 2, 3, 4)
    assert L.qwen_b200_sched_submit(s, ids, 0, 5, ctypes.byref(rid)) == _lib.EINVAL
    assert L.qwen_b200_sched_submit(s, ids, 4, 0, ctypes.byref(rid)) == _lib.EINVAL
    bad = (ctypes.c_uint32 * 1)(151936)
    assert L.qwen_b200_sched_submit(s, bad, 1, 1, ctypes.byref(rid)) == _lib.EINVAL
    assert L.qwen_b200_sched_submit(s, ids, 4, 61, ctypes.byref(rid)) == _lib.ESTATE  # 65 > capacity 64
    assert L.qwen_b200_sched_submit(s, ids, 4, 60, ctypes.byref(rid)) == 0
    first = rid.value
    assert L.qwen_b200_sched_submit(s, ids, 4, 2, ctypes.byref(rid)) == 0 and rid.value == first + 1
    count, done = ctypes.c_uint32(), ctypes.c_int()
    assert L.qwen_b200_sched_result(s, first, None, 0, ctypes.byref(count), ctypes.byref(done)) == 0
    assert count.value == 0 and done.value == 0
    assert L.qwen_b200_sched_result(s, 999, None, 0, ctypes.byref(count), ctypes.byref(done)) == _lib.EINVAL


def test_step_without_a_model_reports_the_engine_error(sched):
    L, h, s = sched
    rid = ctypes.c_uint32()
    ids = (ctypes.c_uint32 * 3)(5, 6, 7)
    assert L.qwen_b200_sched_submit(s, ids, 3, 2, ctypes.byref(rid)) == 0
    running = ctypes.c_uint32()
    assert L.qwen_b200_sched_step(s, ctypes.byref(running)) == _lib.EINVAL
    assert b'no assets' in L.qwen_b200_last_error(h)
